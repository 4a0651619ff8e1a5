"""Slot planner parity: this project's C++ planner (liblocali_core.so) against
(1) a plain-Python SLRU model of the reference's policy, (2) the reference
unit tests' expectations (native/test_locali_core.c:14-80 and
tests/test_locali_native.py:84-122), (3) golden plans recorded from the
reference C core, and (4) the reference C core itself compiled into
oracle/_ref/ when it is present."""

import json
import random
from collections import OrderedDict
from pathlib import Path

import pytest

from locali_b200.native import NativeCache

ROOT = Path(__file__).resolve().parents[1]
REF_LIB = ROOT / "oracle" / "_ref" / "liblocali_core_ref.so"
GOLDEN = ROOT / "tests" / "golden" / "ref_planner.json"


class SlruModel:
    """Python statement of the reference SLRU policy (locali_core.c:79-141)."""

    def __init__(self, slots, protected_capacity):
        self.protected_capacity = protected_capacity
        self.probation_capacity = slots - 1 - protected_capacity
        self.free = list(range(1, slots))
        self.probation = OrderedDict()
        self.protected = OrderedDict()

    def slot_of(self, key):
        return self.probation.get(key, self.protected.get(key, -1))

    def plan(self, key, pinned=(), touch=True):
        if key in self.protected:
            if touch:
                self.protected.move_to_end(key)
            return self.protected[key], True, -1, True
        if key in self.probation:
            slot = self.probation[key]
            if touch and self.protected_capacity:
                del self.probation[key]
                self.protected[key] = slot
                if len(self.protected) > self.protected_capacity:
                    old, old_slot = self.protected.popitem(last=False)
                    self.probation[old] = old_slot
            elif touch:
                self.probation.move_to_end(key)
            return slot, True, -1, True
        full = len(self.probation) >= self.probation_capacity
        victim, src = None, None
        if full or not self.free:
            victim = next((k for k, s in self.probation.items() if s not in pinned), None)
            src = self.probation
        if victim is None and not full and self.free:
            slot, evicted = self.free.pop(), -1
        else:
            if victim is None:
                victim = next((k for k, s in self.protected.items() if s not in pinned), None)
                src = self.protected
            if victim is None:
                return -1, False, -1, False
            slot, evicted = src.pop(victim), victim
        self.probation[key] = slot
        return slot, False, evicted, True


@pytest.mark.parametrize("protected_capacity", [0, 3])
def test_matches_slru_model_fixed_sequence(built, protected_capacity):
    native = NativeCache(64, 8, protected_capacity)
    model = SlruModel(8, protected_capacity)
    seq = [0, 1, 2, 3, 0, 4, 5, 1, 6, 7, 2, 8, 0, 9, 3, 10]
    try:
        for pos, key in enumerate(seq):
            resident = sorted(s for s in range(1, 8) if s in model.probation.values() or s in model.protected.values())
            pinned = resident[:1] if pos % 4 == 3 else []
            exp = model.plan(key, pinned=pinned)
            got = native.plan([key], pinned_slots=pinned)[0]
            assert (got.slot, got.hit, got.evicted_key, got.placed) == exp
            assert native.probation_size == len(model.probation)
            assert native.protected_size == len(model.protected)
            for k in range(11):
                assert native.peek(k) == model.slot_of(k)
    finally:
        native.close()


@pytest.mark.parametrize("seed", range(6))
def test_matches_slru_model_random(built, seed):
    rng = random.Random(seed)
    slots, prot = rng.choice([(3, 0), (5, 2), (8, 3), (16, 7)])
    native = NativeCache(40, slots, prot)
    model = SlruModel(slots, prot)
    try:
        for _ in range(400):
            key = rng.randrange(40)
            resident = [model.slot_of(k) for k in range(40) if model.slot_of(k) > 0]
            pinned = rng.sample(resident, min(len(resident), rng.randrange(3))) if resident else []
            touch = rng.random() < 0.8
            exp = model.plan(key, pinned=pinned, touch=touch)
            got = native.plan([key], pinned_slots=pinned, touch_hits=touch)[0]
            assert (got.slot, got.hit, got.evicted_key, got.placed) == exp
    finally:
        native.close()


def _one(cache, key, touch=True):
    return cache.plan([key], touch_hits=touch)[0]


def test_reference_unit_expectations(built):
    c = NativeCache(16, 4, 0)  # LRU order (test_locali_core.c:14-27)
    assert _one(c, 1).slot == 3 and _one(c, 2).slot == 2 and _one(c, 3).slot == 1
    assert _one(c, 1).hit
    r = _one(c, 4)
    assert not r.hit and r.evicted_key == 2 and r.slot == 2
    assert c.peek(1) == 3 and c.peek(2) == -1
    c.close()
    c = NativeCache(16, 5, 2)  # SLRU reservation and promotion (:29-45)
    assert _one(c, 0).slot == 4 and _one(c, 1).slot == 3
    r = _one(c, 2)
    assert r.evicted_key == 0 and r.slot == 4 and c.probation_size == 2
    assert _one(c, 1).hit and c.probation_size == 1 and c.protected_size == 1
    assert _one(c, 3).slot == 2
    assert _one(c, 2).hit and c.protected_size == 2
    c.close()
    c = NativeCache(8, 3, 0)  # pinned slots are not reused (:47-60)
    first = c.plan([0, 1])
    r = c.plan([2], pinned_slots=[first[0].slot, first[1].slot])[0]
    assert not r.placed and r.slot == -1
    c.close()


def test_lfu_decay_prefers_frequency_then_recency(built):
    c = NativeCache(16, 3, 0, policy="lfu-decay")
    try:
        assert not _one(c, 1).hit
        assert _one(c, 1).hit
        assert not _one(c, 2).hit
        assert _one(c, 3).evicted_key == 2
        for _ in range(16):
            c.note_token()
        assert _one(c, 4).evicted_key == 3
        assert c.peek(1) >= 0
    finally:
        c.close()


def test_invalid_keys_and_arguments(built):
    c = NativeCache(4, 3, 0)
    with pytest.raises(ValueError):
        c.plan([7])
    with pytest.raises(MemoryError):
        NativeCache(4, 1, 0)
    with pytest.raises(ValueError):
        NativeCache(4, 3, 0, policy="fifo")
    c.close()


def _replay(cache, ops):
    out = []
    for op in ops:
        if op[0] == "plan":
            _, keys, pinned, touch = op
            out.append([[r.slot, int(r.hit), r.evicted_key, int(r.placed)] for r in
                        cache.plan(keys, pinned_slots=pinned, touch_hits=bool(touch))])
            out.append([cache.probation_size, cache.protected_size])
        else:
            cache.note_token()
    return out


def test_golden_plans_recorded_from_reference_core(built):
    data = json.loads(GOLDEN.read_text())
    assert data["source"] == "reference native/locali_core.c"
    for case in data["cases"]:
        c = NativeCache(case["keys"], case["slots"], case["protected"], policy=case["policy"])
        try:
            assert _replay(c, case["ops"]) == case["expect"], case["name"]
        finally:
            c.close()


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference core not built into oracle/_ref")
@pytest.mark.parametrize("policy", ["slru", "lfu-decay"])
@pytest.mark.parametrize("seed", range(4))
def test_live_against_reference_core(built, policy, seed):
    from tests.golden.make_golden import random_ops

    case = random_ops(seed + 100, policy)
    ours = NativeCache(case["keys"], case["slots"], case["protected"], policy=policy)
    ref = NativeCache(case["keys"], case["slots"], case["protected"], policy=policy, library=REF_LIB)
    try:
        assert _replay(ours, case["ops"]) == _replay(ref, case["ops"])
    finally:
        ours.close()
        ref.close()
