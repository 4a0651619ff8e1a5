"""Host-side arena behaviour on CPU: slot API, policy, fills from a pack,
device slot table bookkeeping (the arrays live on the CPU here; kernels are
not involved)."""

import numpy as np
import pytest
import torch

from locali_b200 import synth
from locali_b200.arena import ArenaStore
from locali_b200.dsv4_arena import V4ArenaStore
from locali_b200.index import write_pack


def _tiny_cfg():
    return synth.config("c0", hidden=256, inter=64, n_experts=6, top_k=2)


@pytest.fixture()
def pack(tmp_path):
    cfg = _tiny_cfg()
    layers = [synth.make_layer(cfg, seed=s, device="cpu") for s in range(3)]
    idx = write_pack(tmp_path / "pack", [l.experts for l in layers], top_k=cfg.top_k)
    return cfg, layers, idx


def _item_gb(store):
    return store.item["cold"] / 1e9


def test_fill_copies_exact_bytes_and_table(pack):
    cfg, layers, idx = pack
    store = ArenaStore(idx, ceiling_gb=0.01, threads=2, device="cpu")
    try:
        placed = store.slots_for(1, [3, 0, 3])
        assert set(placed) == {3, 0}
        for e, (t, s) in placed.items():
            q = layers[1].experts.gate
            assert torch.equal(store.arena[(t, "gate_proj", "weight")][s], q.weight[e + 1])
            assert torch.equal(store.arena[(t, "down_proj", "scales")][s], layers[1].experts.down.scales[e + 1])
            assert int(store.slot_table[1, e]) == s
        assert int(store.slot_table[1, 1]) == -1
        assert store.stats()["misses"] == 2 and store.stats()["hits"] == 0
        store.slots_for(1, [3])
        assert store.stats()["hits"] == 1
        assert torch.all(store.arena[("cold", "up_proj", "weight")][0] == 0)  # zero slot untouched
    finally:
        store.close()


def test_lru_eviction_updates_table_and_respects_pins(pack):
    cfg, layers, idx = pack
    probe = ArenaStore(idx, ceiling_gb=0.01, threads=1, device="cpu")
    per = _item_gb(probe)
    probe.close()
    store = ArenaStore(idx, ceiling_gb=per * 4.5, threads=1, device="cpu")  # zero slot + 3 usable
    try:
        assert store.slots["cold"] == 4
        a = store.slots_for(0, [0, 1])
        store.slots_for(1, [2])  # a free slot is left
        assert store.evictions == 0
        # layer 2 needs a slot: the least recent entry not pinned by layer 1 goes
        c = store.slots_for(2, [3])
        assert store.evictions == 1
        (s3,) = [s for _, s in c.values()]
        assert s3 == a[0][1]  # (0, 0) was the least recently used
        assert int(store.slot_table[0, 0]) == -1 and int(store.slot_table[2, 3]) == s3
        assert int(store.slot_table[1, 2]) >= 1  # pinned by the previous layer, kept
        with pytest.raises(ValueError):
            store.slots_for(1, [0, 1, 3, 4])  # more missing experts than usable slots
    finally:
        store.close()


def test_native_scheduler_store_matches_python_policy(pack):
    cfg, layers, idx = pack
    probe = ArenaStore(idx, ceiling_gb=0.01, threads=1, device="cpu")
    per = _item_gb(probe)
    probe.close()
    seq = [(0, [0, 1]), (1, [2, 3]), (0, [0, 4]), (2, [5, 1]), (0, [0, 1]), (1, [2, 5])]
    py = V4ArenaStore(idx, native_scheduler=False, ceiling_gb=per * 5.5, threads=1, device="cpu")
    nat = V4ArenaStore(idx, native_scheduler=True, ceiling_gb=per * 5.5, threads=1, device="cpu")
    try:
        assert nat.native_caches and not py.native_caches
        for layer, experts in seq:
            a = py.slots_for(layer, experts)
            b = nat.slots_for(layer, experts)
            assert a == b
        assert py.stats()["hits"] == nat.stats()["hits"]
        assert py.stats()["evictions"] == nat.stats()["evictions"]
        assert nat.stats()["scheduler"] == "c"
        assert np.array_equal(py._table_host, nat._table_host)
    finally:
        py.close()
        nat.close()


def test_prefetch_is_best_effort_and_accounted(pack):
    cfg, layers, idx = pack
    store = ArenaStore(idx, ceiling_gb=0.01, threads=2, device="cpu")
    try:
        store.slots_for(0, [0, 1])
        placed, reads = store.submit(1, [4, 5], prefetch=True)
        store.wait([f for fs in reads.values() for f in fs])
        assert store.prefetched == 2 and store.stats()["misses"] == 2
        store.slots_for(1, [4])
        assert store.prefetch_used == 1
    finally:
        store.close()


def test_v4_quant_inference_and_metadata(pack):
    cfg, layers, idx = pack
    store = V4ArenaStore(idx, ceiling_gb=0.01, threads=1, device="cpu")
    try:
        assert store.quant("cold", "bits") == cfg.bits_gate
        assert store.quant("cold", "group_size", "down_proj") == cfg.group_size
        assert store.quant("cold", "bits", "down_proj") == cfg.bits_down
        assert store.use_f16_moe["cold"] is False
        assert store.tier(2, 5) == "cold"
    finally:
        store.close()


def test_bad_policy_rejected(pack):
    _, _, idx = pack
    with pytest.raises(ValueError):
        ArenaStore(idx, cache_policy="fifo", device="cpu")


def test_demand_that_evicts_its_own_hit_is_refused(pack):
    """The reference policy pins the previous demand's slots, not this call's
    hits; when this call's misses can only take a hit's slot, the store
    refuses instead of handing out a slot that another expert refills."""
    cfg, layers, idx = pack
    probe = ArenaStore(idx, ceiling_gb=1.0, threads=1, device="cpu")
    per = _item_gb(probe)
    probe.close()
    store = ArenaStore(idx, ceiling_gb=per * 5.5, threads=1, device="cpu")  # 4 usable slots
    try:
        assert store.slots["cold"] == 5
        store.slots_for(0, [0, 1])          # pinned: layer 0's two slots
        store.slots_for(1, [4, 5])          # fills the two free slots; pins them
        store.slots_for(0, [0, 1])          # hits; pins layer 0 again
        with pytest.raises(RuntimeError, match="evicted by other experts of the same layer"):
            store.slots_for(1, [4, 5, 2])   # 4, 5 hit; 2 can only evict 4 or 5
    finally:
        store.close()
