"""The layer calls the reference's ArenaMoE splits (arena.py:508-672), on the
device kernels, against the oracle:

* a layer whose experts span two tiers (separate arenas): each tier's own
  routes, then the fp32 scatter-add of y * g in tier order
  (arena.py:625-672);
* ``overlap_hits`` at batch 1: the resident experts run while the missing
  ones are still being filled, and the result equals the one-call path bit
  for bit (arena.py:575-618);
* cross-layer prefetch from a resident layer on the device path: the next
  layer's routing runs on the device and only that small result is waited
  on before its fills are submitted (arena.py:520-541).
"""

import json
import time

import numpy as np
import pytest
import torch

from locali_b200 import synth
from locali_b200.dsv4_arena import V4ArenaMoE, V4ArenaStore
from locali_b200.index import write_pack
from locali_b200.router import V4Gate
from oracle import moe_oracle as O
from oracle.bridge import layer_np, t2np

pytestmark = pytest.mark.gpu


class FixedGate:
    def __init__(self, indices, scores):
        self.indices, self.scores = indices, scores

    def __call__(self, x, input_ids=None):
        return self.indices, self.scores


def _pack(tmp_path, n_layers=2, E=8, k=2, hot=()):
    cfg = synth.config("c0", n_experts=E, top_k=k)
    layers = [synth.make_layer(cfg, seed=s, device="cpu") for s in range(n_layers)]
    idx_path = write_pack(tmp_path / "pack", [l.experts for l in layers], top_k=k)
    if hot:
        idx = json.loads(idx_path.read_text())
        for l in range(n_layers):
            for e in hot:
                idx["experts"][f"L{l}.E{e}"]["tier"] = "hot"
        idx["quantization"]["hot"] = dict(idx["quantization"]["cold"])
        idx_path.write_text(json.dumps(idx))
    return cfg, layers, idx_path


def test_two_tier_layer_matches_oracle(built, tmp_path):
    cfg, layers, idx_path = _pack(tmp_path, hot=(0, 1, 2, 3))
    per = cfg.expert_bytes() / 1e9
    store = V4ArenaStore(idx_path, native_scheduler=False, ceiling_gb=per * 40, threads=2, device="cuda")
    try:
        assert store.tiers == ["cold", "hot"]
        T = 4
        x = synth.make_tokens(cfg, T, seed=3, device="cuda")
        # every token mixes a hot (0-3) and a cold (4-7) expert, in both route orders
        idx = torch.tensor([[5, 1], [0, 7], [2, 3], [6, 4]], dtype=torch.int32, device="cuda")
        w = torch.tensor([[0.6, 0.4], [0.3, 0.7], [0.5, 0.5], [0.2, 0.8]], dtype=torch.float32, device="cuda")
        moe = V4ArenaMoE(store, 0, FixedGate(idx, w), cfg.top_k, swiglu_limit=cfg.swiglu_limit)
        out = moe(x)
        torch.cuda.synchronize()
        assert moe.last_apply == "tiers"
        L = layer_np(layers[0], swiglu_mode="stock")
        _, _, _, y = O.expert_ffn(t2np(x), t2np(idx).astype(np.int64), L, np.float32)
        g = O.round_act(t2np(w), "bf16")
        ref = np.zeros((T, cfg.hidden), np.float32)
        for t in range(T):
            tiers = ["hot" if e < 4 else "cold" for e in t2np(idx)[t]]
            for j in sorted(range(cfg.top_k), key=lambda j: (["cold", "hot"].index(tiers[j]), j)):
                ref[t] += y[t, j] * g[t, j]
        ref = O.round_act(ref, "bf16")
        assert O.rel_l2(t2np(out), ref) < 4e-3
        # a single-tier token batch still takes the one-call path
        idx1 = torch.tensor([[4, 6]], dtype=torch.int32, device="cuda")
        moe.gate = FixedGate(idx1, w[:1])
        moe(x[:1])
        assert moe.last_apply == "single"
    finally:
        store.close()


def test_overlap_hits_equals_one_call_path(built, tmp_path):
    cfg, layers, idx_path = _pack(tmp_path, n_layers=1, E=8, k=3)
    per = cfg.expert_bytes() / 1e9
    x = synth.make_tokens(cfg, 1, seed=4, device="cuda")
    first = torch.tensor([[0, 1, 2]], dtype=torch.int32, device="cuda")
    second = torch.tensor([[1, 5, 2]], dtype=torch.int32, device="cuda")  # 5 is new: filled during the call
    w = torch.tensor([[0.5, 0.3, 0.2]], dtype=torch.float32, device="cuda")
    outs = {}
    for overlap in (False, True):
        store = V4ArenaStore(idx_path, native_scheduler=False, ceiling_gb=per * 9.5, threads=2, device="cuda")
        try:
            fill = store._fill

            def slow_fill(*a, _fill=fill):
                time.sleep(0.2)  # the read is still in flight when the layer call starts
                return _fill(*a)

            moe = V4ArenaMoE(store, 0, FixedGate(first, w), cfg.top_k, swiglu_limit=cfg.swiglu_limit,
                             overlap_hits=overlap)
            moe(x)
            store._fill = slow_fill
            moe.gate = FixedGate(second, w)
            outs[overlap] = moe(x)
            torch.cuda.synchronize()
            assert moe.last_apply == ("overlap" if overlap else "single")
        finally:
            store.close()
    assert torch.equal(outs[True], outs[False])
    ref = O.moe_layer(t2np(x), layer_np(layers[0], swiglu_mode="stock"), idx=t2np(second).astype(np.int64),
                      w=t2np(w))
    assert O.rel_l2(t2np(outs[True]), ref["out"]) < 4e-3


def test_device_path_prefetches_next_layer(built, tmp_path):
    cfg, layers, idx_path = _pack(tmp_path, n_layers=2, E=8, k=2)
    per = cfg.expert_bytes() / 1e9
    # room for layer 0 (8 experts, pinned) and all of layer 1's demand
    store = V4ArenaStore(idx_path, native_scheduler=False, ceiling_gb=per * 16.5, threads=2, device="cuda")
    try:
        store.make_resident([0])
        assert store.layer_resident(0) and not store.layer_resident(1)
        gates = [V4Gate(synth.layer_to(l, "cuda").router) for l in layers]
        m0 = V4ArenaMoE(store, 0, gates[0], cfg.top_k, swiglu_limit=cfg.swiglu_limit, fused_decode=True)
        m1 = V4ArenaMoE(store, 1, gates[1], cfg.top_k, swiglu_limit=cfg.swiglu_limit, fused_decode=True)
        m0.nxt = m1
        x = synth.make_tokens(cfg, 3, seed=5, device="cuda")
        out0 = m0(x)
        torch.cuda.synchronize()
        assert m0.last_path == "device" and m0.last_prefetch == [1]
        assert store.prefetched > 0
        ref0 = O.moe_layer(t2np(x), layer_np(layers[0]), acc=np.float32)
        assert O.rel_l2(t2np(out0), ref0["out"]) < 4e-3
        # the next layer finds (some of) its experts already placed
        out1 = m1(x)
        torch.cuda.synchronize()
        assert store.prefetch_used > 0
        ref1 = O.moe_layer(t2np(x), layer_np(layers[1]), acc=np.float32)
        assert O.rel_l2(t2np(out1), ref1["out"]) < 4e-3
    finally:
        store.close()
