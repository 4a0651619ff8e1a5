"""The reference's own hot-path test geometries, run through the product.

* tests/test_dsv4_arena.py:26-96 of the reference: 4 experts, hidden 128,
  inter 128, top-2, 2-bit affine g128, f16 activations (x = 0.05 * N(0,1)),
  fixed routing through an external gate, then a decode-sized call whose
  experts are one resident and one new (``tier_overlap``).
* tests/test_dsv4_engine_small.py:37-190 of the reference: hidden 128, moe
  inter 128, 4 routed experts, top-2, 4-bit affine g32, sqrt-softplus
  scoring, routed scaling 1.5, normalised top-k, two tokens; routed through
  the device router (V4Gate) on the layer entry point.

MLX is not importable here, so the expected values come from the CPU oracle
(the restatement of ``mx.gather_qmm`` and the V4 gate), at the north_star
tolerances: layer output within 1e-2 relative L2 (held at 4e-3 here),
indices identical except near-ties, weights within rtol 2e-5.
"""

import numpy as np
import pytest
import torch

from locali_b200 import ops, synth
from locali_b200.dsv4_arena import V4ArenaMoE, V4ArenaStore
from locali_b200.router import V4Gate
from oracle import moe_oracle as O
from oracle.bridge import layer_np, t2np

pytestmark = pytest.mark.gpu
TOL = 4e-3


class FixedGate:
    """Routing supplied by the test (reference tests/test_dsv4_arena.py:12-18)."""

    def __init__(self, indices, scores):
        self.indices, self.scores = indices, scores

    def __call__(self, x, input_ids=None):
        return self.indices, self.scores


def _arena_geometry_layer():
    cfg = synth.MoEConfig("ref-arena", 128, 4, 2, 128, 2, 2, 2, 128, swiglu_limit=10.0, routed_scaling=1.0,
                          tokens=3)
    return cfg, synth.make_layer(cfg, seed=7, device="cuda", dtype=torch.float16)


def test_reference_arena_geometry_external_gate():
    cfg, layer = _arena_geometry_layer()
    g = torch.Generator().manual_seed(7)
    x = (torch.randn((3, cfg.hidden), generator=g) * 0.05).to(torch.float16).cuda()
    indices = torch.tensor([[0, 2], [0, 2], [2, 0]], dtype=torch.int32, device="cuda")
    scores = torch.tensor([[0.7, 0.3], [0.4, 0.6], [0.2, 0.8]], dtype=torch.float16, device="cuda")
    store = V4ArenaStore.from_layers([layer.experts], top_k=cfg.top_k, device="cuda")
    # the reference default: stock MLX SwiGLU rounding (fused_decode=False)
    moe = V4ArenaMoE(store, 0, FixedGate(indices, scores), cfg.top_k, swiglu_limit=10.0)
    out = moe(x)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and out.shape == x.shape
    L = layer_np(layer, swiglu_mode="stock", dtype="f16")
    ref = O.moe_layer(t2np(x), L, idx=t2np(indices).astype(np.int64), w=t2np(scores), acc=np.float32)
    assert O.rel_l2(t2np(out), ref["out"]) < TOL

    # decode-sized mixed hit/miss: expert 0 was used above, expert 3 is new
    store.tier_overlap = True
    dx = x[:1]
    di = torch.tensor([[0, 3]], dtype=torch.int32, device="cuda")
    ds = torch.tensor([[0.65, 0.35]], dtype=torch.float16, device="cuda")
    moe.gate = FixedGate(di, ds)
    dout = moe(dx)
    torch.cuda.synchronize()
    dref = O.moe_layer(t2np(dx), L, idx=t2np(di).astype(np.int64), w=t2np(ds), acc=np.float32)
    assert O.rel_l2(t2np(dout), dref["out"]) < TOL


def test_reference_engine_small_geometry_device_router():
    cfg = synth.MoEConfig("ref-small", 128, 4, 2, 128, 4, 4, 4, 32, swiglu_limit=10.0, routed_scaling=1.5,
                          tokens=2, scoring="sqrtsoftplus")
    layer = synth.make_layer(cfg, seed=11, device="cuda")
    store = V4ArenaStore.from_layers([layer.experts], top_k=cfg.top_k, device="cuda")
    gate = V4Gate(layer.router)
    moe = V4ArenaMoE(store, 0, gate, cfg.top_k, swiglu_limit=10.0, fused_decode=True)
    L = layer_np(layer)
    for seed in (3, 4, 5):
        x = synth.make_tokens(cfg, 2, seed=seed, device="cuda")
        out = moe(x)  # device path: router, dispatch and experts in one call
        idx, w = gate(x)
        torch.cuda.synchronize()
        ref = O.moe_layer(t2np(x), L, acc=np.float32)
        ok = ~ref["ties"]
        assert np.array_equal(t2np(idx)[ok], ref["idx"][ok])
        np.testing.assert_allclose(t2np(w)[ok], ref["w"][ok], rtol=2e-5, atol=1e-7)
        assert O.rel_l2(t2np(out), ref["out"]) < TOL


@pytest.mark.parametrize("hidden", [128, 192, 320])
@pytest.mark.parametrize("T", [1, 3, 100])
def test_router_widths_below_and_between_256(hidden, T):
    """Router widths that are multiples of 64 but not of 256 (a partial last
    256-column chunk), through the single-launch decode finisher (T <= 64)
    and the tensor-core logits path (T > 64)."""
    cfg = synth.MoEConfig("ref-router", hidden, 16, 4, 128, 4, 4, 4, 32, routed_scaling=1.5, tokens=T)
    layer = synth.make_layer(cfg, seed=hidden + T, device="cuda")
    x = synth.make_tokens(cfg, T, seed=T, device="cuda")
    idx, w = ops.route(x, layer.router)
    torch.cuda.synchronize()
    ref = O.router(t2np(x), t2np(layer.router.weight), t2np(layer.router.bias), cfg.top_k, "sigmoid",
                   cfg.routed_scaling, True)
    r_idx, r_w, _, biased = ref
    ok = ~O.near_ties(biased, cfg.top_k)
    assert np.array_equal(t2np(idx)[ok], r_idx[ok])
    np.testing.assert_allclose(t2np(w)[ok], r_w[ok], rtol=2e-5, atol=1e-7)


@pytest.mark.parametrize("T", [1, 8, 64])
def test_layer_hidden_128_every_decode_batch(T):
    """The whole layer (device router included) at hidden 128, 2-bit g128
    (the arena test's quantisation), over the decode batch sizes."""
    cfg = synth.MoEConfig("h128", 128, 16, 2, 128, 2, 2, 2, 128, routed_scaling=1.0, tokens=T)
    layer = synth.make_layer(cfg, seed=T, device="cuda")
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit)
    x = synth.make_tokens(cfg, T, seed=T + 1, device="cuda")
    idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
    out = kern(x, idx=idx)
    torch.cuda.synchronize()
    kern.ws.check()
    ref = O.moe_layer(t2np(x), layer_np(layer), acc=np.float32)
    ok = ~ref["ties"]
    assert np.array_equal(t2np(idx)[ok], ref["idx"][ok])
    if ok.all():
        assert O.rel_l2(t2np(out), ref["out"]) < TOL
