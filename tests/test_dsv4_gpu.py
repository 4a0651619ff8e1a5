"""The reference-facing module API on the GPU: V4ArenaMoE over an HBM store
(direct device path and the host path with an external gate, with fills from
a pack on disk), the dsv4_kernels drop-in, and _gather.  Mirrors the
reference's tests/test_dsv4_arena.py and tests/test_dsv4_kernels.py with the
CPU oracle in place of MLX."""

import numpy as np
import pytest
import torch

from locali_b200 import dsv4_kernels, ops, synth
from locali_b200.dsv4_arena import V4ArenaMoE, V4ArenaStore
from locali_b200.index import write_pack
from locali_b200.router import V4Gate
from oracle import moe_oracle as O
from oracle.bridge import layer_np, qproj_np, t2np

pytestmark = pytest.mark.gpu
LAYER_TOL = 1e-2


class FixedGate:
    """Routing supplied by the test (tests/test_dsv4_arena.py:12-18)."""

    def __init__(self, indices, scores):
        self.indices, self.scores = indices, scores

    def __call__(self, x, input_ids=None):
        return self.indices, self.scores


def test_v4_module_direct_path_matches_oracle(built):
    cfg = synth.config("c2")
    layers = [synth.make_layer(cfg, seed=s, device="cuda") for s in range(2)]
    store = V4ArenaStore.from_layers([l.experts for l in layers], top_k=cfg.top_k, device="cuda")
    x = synth.make_tokens(cfg, 4, seed=3, device="cuda")
    for li in range(2):
        moe = V4ArenaMoE(store, li, V4Gate(layers[li].router), cfg.top_k, swiglu_limit=cfg.swiglu_limit,
                         fused_decode=True)
        out = moe(x)
        torch.cuda.synchronize()
        L = layer_np(layers[li])
        ref = O.moe_layer(t2np(x), L, acc=np.float32)
        assert O.rel_l2(t2np(out), ref["out"]) < 4e-3
        # host path with the same routing gives the same bits
        idx, w = V4Gate(layers[li].router)(x)
        moe_h = V4ArenaMoE(store, li, FixedGate(idx, w), cfg.top_k, swiglu_limit=cfg.swiglu_limit,
                           fused_decode=True)
        out_h = moe_h(x)
        torch.cuda.synchronize()
        assert torch.equal(out, out_h)


def test_v4_module_tiled_store_matches_row_major(built):
    """The store's pre-tiled slot copies (stream GEMVs) agree with the
    row-major arrays (bulk-copy GEMVs) within the layer bar; each is
    repeatable bit for bit."""
    cfg = synth.config("c1", n_experts=16)
    layers = [synth.make_layer(cfg, seed=s, device="cuda") for s in range(2)]
    tiled = V4ArenaStore.from_layers([l.experts for l in layers], top_k=cfg.top_k, device="cuda")
    plain = V4ArenaStore.from_layers([l.experts for l in layers], top_k=cfg.top_k, device="cuda", tiled=False)
    assert tiled.tiles and not plain.tiles
    x = synth.make_tokens(cfg, 1, seed=5, device="cuda")
    for li in range(2):
        mods = [V4ArenaMoE(st, li, V4Gate(layers[li].router), cfg.top_k, swiglu_limit=cfg.swiglu_limit,
                           fused_decode=True) for st in (tiled, plain)]
        outs = [m(x) for m in mods]
        again = mods[0](x)
        torch.cuda.synchronize()
        assert O.rel_l2(t2np(outs[0]), t2np(outs[1])) < 4e-3
        assert torch.equal(outs[0], again)
        ref = O.moe_layer(t2np(x), layer_np(layers[li]), acc=np.float32)
        assert O.rel_l2(t2np(outs[0]), ref["out"]) < 4e-3


@pytest.mark.parametrize("native", [True, False])
def test_v4_module_streams_from_pack_with_small_arena(built, tmp_path, native):
    cfg = synth.config("c0", n_experts=8, top_k=2)
    layers = [synth.make_layer(cfg, seed=s, device="cpu") for s in range(3)]
    idx_path = write_pack(tmp_path / "pack", [l.experts for l in layers], top_k=cfg.top_k)
    per = cfg.expert_bytes() / 1e9
    # 8 usable slots: one layer pins up to 4 while the next claims 4 more
    store = V4ArenaStore(idx_path, native_scheduler=native, ceiling_gb=per * 9.5, threads=2, device="cuda",
                         cache_policy="lru")
    try:
        assert store.slots["cold"] == 9
        x = synth.make_tokens(cfg, 2, seed=9, device="cuda")
        for step in range(4):
            li = step % 3
            gate = V4Gate(synth.layer_to(layers[li], "cuda").router)
            idx, w = gate(x)
            moe = V4ArenaMoE(store, li, FixedGate(idx, w), cfg.top_k, swiglu_limit=cfg.swiglu_limit)
            out = moe(x)
            torch.cuda.synchronize()
            L = layer_np(layers[li], swiglu_mode="stock")
            ref = O.moe_layer(t2np(x), L, idx=t2np(idx).astype(np.int64), w=t2np(w))
            assert O.rel_l2(t2np(out), ref["out"]) < 4e-3
        st = store.stats()
        assert st["misses"] > 0 and st["bytes_read"] > 0 and st["evictions"] > 0
        assert store.tiles  # fills repacked the tiled copies the kernels read
        assert st["scheduler"] == ("c" if native else "python")
    finally:
        store.close()


def test_v4_module_raises_when_arena_cannot_hold_a_layer(built, tmp_path):
    cfg = synth.config("c0", n_experts=8, top_k=2)
    layers = [synth.make_layer(cfg, seed=s, device="cpu") for s in range(2)]
    idx_path = write_pack(tmp_path / "pack", [l.experts for l in layers], top_k=cfg.top_k)
    per = cfg.expert_bytes() / 1e9
    store = V4ArenaStore(idx_path, native_scheduler=False, ceiling_gb=per * 5.5, threads=1, device="cuda")
    try:
        x = synth.make_tokens(cfg, 2, seed=9, device="cuda")
        for li in range(2):
            idx = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32, device="cuda") + 4 * li
            w = torch.full((2, 2), 0.5, device="cuda")
            moe = V4ArenaMoE(store, li, FixedGate(idx, w), cfg.top_k)
            if li == 0:
                moe(x)
            else:  # layer 0 still pins all four usable slots
                with pytest.raises(RuntimeError, match="pinned"):
                    moe(x)
    finally:
        store.close()


def test_eligible_is_decode_only(built):
    ex = synth.make_layer(synth.config("c0", hidden=256, inter=128, n_experts=4, bits_gate=2, bits_up=2,
                                       group_size=128), device="cuda").experts
    up = ex.up
    decode = torch.zeros((1, 1, 1, 256), dtype=torch.bfloat16, device="cuda")
    prefill = torch.zeros((2, 1, 1, 256), dtype=torch.bfloat16, device="cuda")
    idx = torch.tensor([[0, 2]], dtype=torch.int32, device="cuda")
    assert dsv4_kernels.eligible(decode, idx, up.weight, up.scales, up.biases, group_size=128, bits=2)
    assert not dsv4_kernels.eligible(prefill, idx.repeat(2, 1), up.weight, up.scales, up.biases,
                                     group_size=128, bits=2)
    assert not dsv4_kernels.eligible(decode, idx, up.weight, up.scales, up.biases, group_size=32, bits=2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_affine2_swiglu_tracks_stock_qmm(built, dtype):
    """tests/test_dsv4_kernels.py:43-75: fused == stock qmm + clip + silu
    (allclose rtol=atol=2e-3), here on the sm_100a kernels."""
    cfg = synth.config("c0", hidden=256, inter=128, n_experts=4, bits_gate=2, bits_up=2, bits_down=2,
                       group_size=128)
    ex = synth.make_layer(cfg, seed=19, device="cuda", dtype=dtype).experts
    g = torch.Generator(device="cuda").manual_seed(19)
    x = (torch.randn((1, 1, 1, 256), generator=g, device="cuda") * 0.05).to(dtype)
    indices = torch.tensor([[1, 4]], dtype=torch.int32, device="cuda")
    got = dsv4_kernels.fused_affine2_swiglu(x, indices, ex.up.weight, ex.up.scales, ex.up.biases, ex.gate.weight,
                                            ex.gate.scales, ex.gate.biases, group_size=128, limit=10.0)
    torch.cuda.synchronize()
    assert got.shape == (1, 2, 1, 128)
    act = "f16" if dtype == torch.float16 else "bf16"
    xs = np.repeat(t2np(x).reshape(1, -1), 2, axis=0)
    s = t2np(indices).reshape(-1)
    up = O.gather_qmm(xs, qproj_np(ex.up), s, act)
    gate = O.gather_qmm(xs, qproj_np(ex.gate), s, act)
    expected = O.swiglu(up, gate, 10.0, "stock", act)
    np.testing.assert_allclose(t2np(got).reshape(2, -1), expected, rtol=2e-3, atol=2e-3)


def test_gather_returns_reference_shape(built):
    cfg = synth.config("c0")
    layer = synth.make_layer(cfg, seed=5, device="cuda")
    store = V4ArenaStore.from_layers([layer.experts], top_k=cfg.top_k, device="cuda")
    moe = V4ArenaMoE(store, 0, V4Gate(layer.router), cfg.top_k, fused_decode=True)
    x = synth.make_tokens(cfg, 3, seed=1, device="cuda")
    slots = torch.tensor([[1, 2], [3, 1], [16, 5]], dtype=torch.int32, device="cuda")
    y = moe._gather("cold", x.reshape(3, 1, 1, -1), slots)
    torch.cuda.synchronize()
    assert y.shape == (3, 2, 1, cfg.hidden)
    L = layer_np(layer)
    L.expert_slot = np.arange(0, cfg.n_experts + 1)  # ids are slots here
    _, _, _, yr = O.expert_ffn(t2np(x), t2np(slots).astype(np.int64), L)
    assert O.rel_l2(t2np(y).reshape(3, 2, -1), yr) < 4e-3


def test_module_output_dtype_follows_input(built):
    cfg = synth.config("c0")
    layer = synth.make_layer(cfg, seed=6, device="cuda")
    store = V4ArenaStore.from_layers([layer.experts], top_k=cfg.top_k, device="cuda")
    moe = V4ArenaMoE(store, 0, V4Gate(layer.router), cfg.top_k)
    x = synth.make_tokens(cfg, 2, seed=2, device="cuda").float().reshape(1, 2, -1)
    out = moe(x)
    assert out.dtype == torch.float32 and out.shape == x.shape


def test_ops_route_matches_oracle(built):
    cfg = synth.config("c1")
    layer = synth.make_layer(cfg, seed=8, device="cuda")
    x = synth.make_tokens(cfg, 100, seed=4, device="cuda")  # > 64 tokens: separate top-k kernel
    idx, w = ops.route(x, layer.router)
    torch.cuda.synchronize()
    L = layer_np(layer)
    ridx, rw, _, biased = O.router(t2np(x), L.router_weight, L.router_bias, cfg.top_k, "sigmoid",
                                   cfg.routed_scaling)
    ok = ~O.near_ties(biased, cfg.top_k)
    assert np.array_equal(t2np(idx)[ok], ridx[ok])
    np.testing.assert_allclose(t2np(w)[ok], rw[ok], rtol=2e-5, atol=1e-7)
