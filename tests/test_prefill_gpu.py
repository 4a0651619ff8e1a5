"""Parity of the prefill path (tcgen05 grouped GEMM) with the CPU oracle.

The prefill path dequantises each weight once to the activation dtype
(rounding the exact scale * q + bias) and contracts on the tensor cores with
fp32 accumulation.  Tolerances:

* against the oracle with the same rounded weights (``weights="rounded"``):
  4e-3 relative L2 on the layer output, < 5% of bf16 last-place mismatches;
* against the exact-weight oracle (the reference arithmetic): the 1e-2
  relative L2 parity bar.

The routing is the kernel's own (the router kernel is shared with the decode
path and pinned by the decode tests), so expert ties cannot matter.
"""

import numpy as np
import pytest
import torch

from locali_b200 import _lib, ops, synth
from oracle import moe_oracle as O
from oracle.bridge import layer_np, t2np

pytestmark = pytest.mark.gpu

LAYER_TOL = 1e-2
ROUNDED_TOL = 4e-3


def _ulp_mismatch(a, b, dtype="bf16"):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if dtype == "bf16":
        return float(np.mean(O.f32_to_bf16_bits(a) != O.f32_to_bf16_bits(b)))
    return float(np.mean(a.astype(np.float16).view(np.uint16) != b.astype(np.float16).view(np.uint16)))


def _run(cfg, T, path="prefill", seed=0, dtype=torch.bfloat16):
    layer = synth.make_layer(cfg, seed=seed, device="cuda", dtype=dtype)
    x = synth.make_tokens(cfg, T, seed=seed + 100, device="cuda", dtype=dtype)
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused", path=path)
    idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device="cuda")
    out = kern(x, idx=idx, w=w)
    torch.cuda.synchronize()
    kern.ws.check()
    return layer, x, kern, out, idx, w


def _check(cfg, T, seed=0, dtype=torch.bfloat16, tokens=None):
    layer, x, _, out, idx, w = _run(cfg, T, "prefill", seed, dtype)
    dname = "bf16" if dtype == torch.bfloat16 else "f16"
    L = layer_np(layer, dtype=dname)
    sel = np.arange(T) if tokens is None else np.asarray(tokens)
    xn = t2np(x)[sel]
    gi = t2np(idx)[sel].astype(np.int64)
    gw = t2np(w)[sel]
    got = t2np(out)[sel]
    ref_r = O.moe_layer(xn, L, idx=gi, w=gw, weights="rounded")["out"]
    ref_e = O.moe_layer(xn, L, idx=gi, w=gw, weights="exact")["out"]
    err_r = O.rel_l2(got, ref_r)
    err_e = O.rel_l2(got, ref_e)
    assert err_r < ROUNDED_TOL, err_r
    assert _ulp_mismatch(got, ref_r, dname) < 0.05
    assert err_e < LAYER_TOL, err_e
    return err_r, err_e


@pytest.mark.parametrize("bits,gs", [(2, 64), (2, 128), (3, 32), (3, 64), (3, 128), (4, 32), (4, 64), (4, 128),
                                     (8, 32), (8, 64), (8, 128)])
def test_prefill_layer_bits(built, bits, gs):
    # the prefill kernels stream scales in blocks of 8 groups: K % (8 * gs) == 0
    inter = 1024 if gs == 128 else 512
    cfg = synth.config("c0", bits_gate=bits, bits_up=bits, bits_down=bits, group_size=gs, inter=inter)
    _check(cfg, 64, seed=bits + gs)


def test_prefill_mixed_bits(built):
    # C2's mix (gate/up 2-bit, down 4-bit) at C0's width, Zipf-skewed routing
    cfg = synth.config("c0", bits_gate=2, bits_up=2, bits_down=4, zipf=True)
    _check(cfg, 96, seed=3)


def test_prefill_f16(built):
    cfg = synth.config("c0", bits_gate=4, bits_up=4, bits_down=4)
    _check(cfg, 48, seed=5, dtype=torch.float16)


@pytest.mark.parametrize("T", [1, 7, 200, 512])
def test_prefill_ragged_and_multi_chunk(built, T):
    """Token counts per expert from 0 to > 128 (several chunks per expert),
    not multiples of 16."""
    cfg = synth.config("c0", n_experts=16)
    _check(cfg, T, seed=T)


def test_prefill_stock_swiglu_and_scalings(built):
    cfg = synth.config("c0", scoring="sqrtsoftplus", routed_scaling=2.5)
    layer = synth.make_layer(cfg, seed=11, device="cuda")
    x = synth.make_tokens(cfg, 80, seed=12, device="cuda")
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "stock", path="prefill")
    idx = torch.empty((80, cfg.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((80, cfg.top_k), dtype=torch.float32, device="cuda")
    out = kern(x, idx=idx, w=w)
    torch.cuda.synchronize()
    kern.ws.check()
    L = layer_np(layer, swiglu_mode="stock")
    ref = O.moe_layer(t2np(x), L, idx=t2np(idx).astype(np.int64), w=t2np(w), weights="rounded")["out"]
    assert O.rel_l2(t2np(out), ref) < ROUNDED_TOL


def test_prefill_and_decode_agree(built):
    """Same layer and tokens through both paths: identical routing, outputs
    within the parity bar of each other and of the exact oracle."""
    cfg = synth.config("c0")
    T = 64
    layer = synth.make_layer(cfg, seed=21, device="cuda")
    x = synth.make_tokens(cfg, T, seed=22, device="cuda")
    outs, idxs = {}, {}
    for path in ("decode", "prefill"):
        kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused", path=path)
        idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
        outs[path] = kern(x, idx=idx).clone()
        idxs[path] = idx
        torch.cuda.synchronize()
        kern.ws.check()
    assert torch.equal(idxs["decode"], idxs["prefill"])
    assert O.rel_l2(t2np(outs["prefill"]), t2np(outs["decode"])) < LAYER_TOL


def test_prefill_auto_switch_and_workspace_reuse(built):
    """AUTO takes the prefill path once the routes reach its threshold; one
    workspace serves both paths in any order."""
    cfg = synth.config("c0")
    layer = synth.make_layer(cfg, seed=31, device="cuda")
    auto = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused")
    for T in (4, 96, 1, 300, 8):
        x = synth.make_tokens(cfg, T, seed=40 + T, device="cuda")
        got = auto(x).clone()
        want_path = "prefill" if _lib.auto_takes_prefill(T, cfg.top_k, cfg.n_experts) else "decode"
        fresh = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused",
                              path=want_path)
        want = fresh(x)
        torch.cuda.synchronize()
        auto.ws.check()
        assert torch.equal(got, want), T


def test_prefill_repeatable(built):
    cfg = synth.config("c0", bits_gate=2, bits_up=2, bits_down=2)
    layer, x, kern, out, _, _ = _run(cfg, 256, seed=7)
    first = out.clone()
    again = kern(x)
    torch.cuda.synchronize()
    assert torch.equal(first, again)


def test_prefill_c3_sampled_tokens(built):
    """The C3 prefill workload at full size (4096 tokens, DeepSeek-V4-Flash
    expert shapes, 2-bit g64, uniform routing): every token through the
    kernels, 4 tokens checked against the oracle."""
    cfg = synth.config("c3")
    _check(cfg, cfg.tokens, seed=0, tokens=[0, 1111, 2222, 4095])


@pytest.mark.parametrize("T", [1, 5])
def test_three_bit_layer_any_batch(built, T):
    """3-bit codes (MLX's continuous LSB-first bit stream, 8 codes per 3 bytes)
    run on the tcgen05 kernels at every token count: AUTO takes that path even
    for decode batches, and the decode path reports them unsupported."""
    cfg = synth.config("c0", bits_gate=3, bits_up=3, bits_down=3)
    layer = synth.make_layer(cfg, seed=40 + T, device="cuda")
    x = synth.make_tokens(cfg, T, seed=50 + T, device="cuda")
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused")
    idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device="cuda")
    out = kern(x, idx=idx, w=w)
    torch.cuda.synchronize()
    kern.ws.check()
    L = layer_np(layer)
    gi, gw = t2np(idx).astype(np.int64), t2np(w)
    ref_r = O.moe_layer(t2np(x), L, idx=gi, w=gw, weights="rounded")["out"]
    ref_e = O.moe_layer(t2np(x), L, idx=gi, w=gw, weights="exact")["out"]
    assert O.rel_l2(t2np(out), ref_r) < ROUNDED_TOL
    assert O.rel_l2(t2np(out), ref_e) < LAYER_TOL
    dec = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused", path="decode")
    with pytest.raises(Exception):
        dec(x)


def test_three_bit_mixed_with_four_bit_down(built):
    cfg = synth.config("c0", bits_gate=3, bits_up=3, bits_down=4, zipf=True)
    _check(cfg, 72, seed=61)


@pytest.mark.parametrize("T", [1, 3])
def test_wide_hidden_decode_batches_take_tcgen05_path(built, T):
    """Hidden 7168 (DeepSeek-V3 width): its 2-bit code rows are 112 16-byte
    chunks, not a power of two, so the decode GEMVs cannot stage them; AUTO
    runs such layers on the tcgen05 kernels at every token count, and the
    decode path reports them unsupported."""
    cfg = synth.config("c0", hidden=7168, inter=512, n_experts=8, bits_gate=2, bits_up=2, bits_down=2)
    layer = synth.make_layer(cfg, seed=70 + T, device="cuda")
    x = synth.make_tokens(cfg, T, seed=80 + T, device="cuda")
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused")
    idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device="cuda")
    out = kern(x, idx=idx, w=w)
    torch.cuda.synchronize()
    kern.ws.check()
    L = layer_np(layer)
    gi, gw = t2np(idx).astype(np.int64), t2np(w)
    assert O.rel_l2(t2np(out), O.moe_layer(t2np(x), L, idx=gi, w=gw, weights="rounded")["out"]) < ROUNDED_TOL
    assert O.rel_l2(t2np(out), O.moe_layer(t2np(x), L, idx=gi, w=gw, weights="exact")["out"]) < LAYER_TOL
    dec = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused", path="decode")
    with pytest.raises(Exception):
        dec(x)
