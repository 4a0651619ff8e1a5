"""The MoE block with the shared expert and the residual add fused into the
combine (lmoe_moe_block), against the oracle restatement of the patched V4
block (dsv4_engine.py:255-261, routed + shared_experts(x)) plus the decoder's
residual add.  Both expert paths; every combine variant (block-local pairs
up to 64 tokens, the counter combine above, the tcgen05 path's combine)."""

import numpy as np
import pytest
import torch

from locali_b200 import ops, synth
from oracle import moe_oracle as O
from oracle.bridge import layer_np, t2np

pytestmark = pytest.mark.gpu


def _setup(T, name="c1", E=32):
    cfg = synth.config(name, n_experts=E, tokens=T)
    layer = synth.make_layer(cfg, seed=40 + T, device="cuda", extra_slots=1)
    shared = E + 1  # the block's shared expert in the slot after the routed experts
    return cfg, layer, shared


@pytest.mark.parametrize("T,path", [(1, "decode"), (8, "decode"), (64, "decode"), (96, "decode"),
                                    (256, "prefill")])
def test_block_matches_oracle(built, T, path):
    cfg, layer, shared = _setup(T)
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, path=path)
    x = synth.make_tokens(cfg, T, seed=7, device="cuda")
    res = synth.make_tokens(cfg, T, seed=8, device="cuda")
    idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
    out = kern.block(x, shared, res, idx=idx)
    torch.cuda.synchronize()
    kern.ws.check()
    ref = O.moe_block(t2np(x), layer_np(layer), shared, t2np(res), acc=np.float32)
    ok = ~ref["ties"]
    assert np.array_equal(t2np(idx)[ok], ref["idx"][ok])
    if ok.all():
        tol = 4e-3 if path == "decode" else 1e-2  # the prefill path rounds each dequantised weight
        assert O.rel_l2(t2np(out), ref["block"]) < tol
    # without the residual the block is routed + shared alone
    out2 = kern.block(x, shared)
    torch.cuda.synchronize()
    ref2 = O.moe_block(t2np(x), layer_np(layer), shared, None, acc=np.float32)
    if ok.all():
        assert O.rel_l2(t2np(out2), ref2["block"]) < (4e-3 if path == "decode" else 1e-2)


@pytest.mark.parametrize("T,path", [(4, "decode"), (96, "decode"), (256, "prefill")])
def test_block_reduces_to_layer_and_in_place_stream(built, T, path):
    cfg, layer, shared = _setup(T)
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, path=path)
    x = synth.make_tokens(cfg, T, seed=9, device="cuda")
    res = synth.make_tokens(cfg, T, seed=10, device="cuda")
    plain = kern(x)
    # no shared expert, no residual: the layer itself, bit for bit
    assert torch.equal(kern.block(x), plain)
    # residual only: one more rounding of (residual + layer)
    want = (res.float() + plain.float()).to(torch.bfloat16)
    assert torch.equal(kern.block(x, -1, res), want)
    # in place: x <- x + block(x), the residual stream of a decoder stack
    full = kern.block(x, shared, x.clone())
    xs = x.clone()
    kern.block(xs, shared, xs, out=xs)
    torch.cuda.synchronize()
    kern.ws.check()
    assert torch.equal(xs, full)


def test_block_rejects_slot_outside_arena(built):
    cfg, layer, _ = _setup(1)
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit)
    x = synth.make_tokens(cfg, 1, seed=1, device="cuda")
    with pytest.raises(Exception):
        kern.block(x, layer.experts.n_slots)
