"""The allocation-free layer entry point (lmoe_moe_layer_static).

It exists for callers that cannot allocate device memory for a workspace;
its scratch is a fixed 8 MiB static device array inside liblmoe.so.  These
tests call it through the C ABI and check it against lmoe_moe_layer (which
uses a caller-allocated workspace) on two calls in a row, within the layer
tolerance the other GPU tests use.  This file is collected last on purpose,
and it also passes when run on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from locali_b200 import _lib, ops, synth
from oracle import moe_oracle as O
from oracle.bridge import t2np

pytestmark = pytest.mark.gpu
LAYER_TOL = 1e-2


@pytest.mark.parametrize("name,T", [("c1", 1), ("c0", 8), ("c2", 16)])
def test_static_entry_matches_workspace_entry_twice(built, name, T):
    cfg = synth.config(name)
    layer = synth.make_layer(cfg, seed=31, device="cuda")
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit)
    xs = [synth.make_tokens(cfg, T, seed=40 + i, device="cuda") for i in range(2)]
    for x in xs:  # two calls in a row through the static scratch
        want = kern(x)
        idx_a = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
        got = kern.call_static(x, idx=idx_a)
        torch.cuda.synchronize()
        assert O.rel_l2(t2np(got), t2np(want)) < LAYER_TOL
        idx_b, _ = kern.route(x)
        torch.cuda.synchronize()
        assert np.array_equal(t2np(idx_a), t2np(idx_b))


def test_static_entry_rejects_oversize_without_launching(built):
    lib = _lib.lmoe()
    cap = lib.lmoe_static_workspace_bytes()
    assert cap == 8 << 20
    cfg = synth.config("c1")
    layer = synth.make_layer(cfg, seed=1, device="cuda")
    # the allocation-free entry always runs the decode path: size with it
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, path="decode")
    big = 1
    while kern.workspace_bytes(big) <= cap:
        big *= 2
    x = torch.zeros((big, cfg.hidden), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    rc = lib.lmoe_moe_layer_static(ctypes.byref(kern.desc), x.data_ptr(), big, out.data_ptr(), None, None,
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LMOE_EWORKSPACE
