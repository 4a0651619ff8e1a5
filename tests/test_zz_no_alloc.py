"""The allocation-free layer entry point (lmoe_moe_layer_static).

It exists for callers that cannot allocate device memory for a workspace;
its scratch is a fixed 8 MiB static device array inside liblmoe.so.  These
tests call it through the C ABI and check it against lmoe_moe_layer (which
uses a caller-allocated workspace) on two calls in a row.  At these token
counts both entry points run the decode kernels, so the outputs must be
identical bit for bit.  This file is collected last on purpose, and it also
passes when run on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from locali_b200 import _lib, ops, synth
from oracle.bridge import t2np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,T", [("c1", 1), ("c0", 8), ("c2", 16)])
def test_static_entry_matches_workspace_entry_twice(built, name, T):
    cfg = synth.config(name)
    layer = synth.make_layer(cfg, seed=31, device="cuda")
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit)
    assert not _lib.auto_takes_prefill(T, cfg.top_k, cfg.n_experts)  # same (decode) path on both
    xs = [synth.make_tokens(cfg, T, seed=40 + i, device="cuda") for i in range(2)]
    for x in xs:  # two calls in a row through the static scratch
        want = kern(x)
        idx_a = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
        got = kern.call_static(x, idx=idx_a)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        idx_b, _ = kern.route(x)
        torch.cuda.synchronize()
        assert np.array_equal(t2np(idx_a), t2np(idx_b))
    ops.static_status()  # no device error was flagged


def test_static_entry_reports_bad_slot(built):
    """A slot table entry outside the arena is flagged on the static scratch
    (LMOE_EINDEX through lmoe_static_status), contributes zeros like the zero
    slot, and the flag is cleared by reading it."""
    cfg = synth.config("c0")
    layer = synth.make_layer(cfg, seed=2, device="cuda")
    bad = layer.expert_slot.clone()
    bad[3] = 10_000
    kern = ops.MoEKernel(layer.router, layer.experts, bad, cfg.swiglu_limit)
    zero = layer.expert_slot.clone()
    zero[3] = 0
    kern0 = ops.MoEKernel(layer.router, layer.experts, zero, cfg.swiglu_limit)
    x = synth.make_tokens(cfg, 8, seed=3, device="cuda")
    idx, _ = kern0.route(x)
    torch.cuda.synchronize()
    assert bool((idx == 3).any())  # expert 3 is selected, so its bad slot is met
    got = kern.call_static(x)
    torch.cuda.synchronize()
    rc = _lib.lmoe().lmoe_static_status(torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LMOE_EINDEX
    ops.static_status()  # cleared by the read above
    want = kern0.call_static(x)
    torch.cuda.synchronize()
    ops.static_status()
    assert torch.equal(got, want)


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
