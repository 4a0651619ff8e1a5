"""Single-token decode with the top-k selected inside the stream gate/up
kernel (the router kernel then only computes the scores).

The fused call must give the routing of the separate finisher (arena.py:501-506:
selection on score + bias, ties to the lower id, weights normalised by the
fp32 sum in selection order, times the routed scaling) and the same layer
output bit for bit.  The staged entry (events after routing and after
gate/up) always takes the separate finisher, so it is the comparison arm.
"""

import dataclasses

import numpy as np
import pytest
import torch

from locali_b200 import ops, synth
from oracle import moe_oracle as O
from oracle.bridge import t2np

pytestmark = pytest.mark.gpu


def _kern(cfg, seed, slot_perm=False, norm=True):
    layer = synth.make_layer(cfg, seed=seed, device="cuda")
    layer.experts.pack_tiles()
    r = layer.router
    if not norm:
        r = dataclasses.replace(r, norm_topk=False)
    slot = layer.expert_slot
    if slot_perm:
        g = torch.Generator().manual_seed(seed)
        slot = (torch.randperm(cfg.n_experts, generator=g) + 1).to(torch.int32).cuda()
    kern = ops.MoEKernel(r, layer.experts, slot, cfg.swiglu_limit, "fused")
    return layer, r, slot, kern


@pytest.mark.parametrize("scoring,E,k,norm,perm", [
    ("sigmoid", 256, 6, True, False),
    ("sigmoid", 256, 8, True, True),
    ("sqrtsoftplus", 64, 6, True, True),
    ("sigmoid", 384, 16, False, True),
    ("sigmoid", 8, 1, True, False),
])
def test_fused_topk_matches_finisher(built, scoring, E, k, norm, perm):
    cfg = synth.config("c1", n_experts=E, top_k=k, scoring=scoring, inter=1024)
    layer, r, slot, kern = _kern(cfg, seed=E + k, slot_perm=perm, norm=norm)
    for s in range(4):
        x = synth.make_tokens(cfg, 1, seed=50 + s, device="cuda")
        idx_f = torch.full((1, k), -7, dtype=torch.int32, device="cuda")
        w_f = torch.full((1, k), -7.0, dtype=torch.float32, device="cuda")
        out_f = kern(x, idx=idx_f, w=w_f).clone()
        out_s = torch.empty_like(out_f)
        e1, e2 = torch.cuda.Event(), torch.cuda.Event()
        kern.staged(x, out_s, e1, e2)
        idx_r, w_r = kern.route(x)
        torch.cuda.synchronize()
        kern.ws.check()
        assert torch.equal(out_f, out_s)
        assert torch.equal(idx_f, idx_r.reshape(1, k).to(torch.int32))
        assert torch.equal(w_f, w_r.reshape(1, k).float())
        # the oracle's selection (fp64 logits; a near-tie may flip)
        ridx, _, _, biased = O.router(t2np(x), t2np(r.weight), t2np(r.bias), k, scoring, r.routed_scaling,
                                      r.norm_topk)
        srt = np.sort(biased[0])[::-1]
        if k == E or srt[k - 1] - srt[k] > 1e-5:
            assert set(t2np(idx_f)[0].tolist()) == set(ridx[0].tolist())


def test_timed_entry_keeps_the_fused_launches(built):
    """lmoe_moe_layer_timed records its events at kernel boundaries without
    switching to the separate finisher: same output and routing as the plain
    call, and as the staged entry that does switch."""
    cfg = synth.config("c1", n_experts=256, top_k=6, inter=1024)
    layer, r, slot, kern = _kern(cfg, seed=21, slot_perm=True)
    for s in range(3):
        x = synth.make_tokens(cfg, 1, seed=70 + s, device="cuda")
        idx_p = torch.full((1, 6), -7, dtype=torch.int32, device="cuda")
        out_p = kern(x, idx=idx_p).clone()
        out_t = torch.empty_like(out_p)
        idx_t = torch.full((1, 6), -7, dtype=torch.int32, device="cuda")
        e1, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        kern.timed(x, out_t, e1, e2, idx=idx_t)
        out_s = torch.empty_like(out_p)
        kern.staged(x, out_s, torch.cuda.Event(), torch.cuda.Event())
        torch.cuda.synchronize()
        kern.ws.check()
        assert torch.equal(out_t, out_p)
        assert torch.equal(out_s, out_p)
        assert torch.equal(idx_t, idx_p)
        assert e0.elapsed_time(e1) >= 0.0 and e1.elapsed_time(e2) > 0.0


def test_fused_topk_host_and_static_entries(built):
    """The pinned-host and static entries take the fused path too."""
    cfg = synth.config("c1", n_experts=64, inter=1024)
    layer, r, slot, kern = _kern(cfg, seed=3, slot_perm=True)
    x = synth.make_tokens(cfg, 1, seed=9, device="cuda")
    want = torch.empty_like(x)
    kern.staged(x, want, torch.cuda.Event(), torch.cuda.Event())
    host = x.cpu().pin_memory()
    got_h = kern(host)
    got_s = kern.call_static(x)
    torch.cuda.synchronize()
    kern.ws.check()
    assert torch.equal(got_h, want.cpu())
    assert torch.equal(got_s, want)
    ops.static_status()  # raises on a device error flag


def test_fused_topk_unmapped_expert_sets_status(built):
    """An expert without an arena slot is an index error on the fused path
    too (reported through the workspace status, the call itself returns)."""
    cfg = synth.config("c1", n_experts=16, top_k=16, inter=1024)
    layer, r, slot, kern = _kern(cfg, seed=5)
    bad = slot.clone()
    bad[3] = 10_000
    kern_bad = ops.MoEKernel(r, layer.experts, bad, cfg.swiglu_limit, "fused")
    x = synth.make_tokens(cfg, 1, seed=2, device="cuda")
    kern_bad(x)
    torch.cuda.synchronize()
    with pytest.raises(Exception):
        kern_bad.ws.check()
