"""Token-id hash routing (the V4 gate's first layers, dsv4_arena.py:149-152)
on the device: the experts come from a token-id table, the weights are their
normalised, routed-scaled scores.  The V4 MoEGate is not in the reference
repository, so this follows the scored layers' weight computation (unpinned).
Tolerances as for the scored router (weights rtol 2e-5) and the layer (the
1e-2 parity bar, 4e-3 at these sizes)."""

import numpy as np
import pytest
import torch

from locali_b200 import ops, synth
from locali_b200.router import V4Gate
from oracle import moe_oracle as O
from oracle.bridge import layer_np, t2np

pytestmark = pytest.mark.gpu


def _table(vocab, E, k, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(vocab)]).to(torch.int32)


@pytest.mark.parametrize("T,scoring", [(1, "sqrtsoftplus"), (5, "sigmoid"), (96, "sqrtsoftplus"), (80, "softmax")])
def test_hashed_router_matches_oracle(built, T, scoring):
    cfg = synth.config("c0", scoring=scoring, routed_scaling=2.5)
    layer = synth.make_layer(cfg, seed=3, device="cuda")
    x = synth.make_tokens(cfg, T, seed=4, device="cuda")
    table = _table(1000, cfg.n_experts, cfg.top_k, 5)
    ids = torch.randint(0, 1000, (T,), generator=torch.Generator().manual_seed(6))
    gate = V4Gate(layer.router, table.cuda())
    idx, w = gate(x, ids.cuda())
    torch.cuda.synchronize()
    L = layer_np(layer)
    ridx, rw, _, _ = O.router(t2np(x), L.router_weight, L.router_bias, cfg.top_k, scoring, 2.5, True,
                              hash_idx=table[ids].numpy())
    assert np.array_equal(t2np(idx), ridx)
    np.testing.assert_allclose(t2np(w), rw, rtol=2e-5, atol=1e-7)
    # without input ids the layer is scored
    idx2, _ = gate(x)
    torch.cuda.synchronize()
    sidx, _, _, biased = O.router(t2np(x), L.router_weight, L.router_bias, cfg.top_k, scoring, 2.5, True)
    ok = ~O.near_ties(biased, cfg.top_k)
    assert np.array_equal(t2np(idx2)[ok], sidx[ok])


@pytest.mark.parametrize("T,path", [(4, "decode"), (64, "decode"), (300, "prefill")])
def test_hashed_layer_matches_oracle(built, T, path):
    cfg = synth.config("c0", scoring="sqrtsoftplus", routed_scaling=2.5)
    layer = synth.make_layer(cfg, seed=7, device="cuda")
    x = synth.make_tokens(cfg, T, seed=8, device="cuda")
    table = _table(500, cfg.n_experts, cfg.top_k, 9)
    ids = torch.randint(0, 500, (T,), generator=torch.Generator().manual_seed(10))
    hidx = table[ids]
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused", path=path)
    idx = torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device="cuda")
    out = kern(x, idx=idx, w=w, hash_idx=hidx.cuda())
    torch.cuda.synchronize()
    kern.ws.check()
    assert torch.equal(idx.cpu(), hidx)
    L = layer_np(layer)
    weights = "rounded" if path == "prefill" else "exact"
    ref = O.moe_layer(t2np(x), L, idx=hidx.numpy().astype(np.int64), w=t2np(w), weights=weights)
    assert O.rel_l2(t2np(out), ref["out"]) < 4e-3
    _, rw, _, _ = O.router(t2np(x), L.router_weight, L.router_bias, cfg.top_k, "sqrtsoftplus", 2.5, True,
                           hash_idx=hidx.numpy())
    np.testing.assert_allclose(t2np(w), rw, rtol=2e-5, atol=1e-7)


def test_v4_module_hash_layer(built):
    """V4ArenaMoE over an HBM store with a hash-routed gate: __call__(x, input_ids)
    equals the kernel layer with the gathered table."""
    from locali_b200.dsv4_arena import V4ArenaMoE, V4ArenaStore

    cfg = synth.config("c0", scoring="sqrtsoftplus", routed_scaling=2.5)
    layer = synth.make_layer(cfg, seed=11, device="cuda")
    store = V4ArenaStore.from_layers([layer.experts], top_k=cfg.top_k, device="cuda")
    table = _table(300, cfg.n_experts, cfg.top_k, 12).cuda()
    gate = V4Gate(layer.router, table)
    moe = V4ArenaMoE(store, 0, gate, cfg.top_k, swiglu_limit=cfg.swiglu_limit, fp32_swiglu=True)
    x = synth.make_tokens(cfg, 6, seed=13, device="cuda")
    ids = torch.tensor([3, 17, 255, 299, 0, 42], device="cuda")
    got = moe(x, ids)
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused")
    want = kern(x, hash_idx=table[ids.long()])
    torch.cuda.synchronize()
    assert torch.equal(got, want)
