"""Expert-parallel exchange on CPU: two gloo ranks run the dispatch plan,
the all-to-all exchanges and the home combine of locali_b200.ep, with the
oracle standing in for the GPU router and expert kernels; the result must
match the single-process oracle layer (the kernels themselves are covered
by the GPU tests)."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from locali_b200 import ep, synth
from oracle import moe_oracle as O
from oracle.bridge import layer_np, t2np

WORLD = 2
CFG = dict(n_experts=8, top_k=3, hidden=256, inter=128)


class OracleRank:
    """Routing and local expert products from the oracle (CPU)."""

    def __init__(self, L, rank, world, n_experts):
        self.L, self.rank, self.world, self.n_experts = L, rank, world, n_experts
        self.lo, self.hi = ep.owned_range(n_experts, rank, world)

    def route(self, x):
        idx, w, _, _ = O.router(t2np(x), self.L.router_weight, self.L.router_bias, self.L.top_k,
                                self.L.scoring, self.L.routed_scaling, self.L.norm_topk)
        return torch.from_numpy(idx.astype(np.int32)), torch.from_numpy(w.astype(np.float32))

    def local_fn(self, xr, ir, wr):
        gid = t2np(ir).astype(np.int64) + self.lo
        assert np.all((gid >= self.lo) & (gid < self.hi))
        out = O.moe_layer(t2np(xr), self.L, idx=gid, w=t2np(wr))["out"]
        return torch.from_numpy(np.asarray(out, np.float32)).to(torch.bfloat16)


def _layer():
    cfg = synth.config("c0", **CFG)
    return cfg, synth.make_layer(cfg, seed=21, device="cpu")


def _worker(rank, world, port, tmp):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, layer = _layer()
        L = layer_np(layer)
        x = synth.make_tokens(cfg, 3 + rank, seed=50 + rank, device="cpu")
        moe = ep.ExpertParallelMoE(OracleRank(L, rank, world, cfg.n_experts))
        got = moe(x)
        want = O.moe_layer(t2np(x), L)["out"]
        err = O.rel_l2(t2np(got), want)
        np.save(os.path.join(tmp, f"r{rank}.npy"), np.array([err, float(np.mean(t2np(got) != want))]))
    finally:
        dist.destroy_process_group()


def test_ep_two_gloo_ranks_match_single_layer(tmp_path):
    port = 29600 + (os.getpid() % 200)
    mp.spawn(_worker, args=(WORLD, port, str(tmp_path)), nprocs=WORLD, join=True)
    for r in range(WORLD):
        err, mism = np.load(tmp_path / f"r{r}.npy")
        assert err < 1e-3, (r, err)
        assert mism < 0.02, (r, mism)


def test_plan_dispatch_dedupes_tokens_per_rank():
    # token 0: experts 0, 1 (rank 0) and 6 (rank 1); token 1: experts 4, 5, 7 (rank 1 only)
    idx = torch.tensor([[0, 6, 1], [4, 5, 7]], dtype=torch.int32)
    w = torch.tensor([[0.5, 0.3, 0.2], [0.1, 0.2, 0.7]])
    x = torch.arange(2 * 4, dtype=torch.float32).reshape(2, 4)
    p = ep.plan_dispatch(x, idx, w, 8, 2)
    assert p.send_counts == [1, 2]
    assert p.tok.tolist() == [0, 0, 1]
    loc = p.meta[:, :3]
    assert loc[0].tolist() == [0, -1, 1]            # rank 0 keeps experts 0 and 1
    assert loc[1].tolist() == [-1, 2, -1]           # rank 1: expert 6 -> local 2
    assert loc[2].tolist() == [0, 1, 3]
    wr = p.meta[:, 3:].contiguous().view(torch.float32)
    assert wr[0].tolist() == pytest.approx([0.5, 0.0, 0.2])


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sized_plan_equals_plan(world):
    """The one-wait planner (device-side counts, nonzero_static) builds the
    same plan as plan_dispatch: rows, their order, metadata and counts; the
    route counts add up to the local routes each destination receives."""
    g = torch.Generator().manual_seed(world)
    E, T, k = 32, 23, 6
    # at 8 ranks only experts 0..15 are chosen: ranks 4..7 receive no rows
    pool = 16 if world == 8 else E
    idx = torch.stack([torch.randperm(pool, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    w = torch.rand((T, k), generator=g)
    x = torch.randn((T, 8), generator=g)
    want = ep.plan_dispatch(x, idx, w, E, world)
    cnt, hits = ep.dispatch_counts(idx, E, world)
    send = cnt[:, 0].tolist()
    got = ep.plan_dispatch_sized(x, idx, w, E, world, hits, send)
    assert send == want.send_counts
    assert torch.equal(got.tok, want.tok)
    assert torch.equal(got.rows, want.rows)
    assert torch.equal(got.meta, want.meta)
    per = E // world
    for d in range(world):
        assert int(cnt[d, 1]) == int(((idx.long() // per) == d).sum())


def test_loopback_matches_distributed_plan():
    cfg, layer = _layer()
    L = layer_np(layer)
    xs = [synth.make_tokens(cfg, 2 + r, seed=70 + r, device="cpu") for r in range(4)]
    ranks = [OracleRank(L, r, 4, cfg.n_experts) for r in range(4)]
    outs = ep.loopback_forward(None, xs, [r.route for r in ranks], [r.local_fn for r in ranks], cfg.n_experts)
    for x, o in zip(xs, outs):
        assert O.rel_l2(t2np(o), O.moe_layer(t2np(x), L)["out"]) < 1e-3
