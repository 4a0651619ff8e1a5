"""Expert-parallel layer with the sm_100a kernels.

* one GPU: N ranks emulated in one process (locali_b200.ep.loopback_forward),
  each with its own expert shard, router workspace and routed-expert kernel;
* two GPUs (skipped otherwise): two NCCL ranks through
  locali_b200.ep.ExpertParallelMoE.

Both must match the single-GPU layer (same routing; the fp32 sums of a
token's routes are associated per rank, so a few last bits may differ).
"""

import os

import numpy as np
import pytest
import torch

from locali_b200 import ep, ops, synth
from oracle import moe_oracle as O
from oracle.bridge import t2np

pytestmark = pytest.mark.gpu


def _single(layer, cfg, x):
    k = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused")
    return k(x)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("tiled", [False, True])
def test_ep_loopback_matches_single_gpu(built, world, tiled):
    cfg = synth.config("c1", n_experts=32)
    layer = synth.make_layer(cfg, seed=12, device="cuda")
    ranks = []
    for r in range(world):
        shard = ep.shard_experts(layer.experts, r, world, cfg.n_experts)
        if tiled:
            shard.pack_tiles()
        ranks.append(ep.EPRank(layer.router, shard, r, world, cfg.n_experts, cfg.swiglu_limit))
    xs = [synth.make_tokens(cfg, 1 + 3 * r, seed=80 + r, device="cuda") for r in range(world)]
    outs = ep.loopback_forward(ranks, xs)
    torch.cuda.synchronize()
    for x, o in zip(xs, outs):
        want = _single(layer, cfg, x)
        torch.cuda.synchronize()
        assert O.rel_l2(t2np(o), t2np(want)) < 1e-3
        assert float(np.mean(t2np(o) != t2np(want))) < 0.02


def _nccl_worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = synth.config("c1", n_experts=32)
        layer = synth.make_layer(cfg, seed=12, device="cuda")
        shard = ep.shard_experts(layer.experts, rank, world, cfg.n_experts).pack_tiles()
        moe = ep.ExpertParallelMoE(ep.EPRank(layer.router, shard, rank, world, cfg.n_experts, cfg.swiglu_limit))
        x = synth.make_tokens(cfg, 4 + rank, seed=90 + rank, device="cuda")
        got = moe(x)
        want = _single(layer, cfg, x)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"r{rank}.npy"),
                np.array([O.rel_l2(t2np(got), t2np(want)), float(np.mean(t2np(got) != t2np(want)))]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_nccl_ranks_match_single_gpu(built, tmp_path):
    import torch.multiprocessing as mp

    port = 29700 + (os.getpid() % 200)
    mp.spawn(_nccl_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        err, mism = np.load(tmp_path / f"r{r}.npy")
        assert err < 1e-3 and mism < 0.02, (r, err, mism)
