"""Expert-parallel layer with the sm_100a kernels.

* the device dispatch writes exactly the rows, trailers and slot table of
  the CPU restatement (oracle/ep_oracle.py);
* the receive side's fp32 partials match the restatement's;
* one GPU: N ranks emulated in one process (locali_b200.ep.loopback_forward),
  each with its own expert shard, on both expert paths;
* two GPUs (skipped otherwise): two NCCL ranks through
  locali_b200.ep.ExpertParallelMoE, eagerly and replayed from a CUDA graph.

The layer must match the single-GPU layer (same routing; the fp32 sums of a
token's routes are associated per rank, so a few last bits may differ).
"""

import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from locali_b200 import ep, ops, synth
from oracle import ep_oracle as EO
from oracle import moe_oracle as O
from oracle.bridge import layer_np, t2np

pytestmark = pytest.mark.gpu


def _single(layer, cfg, x, path="auto"):
    k = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused", path=path)
    return k(x)


def _ranks(layer, cfg, world, tiled=False, path="auto"):
    ranks = []
    for r in range(world):
        shard = ep.shard_experts(layer.experts, r, world, cfg.n_experts)
        if tiled:
            shard.pack_tiles()
        ranks.append(ep.EPRank(layer.router, shard, r, world, cfg.n_experts, cfg.swiglu_limit, path=path))
    return ranks


def _bits(x):
    return x.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("world", [2, 4])
def test_device_dispatch_equals_restatement(built, world):
    cfg = synth.config("c1", n_experts=32)
    layer = synth.make_layer(cfg, seed=12, device="cuda")
    r = _ranks(layer, cfg, world)[0]
    T = 37
    x = synth.make_tokens(cfg, T, seed=3, device="cuda")
    idx, w = r.route(x)
    idx[5, 2] = 99  # out of range: dropped, flagged
    b = r.buffers(T)
    r.dispatch(idx, w, x, b["send"], b["slot_of"])
    torch.cuda.synchronize()
    send, slot_of = EO.dispatch(_bits(x), t2np(idx), t2np(w), cfg.n_experts, world)
    got_send = b["send"].cpu().numpy()
    assert np.array_equal(b["slot_of"].cpu().numpy(), slot_of)
    H = cfg.hidden
    for d in range(world):
        n_real = int((slot_of[:, d] >= 0).sum())
        assert np.array_equal(got_send[d, :n_real], send[d, :n_real])  # rows and trailers
        assert np.array_equal(got_send[d, n_real:, 2 * H:], send[d, n_real:, 2 * H:])  # padding trailers
    with pytest.raises(Exception):
        r.route_ws.check()


@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_device_partials_match_restatement(built, path):
    cfg = synth.config("c1", n_experts=32)
    layer = synth.make_layer(cfg, seed=14, device="cuda")
    world, T = 2, 24
    ranks = _ranks(layer, cfg, world, path=path)
    xs = [synth.make_tokens(cfg, T, seed=30 + s, device="cuda") for s in range(world)]
    bufs = [r.buffers(T) for r in ranks]
    for r, b, x in zip(ranks, bufs, xs):
        idx, w = r.route(x)
        r.dispatch(idx, w, x, b["send"], b["slot_of"])
    d = 1
    for s in range(world):
        bufs[d]["recv"][s].copy_(bufs[s]["send"][d])
    recv = bufs[d]["recv"].view(-1, ranks[d].row_bytes)
    ranks[d].experts_partial(recv, bufs[d]["part"])
    torch.cuda.synchronize()
    ranks[d].check()
    # the rank's shard as an oracle layer: local expert j in slot j + 1
    local = layer_np(SimpleNamespace(router=layer.router, experts=ranks[d].experts,
                                     expert_slot=ranks[d].slot_table, cfg=cfg))
    ref = EO.partials(recv.cpu().numpy(), cfg.hidden, cfg.top_k, local)
    got = bufs[d]["part"].view(-1, cfg.hidden).cpu().numpy()
    real = ~np.isnan(ref[:, 0])
    assert real.any()
    tol = 1e-2 if path == "prefill" else 3e-3  # the prefill path rounds each dequantised weight
    assert O.rel_l2(got[real], ref[real]) < tol


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("tiled", [False, True])
def test_ep_loopback_matches_single_gpu(built, world, tiled):
    cfg = synth.config("c1", n_experts=32)
    layer = synth.make_layer(cfg, seed=12, device="cuda")
    ranks = _ranks(layer, cfg, world, tiled)
    xs = [synth.make_tokens(cfg, 5, seed=80 + r, device="cuda") for r in range(world)]
    outs = ep.loopback_forward(ranks, xs)
    torch.cuda.synchronize()
    for r in ranks:
        r.check()
    for x, o in zip(xs, outs):
        want = _single(layer, cfg, x)
        torch.cuda.synchronize()
        assert O.rel_l2(t2np(o), t2np(want)) < 1e-3
        assert float(np.mean(t2np(o) != t2np(want))) < 0.02


def test_ep_loopback_prefill_path_and_residual(built):
    """Enough tokens that the receive side takes the tcgen05 path, with the
    residual added by the combine; against the single-GPU prefill layer."""
    cfg = synth.config("c2", n_experts=32)
    layer = synth.make_layer(cfg, seed=15, device="cuda")
    world, T = 2, 96
    ranks = _ranks(layer, cfg, world, path="prefill")
    xs = [synth.make_tokens(cfg, T, seed=90 + r, device="cuda") for r in range(world)]
    res = [synth.make_tokens(cfg, T, seed=95 + r, device="cuda") for r in range(world)]
    outs = ep.loopback_forward(ranks, xs, res)
    torch.cuda.synchronize()
    for x, rr, o in zip(xs, res, outs):
        want = (_single(layer, cfg, x, path="prefill").float() + rr.float()).to(torch.bfloat16)
        torch.cuda.synchronize()
        assert O.rel_l2(t2np(o), t2np(want)) < 1e-3
        assert float(np.mean(t2np(o) != t2np(want))) < 0.02


@pytest.mark.parametrize("path,T", [("decode", 24), ("prefill", 128)])
def test_ep_one_rank_residual_and_norm(built, path, T):
    """At one rank the expert-parallel step sums each token's routes in the
    single-GPU combine's order, so with the residual it equals the fused
    block entry bit for bit; the normed output is the weightless LayerNorm of
    that result (the next layer's input)."""
    cfg = synth.config("c2", n_experts=32)
    layer = synth.make_layer(cfg, seed=17, device="cuda")
    (r,) = _ranks(layer, cfg, 1, path=path)
    moe = ep.ExpertParallelMoE(r)
    x = synth.make_tokens(cfg, T, seed=18, device="cuda")
    res = synth.make_tokens(cfg, T, seed=19, device="cuda")
    out, xn = torch.empty_like(x), torch.empty_like(x)
    moe(x, residual=res, out=out, normed=xn)
    kern = ops.MoEKernel(layer.router, layer.experts, layer.expert_slot, cfg.swiglu_limit, "fused", path=path)
    want = kern.block(x, -1, res)
    torch.cuda.synchronize()
    r.check()
    assert torch.equal(out, want)
    ref = EO.normed(t2np(out))
    assert O.rel_l2(t2np(xn), ref) < 2e-3
    assert float(np.mean(t2np(xn) != ref)) < 0.02


def _nccl_worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    graph = None
    try:
        cfg = synth.config("c1", n_experts=32)
        layer = synth.make_layer(cfg, seed=12, device="cuda")
        shard = ep.shard_experts(layer.experts, rank, world, cfg.n_experts).pack_tiles()
        moe = ep.ExpertParallelMoE(ep.EPRank(layer.router, shard, rank, world, cfg.n_experts, cfg.swiglu_limit))
        x = synth.make_tokens(cfg, 6, seed=90 + rank, device="cuda")
        got = moe(x).clone()
        want = _single(layer, cfg, x)
        # the same step replayed from a CUDA graph (NCCL calls captured)
        out = torch.empty_like(x)
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            moe(x, out=out)  # warm-up on the capture stream
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            moe(x, out=out)
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        rec = [O.rel_l2(t2np(got), t2np(want)), float(np.mean(t2np(got) != t2np(want))),
               float(torch.equal(out, got))]
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array(rec))
        dist.barrier()
    finally:
        del graph
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_nccl_ranks_match_single_gpu(built, tmp_path):
    import torch.multiprocessing as mp

    port = 29700 + (os.getpid() % 200)
    mp.spawn(_nccl_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        err, mism, same = np.load(tmp_path / f"r{r}.npy")
        assert err < 1e-3 and mism < 0.02, (r, err, mism)
        assert same == 1.0, r  # the graph replay reproduces the eager step
