"""Expert-parallel exchange on CPU.

Two (and four) gloo ranks run locali_b200.ep.ExpertParallelMoE -- the step's
buffers and its two all-to-alls of equal splits -- with the CPU restatement
of the exchange protocol (oracle/ep_oracle.py) standing in for the device
dispatch, expert and combine kernels (those are checked against the same
restatement by the GPU tests).  The result must match the single-process
oracle layer: the per-rank fp32 association of a token's routes may change
a few last bits."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from locali_b200 import ep, synth
from oracle import ep_oracle as EO
from oracle import moe_oracle as O
from oracle.bridge import layer_np, t2np

CFG = dict(n_experts=8, top_k=3, hidden=256, inter=128)


def _bits(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


class OracleRank:
    """The four per-rank operations of a step on the CPU oracle."""

    def __init__(self, L, rank, world, n_experts):
        self.L, self.rank, self.world, self.n_experts = L, rank, world, n_experts
        self.lo, self.hi = ep.owned_range(n_experts, rank, world)
        self.act_dtype = torch.bfloat16
        self.k, self.H = L.top_k, L.router_weight.shape[1]
        # the rank's experts as a local layer: local expert j -> its arena slot
        self.local = O.LayerNP(**{**L.__dict__, "expert_slot": np.asarray(L.expert_slot)[self.lo:self.hi]})

    def route(self, x):
        idx, w, _, _ = O.router(t2np(x), self.L.router_weight, self.L.router_bias, self.L.top_k,
                                self.L.scoring, self.L.routed_scaling, self.L.norm_topk)
        return torch.from_numpy(idx.astype(np.int32)), torch.from_numpy(w.astype(np.float32))

    def buffers(self, T):
        RB = EO.row_bytes(self.H, self.k)
        return {"send": torch.empty((self.world, T, RB), dtype=torch.uint8),
                "recv": torch.empty((self.world, T, RB), dtype=torch.uint8),
                "part": torch.empty((self.world, T, self.H), dtype=torch.float32),
                "back": torch.empty((self.world, T, self.H), dtype=torch.float32),
                "slot_of": torch.empty((T, self.world), dtype=torch.int32)}

    def dispatch(self, idx, w, x, send, slot_of):
        s, so = EO.dispatch(_bits(x), idx.numpy(), w.numpy(), self.n_experts, self.world)
        send.copy_(torch.from_numpy(s))
        slot_of.copy_(torch.from_numpy(so))

    def experts_partial(self, recv, partial):
        p = EO.partials(recv.numpy(), self.H, self.k, self.local)
        partial.copy_(torch.from_numpy(np.nan_to_num(p)).reshape(partial.shape))

    def combine(self, back, slot_of, out, residual=None, normed=None):
        o = EO.combine(back.numpy(), slot_of.numpy(), "bf16", None if residual is None else t2np(residual))
        out.copy_(torch.from_numpy(o).to(out.dtype))
        if normed is not None:
            normed.copy_(torch.from_numpy(EO.normed(o)).to(normed.dtype))


def _layer():
    cfg = synth.config("c0", **CFG)
    return cfg, synth.make_layer(cfg, seed=21, device="cpu")


def _worker(rank, world, port, tmp, T):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, layer = _layer()
        L = layer_np(layer)
        x = synth.make_tokens(cfg, T, seed=50 + rank, device="cpu")
        res = synth.make_tokens(cfg, T, seed=60 + rank, device="cpu")
        moe = ep.ExpertParallelMoE(OracleRank(L, rank, world, cfg.n_experts))
        got = moe(x)
        got_r = moe(x, residual=res)  # residual added after the single rounding of the layer output
        want = O.moe_layer(t2np(x), L)["out"]
        want_r = O.round_act(O.round_act(want, "bf16") + t2np(res), "bf16")
        rec = [O.rel_l2(t2np(got), want), float(np.mean(t2np(got) != want)),
               O.rel_l2(t2np(got_r), want_r), float(np.mean(t2np(got_r) != want_r))]
        np.save(os.path.join(tmp, f"r{rank}.npy"), np.array(rec))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T", [(2, 5), (4, 3)])
def test_ep_gloo_ranks_match_single_layer(tmp_path, world, T):
    port = 29600 + (os.getpid() % 150) + 7 * world
    mp.spawn(_worker, args=(world, port, str(tmp_path), T), nprocs=world, join=True)
    for r in range(world):
        err, mism, err_r, mism_r = np.load(tmp_path / f"r{r}.npy")
        assert err < 1e-3 and mism < 0.02, (r, err, mism)
        assert err_r < 1e-3 and mism_r < 0.02, (r, err_r, mism_r)


def test_dispatch_layout_by_hand():
    """Token 0: experts 0, 6, 1 (ranks 0, 1, 0); token 1: experts 4, 5, 7
    (rank 1 only); token 2: expert 9 is out of range (dropped), 2, 3."""
    H, k, E, world = 8, 3, 8, 2
    idx = np.array([[0, 6, 1], [4, 5, 7], [9, 2, 3]])
    w = np.array([[0.5, 0.3, 0.2], [0.1, 0.2, 0.7], [0.4, 0.4, 0.2]], np.float32)
    x = np.arange(3 * H, dtype=np.uint16).reshape(3, H)
    send, slot_of = EO.dispatch(x, idx, w, E, world)
    assert slot_of.tolist() == [[0, 0], [-1, 1], [1, -1]]
    xb, ids, ww, tok = EO.parse(send[0], H, k)
    assert tok.tolist() == [0, 2, -1]
    assert ids.tolist() == [[0, -1, 1], [-1, 2, 3], [-1, -1, -1]]
    assert ww[0].tolist() == pytest.approx([0.5, 0.0, 0.2])
    assert np.array_equal(xb[1], x[2])
    xb, ids, ww, tok = EO.parse(send[1], H, k)
    assert tok.tolist() == [0, 1, -1]
    assert ids.tolist() == [[-1, 2, -1], [0, 1, 3], [-1, -1, -1]]
    assert EO.row_bytes(H, k) % 16 == 0


def test_loopback_four_ranks_matches_single_layer():
    cfg, layer = _layer()
    L = layer_np(layer)
    xs = [synth.make_tokens(cfg, 4, seed=70 + r, device="cpu") for r in range(4)]
    ranks = [OracleRank(L, r, 4, cfg.n_experts) for r in range(4)]
    outs = ep.loopback_forward(ranks, xs)
    for x, o in zip(xs, outs):
        assert O.rel_l2(t2np(o), O.moe_layer(t2np(x), L)["out"]) < 1e-3
