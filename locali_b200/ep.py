"""Expert-parallel routed-MoE layer: experts sharded over ranks.

Rank r owns experts ``[r*E/N, (r+1)*E/N)`` of every layer in its own HBM
arena; the router weights are replicated and every rank routes its own
tokens (the same number of tokens on every rank).  One layer step, all on
the device with no host wait (include/lmoe.h, lmoe_ep_*):

1. route the local tokens (``lmoe_route``);
2. ``lmoe_ep_dispatch``: for every destination rank, the rows of the tokens
   with an expert there, each carrying its local expert ids and weights, in
   token order, then padding rows (a fixed ``T`` rows per rank pair);
3. NCCL ``all_to_all_single`` of the rows (equal splits);
4. ``lmoe_ep_experts``: the received routes through the local experts (the
   decode GEMVs or the tcgen05 grouped GEMM), each row's rounded ``y*w``
   terms summed in route order in fp32;
5. NCCL ``all_to_all_single`` of the fp32 partial rows back (equal splits);
6. ``lmoe_ep_combine``: per token, the partials of its owning ranks added in
   rank order, rounded once (plus an optional residual).

Every buffer has a fixed size, so a step can be captured in a CUDA graph
with its NCCL calls.  The reference runs every expert on one device
(``arena.py:508-672``); this module is the expert-parallel deployment of
the same layer (no counterpart in the reference).  The per-rank operations
are methods of :class:`EPRank`, so the same :class:`ExpertParallelMoE`
sequencing runs with NCCL on GPUs, with gloo in the CPU tests (where a test
rank object supplies the four operations), and as a single-process
loopback that emulates N ranks (:func:`loopback_forward`).
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib, ops
from ._lib import check, lmoe


def owned_range(n_experts: int, rank: int, world: int) -> tuple[int, int]:
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per


def shard_experts(experts: ops.ExpertArrays, rank: int, world: int, n_experts: int) -> ops.ExpertArrays:
    """The slots of the experts ``rank`` owns, from an arena whose slot
    ``1 + e`` holds expert ``e`` (slot 0 zero).  Returns a new arena with slot
    0 zero and slot ``1 + j`` = local expert ``j``."""
    lo, hi = owned_range(n_experts, rank, world)

    def cut(q: ops.QProjArrays) -> ops.QProjArrays:
        def take(a):
            return torch.cat([a[:1], a[1 + lo:1 + hi]]).contiguous()

        return ops.QProjArrays(take(q.weight), take(q.scales), take(q.biases), q.bits, q.group_size)

    return ops.ExpertArrays(cut(experts.gate), cut(experts.up), cut(experts.down))


def row_bytes(hidden: int, top_k: int) -> int:
    """Bytes of one exchanged row (``lmoe_ep_row_bytes``)."""
    n = int(lmoe().lmoe_ep_row_bytes(int(hidden), int(top_k)))
    if n == 0:
        raise _lib.LmoeError(_lib.LMOE_EINVAL, f"exchange row of hidden {hidden}, top_k {top_k}")
    return n


class EPRank:
    """The per-rank state on the GPU: replicated router, local expert shard
    (slot ``1 + j`` = local expert ``j``), workspaces."""

    def __init__(self, router: ops.RouterArrays, local_experts: ops.ExpertArrays, rank: int, world: int,
                 n_experts: int, swiglu_limit: float = 10.0, swiglu_mode: str = "fused", path: str = "auto"):
        ops._need_cuda(router.weight, local_experts.gate.weight)
        self.router, self.rank, self.world, self.n_experts = router, rank, world, n_experts
        self.lo, self.hi = owned_range(n_experts, rank, world)
        self.n_local = self.hi - self.lo
        self.top_k = router.top_k
        self.experts = local_experts
        self.hidden = local_experts.hidden
        self.act_dtype = local_experts.dtype
        self.path = path
        dev = router.weight.device
        self.device = dev
        self.slot_table = torch.arange(1, self.n_local + 1, dtype=torch.int32, device=dev)
        # the local layer: the shard's experts with the route width top_k; its
        # router is never evaluated (weight pointer unused)
        local_router = _lib.Router(router.weight.data_ptr(), None, self.n_local, int(self.top_k), 0, 1, 1.0)
        self.local = _lib.Layer(local_router, local_experts.ctype(), self.slot_table.data_ptr(), float(swiglu_limit),
                                _lib.SWIGLU_MODE[swiglu_mode])
        self.route_ws = ops.Workspace(dev)
        self.ws = ops.Workspace(dev)
        self.row_bytes = row_bytes(self.hidden, self.top_k)

    # ---- the four per-rank operations of a step
    def route(self, x: torch.Tensor):
        return ops.route(x, self.router, self.route_ws)

    def dispatch(self, idx: torch.Tensor, w: torch.Tensor, x: torch.Tensor, send: torch.Tensor,
                 slot_of: torch.Tensor) -> None:
        T = x.shape[0]
        check(lmoe().lmoe_ep_dispatch(idx.data_ptr(), w.data_ptr(), x.data_ptr(), T, self.hidden, int(self.top_k),
                                      self.n_experts, self.world, send.data_ptr(), slot_of.data_ptr(),
                                      self.route_ws.ptr(), ops._stream()), "lmoe_ep_dispatch")

    def workspace_bytes(self, rows: int) -> int:
        n = int(lmoe().lmoe_ep_workspace_size(ctypes.byref(self.local), int(rows), self.world,
                                              _lib.PATH[self.path]))
        if n == 0:
            raise _lib.LmoeError(_lib.LMOE_EUNSUPPORTED, "expert-parallel local layer")
        return n

    def experts_partial(self, recv: torch.Tensor, partial: torch.Tensor) -> None:
        rows = recv.shape[0] if recv.dim() == 2 else recv.shape[0] * recv.shape[1]
        self.ws.ensure(self.workspace_bytes(rows))
        check(lmoe().lmoe_ep_experts(ctypes.byref(self.local), recv.data_ptr(), rows, self.world,
                                     partial.data_ptr(), self.ws.ptr(), self.ws.nbytes, ops._stream(),
                                     _lib.PATH[self.path]), "lmoe_ep_experts")

    def combine(self, back: torch.Tensor, slot_of: torch.Tensor, out: torch.Tensor,
                residual: torch.Tensor | None = None, normed: torch.Tensor | None = None,
                eps: float = 1e-6) -> None:
        T = slot_of.shape[0]
        check(lmoe().lmoe_ep_combine(back.data_ptr(), T, self.world, self.hidden, ops._ACT[self.act_dtype],
                                     slot_of.data_ptr(), ops._ptr(residual), out.data_ptr(), ops._ptr(normed),
                                     float(eps), ops._stream()), "lmoe_ep_combine")

    def buffers(self, T: int) -> dict:
        """Fixed-size exchange buffers of a step with T tokens per rank."""
        dev, N, H = self.device, self.world, self.hidden
        return {
            "send": torch.empty((N, T, self.row_bytes), dtype=torch.uint8, device=dev),
            "recv": torch.empty((N, T, self.row_bytes), dtype=torch.uint8, device=dev),
            "part": torch.empty((N, T, H), dtype=torch.float32, device=dev),
            "back": torch.empty((N, T, H), dtype=torch.float32, device=dev),
            "slot_of": torch.empty((T, N), dtype=torch.int32, device=dev),
        }

    def check(self) -> None:
        """Synchronise and raise if a kernel flagged a bad expert id or slot."""
        self.route_ws.check()
        self.ws.check()


class ExpertParallelMoE:
    """One expert-parallel layer step under ``torch.distributed`` (NCCL on
    GPUs).  ``rank_state`` supplies route / dispatch / experts_partial /
    combine / buffers (:class:`EPRank` on a GPU).  Every rank calls it with
    the same number of tokens."""

    def __init__(self, rank_state, group=None):
        self.r = rank_state
        self.group = group
        self._bufs: dict[int, dict] = {}

    def _exchange(self, dst: torch.Tensor, src: torch.Tensor) -> None:
        if self.r.world == 1:
            dst.copy_(src)
            return
        import torch.distributed as dist

        dist.all_to_all_single(dst, src, group=self.group)

    def __call__(self, x: torch.Tensor, residual: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, normed: torch.Tensor | None = None) -> torch.Tensor:
        """``out = residual + moe(x)`` (without residual: ``moe(x)``); with
        ``normed``, also its weightless LayerNorm (the next layer's input)."""
        flat = x.reshape(-1, x.shape[-1])
        if flat.dtype != self.r.act_dtype:
            flat = flat.to(self.r.act_dtype)
        flat = flat.contiguous()
        T = flat.shape[0]
        b = self._bufs.get(T)
        if b is None:
            b = self._bufs[T] = self.r.buffers(T)
        idx, w = self.r.route(flat)
        self.r.dispatch(idx, w, flat, b["send"], b["slot_of"])
        self._exchange(b["recv"], b["send"])
        self.r.experts_partial(b["recv"].view(-1, b["recv"].shape[-1]), b["part"])
        self._exchange(b["back"], b["part"])
        if out is None:
            out = torch.empty_like(flat)
        res = None if residual is None else residual.reshape(flat.shape).to(flat.dtype).contiguous()
        if normed is None:
            self.r.combine(b["back"], b["slot_of"], out, res)
        else:
            self.r.combine(b["back"], b["slot_of"], out, res, normed)
        return out.reshape(x.shape)


def loopback_forward(ranks: Sequence, xs: Sequence[torch.Tensor],
                     residuals: Sequence[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """The same step for N ranks emulated in one process (the exchanges are
    block copies between the ranks' buffers).  ``ranks`` are objects with the
    :class:`EPRank` operations; every x holds the same number of tokens."""
    world = len(ranks)
    T = xs[0].shape[0]
    if any(x.shape[0] != T for x in xs):
        raise ValueError("every rank holds the same number of tokens")
    bufs = [r.buffers(T) for r in ranks]
    flats = [x.reshape(T, -1).contiguous() for x in xs]
    for r, b, x in zip(ranks, bufs, flats):
        idx, w = r.route(x)
        r.dispatch(idx, w, x, b["send"], b["slot_of"])
    for d in range(world):  # rank d receives block d of every sender, in sender order
        for s in range(world):
            bufs[d]["recv"][s].copy_(bufs[s]["send"][d])
    for r, b in zip(ranks, bufs):
        r.experts_partial(b["recv"].view(-1, b["recv"].shape[-1]), b["part"])
    for s in range(world):  # partials of sender s's rows go back to s, in rank order
        for d in range(world):
            bufs[s]["back"][d].copy_(bufs[d]["part"][s])
    outs = []
    for i, (r, b, x) in enumerate(zip(ranks, bufs, flats)):
        out = torch.empty_like(x)
        res = None if residuals is None else residuals[i].reshape(x.shape).contiguous()
        r.combine(b["back"], b["slot_of"], out, res)
        outs.append(out)
    return outs
