"""Expert-parallel routed-MoE layer: experts sharded over ranks.

Rank r owns experts ``[r*E/N, (r+1)*E/N)`` in its own HBM arena; the router
weights are replicated and every rank routes its own tokens (data parallel).
One layer step:

1. route the local tokens (``lmoe_route``);
2. plan the dispatch: a token goes once to every rank that owns at least one
   of its experts, with its local expert ids there and their combine weights
   (``-1`` / 0 for routes owned elsewhere);
3. exchange counts, token rows and route metadata (all-to-all);
4. run the received routes through the local experts (one
   ``lmoe_moe_routed`` call, one route per entry) and sum each received row's
   routes in route order in fp32;
5. send the fp32 partial rows home (all-to-all) and add them per token in
   rank order, then round once.

The reference runs every expert on one device (``arena.py:508-672``); this
module is the expert-parallel deployment of the same layer (no counterpart
in the reference).  The per-rank phases are plain methods so the same code
runs under ``torch.distributed`` (:class:`ExpertParallelMoE`, NCCL on GPUs,
gloo in the CPU tests) and under a single-process loopback that emulates N
ranks (:func:`loopback_forward`).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch

from . import ops


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


@dataclass
class DispatchPlan:
    tok: torch.Tensor          # [S] token of each sent row, grouped by destination rank
    send_counts: list[int]     # rows per destination rank
    rows: torch.Tensor         # [S, H] the token rows
    meta: torch.Tensor         # [S, 2k] int32: local expert ids (-1 = elsewhere), fp32 weight bits


def plan_dispatch(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, n_experts: int, world: int) -> DispatchPlan:
    """Step 2: one row per (token, destination rank that owns one of its
    experts), in (destination, token) order."""
    T, k = idx.shape
    per = n_experts // world
    idx = idx.to(torch.int64)
    owner = idx // per                                            # [T, k]
    ranks = torch.arange(world, device=idx.device)
    hits = (owner.unsqueeze(-1) == ranks).any(1)                  # [T, world]
    dst, tok = hits.t().nonzero(as_tuple=True)                    # destination-major, then token
    own = owner[tok] == dst.unsqueeze(1)                          # [S, k]
    local = torch.where(own, idx[tok] - dst.unsqueeze(1) * per, torch.full_like(idx[tok], -1))
    wsel = torch.where(own, w[tok].to(torch.float32), torch.zeros_like(w[tok], dtype=torch.float32))
    meta = torch.cat([local.to(torch.int32), wsel.view(torch.int32)], dim=1)
    counts = hits.sum(0).tolist()
    return DispatchPlan(tok, counts, x[tok], meta)


def dispatch_counts(idx: torch.Tensor, n_experts: int, world: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per destination rank: the token rows it receives from this rank and
    the routes those rows carry, as one int64 [world, 2] tensor on the
    device, together with the token x destination hit mask."""
    per = n_experts // world
    owner = idx.to(torch.int64) // per                                            # [T, k]
    own = owner.unsqueeze(-1) == torch.arange(world, device=idx.device)           # [T, k, world]
    hits = own.any(1)                                                             # [T, world]
    return torch.stack([hits.sum(0), own.sum((0, 1))], 1), hits


def plan_dispatch_sized(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, n_experts: int, world: int,
                        hits: torch.Tensor, send_counts: list[int]) -> DispatchPlan:
    """plan_dispatch with the per-destination row counts already on the host
    (no host wait)."""
    T, k = idx.shape
    per = n_experts // world
    idx = idx.to(torch.int64)
    owner = idx // per
    dst, tok = torch.nonzero_static(hits.t(), size=sum(send_counts)).unbind(1)
    own = owner[tok] == dst.unsqueeze(1)
    local = torch.where(own, idx[tok] - dst.unsqueeze(1) * per, torch.full_like(idx[tok], -1))
    wsel = torch.where(own, w[tok].to(torch.float32), torch.zeros_like(w[tok], dtype=torch.float32))
    meta = torch.cat([local.to(torch.int32), wsel.view(torch.int32)], dim=1)
    return DispatchPlan(tok, list(send_counts), x[tok], meta)


def expert_partials(recv_rows: torch.Tensor, recv_meta: torch.Tensor, k: int,
                    local_fn: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                    n_routes: int | None = None) -> torch.Tensor:
    """Step 4: each received row's routes through the local experts, summed in
    route order in fp32.  ``local_fn(x [R,H], idx [R,1], w [R,1])`` returns the
    rounded per-route products ``T(T(y)*T(w))`` [R, H].  Every local (row,
    route) pair goes through one ``local_fn`` call; the products are placed
    at their route position and summed over the routes in order 0..k-1
    (absent routes add exact zeros).  ``n_routes``, the number of local
    routes when the caller knows it, saves a host wait."""
    n, H = recv_rows.shape
    out = torch.zeros((n, H), dtype=torch.float32, device=recv_rows.device)
    if n == 0:
        return out
    loc = recv_meta[:, :k]
    wr = recv_meta[:, k:].contiguous().view(torch.float32)
    if n_routes is None:
        rows, js = (loc >= 0).nonzero(as_tuple=True)
    else:
        rows, js = torch.nonzero_static(loc >= 0, size=n_routes).unbind(1)
    if rows.numel() == 0:
        return out
    y = local_fn(recv_rows[rows], loc[rows, js].unsqueeze(1), wr[rows, js].unsqueeze(1))
    per_route = torch.zeros((n, k, H), dtype=torch.float32, device=recv_rows.device)
    per_route[rows, js] = y.float()
    for j in range(k):  # route order j = 0..k-1, fp32
        out += per_route[:, j]
    return out


def combine_home(T: int, H: int, tok: torch.Tensor, back: torch.Tensor, send_counts: Sequence[int],
                 dtype: torch.dtype) -> torch.Tensor:
    """Step 5: add the partial rows per token in rank order (fp32), round once."""
    out = torch.zeros((T, H), dtype=torch.float32, device=back.device)
    start = 0
    for n in send_counts:  # rank order
        if n:
            out[tok[start:start + n]] += back[start:start + n]
        start += n
    return out.to(dtype)


class EPRank:
    """The per-rank state: replicated router, local expert shard."""

    def __init__(self, router: ops.RouterArrays, local_experts: ops.ExpertArrays, rank: int, world: int,
                 n_experts: int, swiglu_limit: float = 10.0, swiglu_mode: str = "fused"):
        self.router, self.rank, self.world, self.n_experts = router, rank, world, n_experts
        self.lo, self.hi = owned_range(n_experts, rank, world)
        n_local = self.hi - self.lo
        dev = router.weight.device
        # a top-1 layer over the local experts for the routed products; its
        # router is never evaluated
        local_router = ops.RouterArrays(torch.zeros((n_local, router.weight.shape[1]), dtype=torch.bfloat16,
                                                    device=dev), None, 1)
        self.slot_table = torch.arange(1, n_local + 1, dtype=torch.int32, device=dev)
        self.local = ops.MoEKernel(local_router, local_experts, self.slot_table, swiglu_limit, swiglu_mode)
        self.route_ws = ops.Workspace(dev)

    def route(self, x: torch.Tensor):
        return ops.route(x, self.router, self.route_ws)

    def local_fn(self, xr: torch.Tensor, ir: torch.Tensor, wr: torch.Tensor) -> torch.Tensor:
        return self.local.routed(xr, ir, wr)


class ExpertParallelMoE:
    """One expert-parallel layer step under ``torch.distributed``."""

    def __init__(self, rank_state: EPRank, group=None):
        self.r = rank_state
        self.group = group

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        flat = x.reshape(-1, x.shape[-1])
        T, H = flat.shape
        idx, w = self.r.route(flat)
        k = idx.shape[1]
        world = self.r.world
        # rows and routes per destination, exchanged as one [world, 2] tensor;
        # one host wait then gives every split size of the step
        cnt, hits = dispatch_counts(idx, self.r.n_experts, world)
        recv_cnt = torch.empty_like(cnt)
        dist.all_to_all_single(recv_cnt, cnt, group=self.group)
        host = torch.cat([cnt.reshape(-1), recv_cnt.reshape(-1)]).tolist()
        send_counts, rc = host[0:2 * world:2], host[2 * world::2]
        n_routes = sum(host[2 * world + 1::2])
        plan = plan_dispatch_sized(flat, idx, w, self.r.n_experts, world, hits, send_counts)
        recv_rows = flat.new_empty((sum(rc), H))
        dist.all_to_all_single(recv_rows, plan.rows, rc, plan.send_counts, group=self.group)
        recv_meta = plan.meta.new_empty((sum(rc), 2 * k))
        dist.all_to_all_single(recv_meta, plan.meta, rc, plan.send_counts, group=self.group)
        part = expert_partials(recv_rows, recv_meta, k, self.r.local_fn, n_routes)
        back = part.new_empty((sum(plan.send_counts), H))
        dist.all_to_all_single(back, part, plan.send_counts, rc, group=self.group)
        return combine_home(T, H, plan.tok, back, plan.send_counts, flat.dtype).reshape(x.shape)


def loopback_forward(ranks: Sequence, xs: Sequence[torch.Tensor], route_fns=None, local_fns=None,
                     n_experts: int | None = None) -> list[torch.Tensor]:
    """The same step for N ranks emulated in one process (the exchanges are
    list shuffles).  ``ranks`` are :class:`EPRank` objects, or ``None`` when
    ``route_fns`` / ``local_fns`` supply the per-rank routing and expert
    products."""
    world = len(xs)
    E = n_experts if n_experts is not None else ranks[0].n_experts
    plans, ks = [], []
    for r in range(world):
        route = route_fns[r] if route_fns else ranks[r].route
        idx, w = route(xs[r])
        ks.append(idx.shape[1])
        plans.append(plan_dispatch(xs[r], idx, w, E, world))
    k = ks[0]
    # rows each destination receives, in source-rank order
    starts = []
    for p in plans:
        s, acc = [], 0
        for n in p.send_counts:
            s.append(acc)
            acc += n
        starts.append(s)
    backs = [[None] * world for _ in range(world)]
    for d in range(world):
        rows = [plans[s].rows[starts[s][d]:starts[s][d] + plans[s].send_counts[d]] for s in range(world)]
        metas = [plans[s].meta[starts[s][d]:starts[s][d] + plans[s].send_counts[d]] for s in range(world)]
        fn = local_fns[d] if local_fns else ranks[d].local_fn
        part = expert_partials(torch.cat(rows), torch.cat(metas), k, fn)
        o = 0
        for s in range(world):
            n = plans[s].send_counts[d]
            backs[s][d] = part[o:o + n]
            o += n
    outs = []
    for s in range(world):
        back = torch.cat(backs[s])
        T, H = xs[s].shape
        outs.append(combine_home(T, H, plans[s].tok, back, plans[s].send_counts, xs[s].dtype))
    return outs
