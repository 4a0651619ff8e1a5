"""DeepSeek-V4 routed experts over the HBM arena (the reference's
dsv4_arena.py module interface: ``V4ArenaStore`` and ``V4ArenaMoE``).

``V4ArenaMoE(store, layer, gate, top_k, swiglu_limit=10.0, fused_decode=False,
overlap_hits=False, fp32_swiglu=False)`` keeps the reference constructor
(dsv4_arena.py:155-163) and call convention (``__call__(x, input_ids=None)``
returns a tensor shaped and typed like ``x``, arena.py:508-547).  When the gate
is a :class:`~locali_b200.router.V4Gate` and every expert of the layer is
resident, the whole layer -- router, dispatch, gate/up + clamped SwiGLU,
down + weighted combine -- is one device pipeline with no host
synchronisation (experts resolve to slots through the store's device slot
table).  Otherwise the reference's host sequence runs: route, host list of
experts, ``submit``/``slots_for``, optional cross-layer prefetch, wait for
the fills, then the same expert kernels with the caller's routing.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from . import ops
from .arena import ARRS, PROJS, ArenaMoE, ArenaStore
from .native import NativeCache
from .native import available as native_available
from .router import V4Gate


class V4ArenaStore(ArenaStore):
    """The arena with V4 quantization metadata validated (dsv4_arena.py:17-143)."""

    def __init__(self, index_path=None, native_scheduler=True, *, index=None, **kwargs):
        config = index if index is not None else json.loads(Path(index_path).read_text())
        self.expert_quant = config.get("quantization", {})
        for tier, quant in self.expert_quant.items():
            if quant.get("mode", "affine") != "affine":
                raise ValueError(f"DeepSeek V4 streaming requires affine MLX weights, got {quant.get('mode')!r} "
                                 f"for tier {tier}")
        super().__init__(index_path, index=config, **kwargs)
        self.use_f16_moe = {}
        for tier in self.tiers:
            m = self.sample[tier]
            dts = {m[p][k][5] for p in PROJS for k in ("scales", "biases")}
            self.use_f16_moe[tier] = dts == {"F16"}
        self.native_caches = {}
        if native_scheduler and native_available():
            for tier in self.tiers:
                self.native_caches[tier] = NativeCache(
                    self.layers * self.E, self.slots[tier], self.protected_cap[tier],
                    policy="lfu-decay" if self.cache_policy == "lfu-decay" else "slru")
        elif self.cache_policy == "lfu-decay":
            raise RuntimeError("lfu-decay requires the compiled planner (liblocali_core.so)")

    @classmethod
    def from_layers(cls, experts_per_layer, top_k, device=None, **kw):
        """All-resident V4 store over in-memory arrays (see ArenaStore.from_layers);
        placement is fixed, so no planner is attached."""
        idx = ArenaStore._resident_index(experts_per_layer, top_k)
        L, E = idx["layers"], idx["num_experts"]
        store = cls.__new__(cls)
        V4ArenaStore.__init__(store, None, native_scheduler=False, index=idx, ceiling_gb=0.0, threads=2,
                              device=device, slots={"cold": L * E + 1}, **kw)
        for l, ex in enumerate(experts_per_layer):
            for p, q in zip(PROJS, (ex.gate, ex.up, ex.down)):
                for k, a in zip(ARRS, (q.weight, q.scales, q.biases)):
                    store.arena[("cold", p, k)][1 + l * E:1 + (l + 1) * E].copy_(a[1:])
        for l in range(L):
            for e in range(E):
                s = 1 + l * E + e
                store.lru["cold"][(l, e)] = s
                store._set_table((l, e), s)
        store.free["cold"] = []
        store._pack("cold", 0, L * E + 1)
        store.sync_table()
        torch.cuda.synchronize(store.device)
        return store

    def _key_id(self, key):
        layer, expert = key
        return layer * self.E + expert

    def _decode_key(self, key_id):
        return divmod(key_id, self.E)

    def quant(self, tier, field, proj=None):
        """Tier metadata from the index (defaults 2-bit, group 128, affine,
        dsv4_arena.py:64-66); with ``proj`` the geometry is inferred from the
        arena shapes instead, which also covers mixed per-projection bits."""
        if proj is not None:
            return super().quant(tier, field, proj)
        defaults = {"bits": 2, "group_size": 128, "mode": "affine"}
        return self.expert_quant.get(tier, {}).get(field, defaults[field])

    def _place_keys(self, layer, want, prefetch):
        if not self.native_caches:
            return super()._place_keys(layer, want, prefetch)
        if not want:
            return {}, [], {tier: [] for tier in self.tiers}
        tiers = {self.tier(layer, e) for e in want}
        if len(tiers) != 1:
            raise ValueError(f"layer {layer} spans multiple expert tiers: {tiers}")
        tier = tiers.pop()
        cache = self.native_caches[tier]
        if layer == 0 and not prefetch and len(want) <= self.top_k:
            for c in self.native_caches.values():
                c.note_token()
        if not prefetch and len(want) > self.slots[tier] - 1:
            raise ValueError(f"layer {layer} needs {len(want)} {tier} experts but the arena has "
                             f"{self.slots[tier] - 1}; raise --ceiling-gb")
        results = cache.plan([layer * self.E + e for e in want], pinned_slots=tuple(self.pinned.get(tier, ())),
                             touch_hits=not prefetch)
        out, issued = {}, []
        waits = {name: [] for name in self.tiers}
        for e, r in zip(want, results):
            key = (layer, e)
            if r.hit:
                if not prefetch:
                    self.hits += 1
                    if key in self.pf_keys:
                        self.pf_keys.discard(key)
                        self.prefetch_used += 1
                futs = self.inflight.get(key)
                if futs:
                    if all(f.done() for f in futs):
                        del self.inflight[key]
                    elif not prefetch:
                        waits[tier].extend(futs)
            else:
                if not prefetch:
                    self.misses += 1
                if r.evicted_key >= 0:
                    self._evicted(self._decode_key(r.evicted_key))
                if r.placed:
                    issued.append((e, tier, r.slot))
            if r.placed:
                out[e] = (tier, r.slot)
            elif not prefetch:
                raise RuntimeError(f"native scheduler could not place demanded L{layer}.E{e}")
        if not prefetch:
            self.pinned = {tier: {slot for _, slot in out.values()}}
        return out, issued, waits

    def _protected_size(self, tier):
        if tier in self.native_caches:
            return self.native_caches[tier].protected_size
        return super()._protected_size(tier)

    def stats(self):
        s = super().stats()
        s["scheduler"] = "c" if self.native_caches else "python"
        return s

    def close(self):
        for c in self.native_caches.values():
            c.close()
        self.native_caches = {}
        super().close()


class V4ArenaMoE(ArenaMoE):
    """V4 top-k routing and clamped SwiGLU over the HBM arena."""

    def __init__(self, store: V4ArenaStore, layer: int, gate, top_k: int, swiglu_limit: float = 10.0,
                 fused_decode: bool = False, overlap_hits: bool = False, fp32_swiglu: bool = False):
        super().__init__(store, layer, gate, bias=None, top_k=top_k)
        self.swiglu_limit = swiglu_limit
        self.scores_follow_output = True
        self.fused_decode = fused_decode
        self.overlap_hits = overlap_hits
        self.fp32_swiglu = fp32_swiglu
        self._kernels = {}

    # rounding of the SwiGLU product: the fused decode kernel and fp32_swiglu
    # round once (dsv4_kernels.py:165-170, dsv4_arena.py:228-232); the stock
    # MLX path rounds op by op (dsv4_arena.py:234)
    def _swiglu_mode(self) -> str:
        return "fused" if (self.fused_decode or self.fp32_swiglu) else "stock"

    def route(self, x, input_ids=None):
        return self.gate(x, input_ids)

    def experts(self, tier) -> ops.ExpertArrays:
        q = self.store._qproj
        return ops.ExpertArrays(q(tier, "gate_proj"), q(tier, "up_proj"), q(tier, "down_proj"))

    def kernel(self, tier) -> ops.MoEKernel:
        k = self._kernels.get(tier)
        if k is None:
            router = self.gate.router if isinstance(self.gate, V4Gate) else ops.RouterArrays(
                torch.zeros((self.store.E, self.store.cols(tier, "gate_proj")), dtype=torch.bfloat16,
                            device=self.store.device), None, self.top_k)
            k = ops.MoEKernel(router, self.experts(tier), self.store.slot_table[self.layer], self.swiglu_limit,
                              self._swiglu_mode())
            self._kernels[tier] = k
        return k

    def _prefetch_routes(self, x, input_ids, blocks):
        """The next layers' routing for their cross-layer prefetch
        (arena.py:520-541), launched on the device; each result is copied to
        pinned host memory behind an event, so only that small copy is ever
        waited on.  Candidates are cut to the ``k`` highest gates."""
        pend = []
        for blk, k in blocks:
            pi, pg = blk.route(x, input_ids)
            pi = pi.reshape(-1, self.top_k)
            if k and k < self.top_k:
                order = torch.argsort(-pg.reshape(-1, self.top_k).float(), dim=-1)
                pi = torch.gather(pi, -1, order[:, :k])
            if pi.is_cuda:
                host = torch.empty(pi.shape, dtype=pi.dtype, pin_memory=True)
                host.copy_(pi, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record()
                pend.append((blk, host, ev))
            else:
                pend.append((blk, pi, None))
        return pend

    def _submit_prefetch(self, pend):
        for blk, host, ev in pend:
            if ev is not None:
                ev.synchronize()
            self.store.submit(blk.layer, [int(e) for e in host.reshape(-1).tolist()], prefetch=True)
        self.last_prefetch = [blk.layer for blk, _, _ in pend]

    def __call__(self, x, input_ids=None):
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        # the layer's tier and residency only change with the slot table
        ver = self.store.table_version
        if self.__dict__.get("_ver") != ver:
            self._tier = self.store.tier(self.layer, 0)
            self._resident = self.store.layer_resident(self.layer)
            self._ver = ver
        tier = self._tier
        blocks = [(b, k) for b, k in ((self.nxt, self.prefetch_k), (self.nxt2, self.prefetch_k2)) if b is not None]
        # a next layer whose experts are all resident needs no prefetch (its
        # submit would claim nothing)
        blocks = [(b, k) for b, k in blocks if not self.store.layer_resident(b.layer)]
        if self._resident and isinstance(self.gate, V4Gate):
            # device path: router, dispatch and experts in one call with the
            # slot table on the device, no host synchronisation for this layer
            pend = self._prefetch_routes(x, input_ids, blocks) if blocks else []
            self.store.sync_table()
            out = self.kernel(tier)(flat, hash_idx=self.gate.hash_idx(input_ids)).reshape(shape)
            if pend:
                self._submit_prefetch(pend)
            self.last_path = "device"
            return out if out.dtype == x.dtype else out.to(x.dtype)
        self.last_path = "host"
        inds, gates = self.route(x, input_ids)
        ii = inds.reshape(-1, self.top_k)
        ii_host = ii.tolist()  # host sync, as arena.py:513
        experts = [e for row in ii_host for e in row]
        if self.store.tier_overlap:
            placed, reads = self.store.submit(self.layer, experts)
        else:
            placed, reads = self.store.slots_for(self.layer, experts), None
        missing = sorted(set(experts) - set(placed))
        if missing:
            raise RuntimeError(f"arena could not place demanded experts {missing} of layer {self.layer}: every "
                               "usable slot is pinned; raise the ceiling")
        if blocks:
            self._submit_prefetch(self._prefetch_routes(x, input_ids, blocks))
        self.store.sync_table()
        w = gates.reshape(-1, self.top_k)
        out = self._apply(flat, ii, ii_host, placed, w, reads)
        return out.reshape(shape).to(x.dtype)

    def _apply(self, flat, ii, ii_host, placed, w, reads):
        """``ArenaMoE._apply`` (arena.py:549-672) on the device kernels."""
        T, k = len(ii_host), self.top_k
        present = [t for t in self.store.tiers if any(placed[e][0] == t for row in ii_host for e in row)]
        ii = ii.to(torch.int32)
        if len(present) == 1:
            t = present[0]
            pending = getattr(reads, "pending_experts", ()) if reads else ()
            if self.overlap_hits and T == 1 and pending and len(pending) < k:
                # resident experts first, then the ones still being filled
                # (arena.py:575-618); the per-route products are combined
                # once in route order, so the result equals the fused path
                ready = torch.tensor([[e not in pending for e in ii_host[0]]], device=ii.device)
                prod = torch.empty((k, flat.shape[1]), dtype=flat.dtype, device=flat.device)
                kern = self.kernel(t)
                kern.products(flat, torch.where(ready, ii, -1), w, prod)
                self.store.wait(reads[t])
                kern.products(flat, torch.where(ready, -1, ii), w, prod)
                self.last_apply = "overlap"
                return ops.combine_routes(prod, k)
            if reads is not None:
                self.store.wait(reads[t])
            self.last_apply = "single"
            return self.kernel(t).routed(flat, ii, w)
        # Several tiers (arena.py:625-672): each tier's own routes, unweighted
        # rows, then the fp32 sum of y * g in tier order and route order,
        # with g the weights rounded to the activation dtype; one rounding.
        tier_pos = {t: i for i, t in enumerate(present)}
        tier_of = torch.tensor([[tier_pos[placed[e][0]] for e in row] for row in ii_host], device=ii.device)
        order = torch.tensor([sorted(range(k), key=lambda j, row=row: (tier_pos[placed[row[j]][0]], j))
                              for row in ii_host], dtype=torch.int32, device=ii.device)
        prod = torch.empty((T * k, flat.shape[1]), dtype=flat.dtype, device=flat.device)
        for i, t in enumerate(present):
            if reads is not None:
                self.store.wait(reads[t])
            self.kernel(t).products(flat, torch.where(tier_of == i, ii, -1), None, prod)
        g = w.to(flat.dtype).float()
        self.last_apply = "tiers"
        return ops.combine_routes(prod, k, w=g, order=order)

    def _gather(self, tier, inputs, indices):
        """Expert products for [T, k] slot indices (dsv4_arena.py:168-235):
        inputs [T, 1, 1, hidden] -> [T, k, 1, hidden]."""
        T = inputs.shape[0]
        ex = self.experts(tier)
        x = inputs.reshape(T, -1)
        slots = indices.reshape(T, -1).to(torch.int32)
        h = ops.gateup_swiglu(x, slots, ex, self.swiglu_limit, self._swiglu_mode())
        y = ops.gather_qmm(h, slots.reshape(-1), ex.down)
        return y.reshape(T, slots.shape[1], 1, -1)
