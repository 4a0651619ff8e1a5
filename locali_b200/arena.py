"""Expert arena in HBM behind the reference's slot API.

``ArenaStore`` keeps the reference's interface (arena.py:64-457): the index
JSON format (records ``[root, shard, offset, nbytes, shape, dtype]``), one
stacked ``[n_slots, *shape]`` array per (tier, projection, kind) with slot 0
reserved as zeros, slot claim/evict under LRU or SLRU with pinning,
``submit``/``wait``/``slots_for``/``stats``/``close``.  What changes on B200:

* the arrays are CUDA tensors in HBM (180 GB holds every expert of the
  reference model, so the usual configuration is "all resident");
* a device table ``slot_table[layer, expert]`` (int32, -1 = not resident)
  mirrors every placement, so kernels resolve experts to slots on the GPU and
  the per-layer host synchronisation of arena.py:513 is not needed;
* fills read the expert's bytes from disk into pinned host buffers on a thread
  pool and copy them host->device on a dedicated stream; a fill's completion is
  a CUDA event, and ``wait`` makes the compute stream wait on it (no host
  block for the copy itself).
"""

from __future__ import annotations

import json
import os
import queue
import time
from collections import OrderedDict
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

PROJS = ("gate_proj", "up_proj", "down_proj")
ARRS = ("weight", "scales", "biases")
TORCH_DT = {"U32": torch.int32, "I32": torch.int32, "F16": torch.float16, "BF16": torch.bfloat16,
            "F32": torch.float32, "U8": torch.uint8}
DT_NAME = {torch.int32: "U32", torch.float16: "F16", torch.bfloat16: "BF16", torch.float32: "F32",
           torch.uint8: "U8"}
POLICIES = ("lru", "slru-cold", "slru-all", "lfu-decay")


class ReadPlan(dict):
    """Per-tier fill completions plus the experts whose slots are not ready."""

    def __init__(self, *args, pending_experts=(), **kwargs):
        super().__init__(*args, **kwargs)
        self.pending_experts = frozenset(pending_experts)


class _Fill:
    """Completion of one expert fill: a future for the disk read whose result
    is the CUDA event recorded after the host->device copies."""

    def __init__(self, future):
        self.future = future

    def done(self) -> bool:
        if not self.future.done():
            return False
        ev = self.future.result()
        return ev is None or ev.query()

    def result(self):
        return self.future.result()


class ArenaStore:
    def __init__(self, index_path=None, ceiling_gb=8.0, hot_share=0.33, threads=8, nocache=True,
                 cache_policy="lru", *, device=None, index: dict | None = None, slots: dict | None = None,
                 tiled: bool = True):
        idx = index if index is not None else json.loads(Path(index_path).read_text())
        if cache_policy not in POLICIES:
            raise ValueError("cache_policy must be 'lru', 'slru-cold', 'slru-all', or 'lfu-decay'")
        self.meta = idx["experts"]
        self.layers, self.E = int(idx["layers"]), int(idx["num_experts"])
        self.top_k = int(idx["top_k"])
        self.cache_policy = cache_policy
        self.ceiling = int(ceiling_gb * 1e9)
        self.tier_overlap = bool(idx.get("pack"))
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._nocache = nocache
        self.fds = {}
        self.pool = ThreadPoolExecutor(max_workers=max(1, threads))
        self.hits = self.misses = self.evictions = self.bytes_read = 0
        self.t_stall = 0.0
        self.pinned, self.inflight, self.pf_keys = {}, {}, set()
        self.prefetched = self.prefetch_used = self.prefetch_wasted = 0

        sample = {}
        for m in self.meta.values():
            sample.setdefault(m["tier"], m)
        self.tiers = sorted(sample)
        self.sample = sample
        share = {self.tiers[0]: 1.0} if len(self.tiers) == 1 else {"hot": hot_share, "cold": 1.0 - hot_share}
        self.arena, self.item, self.slots = {}, {}, {}
        self.lru, self.protected, self.protected_cap, self.free = {}, {}, {}, {}
        for t in self.tiers:
            m = sample[t]
            per = sum(m[p][k][3] for p in PROJS for k in ARRS)
            self.item[t] = per
            n = int(slots[t]) if slots and t in slots else int(self.ceiling * share.get(t, 0.5) / per)
            if n < 2:
                raise ValueError(f"{ceiling_gb:.2f} GB gives tier {t} no usable expert slot after its reserved "
                                 "zero slot; raise --ceiling-gb or adjust --hot-share")
            self.slots[t] = n
            self.lru[t], self.protected[t] = OrderedDict(), OrderedDict()
            slru = cache_policy == "slru-all" or (cache_policy == "slru-cold" and t == "cold")
            self.protected_cap[t] = (n - 1) // 2 if slru else 0
            self.free[t] = list(range(1, n))
            for p in PROJS:
                for k in ARRS:
                    shape, dt = m[p][k][4], m[p][k][5]
                    self.arena[(t, p, k)] = torch.zeros((n, *shape), dtype=TORCH_DT[dt], device=self.device)
        self.resident = sum(self.slots[t] * self.item[t] for t in self.tiers)
        self.slot_table = torch.full((self.layers, self.E), -1, dtype=torch.int32, device=self.device)
        self._table_host = np.full((self.layers, self.E), -1, dtype=np.int32)
        self._table_dirty = set()
        self.table_version = 0  # bumped on every slot-table change
        self.copy_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self._staging: dict[str, queue.Queue] = {}
        # Pre-tiled copy of every slot (16-row tiles of codes + scales +
        # biases, one bulk copy each for the decode GEMV), kept in step with
        # the row-major slot arrays by repacking a slot whenever it is filled.
        # Device arenas only; no counterpart in the reference.
        self.tiles = {}
        if tiled and self.device.type == "cuda":
            for t in self.tiers:
                for p in PROJS:
                    nb = self._qproj(t, p).tile_bytes()
                    if nb:
                        self.tiles[(t, p)] = torch.zeros((self.slots[t], nb), dtype=torch.uint8, device=self.device)

    # ------------------------------------------------------------ metadata
    def tier(self, layer, expert):
        return self.meta[f"L{layer}.E{expert}"]["tier"]

    def quant(self, tier, field, proj=None):
        """Per-tier (or per-projection) quantisation inferred from the arena shapes
        (bits = packed*32/cols, group = cols/groups; dsv4_engine.py:162-171)."""
        proj = proj or "gate_proj"
        w = self.arena[(tier, proj, "weight")]
        s = self.arena[(tier, proj, "scales")]
        cols = self.cols(tier, proj)
        if field == "bits":
            return int(w.shape[-1]) * 32 // cols
        if field == "group_size":
            return cols // int(s.shape[-1])
        if field == "mode":
            return "affine"
        raise KeyError(field)

    def _qproj(self, tier, proj):
        """Kernel descriptor of one projection of all slots of a tier."""
        from . import ops

        a = self.arena
        return ops.QProjArrays(a[(tier, proj, "weight")], a[(tier, proj, "scales")], a[(tier, proj, "biases")],
                               self.quant(tier, "bits", proj), self.quant(tier, "group_size", proj),
                               getattr(self, "tiles", {}).get((tier, proj)))

    def _pack(self, tier, s0, n=1):
        """Repack slots [s0, s0 + n) of a tier into its tiles (current stream)."""
        for p in PROJS:
            if (tier, p) in self.tiles:
                self._qproj(tier, p).pack_tiles(s0, n)

    def cols(self, tier, proj):
        """Logical input width of a projection (hidden for gate/up, inter for down)."""
        gate = self.arena[(tier, "gate_proj", "weight")]
        inter = int(gate.shape[-2])
        if proj == "down_proj":
            return inter
        return int(self.arena[(tier, "down_proj", "weight")].shape[-2])

    # ------------------------------------------------------------ policy
    def _protected_size(self, t):
        return len(self.protected[t])

    def _resident(self, t, key):
        return key in self.lru[t] or key in self.protected[t]

    def _slot(self, t, key):
        return self.protected[t].get(key, self.lru[t].get(key))

    def _touch(self, t, key):
        if key in self.protected[t]:
            self.protected[t].move_to_end(key)
        elif self.protected_cap[t] == 0:
            self.lru[t].move_to_end(key)
        else:
            self.protected[t][key] = self.lru[t].pop(key)
            if len(self.protected[t]) > self.protected_cap[t]:
                old, old_slot = self.protected[t].popitem(last=False)
                self.lru[t][old] = old_slot

    def _evicted(self, victim):
        self.inflight.pop(victim, None)
        if victim in self.pf_keys:
            self.pf_keys.discard(victim)
            self.prefetch_wasted += 1
        self.evictions += 1
        self._set_table(victim, -1)

    def _claim(self, t, key):
        """A slot for ``key``: a free one while probation has room, else the least
        recently used unpinned probation entry, then protected (arena.py:212-263).
        None when every candidate is pinned."""
        pin = self.pinned.get(t, ())
        full = len(self.lru[t]) >= self.slots[t] - 1 - self.protected_cap[t]
        victim, seg = None, None
        if full or not self.free[t]:
            victim = next((k for k, s in self.lru[t].items() if s not in pin), None)
            seg = self.lru[t]
        if victim is None and not full and self.free[t]:
            s = self.free[t].pop()
        else:
            if victim is None:
                victim = next((k for k, s in self.protected[t].items() if s not in pin), None)
                seg = self.protected[t]
            if victim is None:
                return None
            s = seg.pop(victim)
            self._evicted(victim)
        self.lru[t][key] = s
        return s

    def _set_table(self, key, slot):
        layer, expert = key
        if 0 <= layer < self.layers and 0 <= expert < self.E:
            self._table_host[layer, expert] = slot
            self._table_dirty.add(layer)
            self.table_version += 1

    def sync_table(self, stream=None):
        """Push changed rows of the slot table to the device (async, small)."""
        if not self._table_dirty:
            return
        if self.device.type != "cuda":
            for layer in sorted(self._table_dirty):
                self.slot_table[layer].copy_(torch.from_numpy(self._table_host[layer].copy()))
            self._table_dirty.clear()
            return
        st = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(st):
            for layer in sorted(self._table_dirty):
                row = torch.from_numpy(self._table_host[layer].copy()).pin_memory()
                self.slot_table[layer].copy_(row, non_blocking=True)
        self._table_dirty.clear()

    def _place_keys(self, layer, want, prefetch):
        out, miss = {}, []
        waits = {t: [] for t in self.tiers}
        for e in want:
            key = (layer, e)
            t = self.tier(layer, e)
            if self._resident(t, key):
                out[e] = (t, self._slot(t, key))
                if not prefetch:
                    self.hits += 1
                    self._touch(t, key)
                    if key in self.pf_keys:
                        self.pf_keys.discard(key)
                        self.prefetch_used += 1
                futs = self.inflight.get(key)
                if futs:
                    if all(f.done() for f in futs):
                        del self.inflight[key]
                    elif not prefetch:
                        waits[t].extend(futs)
            else:
                if not prefetch:
                    self.misses += 1
                miss.append((e, t))
        if not prefetch:
            need = {}
            for _, t in miss:
                need[t] = need.get(t, 0) + 1
            for t, n in need.items():
                if n > self.slots[t] - 1:
                    raise ValueError(f"layer {layer} needs {n} {t} experts but the arena has {self.slots[t] - 1}; "
                                     "raise --ceiling-gb or --hot-share")
        issued = []
        for e, t in miss:
            s = self._claim(t, (layer, e))
            if s is None:
                continue
            out[e] = (t, s)
            issued.append((e, t, s))
        if not prefetch:
            pin = {t: set() for t in self.tiers}
            for t, s in out.values():
                pin[t].add(s)
            self.pinned = pin
        return out, issued, waits

    # ------------------------------------------------------------ fills
    def _fd(self, root, shard):
        key = (root, shard)
        if key not in self.fds:
            self.fds[key] = os.open(os.path.join(root, shard), os.O_RDONLY)
            if self._nocache and hasattr(os, "posix_fadvise"):
                os.posix_fadvise(self.fds[key], 0, 0, os.POSIX_FADV_DONTNEED)
        return self.fds[key]

    def _staging_buffer(self, t):
        q = self._staging.setdefault(t, queue.Queue())
        try:
            return q.get_nowait()
        except queue.Empty:
            return torch.empty(self.item[t], dtype=torch.uint8, pin_memory=self.copy_stream is not None)

    def _fill(self, t, s, recs):
        """Read one expert's nine records into pinned memory, copy them into slot
        ``s`` on the copy stream; returns the completion event."""
        buf = self._staging_buffer(t)
        host = buf.numpy()
        off = 0
        views = []
        for rec in recs:
            root, shard, pos, nbytes, _, _ = rec
            got = os.preadv(self._fd(root, shard), [memoryview(host[off:off + nbytes])], pos)
            if got != nbytes:
                raise IOError(f"short read {got}/{nbytes} at {shard}+{pos}")
            views.append((off, nbytes))
            off += nbytes
        ev = None
        if self.copy_stream is not None:
            with torch.cuda.stream(self.copy_stream):
                for (o, n), (p, k) in zip(views, [(p, k) for p in PROJS for k in ARRS]):
                    dst = self.arena[(t, p, k)][s].view(-1).view(torch.uint8)
                    dst.copy_(buf[o:o + n], non_blocking=True)
                self._pack(t, s)
                ev = torch.cuda.Event()
                ev.record(self.copy_stream)
            ev.synchronize()  # the staging buffer is reusable once its copies are done
        else:
            for (o, n), (p, k) in zip(views, [(p, k) for p in PROJS for k in ARRS]):
                self.arena[(t, p, k)][s].view(-1).view(torch.uint8).copy_(buf[o:o + n])
        self._staging[t].put(buf)
        return ev

    def submit(self, layer, experts, prefetch=False):
        """Claim slots now, return before the bytes arrive (arena.py:356-435)."""
        want = list(dict.fromkeys(int(e) for e in experts))
        out, issued, waits = self._place_keys(layer, want, prefetch)
        by_tier = ReadPlan({t: [] for t in self.tiers})
        for e, t, s in issued:
            m = self.meta[f"L{layer}.E{e}"]
            recs = [m[p][k] for p in PROJS for k in ARRS]
            fill = _Fill(self.pool.submit(self._fill, t, s, recs))
            self.inflight.setdefault((layer, e), []).append(fill)
            by_tier[t].append(fill)
            self.bytes_read += self.item[t]
            self._set_table((layer, e), s)
        if not prefetch:
            # The placement follows the reference policy (arena.py:305-354),
            # which pins the previous demand's slots but not this call's hits:
            # in an arena too small for both, a miss can evict a hit of the
            # same call and take its slot.  The reference would then compute
            # with the refilled slot; refuse instead of computing garbage.
            lost = [e for e, (t, s) in out.items() if self._table_host[layer, e] != s]
            if lost:
                raise RuntimeError(f"layer {layer}: demanded experts {sorted(lost)} were evicted by other experts of "
                                   "the same layer (the arena is too small beside the pinned slots); raise the "
                                   "ceiling")
        for t in self.tiers:
            by_tier[t] = by_tier[t] + waits[t]
        by_tier.pending_experts = frozenset(
            e for e in want if any(not f.done() for f in self.inflight.get((layer, e), ())))
        if prefetch:
            self.prefetched += len(issued)
            self.pf_keys.update((layer, e) for e, _, _ in issued)
        self.sync_table()
        return out, by_tier

    def wait(self, futs, stream=None):
        """Block on the disk reads, then make ``stream`` wait (on the GPU) for
        the host->device copies."""
        if not futs:
            return
        t0 = time.perf_counter()
        st = stream or (torch.cuda.current_stream(self.device) if self.copy_stream is not None else None)
        for f in futs:
            ev = f.result()
            if ev is not None and st is not None:
                st.wait_event(ev)
        self.t_stall += time.perf_counter() - t0

    def slots_for(self, layer, experts):
        placed, by_tier = self.submit(layer, experts)
        self.wait([f for futs in by_tier.values() for f in futs])
        return placed

    def make_resident(self, layers=None):
        """Fill every expert of the given layers (all by default) and pin the
        placement in the device slot table."""
        for layer in (range(self.layers) if layers is None else layers):
            self.slots_for(layer, range(self.E))
        self.sync_table()

    def layer_resident(self, layer) -> bool:
        return bool((self._table_host[layer] >= 0).all())

    def stats(self):
        n = self.hits + self.misses
        return {"hits": self.hits, "misses": self.misses, "hit_rate": self.hits / n if n else 0.0,
                "evictions": self.evictions, "bytes_read": self.bytes_read, "resident": self.resident,
                "peak": self.resident, "slots": dict(self.slots), "t_stall": self.t_stall, "t_convert": 0.0,
                "t_eval": 0.0, "prefetched": self.prefetched, "prefetch_used": self.prefetch_used,
                "prefetch_wasted": self.prefetch_wasted, "cache_policy": self.cache_policy,
                "protected": {t: self._protected_size(t) for t in self.tiers}}

    def close(self):
        self.pool.shutdown()
        for fd in self.fds.values():
            os.close(fd)
        self.fds.clear()

    # ------------------------------------------------------------ resident stores
    @classmethod
    def _resident_index(cls, experts_per_layer, top_k, tier="cold"):
        ex = experts_per_layer[0]
        layers, E = len(experts_per_layer), int(ex.gate.weight.shape[0]) - 1
        rec = {}
        for p, q in zip(PROJS, (ex.gate, ex.up, ex.down)):
            rec[p] = {}
            for k, a in zip(ARRS, (q.weight, q.scales, q.biases)):
                nb = a[0].numel() * a.element_size()
                rec[p][k] = ["", "", 0, nb, list(a.shape[1:]), DT_NAME[a.dtype]]
        experts = {f"L{l}.E{e}": dict(rec, tier=tier) for l in range(layers) for e in range(E)}
        return {"format": 1, "layers": layers, "num_experts": E, "top_k": top_k, "experts": experts,
                "quantization": {tier: {"bits": ex.gate.bits, "group_size": ex.gate.group_size, "mode": "affine"}}}

    @classmethod
    def from_layers(cls, experts_per_layer, top_k, device=None, **kw):
        """An all-resident store over in-memory expert arrays (one
        ``ops.ExpertArrays`` per layer, each ``[E + 1, ...]`` with slot 0 zero):
        expert e of layer l goes to slot ``1 + l*E + e``."""
        idx = cls._resident_index(experts_per_layer, top_k)
        L, E = idx["layers"], idx["num_experts"]
        n = L * E + 1
        store = cls.__new__(cls)
        store._init_resident(idx, n, device, **kw)
        for l, ex in enumerate(experts_per_layer):
            for p, q in zip(PROJS, (ex.gate, ex.up, ex.down)):
                for k, a in zip(ARRS, (q.weight, q.scales, q.biases)):
                    store.arena[("cold", p, k)][1 + l * E:1 + (l + 1) * E].copy_(a[1:])
        for l in range(L):
            for e in range(E):
                key, s = (l, e), 1 + l * E + e
                store.lru["cold"][key] = s
                store._set_table(key, s)
        store.free["cold"] = []
        store._pack("cold", 0, n)
        store.sync_table()
        torch.cuda.synchronize(store.device)
        return store

    def _init_resident(self, idx, n_slots, device, cache_policy="lru", threads=2, tiled=True):
        ArenaStore.__init__(self, None, ceiling_gb=0.0, threads=threads, cache_policy=cache_policy, device=device,
                            index=idx, slots={t: n_slots for t in sorted({m["tier"] for m in idx["experts"].values()})},
                            tiled=tiled)


class ArenaMoE:
    """Generic MoE block over the arena (arena.py:460-681): route, resolve
    experts to slots, run the expert products, weighted combine."""

    def __init__(self, store: ArenaStore, layer: int, gate, bias, top_k: int):
        self.store, self.layer, self.gate = store, layer, gate
        self.bias, self.top_k = bias, top_k
        self.scores_follow_output = False
        self.nxt = None
        self.nxt2 = None
        self.prefetch_k = None
        self.prefetch_k2 = None
        self.overlap_hits = False

    def route(self, x, input_ids=None):
        """``arena.py:501-506`` on the GPU: sigmoid scores, selection on
        score + bias, weights normalised by sum + 1e-20."""
        scores = torch.sigmoid(self.gate(x.float()))
        biased = scores + (self.bias if self.bias is not None else 0.0)
        inds = torch.topk(biased, self.top_k, dim=-1).indices
        g = torch.gather(scores, -1, inds)
        return inds.to(torch.int32), g / (g.sum(-1, keepdim=True) + 1e-20)
