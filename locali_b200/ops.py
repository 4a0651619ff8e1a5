"""Tensor-level wrappers over the C ABI (torch CUDA tensors in, out).

These are thin: they build the plain-pointer descriptors of include/lmoe.h
from torch tensors, own a device workspace, and enqueue the kernels on the
current CUDA stream.  No host synchronisation happens unless asked for
(:meth:`Workspace.check`).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, lmoe

_ACT = {torch.bfloat16: _lib.LMOE_BF16, torch.float16: _lib.LMOE_F16}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    """Raw cudaStream_t of the current device's current stream."""
    return torch._C._cuda_getCurrentRawStream(torch.cuda.current_device())


def _event(ev: torch.cuda.Event | None) -> int | None:
    """Raw cudaEvent_t of a torch event (created on first use)."""
    if ev is None:
        return None
    if ev.cuda_event == 0:
        ev.record()  # forces creation of the underlying event
    return ev.cuda_event


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("locali_b200 kernels need CUDA tensors (no CPU fallback)")


@dataclass
class QProjArrays:
    """One projection of all arena slots (MLX SwitchGLU layout).

    weight int32/uint32 [n_slots, rows, cols*bits/32]; scales/biases
    [n_slots, rows, cols/group_size] in the activation dtype.
    """

    weight: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    bits: int
    group_size: int
    # optional pre-tiled copy (uint8 [n_slots, tile_bytes]); the expert GEMVs
    # stream it with one bulk copy per 16-row tile instead of the arrays above
    tiles: torch.Tensor | None = None

    @property
    def n_slots(self) -> int:
        return int(self.weight.shape[0])

    @property
    def rows(self) -> int:
        return int(self.weight.shape[-2])

    @property
    def cols(self) -> int:
        return int(self.scales.shape[-1]) * self.group_size

    @staticmethod
    def infer(weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, cols: int) -> "QProjArrays":
        """Infer bits = packed*32/cols and group = cols/groups (dsv4_engine.py:162-171)."""
        packed = int(weight.shape[-1])
        groups = int(scales.shape[-1])
        if (packed * 32) % cols or cols % groups:
            raise ValueError(f"cannot infer affine quantization: weight {tuple(weight.shape)}, "
                             f"scales {tuple(scales.shape)}, cols {cols}")
        return QProjArrays(weight, scales, biases, packed * 32 // cols, cols // groups)

    def ctype(self) -> _lib.QProj:
        for t in (self.weight, self.scales, self.biases):
            if not t.is_contiguous():
                raise ValueError("arena arrays must be contiguous")
        return _lib.QProj(self.weight.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr(),
                          int(self.bits), int(self.group_size), _ptr(self.tiles))

    def tile_bytes(self) -> int:
        """Bytes per slot of the pre-tiled copy (0: geometry has no tile layout)."""
        return int(lmoe().lmoe_tile_bytes(self.rows, self.cols, int(self.bits), int(self.group_size)))

    def pack_tiles(self, slot_begin: int = 0, slot_count: int | None = None) -> "QProjArrays":
        """(Re)pack slots [slot_begin, slot_begin + slot_count) into ``tiles``.

        Allocates ``tiles`` on first use.  Enqueued on the current stream;
        call again for slots whose row-major arrays were rewritten.
        """
        _need_cuda(self.weight, self.scales, self.biases)
        nb = self.tile_bytes()
        if nb == 0:
            raise ValueError(f"no tile layout for [{self.rows}, {self.cols}] bits={self.bits} gs={self.group_size}")
        if self.tiles is None:
            self.tiles = torch.empty((self.n_slots, nb), dtype=torch.uint8, device=self.weight.device)
        if slot_count is None:
            slot_count = self.n_slots - slot_begin
        q = _lib.QProj(self.weight.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr(),
                       int(self.bits), int(self.group_size), None)
        check(lmoe().lmoe_tile_pack(ctypes.byref(q), self.n_slots, self.rows, self.cols, int(slot_begin),
                                    int(slot_count), self.tiles.data_ptr(), _stream()), "lmoe_tile_pack")
        return self


@dataclass
class ExpertArrays:
    gate: QProjArrays
    up: QProjArrays
    down: QProjArrays

    @property
    def n_slots(self) -> int:
        return int(self.gate.weight.shape[0])

    @property
    def hidden(self) -> int:
        return self.gate.cols

    @property
    def inter(self) -> int:
        return self.gate.rows

    @property
    def dtype(self) -> torch.dtype:
        return self.gate.scales.dtype

    def pack_tiles(self, slot_begin: int = 0, slot_count: int | None = None) -> "ExpertArrays":
        """Pre-tile the projections that have a tile layout (see
        :meth:`QProjArrays.pack_tiles`; 3-bit rows have none: those
        projections run on the prefill kernels, which read the row-major
        arrays)."""
        for q in (self.gate, self.up, self.down):
            if q.tile_bytes():
                q.pack_tiles(slot_begin, slot_count)
        return self

    def ctype(self) -> _lib.Experts:
        if self.dtype not in _ACT:
            raise ValueError(f"unsupported scale dtype {self.dtype}")
        return _lib.Experts(self.n_slots, self.hidden, self.inter, _ACT[self.dtype],
                            self.gate.ctype(), self.up.ctype(), self.down.ctype())


@dataclass
class RouterArrays:
    weight: torch.Tensor            # [E, H] bf16
    bias: torch.Tensor | None       # [E] fp32 selection-only bias
    top_k: int
    scoring: str = "sigmoid"
    routed_scaling: float = 1.0
    norm_topk: bool = True

    @property
    def n_experts(self) -> int:
        return int(self.weight.shape[0])

    def ctype(self) -> _lib.Router:
        if self.weight.dtype != torch.bfloat16:
            raise ValueError("router weight must be bf16")
        if self.bias is not None and self.bias.dtype != torch.float32:
            raise ValueError("router bias must be fp32")
        return _lib.Router(self.weight.data_ptr(), _ptr(self.bias), self.n_experts, int(self.top_k),
                           _lib.SCORING[self.scoring], int(bool(self.norm_topk)), float(self.routed_scaling))


class Workspace:
    """Caller-owned device scratch for the kernels; zeroed once when (re)sized.

    Kernels leave it reusable (their combine counters return to zero), so a
    workspace may be used by any number of calls on one stream.  Calls that
    overlap on different streams need different workspaces.
    """

    def __init__(self, device: torch.device | str | int | None = None):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.buf: torch.Tensor | None = None

    @property
    def nbytes(self) -> int:
        return 0 if self.buf is None else self.buf.numel()

    def ensure(self, nbytes: int) -> "Workspace":
        if nbytes <= 0:
            raise _lib.LmoeError(_lib.LMOE_EINVAL, "workspace size")
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.empty(int(nbytes), dtype=torch.uint8, device=self.device)
            check(lmoe().lmoe_workspace_init(self.buf.data_ptr(), self.buf.numel(), _stream()), "workspace init")
        return self

    def ptr(self) -> int:
        return self.buf.data_ptr()

    def check(self) -> None:
        """Synchronise and raise if a kernel flagged a bad expert id or slot."""
        if self.buf is not None:
            check(lmoe().lmoe_workspace_status(self.buf.data_ptr(), _stream()), "kernel status")


class MoEKernel:
    """One routed-MoE layer bound to its arena arrays and router.

    ``expert_slot`` (int32 [E] on the device) maps expert ids to arena slots,
    so routing, dispatch and the expert products all stay on the GPU.
    """

    def __init__(self, router: RouterArrays, experts: ExpertArrays, expert_slot: torch.Tensor,
                 swiglu_limit: float = 10.0, swiglu_mode: str = "fused", path: str = "auto"):
        _need_cuda(router.weight, experts.gate.weight, expert_slot)
        if path not in _lib.PATH:
            raise ValueError(f"path must be one of {sorted(_lib.PATH)}")
        # "decode": fused dequant GEMVs; "prefill": tcgen05 grouped GEMM;
        # "auto": prefill once the routes reach 256 and 1.75 * n_experts
        self.path = path
        if expert_slot.dtype != torch.int32 or not expert_slot.is_contiguous():
            raise ValueError("expert_slot must be contiguous int32")
        self.router, self.experts, self.expert_slot = router, experts, expert_slot
        self.swiglu_limit, self.swiglu_mode = float(swiglu_limit), swiglu_mode
        self.desc = _lib.Layer(router.ctype(), experts.ctype(), expert_slot.data_ptr(),
                               self.swiglu_limit, _lib.SWIGLU_MODE[swiglu_mode])
        self.act_dtype = experts.dtype
        self.ws = Workspace(expert_slot.device)
        # per-call fast path of __call__: the bound entry point, the
        # descriptor reference, and the (workspace, tokens) last sized for
        self._layer_fn = lmoe().lmoe_moe_layer_path
        self._desc_ref = ctypes.byref(self.desc)
        self._ready: tuple | None = None
        self._stage: torch.Tensor | None = None  # device rows for host-buffer calls

    def workspace_bytes(self, tokens: int) -> int:
        cache = self.__dict__.setdefault("_ws_bytes", {})
        n = cache.get((tokens, self.path))
        if n is None:
            n = int(lmoe().lmoe_workspace_size_path(ctypes.byref(self.desc), int(tokens), _lib.PATH[self.path]))
            if n == 0:
                raise _lib.LmoeError(_lib.LMOE_EUNSUPPORTED, "layer descriptor")
            cache[(tokens, self.path)] = n
        return n

    def _x(self, x: torch.Tensor) -> torch.Tensor:
        _need_cuda(x)
        if x.dtype != self.act_dtype:
            x = x.to(self.act_dtype)
        return x.reshape(-1, x.shape[-1]).contiguous()

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, idx: torch.Tensor | None = None,
                 w: torch.Tensor | None = None, hash_idx: torch.Tensor | None = None) -> torch.Tensor:
        """The whole layer.  ``hash_idx`` [T, top_k] selects the experts of
        each token (token-id hash routing) instead of the router's top-k."""
        if (out is None and idx is None and w is None and hash_idx is None and x.dtype is self.act_dtype
                and x.dim() == 2 and not x.is_cuda and x.is_contiguous() and x.is_pinned()):
            # host buffers: the rows are staged on the device by a kernel and
            # the result is written into pinned host memory by the combine
            # (returned tensor: filled when the current stream reaches the end
            # of this call; x must stay unchanged until then)
            T = x.shape[0]
            ready = self._ready
            if ready is None or ready[0] is not self.ws or ready[1] != T:
                self.ws.ensure(self.workspace_bytes(T))
                self._ready = (self.ws, T)
            stage = self._stage
            if stage is None or stage.numel() < x.numel():
                self._stage = stage = torch.empty(x.numel(), dtype=x.dtype, device=self.ws.device)
            buf = self.ws.buf
            out = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
            rc = lmoe().lmoe_moe_layer_host(self._desc_ref, x.data_ptr(), T, out.data_ptr(), stage.data_ptr(),
                                            buf.data_ptr(), buf.numel(), _stream(), _lib.PATH[self.path])
            if rc != _lib.LMOE_OK:
                check(rc, "lmoe_moe_layer_host")
            return out
        if (out is None and idx is None and w is None and hash_idx is None and x.dtype is self.act_dtype
                and x.dim() == 2 and x.is_cuda and x.is_contiguous()):
            # steady-state decode call: no reshapes or casts, the workspace
            # already sized for this token count
            T = x.shape[0]
            ready = self._ready
            if ready is None or ready[0] is not self.ws or ready[1] != T:
                self.ws.ensure(self.workspace_bytes(T))
                self._ready = (self.ws, T)
            buf = self.ws.buf
            out = torch.empty_like(x)
            rc = self._layer_fn(self._desc_ref, x.data_ptr(), T, out.data_ptr(), None, None, buf.data_ptr(),
                                buf.numel(), _stream(), _lib.PATH[self.path], None, None)
            if rc != _lib.LMOE_OK:
                check(rc, "lmoe_moe_layer")
            return out
        flat = self._x(x)
        T = flat.shape[0]
        if out is None:
            out = torch.empty_like(flat)
        self.ws.ensure(self.workspace_bytes(T))
        h = _hash(hash_idx, T, self.router.top_k)
        if h is not None:
            check(lmoe().lmoe_moe_layer_hashed(ctypes.byref(self.desc), flat.data_ptr(), T, h.data_ptr(),
                                               out.data_ptr(), _ptr(idx), _ptr(w), self.ws.ptr(), self.ws.nbytes,
                                               _stream(), _lib.PATH[self.path]), "lmoe_moe_layer_hashed")
            return out.reshape(x.shape)
        check(lmoe().lmoe_moe_layer_path(ctypes.byref(self.desc), flat.data_ptr(), T, out.data_ptr(), _ptr(idx),
                                         _ptr(w), self.ws.ptr(), self.ws.nbytes, _stream(), _lib.PATH[self.path],
                                         None, None), "lmoe_moe_layer")
        return out.reshape(x.shape)

    def block(self, x: torch.Tensor, shared_slot: int = -1, residual: torch.Tensor | None = None,
              out: torch.Tensor | None = None, idx: torch.Tensor | None = None,
              w: torch.Tensor | None = None) -> torch.Tensor:
        """The DeepSeek-V4 MoE block with the decoder's residual add, fused
        into the combine (``lmoe_moe_block``): ``residual + (routed +
        shared_expert(x))``, each sum rounded once.  The shared expert is the
        expert in arena slot ``shared_slot`` (-1: none); ``residual`` (None:
        none) may be ``out`` and ``x`` itself (in-place residual stream)."""
        flat = self._x(x)
        T = flat.shape[0]
        if out is None:
            out = torch.empty_like(flat)
        res = None
        if residual is not None:
            res = residual.reshape(flat.shape)
            if res.dtype != flat.dtype or not res.is_contiguous():
                res = res.to(flat.dtype).contiguous()
        cache = self.__dict__.setdefault("_blk_bytes", {})
        n = cache.get((T, self.path))
        if n is None:
            n = int(lmoe().lmoe_workspace_size_block(ctypes.byref(self.desc), int(T), _lib.PATH[self.path]))
            if n == 0:
                raise _lib.LmoeError(_lib.LMOE_EUNSUPPORTED, "layer descriptor")
            cache[(T, self.path)] = n
        self.ws.ensure(n)
        check(lmoe().lmoe_moe_block(ctypes.byref(self.desc), int(shared_slot), flat.data_ptr(), T, _ptr(res),
                                    out.data_ptr(), _ptr(idx), _ptr(w), self.ws.ptr(), self.ws.nbytes, _stream(),
                                    _lib.PATH[self.path]), "lmoe_moe_block")
        return out.reshape(x.shape)

    def call_static(self, x: torch.Tensor, out: torch.Tensor | None = None, idx: torch.Tensor | None = None,
                    w: torch.Tensor | None = None) -> torch.Tensor:
        """The layer through ``lmoe_moe_layer_static``: no workspace is
        allocated; the library's fixed 8 MiB device scratch is used instead
        (for callers that cannot allocate device memory).  It always runs the
        decode path.  Calls that overlap on the GPU share that scratch and
        must not run concurrently.  :func:`static_status` reports the device
        error flag of the latest such call."""
        flat = self._x(x)
        T = flat.shape[0]
        if out is None:
            out = torch.empty_like(flat)
        check(lmoe().lmoe_moe_layer_static(ctypes.byref(self.desc), flat.data_ptr(), T, out.data_ptr(), _ptr(idx),
                                           _ptr(w), _stream()), "lmoe_moe_layer_static")
        return out.reshape(x.shape)

    def staged(self, x: torch.Tensor, out: torch.Tensor, ev_routed: torch.cuda.Event,
               ev_gateup: torch.cuda.Event, idx: torch.Tensor | None = None) -> torch.Tensor:
        """The layer with CUDA events recorded after routing and after gate/up
        (for per-kernel timing on the launching stream)."""
        flat = self._x(x)
        T = flat.shape[0]
        self.ws.ensure(self.workspace_bytes(T))
        check(lmoe().lmoe_moe_layer_path(ctypes.byref(self.desc), flat.data_ptr(), T, out.data_ptr(), _ptr(idx),
                                         None, self.ws.ptr(), self.ws.nbytes, _stream(), _lib.PATH[self.path],
                                         _event(ev_routed), _event(ev_gateup)), "lmoe_moe_layer_staged")
        return out

    def timed(self, x: torch.Tensor, out: torch.Tensor, ev_router: torch.cuda.Event,
              ev_experts: torch.cuda.Event, idx: torch.Tensor | None = None) -> torch.Tensor:
        """The launches of ``__call__`` (AUTO path) with CUDA events at kernel
        boundaries: after the routing kernel and after the first expert
        kernel (``lmoe_moe_layer_timed``).  Unlike :meth:`staged`, the routing
        is not complete at ``ev_router`` when the top-k runs in the expert
        kernel, so the timed launches are exactly the untimed ones."""
        flat = self._x(x)
        T = flat.shape[0]
        self.ws.ensure(self.workspace_bytes(T))
        check(lmoe().lmoe_moe_layer_timed(ctypes.byref(self.desc), flat.data_ptr(), T, out.data_ptr(), _ptr(idx),
                                          None, self.ws.ptr(), self.ws.nbytes, _stream(), _event(ev_router),
                                          _event(ev_experts)), "lmoe_moe_layer_timed")
        return out

    def route(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return route(self._x(x), self.router, self.ws)

    def products(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor | None,
                 out: torch.Tensor) -> torch.Tensor:
        """``lmoe_moe_products``: into ``out`` [T*top_k, hidden], the rounded
        ``y * w`` row (``y`` when ``w`` is None) of every route whose expert
        id is >= 0; rows of the routes marked -1 are left untouched."""
        flat = self._x(x)
        T = flat.shape[0]
        idx = idx.reshape(T, -1).to(torch.int32).contiguous()
        if idx.shape[1] != self.router.top_k:
            raise ValueError("routing width must equal top_k")
        wf = None if w is None else w.reshape(T, -1).to(torch.float32).contiguous()
        self.ws.ensure(self.workspace_bytes(T))
        check(lmoe().lmoe_moe_products(ctypes.byref(self.desc), flat.data_ptr(), T, idx.data_ptr(), _ptr(wf),
                                       out.data_ptr(), self.ws.ptr(), self.ws.nbytes, _stream()), "lmoe_moe_products")
        return out

    def routed(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
        flat = self._x(x)
        T = flat.shape[0]
        idx = idx.reshape(T, -1).to(torch.int32).contiguous()
        w = w.reshape(T, -1).to(torch.float32).contiguous()
        if idx.shape[1] != self.router.top_k:
            raise ValueError("routing width must equal top_k")
        if out is None:
            out = torch.empty_like(flat)
        self.ws.ensure(self.workspace_bytes(T))
        check(lmoe().lmoe_moe_routed(ctypes.byref(self.desc), flat.data_ptr(), T, idx.data_ptr(), w.data_ptr(),
                                     out.data_ptr(), self.ws.ptr(), self.ws.nbytes, _stream()), "lmoe_moe_routed")
        return out.reshape(x.shape)


def combine_routes(products: torch.Tensor, top_k: int, w: torch.Tensor | None = None,
                   order: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``lmoe_combine_routes``: per token, the fp32 sum of its ``top_k`` route
    rows (times ``w`` when given), in ``order`` ([T, top_k] route positions;
    route order by default), rounded once."""
    _need_cuda(products)
    R, H = products.shape
    T = R // top_k
    if out is None:
        out = torch.empty((T, H), dtype=products.dtype, device=products.device)
    wf = None if w is None else w.reshape(-1).to(torch.float32).contiguous()
    of = None if order is None else order.reshape(-1).to(torch.int32).contiguous()
    check(lmoe().lmoe_combine_routes(products.data_ptr(), _ptr(wf), _ptr(of), T, int(top_k), H,
                                     _ACT[products.dtype], out.data_ptr(), _stream()), "lmoe_combine_routes")
    return out


def static_status() -> None:
    """Synchronise and raise if the latest ``lmoe_moe_layer_static`` call on
    the current device flagged a bad expert id or slot (clears the flag)."""
    check(lmoe().lmoe_static_status(_stream()), "static scratch status")


def _hash(hash_idx: torch.Tensor | None, T: int, k: int) -> torch.Tensor | None:
    if hash_idx is None:
        return None
    _need_cuda(hash_idx)
    h = hash_idx.reshape(T, -1)
    if h.shape[1] != k:
        raise ValueError(f"hash_idx must hold top_k={k} experts per token")
    return h.to(torch.int32).contiguous()


def route(x: torch.Tensor, router: RouterArrays, ws: Workspace | None = None,
          hash_idx: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Router kernel only: x [T, hidden] -> (idx int32 [T, k], w fp32 [T, k]).

    ``hash_idx`` [T, k] (token-id hash routing): the experts are given; the
    weights are their normalised, routed-scaled scores."""
    _need_cuda(x, router.weight)
    if x.dtype not in _ACT:
        raise ValueError(f"unsupported activation dtype {x.dtype}")
    flat = x.reshape(-1, x.shape[-1]).contiguous()
    T, H = flat.shape
    k = router.top_k
    idx = torch.empty((T, k), dtype=torch.int32, device=flat.device)
    w = torch.empty((T, k), dtype=torch.float32, device=flat.device)
    desc = router.ctype()
    n = lmoe().lmoe_workspace_size_route(ctypes.byref(desc), H, T)
    if n == 0:
        raise _lib.LmoeError(_lib.LMOE_EUNSUPPORTED, "router descriptor")
    ws = (ws or Workspace(flat.device)).ensure(int(n))
    h = _hash(hash_idx, T, k)
    if h is None:
        check(lmoe().lmoe_route(ctypes.byref(desc), H, _ACT[flat.dtype], flat.data_ptr(), T, idx.data_ptr(),
                                w.data_ptr(), ws.ptr(), ws.nbytes, _stream()), "lmoe_route")
    else:
        check(lmoe().lmoe_route_hashed(ctypes.byref(desc), H, _ACT[flat.dtype], flat.data_ptr(), T, h.data_ptr(),
                                       idx.data_ptr(), w.data_ptr(), ws.ptr(), ws.nbytes, _stream()),
              "lmoe_route_hashed")
    return idx, w


_route_ws: dict[int, Workspace] = {}


def _routes_ws(device: torch.device, routes: int, hidden: int, inter: int, n_slots: int) -> Workspace:
    key = device.index if device.index is not None else torch.cuda.current_device()
    ws = _route_ws.get(key)
    if ws is None:
        ws = _route_ws[key] = Workspace(torch.device("cuda", key))
    n = lmoe().lmoe_workspace_size_routes(int(routes), int(hidden), int(inter), int(n_slots))
    return ws.ensure(int(n))


def gateup_swiglu(x: torch.Tensor, slots: torch.Tensor, experts: ExpertArrays, limit: float,
                  mode: str = "fused") -> torch.Tensor:
    """Fused gate/up + clamped SwiGLU for [T, k] routes -> [T*k, inter]."""
    _need_cuda(x, slots)
    T = x.shape[0]
    slots = slots.reshape(T, -1).to(torch.int32).contiguous()
    k = slots.shape[1]
    x = x.reshape(T, -1).to(experts.dtype).contiguous()
    h = torch.empty((T * k, experts.inter), dtype=experts.dtype, device=x.device)
    ws = _routes_ws(x.device, T * k, experts.hidden, experts.inter, experts.n_slots)
    desc = experts.ctype()
    check(lmoe().lmoe_gateup_swiglu(ctypes.byref(desc), x.data_ptr(), T, k, slots.data_ptr(), float(limit),
                                    _lib.SWIGLU_MODE[mode], h.data_ptr(), ws.ptr(), ws.nbytes, _stream()),
          "lmoe_gateup_swiglu")
    return h


def gather_qmm(x: torch.Tensor, slots: torch.Tensor, proj: QProjArrays) -> torch.Tensor:
    """``mx.gather_qmm(x, w, s, b, rhs_indices=slots, transpose=True)`` with one
    input row per route: x [R, cols], slots [R] -> [R, rows]."""
    _need_cuda(x, slots)
    R = x.shape[0]
    slots = slots.reshape(-1).to(torch.int32).contiguous()
    if slots.numel() != R:
        raise ValueError("one slot per input row")
    x = x.reshape(R, -1).to(proj.scales.dtype).contiguous()
    y = torch.empty((R, proj.rows), dtype=proj.scales.dtype, device=x.device)
    ws = _routes_ws(x.device, R, proj.cols, proj.rows, int(proj.weight.shape[0]))
    desc = proj.ctype()
    check(lmoe().lmoe_gather_qmm(ctypes.byref(desc), int(proj.weight.shape[0]), proj.rows, proj.cols,
                                 _ACT[proj.scales.dtype], x.data_ptr(), R, slots.data_ptr(), y.data_ptr(),
                                 ws.ptr(), ws.nbytes, _stream()), "lmoe_gather_qmm")
    return y
