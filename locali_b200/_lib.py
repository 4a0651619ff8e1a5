"""ctypes bindings of liblmoe.so (include/lmoe.h) and liblocali_core.so.

The libraries are built in-tree by ``locali_b200.csrc.build``.  Loading fails
loudly: there is no CPU or pure-PyTorch fallback for any kernel.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
# LMOE_LIBRARY overrides the library path (for comparing builds)
LMOE_PATH = Path(os.environ["LMOE_LIBRARY"]) if os.environ.get("LMOE_LIBRARY") else PKG / "liblmoe.so"
CORE_PATH = PKG / "liblocali_core.so"

LMOE_OK = 0
LMOE_EINVAL = -1
LMOE_EUNSUPPORTED = -2
LMOE_EINDEX = -3
LMOE_ECUDA = -4
LMOE_EWORKSPACE = -5

LMOE_BF16 = 0
LMOE_F16 = 1

SCORING = {"sigmoid": 0, "softmax": 1, "sqrtsoftplus": 2}
SWIGLU_MODE = {"fused": 0, "stock": 1}
# expert-product path of a layer call (LMOE_PATH_*)
PATH = {"auto": 0, "decode": 1, "prefill": 2}
PREFILL_MIN_ROUTES = 256
PREFILL_ROUTES_PER_4_EXPERTS = 7


def auto_takes_prefill(tokens: int, top_k: int, n_experts: int) -> bool:
    """LMOE_PATH_AUTO's choice for a layer where both paths are available."""
    routes = tokens * top_k
    return routes >= PREFILL_MIN_ROUTES and 4 * routes >= PREFILL_ROUTES_PER_4_EXPERTS * n_experts


class QProj(ctypes.Structure):
    _fields_ = [
        ("weight", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("biases", ctypes.c_void_p),
        ("bits", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("tiles", ctypes.c_void_p),
    ]


class Experts(ctypes.Structure):
    _fields_ = [
        ("n_slots", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("inter", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("gate", QProj),
        ("up", QProj),
        ("down", QProj),
    ]


class Router(ctypes.Structure):
    _fields_ = [
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("n_experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("scoring", ctypes.c_int32),
        ("norm_topk", ctypes.c_int32),
        ("routed_scaling", ctypes.c_float),
    ]


class Layer(ctypes.Structure):
    _fields_ = [
        ("router", Router),
        ("experts", Experts),
        ("expert_slot", ctypes.c_void_p),
        ("swiglu_limit", ctypes.c_float),
        ("swiglu_mode", ctypes.c_int32),
    ]


class LmoeError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: {strerror(status)} ({status})" if what else strerror(status))


_VP = ctypes.c_void_p
_SIGS = {
    "lmoe_version": ([], ctypes.c_int),
    "lmoe_strerror": ([ctypes.c_int], ctypes.c_char_p),
    "lmoe_workspace_size": ([ctypes.POINTER(Layer), ctypes.c_int32], ctypes.c_size_t),
    "lmoe_workspace_size_routes": ([ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32],
                                   ctypes.c_size_t),
    "lmoe_workspace_init": ([_VP, ctypes.c_size_t, _VP], ctypes.c_int),
    "lmoe_workspace_status": ([_VP, _VP], ctypes.c_int),
    "lmoe_route": ([ctypes.POINTER(Router), ctypes.c_int32, ctypes.c_int32, _VP, ctypes.c_int32, _VP, _VP, _VP,
                    ctypes.c_size_t, _VP], ctypes.c_int),
    "lmoe_workspace_size_route": ([ctypes.POINTER(Router), ctypes.c_int32, ctypes.c_int32], ctypes.c_size_t),
    "lmoe_route_hashed": ([ctypes.POINTER(Router), ctypes.c_int32, ctypes.c_int32, _VP, ctypes.c_int32, _VP, _VP, _VP,
                           _VP, ctypes.c_size_t, _VP], ctypes.c_int),
    "lmoe_moe_layer_hashed": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, _VP, _VP, ctypes.c_size_t,
                               _VP, ctypes.c_int32], ctypes.c_int),
    "lmoe_moe_layer": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, _VP, ctypes.c_size_t,
                        _VP], ctypes.c_int),
    "lmoe_moe_layer_staged": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, _VP, ctypes.c_size_t,
                               _VP, _VP, _VP], ctypes.c_int),
    "lmoe_moe_layer_path": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, _VP, ctypes.c_size_t,
                             _VP, ctypes.c_int32, _VP, _VP], ctypes.c_int),
    "lmoe_moe_layer_timed": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, _VP, ctypes.c_size_t,
                              _VP, _VP, _VP], ctypes.c_int),
    "lmoe_workspace_size_path": ([ctypes.POINTER(Layer), ctypes.c_int32, ctypes.c_int32], ctypes.c_size_t),
    "lmoe_moe_layer_static": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, _VP], ctypes.c_int),
    "lmoe_static_workspace_bytes": ([], ctypes.c_size_t),
    "lmoe_static_status": ([_VP], ctypes.c_int),
    "lmoe_moe_layer_host": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, ctypes.c_size_t, _VP,
                             ctypes.c_int32], ctypes.c_int),
    "lmoe_moe_routed": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, _VP, ctypes.c_size_t,
                         _VP], ctypes.c_int),
    "lmoe_gateup_swiglu": ([ctypes.POINTER(Experts), _VP, ctypes.c_int32, ctypes.c_int32, _VP, ctypes.c_float,
                            ctypes.c_int32, _VP, _VP, ctypes.c_size_t, _VP], ctypes.c_int),
    "lmoe_gather_qmm": ([ctypes.POINTER(QProj), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                         _VP, ctypes.c_int32, _VP, _VP, _VP, ctypes.c_size_t, _VP], ctypes.c_int),
    "lmoe_tile_bytes": ([ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32], ctypes.c_size_t),
    "lmoe_tile_pack": ([ctypes.POINTER(QProj), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                        ctypes.c_int32, _VP, _VP], ctypes.c_int),
    "lmoe_moe_products": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, _VP, _VP, _VP, _VP, ctypes.c_size_t, _VP],
                          ctypes.c_int),
    "lmoe_combine_routes": ([_VP, _VP, _VP, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _VP,
                             _VP], ctypes.c_int),
    "lmoe_moe_block": ([ctypes.POINTER(Layer), ctypes.c_int32, _VP, ctypes.c_int32, _VP, _VP, _VP, _VP, _VP,
                        ctypes.c_size_t, _VP, ctypes.c_int32], ctypes.c_int),
    "lmoe_workspace_size_block": ([ctypes.POINTER(Layer), ctypes.c_int32, ctypes.c_int32], ctypes.c_size_t),
    "lmoe_ep_row_bytes": ([ctypes.c_int32, ctypes.c_int32], ctypes.c_size_t),
    "lmoe_ep_dispatch": ([_VP, _VP, _VP, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                          ctypes.c_int32, _VP, _VP, _VP, _VP], ctypes.c_int),
    "lmoe_ep_workspace_size": ([ctypes.POINTER(Layer), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32],
                               ctypes.c_size_t),
    "lmoe_ep_experts": ([ctypes.POINTER(Layer), _VP, ctypes.c_int32, ctypes.c_int32, _VP, _VP, ctypes.c_size_t,
                         _VP, ctypes.c_int32], ctypes.c_int),
    "lmoe_ep_combine": ([_VP, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _VP, _VP, _VP, _VP,
                         ctypes.c_float, _VP], ctypes.c_int),
}

CORE_SYMBOLS = [
    "locali_cache_create",
    "locali_cache_create_policy",
    "locali_cache_destroy",
    "locali_cache_note_token",
    "locali_cache_plan",
    "locali_cache_peek",
    "locali_cache_probation_size",
    "locali_cache_protected_size",
]

_lmoe = None


def lmoe() -> ctypes.CDLL:
    """The loaded liblmoe.so; raises if it has not been built."""
    global _lmoe
    if _lmoe is None:
        if not LMOE_PATH.is_file():
            raise RuntimeError(
                f"{LMOE_PATH} is missing: build it with `python -m locali_b200.csrc.build` "
                "(no CPU fallback exists for the routed-MoE kernels)"
            )
        lib = ctypes.CDLL(str(LMOE_PATH))
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        if lib.lmoe_version() != 2:
            raise RuntimeError("liblmoe.so ABI version mismatch; rebuild it")
        _lmoe = lib
    return _lmoe


def strerror(status: int) -> str:
    try:
        return lmoe().lmoe_strerror(status).decode()
    except Exception:  # library missing: still give a message
        return f"status {status}"


def check(status: int, what: str = "") -> None:
    if status != LMOE_OK:
        raise LmoeError(status, what)
