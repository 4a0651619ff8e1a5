"""ctypes binding of the slot-residency planner (include/locali_core.h).

Same Python surface as the reference's locali_native.py (NativeCache :58,
plan :113, peek, note_token, probation/protected sizes, close), loading this
project's own liblocali_core.so.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

from ._lib import CORE_PATH

DEFAULT_LIBRARY = CORE_PATH


class _Result(ctypes.Structure):
    _fields_ = [
        ("key", ctypes.c_int32),
        ("slot", ctypes.c_int32),
        ("evicted_key", ctypes.c_int32),
        ("hit", ctypes.c_uint8),
        ("placed", ctypes.c_uint8),
    ]


@dataclass(frozen=True)
class CacheResult:
    key: int
    slot: int
    evicted_key: int
    hit: bool
    placed: bool


def available(path: Path = DEFAULT_LIBRARY) -> bool:
    return Path(path).is_file()


def ensure_available(path: Path = DEFAULT_LIBRARY) -> bool:
    """Build the planner library on first use when it is missing."""
    if available(path):
        return True
    try:
        from .csrc.build import build_core

        build_core()
    except Exception:
        return False
    return available(path)


_POLICIES = {"slru": 0, "lfu-decay": 1}


class NativeCache:
    def __init__(self, key_capacity: int, slots: int, protected_capacity: int, *, policy: str = "slru",
                 library: Path = DEFAULT_LIBRARY):
        self._cache = None
        if policy not in _POLICIES:
            raise ValueError(f"unknown native cache policy: {policy}")
        lib = ctypes.CDLL(str(library))
        i32, vp = ctypes.c_int32, ctypes.c_void_p
        lib.locali_cache_create_policy.argtypes = [i32, i32, i32, i32]
        lib.locali_cache_create_policy.restype = vp
        lib.locali_cache_destroy.argtypes = [vp]
        lib.locali_cache_note_token.argtypes = [vp]
        lib.locali_cache_plan.argtypes = [vp, ctypes.POINTER(i32), ctypes.c_size_t, ctypes.POINTER(i32),
                                          ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(_Result)]
        lib.locali_cache_plan.restype = ctypes.c_int
        lib.locali_cache_peek.argtypes = [vp, i32]
        lib.locali_cache_peek.restype = i32
        lib.locali_cache_probation_size.argtypes = [vp]
        lib.locali_cache_probation_size.restype = i32
        lib.locali_cache_protected_size.argtypes = [vp]
        lib.locali_cache_protected_size.restype = i32
        self._lib = lib
        self._cache = lib.locali_cache_create_policy(key_capacity, slots, protected_capacity, _POLICIES[policy])
        if not self._cache:
            raise MemoryError("failed to create the native slot planner")

    def note_token(self) -> None:
        self._lib.locali_cache_note_token(self._cache)

    def plan(self, keys, *, pinned_slots=(), touch_hits: bool = True) -> list[CacheResult]:
        keys = list(keys)
        if not keys:
            return []
        pinned_slots = list(pinned_slots)
        karr = (ctypes.c_int32 * len(keys))(*keys)
        parr = (ctypes.c_int32 * len(pinned_slots))(*pinned_slots) if pinned_slots else None
        res = (_Result * len(keys))()
        rc = self._lib.locali_cache_plan(self._cache, karr, len(keys), parr, len(pinned_slots), int(touch_hits), res)
        if rc:
            raise ValueError(f"native cache plan failed with error {rc}")
        return [CacheResult(r.key, r.slot, r.evicted_key, bool(r.hit), bool(r.placed)) for r in res]

    def peek(self, key: int) -> int:
        return int(self._lib.locali_cache_peek(self._cache, key))

    @property
    def probation_size(self) -> int:
        return int(self._lib.locali_cache_probation_size(self._cache))

    @property
    def protected_size(self) -> int:
        return int(self._lib.locali_cache_protected_size(self._cache))

    def close(self) -> None:
        if getattr(self, "_cache", None):
            self._lib.locali_cache_destroy(self._cache)
            self._cache = None

    def __del__(self):
        self.close()
