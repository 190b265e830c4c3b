"""ctypes bindings of the native host runtime (csrc/runtime/host_runtime.cpp)."""
from __future__ import annotations

import ctypes
import threading

import numpy as np

from .. import _build

_lib = None
_lock = threading.Lock()

_I32P = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")


def lib():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            L = ctypes.CDLL(_build.build_hostlib())
            L.sched_alloc_create.restype = ctypes.c_void_p
            L.sched_alloc_create.argtypes = [ctypes.c_int32]
            L.sched_alloc_destroy.argtypes = [ctypes.c_void_p]
            L.sched_alloc_free_count.restype = ctypes.c_int32
            L.sched_alloc_free_count.argtypes = [ctypes.c_void_p]
            L.sched_alloc_take.restype = ctypes.c_int32
            L.sched_alloc_take.argtypes = [ctypes.c_void_p, ctypes.c_int32, _I32P]
            L.sched_alloc_give.restype = ctypes.c_int32
            L.sched_alloc_give.argtypes = [ctypes.c_void_p, ctypes.c_int32, _I32P]
            L.sched_plan_decode.restype = ctypes.c_int32
            L.sched_plan_decode.argtypes = [ctypes.c_int32, _I32P, ctypes.c_int32, ctypes.c_int32,
                                            _I32P, _I32P, _I32P]
            L.sched_plan_task_costs.argtypes = [ctypes.c_int32, _I32P, ctypes.c_int32, _F32P]
            L.sched_order_grouped_lpt.argtypes = [_F32P, ctypes.c_int32, ctypes.c_int32, _I32P]
            L.sched_order_region.argtypes = [_F32P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _I32P]
            _lib = L
    return _lib


class PageAllocator:
    """KV page free list (native). ``take`` is all-or-nothing."""

    def __init__(self, num_pages: int):
        self.num_pages = int(num_pages)
        self._h = lib().sched_alloc_create(self.num_pages)
        if not self._h:
            raise MemoryError("page allocator creation failed")

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            _lib.sched_alloc_destroy(h)

    @property
    def free(self) -> int:
        return lib().sched_alloc_free_count(self._h)

    def take(self, n: int) -> np.ndarray | None:
        out = np.empty(max(0, n), dtype=np.int32)
        if lib().sched_alloc_take(self._h, int(n), out) != 0:
            return None
        return out

    def give(self, pages) -> None:
        arr = np.ascontiguousarray(pages, dtype=np.int32)
        if arr.size and lib().sched_alloc_give(self._h, arr.size, arr) != 0:
            raise ValueError("returning a page that is not allocated (double free)")


def plan_decode(seq_lens: np.ndarray, splits: int, blk: int = 128):
    """Decode work items [B*S, 4], merge_req [B], merge_begin [B+1]."""
    B = int(seq_lens.size)
    s = max(1, int(splits))
    items = np.empty((B * s, 4), dtype=np.int32)
    mreq = np.empty(max(B, 1), dtype=np.int32)
    mbeg = np.empty(B + 1, dtype=np.int32)
    lib().sched_plan_decode(B, np.ascontiguousarray(seq_lens, dtype=np.int32), s, blk, items, mreq, mbeg)
    return items, mreq[:B], mbeg


def task_costs(items: np.ndarray, n_items: int, hkv: int) -> np.ndarray:
    out = np.empty(n_items * hkv, dtype=np.float32)
    lib().sched_plan_task_costs(n_items, np.ascontiguousarray(items[:n_items]), hkv, out)
    return out


def grouped_lpt(cost: np.ndarray, block: int = 16) -> np.ndarray:
    c = np.ascontiguousarray(cost, dtype=np.float32)
    out = np.empty(c.size, dtype=np.int32)
    lib().sched_order_grouped_lpt(c, c.size, int(block), out)
    return out


def region_order(cost: np.ndarray, R: int, block: int = 16) -> np.ndarray:
    c = np.ascontiguousarray(cost, dtype=np.float32)
    out = np.empty(c.size, dtype=np.int32)
    lib().sched_order_region(c, c.size, int(R), int(block), out)
    return out
