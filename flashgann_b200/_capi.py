"""ctypes declarations of libflashgann.so (include/flashgann.h).

The library is built in-tree (``make lib`` or ``__graft_entry__.build()``)
and loaded from this directory; a missing library raises ImportError.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

FG_OK = 0
FG_ERR_IO = 1
FG_ERR_FORMAT = 2
FG_ERR_ARG = 3
FG_ERR_CUDA = 4
FG_ERR_OOM = 5
FG_ERR_UNSUPPORTED = 6
FG_ERR_NO_DEVICE = 7
FG_METRIC_L2 = 0
FG_METRIC_IP = 1
FG_ASYNC_SLOTS = 4
FG_GOAL_LATENCY = 0
FG_GOAL_THROUGHPUT = 1
FG_PLAN_KERNELS = {0: "cta", 1: "warp", 2: "staged", 3: "pair"}

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libflashgann.so")


class FlashGANNError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class Layout(ctypes.Structure):
    _fields_ = [("num_nodes", ctypes.c_uint64), ("dim", ctypes.c_uint64), ("padded_dim", ctypes.c_uint64),
                ("code_offset", ctypes.c_uint64), ("factor_offset", ctypes.c_uint64),
                ("neighbor_offset", ctypes.c_uint64), ("row_offset", ctypes.c_uint64), ("degree", ctypes.c_int32),
                ("entry_point", ctypes.c_uint32), ("metric", ctypes.c_int32), ("device", ctypes.c_int32)]


class QueryStats(ctypes.Structure):
    _fields_ = [("iterations", ctypes.c_uint32), ("expansions", ctypes.c_uint32), ("evaluations", ctypes.c_uint32),
                ("estimates", ctypes.c_uint32)]


# (name, restype, argtypes) for every entry point of include/flashgann.h
_vp = ctypes.c_void_p
_u64 = ctypes.c_uint64
_i32 = ctypes.c_int32
_u32 = ctypes.c_uint32
_f64 = ctypes.c_double
_cs = ctypes.c_char_p
SIGNATURES = [
    ("fg_status_string", ctypes.c_char_p, [ctypes.c_int]),
    ("fg_last_error", ctypes.c_char_p, []),
    ("fg_index_load", ctypes.c_int, [_cs, _u64, _u64, _i32, _i32, _i32, ctypes.POINTER(_vp)]),
    ("fg_index_create", ctypes.c_int, [_vp, _vp, _u32, _u64, _u64, _i32, _i32, _i32, ctypes.POINTER(_vp)]),
    ("fg_index_create_device", ctypes.c_int, [_vp, _vp, _u32, _u64, _u64, _i32, _i32, _i32, ctypes.POINTER(_vp)]),
    ("fg_index_free", ctypes.c_int, [_vp]),
    ("fg_index_layout", ctypes.c_int, [_vp, ctypes.POINTER(Layout)]),
    ("fg_index_set_metric", ctypes.c_int, [_vp, _i32]),
    ("fg_index_set_plan_goal", ctypes.c_int, [_vp, _i32]),
    ("fg_search_plan", ctypes.c_int, [_vp, _i32, _i32, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    ("fg_search", ctypes.c_int, [_vp, _i32, _vp, _i32, _vp, _i32, ctypes.POINTER(_f64)]),
    ("fg_search_noalloc", ctypes.c_int, [_vp, _i32, _vp, _i32, _vp, _i32, ctypes.POINTER(_f64)]),
    ("fg_search_async", ctypes.c_int, [_vp, _i32, _i32, _vp, _i32, _vp, _i32, _vp]),
    ("fg_search_multi", ctypes.c_int, [ctypes.POINTER(_vp), _i32, _i32, _vp, _i32, _vp, _vp, _i32, ctypes.POINTER(_f64)]),
    ("fg_search_device", ctypes.c_int, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _vp]),
    ("fg_search_device_ex", ctypes.c_int, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _i32]),
    ("fg_query_prepare_device", ctypes.c_int, [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("fg_beam_merge_device", ctypes.c_int, [_vp, _vp, _i32, _i32, _i32, _i32, _vp]),
    ("fg_shard_merge_device", ctypes.c_int, [_vp, _vp, ctypes.POINTER(_u32), _i32, _i32, _i32, _i32, _vp, _vp, _vp]),
    ("fg_effective_sort_beam_size", _u32, [_u32]),
    ("fg_entry_point_centroid", _u32, [_vp, _u64, _u64, _u64, _i32]),
    ("fg_compute_recall", ctypes.c_float, [_vp, _vp, _u64, _i32, _i32]),
    ("fg_append_run_stats_csv", ctypes.c_int, [_cs, _i32, _i32, _f64, _f64, _f64, _f64]),
    ("fg_infer_metric_from_path", _i32, [_cs]),
    ("fg_vecs_info", ctypes.c_int, [_cs, ctypes.POINTER(_u64), ctypes.POINTER(_i32)]),
    ("fg_vecs_read", ctypes.c_int, [_cs, _vp, _u64, _i32]),
]

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load libflashgann.so (in-tree) and declare its signatures."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make lib` (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def device_ptr(x) -> Optional[int]:
    """Raw device address of a torch CUDA tensor, an int, or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if hasattr(x, "is_cuda") and not x.is_cuda:
            raise FlashGANNError(FG_ERR_ARG, "expected a CUDA tensor")
        return x.data_ptr()
    raise FlashGANNError(FG_ERR_ARG, f"cannot take a device pointer of {type(x)!r}")
