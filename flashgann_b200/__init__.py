"""FlashGANN-B200: GPU graph ANN search for NVIDIA B200 (sm_100a).

Python mirror of the reference's host interface (SophiaSun18/FlashGANN):

* ``QuantizationGraph(num_nodes, dim, degree, codebook_path)`` with
  ``set_metric`` and ``gpu_search_adaptive(nq, queries, K, result_idx,
  beam_sz) -> elapsed`` (include/qg.hpp:17-63, gpu_search_adaptive.cu:12-114);
* ``load_fvecs`` / ``load_ivecs`` (include/data_io.hpp), ``compute_recall`` and
  ``append_run_stats_to_csv`` (include/common.hpp:49-94),
  ``infer_metric_from_dataset_path`` (include/metric.hpp:13-28).

All search work runs in libflashgann.so (flashgann_b200/csrc); there is no
CPU fallback -- without the library every call raises.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

from . import _capi
from ._capi import (FG_ERR_ARG, FG_ERR_CUDA, FG_ERR_FORMAT, FG_ERR_IO, FG_ERR_NO_DEVICE, FG_ERR_OOM,
                    FG_ERR_UNSUPPORTED, FG_METRIC_IP, FG_METRIC_L2, FG_OK, FlashGANNError, QueryStats, lib)

METRIC_L2 = FG_METRIC_L2
METRIC_IP = FG_METRIC_IP

__all__ = [
    "QuantizationGraph", "FlashGANNError", "QueryStats", "lib", "load_fvecs", "load_ivecs", "compute_recall",
    "append_run_stats_to_csv", "infer_metric_from_dataset_path", "effective_sort_beam_size", "METRIC_L2",
    "METRIC_IP",
    "search_multi",
]


def _check(rc: int, what: str) -> None:
    if rc != FG_OK:
        L = lib()
        raise FlashGANNError(rc, f"{what}: {L.fg_status_string(rc).decode()} ({L.fg_last_error().decode()})")


class QuantizationGraph:
    """A qg_codebook resident on one GPU (include/qg.hpp:14-89).

    Unlike the reference class, which re-uploads the codebook on every
    search call, the codebook is uploaded once here and stays on the device
    until ``close()``.
    """

    def __init__(self, num_node: int, dim: int, degree: int, codebook_path: str, device: int = 0,
                 metric: int = METRIC_L2):
        self._h = ctypes.c_void_p()
        _check(lib().fg_index_load(os.fsencode(codebook_path), num_node, dim, degree, metric, device,
                                   ctypes.byref(self._h)), "fg_index_load")
        self._fill_layout()

    @classmethod
    def from_arrays(cls, rows: np.ndarray, signs: np.ndarray, entry_point: int, dim: int, degree: int,
                    device: int = 0, metric: int = METRIC_L2) -> "QuantizationGraph":
        self = cls.__new__(cls)
        self._h = ctypes.c_void_p()
        rows = np.ascontiguousarray(rows, dtype=np.float32)
        signs = np.ascontiguousarray(signs, dtype=np.float32)
        _check(lib().fg_index_create(rows.ctypes.data_as(ctypes.c_void_p), signs.ctypes.data_as(ctypes.c_void_p),
                                     entry_point & 0xFFFFFFFF, rows.shape[0], dim, degree, metric, device,
                                     ctypes.byref(self._h)), "fg_index_create")
        self._fill_layout()
        return self

    @classmethod
    def from_device(cls, rows, signs, entry_point: int, dim: int, degree: int, metric: int = METRIC_L2
                    ) -> "QuantizationGraph":
        """An index from a codebook already on a GPU (fg_index_create_device):
        rows float32 [n, row_offset] and signs float32 [padded_dim], CUDA
        tensors on the device the index will live on (copied there; the
        tensors may be freed afterwards)."""
        self = cls.__new__(cls)
        self._h = ctypes.c_void_p()
        rows = rows.contiguous()
        signs = signs.contiguous()
        _check(lib().fg_index_create_device(_capi.device_ptr(rows), _capi.device_ptr(signs), entry_point & 0xFFFFFFFF,
                                            rows.shape[0], dim, degree, metric, rows.device.index or 0,
                                            ctypes.byref(self._h)), "fg_index_create_device")
        self._fill_layout()
        return self

    def _fill_layout(self) -> None:
        L = _capi.Layout()
        _check(lib().fg_index_layout(self._h, ctypes.byref(L)), "fg_index_layout")
        self.num_nodes = L.num_nodes
        self.dim = L.dim
        self.padded_dim = L.padded_dim
        self.code_offset = L.code_offset
        self.factor_offset = L.factor_offset
        self.neighbor_offset = L.neighbor_offset
        self.row_offset = L.row_offset
        self.degree = L.degree
        self.entry_point = L.entry_point
        self.metric = L.metric
        self.device = L.device

    # getters of include/qg.hpp:49-60
    def get_code_offset(self) -> int: return self.code_offset
    def get_factor_offset(self) -> int: return self.factor_offset
    def get_neighbor_offset(self) -> int: return self.neighbor_offset
    def get_row_offset(self) -> int: return self.row_offset
    def get_entry_point(self) -> int: return self.entry_point
    def get_metric(self) -> int: return self.metric
    def get_data_bytes(self) -> int: return self.num_nodes * self.row_offset * 4
    def get_signs_bytes(self) -> int: return self.padded_dim * 4

    def set_metric(self, metric: int) -> None:
        _check(lib().fg_index_set_metric(self._h, metric), "fg_index_set_metric")
        self.metric = metric

    def set_plan_goal(self, goal: str) -> None:
        """What the kernel planner aims for: "latency" (the default: the
        shortest time of one batch on an idle GPU) or "throughput" (the most
        queries per second while batches are kept in flight on several
        streams).  Results do not depend on it (fg_index_set_plan_goal)."""
        from ._capi import FG_GOAL_LATENCY, FG_GOAL_THROUGHPUT
        goals = {"latency": FG_GOAL_LATENCY, "throughput": FG_GOAL_THROUGHPUT}
        if goal not in goals:
            raise ValueError(f"plan goal must be 'latency' or 'throughput', not {goal!r}")
        _check(lib().fg_index_set_plan_goal(self._h, goals[goal]), "fg_index_set_plan_goal")

    def search_plan(self, nq: int, K: int, beam: int):
        """(kernel name, queries resident at once) that a batch of nq queries
        would run with under the current goal (fg_search_plan)."""
        from ._capi import FG_PLAN_KERNELS
        k, r = ctypes.c_int32(-1), ctypes.c_int32(0)
        _check(lib().fg_search_plan(self._h, nq, K, beam, ctypes.byref(k), ctypes.byref(r)), "fg_search_plan")
        return FG_PLAN_KERNELS[k.value], r.value

    def gpu_search_adaptive(self, nq: int, queries: np.ndarray, K: int, result_idx: np.ndarray,
                            beam_sz: int) -> float:
        """Search nq queries; fills result_idx[nq*K] (uint32) and returns the
        elapsed seconds of the launch + synchronisation, as the reference
        reports it (gpu_search_adaptive.cu:98-107)."""
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.size < nq * self.dim:
            raise FlashGANNError(FG_ERR_ARG, "queries buffer smaller than nq*dim")
        if result_idx.dtype != np.uint32 or not result_idx.flags.c_contiguous or result_idx.size < nq * K:
            raise FlashGANNError(FG_ERR_ARG, "result_idx must be a contiguous uint32 array of nq*K")
        elapsed = ctypes.c_double()
        _check(lib().fg_search(self._h, nq, q.ctypes.data_as(ctypes.c_void_p), K,
                               result_idx.ctypes.data_as(ctypes.c_void_p), beam_sz, ctypes.byref(elapsed)),
               "fg_search")
        return elapsed.value

    def search(self, queries: np.ndarray, K: int, beam: int) -> np.ndarray:
        q = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, self.dim)
        out = np.empty((q.shape[0], K), dtype=np.uint32)
        self.gpu_search_adaptive(q.shape[0], q, K, out, beam)
        return out

    def search_async(self, slot: int, nq: int, queries: np.ndarray, K: int, result_idx: np.ndarray, beam: int,
                     stream) -> None:
        """Enqueue one host-buffer batch on `stream` (fg_search_async): upload,
        search and download of the ids into result_idx, without waiting.
        `slot` (0 .. FG_ASYNC_SLOTS-1) picks the index's device buffers; keep
        `queries` and `result_idx` alive (and pinned, for overlap) until the
        stream has been synchronised."""
        if result_idx.dtype != np.uint32 or not result_idx.flags.c_contiguous or result_idx.size < nq * K:
            raise FlashGANNError(FG_ERR_ARG, "result_idx must be a contiguous uint32 array of nq*K")
        if queries.dtype != np.float32 or not queries.flags.c_contiguous or queries.size < nq * self.dim:
            raise FlashGANNError(FG_ERR_ARG, "queries must be a contiguous float32 array of nq*dim")
        s = getattr(stream, "cuda_stream", stream) or 0
        _check(lib().fg_search_async(self._h, slot, nq, queries.ctypes.data_as(ctypes.c_void_p), K,
                                     result_idx.ctypes.data_as(ctypes.c_void_p), beam, ctypes.c_void_p(s)),
               "fg_search_async")

    def search_stream(self, batches, K: int, beam: int, depth: int = 2):
        """Pipelined search of an iterable of query batches (float32 [m, dim]
        each): yields the ids (uint32 [m, K]) of every batch in order.  Up to
        `depth` batches are in flight, each with its own slot, stream and
        pinned staging buffers, so one batch's upload and download overlap
        another's search."""
        import torch
        if not 1 <= depth <= _capi.FG_ASYNC_SLOTS:
            raise FlashGANNError(FG_ERR_ARG, f"depth must be in [1, {_capi.FG_ASYNC_SLOTS}]")
        streams = [torch.cuda.Stream(device=self.device) for _ in range(depth)]
        staged = [None] * depth  # (pinned queries, pinned ids, m) per slot
        pending = []  # slots in submission order

        def take(slot):
            streams[slot].synchronize()
            _, hres, m = staged[slot]
            return hres[:m * K].reshape(m, K).copy()

        n = 0
        for b in batches:
            q = np.ascontiguousarray(b, dtype=np.float32).reshape(-1, self.dim)
            m = q.shape[0]
            slot = n % depth
            if len(pending) == depth:
                yield take(pending.pop(0))
            cur = staged[slot]
            if cur is None or cur[0].size < q.size or cur[1].size < m * K:
                hq = torch.empty(max(q.size, 1), dtype=torch.float32).pin_memory().numpy()
                hr = torch.empty(max(m * K, 1), dtype=torch.int32).pin_memory().numpy().view(np.uint32)
                cur = (hq, hr, m)
            hq, hr, _ = cur
            hq[:q.size] = q.reshape(-1)
            staged[slot] = (hq, hr, m)
            self.search_async(slot, m, hq, K, hr, beam, streams[slot])
            pending.append(slot)
            n += 1
        while pending:
            yield take(pending.pop(0))

    def search_device(self, d_queries, K: int, beam: int, d_out=None, d_dists=None, stream=None, d_stats=None,
                      d_trace=None, d_trace_count=None, trace_cap: int = 0):
        """Asynchronous search on device buffers (torch CUDA tensors or raw
        device pointers as ints) on `stream` (torch stream or handle)."""
        ptr = _capi.device_ptr
        nq = int(d_queries.shape[0]) if hasattr(d_queries, "shape") else None
        if nq is None:
            raise FlashGANNError(FG_ERR_ARG, "search_device needs a tensor with a shape")
        s = getattr(stream, "cuda_stream", stream) or 0
        _check(lib().fg_search_device_ex(self._h, nq, ptr(d_queries), K, ptr(d_out), ptr(d_dists), beam,
                                         ctypes.c_void_p(s), ptr(d_stats), ptr(d_trace), ptr(d_trace_count),
                                         trace_cap), "fg_search_device_ex")
        return d_out

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            lib().fg_index_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()



def search_multi(graphs, queries: np.ndarray, K: int, beam: int, with_dists: bool = False):
    """One batch over several QuantizationGraph handles of the same codebook,
    each on its own device (fg_search_multi): the batch is split into balanced
    contiguous slices searched concurrently.  Returns (ids uint32 [nq, K],
    dists float32 [nq, K] or None, elapsed seconds)."""
    q = np.ascontiguousarray(queries, dtype=np.float32)
    nq = q.shape[0]
    hs = (ctypes.c_void_p * len(graphs))(*[g._h.value for g in graphs])
    ids = np.empty((nq, K), dtype=np.uint32)
    dists = np.empty((nq, K), dtype=np.float32) if with_dists else None
    el = ctypes.c_double()
    _check(lib().fg_search_multi(hs, len(graphs), nq, q.ctypes.data_as(ctypes.c_void_p), K,
                                 ids.ctypes.data_as(ctypes.c_void_p),
                                 dists.ctypes.data_as(ctypes.c_void_p) if with_dists else None, beam,
                                 ctypes.byref(el)), "fg_search_multi")
    return ids, dists, el.value


def effective_sort_beam_size(beam: int) -> int:
    return int(lib().fg_effective_sort_beam_size(beam))


def _load_vecs(path: str, dtype) -> np.ndarray:
    L = lib()
    count = ctypes.c_uint64()
    dim = ctypes.c_int32()
    _check(L.fg_vecs_info(os.fsencode(path), ctypes.byref(count), ctypes.byref(dim)), f"fg_vecs_info({path})")
    out = np.empty((count.value, max(dim.value, 0)), dtype=dtype)
    _check(L.fg_vecs_read(os.fsencode(path), out.ctypes.data_as(ctypes.c_void_p), count.value, dim.value),
           f"fg_vecs_read({path})")
    return out


def load_fvecs(path: str) -> np.ndarray:
    """include/data_io.hpp:18-47: count = file_size / (4 + 4*dim)."""
    return _load_vecs(path, np.float32)


def load_ivecs(path: str) -> np.ndarray:
    """include/data_io.hpp:49-77."""
    return _load_vecs(path, np.int32)


def compute_recall(predicted: np.ndarray, groundtruth: np.ndarray, topk: int) -> float:
    """include/common.hpp:49-66 (fraction; duplicates in a row all count)."""
    p = np.ascontiguousarray(predicted, dtype=np.uint32)
    g = np.ascontiguousarray(groundtruth, dtype=np.int32)
    return float(lib().fg_compute_recall(p.ctypes.data_as(ctypes.c_void_p), g.ctypes.data_as(ctypes.c_void_p),
                                         p.shape[0], topk, g.shape[1]))


def append_run_stats_to_csv(filename: str, k: int, beam: int, runtime: float, latency: float, throughput: float,
                            recall: float) -> None:
    """include/common.hpp:68-94."""
    _check(lib().fg_append_run_stats_csv(os.fsencode(filename), k, beam, runtime, latency, throughput, recall),
           "fg_append_run_stats_csv")


def infer_metric_from_dataset_path(path: str) -> int:
    """include/metric.hpp:13-28."""
    return int(lib().fg_infer_metric_from_path(os.fsencode(path)))
