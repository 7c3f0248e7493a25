"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA search path and the CPU
baseline timed by bench.py.  Only tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference legs import this package; the product
(flashgann_b200) never does.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

c_u32p = ctypes.POINTER(ctypes.c_uint32)
c_i32p = ctypes.POINTER(ctypes.c_int32)
c_f32p = ctypes.POINTER(ctypes.c_float)
c_u8p = ctypes.POINTER(ctypes.c_uint8)


class Knobs(ctypes.Structure):
    _fields_ = [
        ("block_size", ctypes.c_int), ("search_width", ctypes.c_int), ("theta_min", ctypes.c_int),
        ("theta_max", ctypes.c_int), ("rho_min", ctypes.c_float), ("rho_max", ctypes.c_float),
        ("min_phase2_keep", ctypes.c_int), ("check_interval", ctypes.c_int),
        ("buffer_bound", ctypes.c_int), ("phase1_theta", ctypes.c_int), ("phase1_rho", ctypes.c_float),
        ("phase2_theta", ctypes.c_int), ("stall_iters", ctypes.c_int), ("max_iterations", ctypes.c_int),
        ("reset_interval", ctypes.c_int), ("hash_base_bitlen", ctypes.c_int),
    ]


class Layout(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_uint64), ("padded_dim", ctypes.c_uint64), ("code_off", ctypes.c_uint64),
                ("factor_off", ctypes.c_uint64), ("nbr_off", ctypes.c_uint64), ("row", ctypes.c_uint64),
                ("degree", ctypes.c_int)]


class Index(ctypes.Structure):
    _fields_ = [("L", Layout), ("n", ctypes.c_uint64), ("data", c_f32p), ("signs", c_f32p),
                ("entry_point", ctypes.c_uint32), ("use_ip", ctypes.c_int)]


class QFactors(ctypes.Structure):
    _fields_ = [("low", ctypes.c_float), ("high", ctypes.c_float), ("width", ctypes.c_float),
                ("sum_q", ctypes.c_int32)]


class Stats(ctypes.Structure):
    _fields_ = [("iterations", ctypes.c_uint64), ("expansions", ctypes.c_uint64),
                ("evaluations", ctypes.c_uint64), ("estimates", ctypes.c_uint64),
                ("phase2_iter", ctypes.c_uint64)]


class Trace(ctypes.Structure):
    _fields_ = [("trace", c_u32p), ("trace_count", c_i32p), ("trace_cap", ctypes.c_int),
                ("n_iters", ctypes.c_int)]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise ImportError(f"oracle library missing: build it with `make -C {_HERE}`")
        L = ctypes.CDLL(_LIB_PATH)
        L.og_default_knobs.argtypes = [ctypes.POINTER(Knobs)]
        L.og_compute_layout.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.POINTER(Layout)]
        L.og_query_prepare.argtypes = [c_f32p, c_f32p, ctypes.c_int, ctypes.c_int, c_f32p, c_u8p, c_u8p,
                                       ctypes.POINTER(QFactors)]
        L.og_search_one.argtypes = [ctypes.POINTER(Index), ctypes.POINTER(Knobs), c_f32p, ctypes.c_int,
                                    ctypes.c_int, c_u32p, c_f32p, ctypes.POINTER(Stats), ctypes.POINTER(Trace)]
        L.og_search_batch.argtypes = [ctypes.POINTER(Index), ctypes.POINTER(Knobs), ctypes.c_int, c_f32p,
                                      ctypes.c_int, ctypes.c_int, c_u32p, ctypes.c_int, ctypes.POINTER(Stats)]
        L.og_hash_bitlen.argtypes = [ctypes.c_uint32] * 4
        L.og_hash_bitlen.restype = ctypes.c_uint32
        L.og_beam_merge.argtypes = [c_u32p, c_f32p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int, ctypes.c_int]
        L.og_candidate_sort.argtypes = [c_u32p, c_f32p, ctypes.c_uint32]
        L.og_estimate.argtypes = [c_u8p, ctypes.POINTER(QFactors), c_u8p, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int]
        L.og_estimate.restype = ctypes.c_float
        L.og_warp_distance.argtypes = [ctypes.c_int, c_f32p, c_f32p, ctypes.c_int]
        L.og_warp_distance.restype = ctypes.c_float
        L.og_effective_sort_beam.argtypes = [ctypes.c_uint32]
        L.og_effective_sort_beam.restype = ctypes.c_uint32
        L.og_candidate_buffer_size.argtypes = [ctypes.c_int, ctypes.POINTER(Knobs)]
        L.og_candidate_buffer_size.restype = ctypes.c_uint32
        L.og_entry_point_centroid.argtypes = [c_f32p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int]
        L.og_entry_point_centroid.restype = ctypes.c_uint32
        L.og_rho_update.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_uint32,
                                    ctypes.c_int, ctypes.c_uint32, ctypes.POINTER(Knobs), c_f32p,
                                    ctypes.POINTER(ctypes.c_int)]
        L.og_compute_recall.argtypes = [c_u32p, c_i32p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
        L.og_compute_recall.restype = ctypes.c_float
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def default_knobs() -> Knobs:
    k = Knobs()
    lib().og_default_knobs(ctypes.byref(k))
    return k


class OracleIndex:
    """A codebook held in host memory for the CPU oracle."""

    def __init__(self, rows: np.ndarray, signs: np.ndarray, entry: int, dim: int, degree: int,
                 use_ip: bool = False):
        self.rows = np.ascontiguousarray(rows, dtype=np.float32)
        self.signs = np.ascontiguousarray(signs, dtype=np.float32)
        L = Layout()
        lib().og_compute_layout(dim, degree, ctypes.byref(L))
        if self.rows.shape[1] != L.row:
            raise ValueError(f"row width {self.rows.shape[1]} != layout row {L.row}")
        if entry == 0xFFFFFFFF:
            entry = int(lib().og_entry_point_centroid(_p(self.rows, c_f32p), self.rows.shape[0], dim, L.row,
                                                      int(use_ip)))
        self.entry = entry
        self.c = Index(L, self.rows.shape[0], _p(self.rows, c_f32p), _p(self.signs, c_f32p), entry, int(use_ip))
        self.dim = dim
        self.degree = degree

    def search_one(self, query: np.ndarray, K: int, beam: int, knobs: Optional[Knobs] = None,
                   trace_cap: int = 0):
        kn = knobs or default_knobs()
        q = np.ascontiguousarray(query, dtype=np.float32)
        ids = np.zeros(K, dtype=np.uint32)
        dists = np.zeros(K, dtype=np.float32)
        st = Stats()
        tr = None
        tbuf = tcnt = None
        if trace_cap:
            tbuf = np.full(trace_cap * kn.search_width, 0xFFFFFFFF, dtype=np.uint32)
            tcnt = np.zeros(trace_cap, dtype=np.int32)
            tr = Trace(_p(tbuf, c_u32p), _p(tcnt, c_i32p), trace_cap, 0)
        rc = lib().og_search_one(ctypes.byref(self.c), ctypes.byref(kn), _p(q, c_f32p), K, beam,
                                 _p(ids, c_u32p), _p(dists, c_f32p), ctypes.byref(st),
                                 ctypes.byref(tr) if tr is not None else None)
        if rc != 0:
            raise ValueError(f"oracle search failed ({rc})")
        out = dict(ids=ids, dists=dists, stats=st)
        if tr is not None:
            n = tr.n_iters
            out["trace"] = tbuf.reshape(trace_cap, kn.search_width)[:n].copy()
            out["trace_count"] = tcnt[:n].copy()
        return out

    def search(self, queries: np.ndarray, K: int, beam: int, threads: int = 0,
               knobs: Optional[Knobs] = None) -> Tuple[np.ndarray, Stats]:
        kn = knobs or default_knobs()
        q = np.ascontiguousarray(queries, dtype=np.float32)
        nq = q.shape[0]
        ids = np.zeros((nq, K), dtype=np.uint32)
        st = Stats()
        rc = lib().og_search_batch(ctypes.byref(self.c), ctypes.byref(kn), nq, _p(q, c_f32p), K, beam,
                                   _p(ids, c_u32p), threads, ctypes.byref(st))
        if rc != 0:
            raise ValueError(f"oracle search failed ({rc})")
        return ids, st


def query_prepare(query: np.ndarray, signs: np.ndarray, dim: int, D: int):
    q = np.ascontiguousarray(query, dtype=np.float32)
    s = np.ascontiguousarray(signs, dtype=np.float32)
    rot = np.zeros(D, dtype=np.float32)
    quant = np.zeros(D, dtype=np.uint8)
    lut = np.zeros(4 * D, dtype=np.uint8)
    qf = QFactors()
    lib().og_query_prepare(_p(q, c_f32p), _p(s, c_f32p), dim, D, _p(rot, c_f32p), _p(quant, c_u8p),
                           _p(lut, c_u8p), ctypes.byref(qf))
    return dict(rotated=rot, quant=quant, lut=lut, low=qf.low, high=qf.high, width=qf.width, sum_q=qf.sum_q)


def beam_merge(idx: np.ndarray, dist: np.ndarray, cbs: int, itopk: int, first: bool, block_size: int = 256):
    i = np.ascontiguousarray(idx, dtype=np.uint32).copy()
    d = np.ascontiguousarray(dist, dtype=np.float32).copy()
    rc = lib().og_beam_merge(_p(i, c_u32p), _p(d, c_f32p), cbs, itopk, int(first), block_size)
    if rc != 0:
        raise ValueError("bad merge arguments")
    return i, d


def candidate_sort(idx: np.ndarray, dist: np.ndarray, cbs: int):
    i = np.ascontiguousarray(idx, dtype=np.uint32).copy()
    d = np.ascontiguousarray(dist, dtype=np.float32).copy()
    lib().og_candidate_sort(_p(i, c_u32p), _p(d, c_f32p), cbs)
    return i, d


def warp_distance(a: np.ndarray, b: np.ndarray, use_ip: bool = False) -> float:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return float(lib().og_warp_distance(a.shape[0], _p(a, c_f32p), _p(b, c_f32p), int(use_ip)))


def compute_recall(pred: np.ndarray, gt: np.ndarray, topk: int) -> float:
    p = np.ascontiguousarray(pred, dtype=np.uint32)
    g = np.ascontiguousarray(gt, dtype=np.int32)
    return float(lib().og_compute_recall(_p(p, c_u32p), _p(g, c_i32p), p.shape[0], topk, g.shape[1]))
