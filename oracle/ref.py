"""ctypes binding of oracle/_ref/libfgref.so: the reference's own sm_100a
build plus the harness kernels of oracle/ref_harness.cu.

TEST INFRASTRUCTURE ONLY (golden-vector generation and bench.py's reference
leg).  Needs a GPU; device buffers are torch tensors.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import sys

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libfgref.so")
CLI_PATH = os.path.join(_HERE, "_ref", "gpu_flashgann_ref")

_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not available():
            raise ImportError(f"{LIB_PATH} missing: build it with `make -C oracle ref` where the reference is mounted")
        L = ctypes.CDLL(LIB_PATH)
        vp, sz, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
        L.ref_qg_create.restype = vp
        L.ref_qg_create.argtypes = [ctypes.c_char_p, sz, sz, i, i]
        L.ref_qg_search.argtypes = [vp, i, vp, i, vp, i, ctypes.POINTER(ctypes.c_double)]
        L.ref_qg_free.argtypes = [vp]
        L.ref_internal_topk.restype = i
        L.ref_query_prep.argtypes = [vp, i, i, i, vp, vp, vp, vp, vp]
        L.ref_scan.argtypes = [vp, sz, sz, sz, i, i, i, vp, vp, vp, vp, vp, vp, vp]
        L.ref_l2.argtypes = [vp, i, vp, sz, vp, vp, i, i, vp]
        L.ref_merge.argtypes = [vp, vp, i, i, i, i]
        L.ref_ctrl.argtypes = [i, vp, vp, vp, vp, vp, vp, vp, vp, vp]
        _lib = L
    return _lib


@contextlib.contextmanager
def quiet_stdout():
    """The reference prints progress to stdout; silence it at the fd level."""
    sys.stdout.flush()
    fd = os.dup(1)
    with open(os.devnull, "wb") as dn:
        os.dup2(dn.fileno(), 1)
    try:
        yield
    finally:
        sys.stdout.flush()
        os.dup2(fd, 1)
        os.close(fd)


class RefGraph:
    """The reference's QuantizationGraph (include/qg.hpp) over a codebook file."""

    def __init__(self, path: str, n: int, dim: int, degree: int, use_ip: bool = False, quiet: bool = True):
        self.quiet = quiet
        with (quiet_stdout() if quiet else contextlib.nullcontext()):
            self.h = lib().ref_qg_create(os.fsencode(path), n, dim, degree, int(use_ip))
        self.dim = dim

    def search(self, queries: np.ndarray, K: int, beam: int):
        q = np.ascontiguousarray(queries, dtype=np.float32)
        nq = q.shape[0]
        out = np.zeros((nq, K), dtype=np.uint32)
        el = ctypes.c_double()
        with (quiet_stdout() if self.quiet else contextlib.nullcontext()):
            lib().ref_qg_search(self.h, nq, q.ctypes.data_as(ctypes.c_void_p), K,
                                out.ctypes.data_as(ctypes.c_void_p), beam, ctypes.byref(el))
        return out, el.value

    def close(self):
        if self.h:
            lib().ref_qg_free(self.h)
            self.h = None


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def query_prep(queries: np.ndarray, signs: np.ndarray, dim: int, D: int):
    import torch
    q = torch.from_numpy(np.ascontiguousarray(queries, dtype=np.float32)).cuda()
    s = torch.from_numpy(np.ascontiguousarray(signs, dtype=np.float32)).cuda()
    nq = q.shape[0]
    rot = torch.zeros((nq, D), dtype=torch.float32, device="cuda")
    lut = torch.zeros((nq, 4 * D), dtype=torch.uint8, device="cuda")
    fac = torch.zeros((nq, 3), dtype=torch.float32, device="cuda")
    sq = torch.zeros(nq, dtype=torch.int32, device="cuda")
    rc = lib().ref_query_prep(_p(q), nq, dim, D, _p(s), _p(rot), _p(lut), _p(fac), _p(sq))
    assert rc == 0, rc
    return rot.cpu().numpy(), lut.cpu().numpy(), fac.cpu().numpy(), sq.cpu().numpy()


def scan(rows: np.ndarray, layout, parents: np.ndarray, pdists: np.ndarray, luts: np.ndarray, qfacs: np.ndarray,
         sumqs: np.ndarray):
    import torch
    r = torch.from_numpy(np.ascontiguousarray(rows)).cuda()
    nb = parents.shape[0]
    deg = layout.degree
    par = torch.from_numpy(parents.astype(np.uint32).view(np.int32)).cuda()
    pd = torch.from_numpy(pdists.astype(np.float32)).cuda()
    lt = torch.from_numpy(np.ascontiguousarray(luts, dtype=np.uint8)).cuda()
    qf = torch.from_numpy(np.ascontiguousarray(qfacs, dtype=np.float32)).cuda()
    sq = torch.from_numpy(np.ascontiguousarray(sumqs, dtype=np.int32)).cuda()
    l8 = torch.zeros((nb, deg), dtype=torch.float32, device="cuda")
    sqo = torch.zeros((nb, deg), dtype=torch.float32, device="cuda")
    rc = lib().ref_scan(_p(r), layout.row, layout.code_off, layout.factor_off, deg, layout.padded_dim, nb, _p(par),
                        _p(pd), _p(lt), _p(qf), _p(sq), _p(l8), _p(sqo))
    assert rc == 0, rc
    return l8.cpu().numpy(), sqo.cpu().numpy()


def l2(queries: np.ndarray, rows: np.ndarray, row_floats: int, qidx: np.ndarray, nodes: np.ndarray, use_ip: bool):
    import torch
    q = torch.from_numpy(np.ascontiguousarray(queries, dtype=np.float32)).cuda()
    r = torch.from_numpy(np.ascontiguousarray(rows)).cuda()
    qi = torch.from_numpy(qidx.astype(np.int32)).cuda()
    nd = torch.from_numpy(nodes.astype(np.int32)).cuda()
    out = torch.zeros(len(nodes), dtype=torch.float32, device="cuda")
    rc = lib().ref_l2(_p(q), q.shape[1], _p(r), row_floats, _p(qi), _p(nd), len(nodes), int(use_ip), _p(out))
    assert rc == 0, rc
    return out.cpu().numpy()


def merge(idx: np.ndarray, dist: np.ndarray, itopk: int, cbs: int, first: bool):
    import torch
    i = torch.from_numpy(np.ascontiguousarray(idx, dtype=np.uint32).view(np.int32)).cuda()
    d = torch.from_numpy(np.ascontiguousarray(dist, dtype=np.float32)).cuda()
    rc = lib().ref_merge(_p(i), _p(d), idx.shape[0], itopk, cbs, int(first))
    assert rc == 0, rc
    return i.cpu().numpy().view(np.uint32), d.cpu().numpy()


def ctrl(rho_prev, policy, rate, p2rho, active, cut, near):
    import torch
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dtype=dt)).cuda()
    n = len(rho_prev)
    ro = torch.zeros(n, dtype=torch.float32, device="cuda")
    ko = torch.zeros(n, dtype=torch.int32, device="cuda")
    args = [t(rho_prev, np.float32), t(policy, np.int32), t(rate, np.float32), t(p2rho, np.float32),
            t(np.asarray(active, dtype=np.uint32).view(np.int32), np.int32), t(cut, np.int32),
            t(np.asarray(near, dtype=np.uint32).view(np.int32), np.int32)]
    rc = lib().ref_ctrl(n, *[_p(a) for a in args], _p(ro), _p(ko))
    assert rc == 0, rc
    return ro.cpu().numpy(), ko.cpu().numpy()
