"""Seeded synthetic data and SymphonyQG-layout codebooks.

The reference ships no index builder: its search reads a prebuilt
"SymphonyQG-style codebook with data layout adjustment" (README.md:13) whose
byte layout is fixed by include/qg.hpp:17-42,66-73.  This module writes files
in exactly that layout so the reference build and this build can be run on
identical inputs:

    uint32 entry_point
    n rows x row floats, row = [dim raw floats][deg*D/8 code bytes]
                                [deg triple_x][deg f_dq][deg f_vq][deg uint32 ids]
    D float signs (only the first dim are applied, include/utils.cuh:795-797)

Codes and factors follow the estimator the kernel evaluates
(include/utils.cuh:989-993): for a parent c and neighbour o, with
u = H_D (s * pad(o - c)) (unnormalised Walsh-Hadamard, signs s), bits b = u > 0:

    L2:  triple_x = |o-c|^2 + 2<o-c, c>,  f_dq = -2 |u|^2 / (D <sign(u), u>)
    IP:  triple_x = 0,                     f_dq = -1 |u|^2 / (D <sign(u), u>)
    f_vq = f_dq * sum(2b - 1)

so that triple_x + d(q, c) + f_dq*width*(2*sum_b q - sum q) + f_vq*low
estimates d(q, o).  Invalid neighbour slots hold id 0xFFFFFFFF and
triple_x = FLT_MAX (the kernel's gates at adaptive_search.cuh:233,372 and
utils.cuh:951,1000).

Graph: exact k-NN, merged with reverse k-NN edges, relative-neighbourhood
pruned and filled with the nearest pruned candidates, plus a few seeded random
long edges per node so a single entry point reaches every mixture component.  The graph builder is offline
test/bench infrastructure, not the search path; it uses torch (GPU when
present) for the brute-force distance work.
"""

from __future__ import annotations

import dataclasses
import hashlib
import math
import os
import struct
from typing import Optional, Tuple

import numpy as np
import torch

FLT_MAX = np.float32(3.4028234663852886e38)
INVALID_ID = np.uint32(0xFFFFFFFF)


# --------------------------------------------------------------------------
# layout (include/qg.hpp:66-73)
# --------------------------------------------------------------------------
def padded_dim(dim: int) -> int:
    d = 1
    while d < dim:
        d <<= 1
    return d


@dataclasses.dataclass(frozen=True)
class Layout:
    dim: int
    degree: int
    padded_dim: int
    code_off: int
    factor_off: int
    nbr_off: int
    row: int

    @property
    def code_bytes(self) -> int:
        return self.padded_dim // 8


def layout(dim: int, degree: int) -> Layout:
    D = padded_dim(dim)
    code_off = dim
    factor_off = code_off + (D // 64) * 2 * degree
    nbr_off = factor_off + 3 * degree
    return Layout(dim, degree, D, code_off, factor_off, nbr_off, nbr_off + degree)


# --------------------------------------------------------------------------
# synthetic data
# --------------------------------------------------------------------------
@dataclasses.dataclass(frozen=True)
class DatasetSpec:
    name: str
    n: int
    nq: int
    dim: int
    n_comp: int
    sigma: float
    lo: float
    hi: float
    degree: int
    K: int
    beams: Tuple[int, ...]
    seed: int
    kind: str = "int_gmm"      # int_gmm | int_gmm_dup | norm_aniso | lowrank
    knn_k: int = 64
    gt_k: int = 100
    knn: str = "exact"         # graph candidates: exact | exact_tf32 | partitioned (see build_graph)
    block: int = 0             # > 0: the base is drawn in blocks of this many rows, each from a stream of its own
    random_links: int = -1     # seeded random long edges per node (-1: max(2, degree // 8), see build_graph)


SPECS = {
    # the reference's own CPU-runnable plumbing case
    "c1_100k": DatasetSpec("c1_100k", 100_000, 1_000, 128, 50, 20.0, 0.0, 255.0, 16, 10,
                           (16, 32, 64, 128, 256, 512), seed=1),
    # the headline case
    "c2_1m": DatasetSpec("c2_1m", 1_000_000, 10_000, 128, 200, 25.0, 0.0, 255.0, 32, 100,
                         (100, 128, 256, 384, 512, 640, 768, 896, 1024), seed=2),
    # BASELINE.json configs[2] (10M x 96, L2-normalised anisotropic mixture) at a tenth of the base size
    "c3s_1m": DatasetSpec("c3s_1m", 1_000_000, 10_000, 96, 1000, 0.0, 0.0, 0.0, 32, 100,
                          (100, 128, 256, 384, 512, 640, 768, 896, 1024), seed=5, kind="norm_aniso"),
    # BASELINE.json configs[3] (1M x 1536, L2-normalised low-rank) at a fifth of the base size
    "c4s_200k": DatasetSpec("c4s_200k", 200_000, 1_000, 1536, 1, 0.0, 0.0, 0.0, 32, 100,
                            (100, 128, 256, 384, 512, 640, 768, 896, 1024), seed=4, kind="lowrank"),
    # BASELINE.json configs[2] at full size: 10M x 96, L2-normalised anisotropic mixture
    "c3_10m": DatasetSpec("c3_10m", 10_000_000, 10_000, 96, 1000, 0.0, 0.0, 0.0, 32, 100,
                          (100, 128, 256, 384, 512, 640, 768, 896, 1024), seed=3, kind="norm_aniso",
                          knn="partitioned"),
    # BASELINE.json configs[3] at full size: 1M x 1536, L2-normalised low-rank model
    "c4_1m": DatasetSpec("c4_1m", 1_000_000, 1_000, 1536, 1, 0.0, 0.0, 0.0, 32, 100,
                         (100, 128, 256, 384, 512, 640, 768, 896, 1024), seed=4, kind="lowrank",
                         knn="exact_tf32", random_links=0),
    # 100M x 100 integers in [-128, 127] from a 5,000-component mixture,
    # only ever materialised as shards (one per GPU, each built on its own GPU; see materialize_shard_device)
    "c5_100m": DatasetSpec("c5_100m", 100_000_000, 10_000, 100, 5000, 18.0, -128.0, 127.0, 32, 100,
                           (128, 256, 512, 1024), seed=5, knn="partitioned", block=500_000, random_links=12),
    # the same distribution at a tenth of the size (10M rows, 20 blocks): the sharded mode on 2-8 GPUs
    "c5s_10m": DatasetSpec("c5s_10m", 10_000_000, 10_000, 100, 5000, 18.0, -128.0, 127.0, 32, 100,
                           (128, 256, 512, 1024), seed=5, knn="partitioned", block=500_000, random_links=12),
    # the headline config's per-component structure (5,000 points per component, degree 32)
    # at a fifth of the size, for profiling captures that must stay small
    "p_200k": DatasetSpec("p_200k", 200_000, 2_000, 128, 40, 25.0, 0.0, 255.0, 32, 100,
                          (100, 128, 256, 384, 512, 640, 768, 896, 1024), seed=3),
    # a blocked spec small enough for tests of the device-built shards
    "t_blk40k": DatasetSpec("t_blk40k", 40_000, 100, 100, 40, 18.0, -128.0, 127.0, 32, 100,
                            (128, 256, 512), seed=21, knn="partitioned", block=10_000),
    # small cases for the parity tests (same generators, sizes the oracle finishes in seconds)
    "t_20k": DatasetSpec("t_20k", 20_000, 200, 128, 8, 25.0, 0.0, 255.0, 32, 100,
                         (100, 128, 256, 512, 1024), seed=11),
    "t_8k16": DatasetSpec("t_8k16", 8_000, 200, 128, 4, 20.0, 0.0, 255.0, 16, 10,
                          (16, 32, 64, 96, 128, 256, 512), seed=12),
    "t_4k96f": DatasetSpec("t_4k96f", 4_000, 100, 96, 8, 0.0, 0.0, 0.0, 32, 100,
                           (100, 256), seed=13, kind="norm_aniso"),
    "t_2k": DatasetSpec("t_2k", 2_000, 64, 128, 4, 25.0, 0.0, 255.0, 32, 100,
                        (32, 100, 128, 200, 256), seed=14),
    # every vector four times: equal distances everywhere (tie paths of the merges)
    "t_2kdup": DatasetSpec("t_2kdup", 2_000, 64, 128, 4, 25.0, 0.0, 255.0, 32, 100,
                           (100, 200, 256, 512), seed=17, kind="int_gmm_dup"),
    # padded dimensions above 256 (the one-CTA-per-query kernel): 300 -> 512, 1536 -> 2048
    "t_2k300": DatasetSpec("t_2k300", 2_000, 48, 300, 4, 25.0, 0.0, 255.0, 32, 100,
                           (100, 256), seed=15),
    "t_1k1536": DatasetSpec("t_1k1536", 1_000, 24, 1536, 1, 0.0, 0.0, 0.0, 32, 10,
                            (32, 128), seed=16, kind="lowrank"),
    # ragged dimensions for the one-warp-per-query kernel: 50 -> 64 (two code words per
    # neighbour) and 130 -> 256 (rows and codes not 16-byte aligned: scalar code loads)
    "t_2k50": DatasetSpec("t_2k50", 2_000, 48, 50, 4, 25.0, 0.0, 255.0, 32, 100,
                          (64, 128, 256), seed=18),
    "t_2k130": DatasetSpec("t_2k130", 2_000, 48, 130, 4, 25.0, 0.0, 255.0, 32, 100,
                           (64, 128, 256), seed=19),
}


def _rng(seed: int, stream: int) -> np.random.Generator:
    return np.random.default_rng([seed, stream])


def generate_vectors(spec: DatasetSpec) -> Tuple[np.ndarray, np.ndarray]:
    """Base and query vectors (float32) for a spec; deterministic in the seed."""
    return _draw(spec, 1, spec.n), _draw(spec, 2, spec.nq)


def generate_block(spec: DatasetSpec, b: int) -> np.ndarray:
    """Rows [b*block, (b+1)*block) of a blocked spec's base (stream 100 + b):
    any range of whole blocks can be drawn without the rest of the base."""
    if spec.block <= 0:
        raise ValueError(f"{spec.name} is not drawn in blocks")
    m = min(spec.block, spec.n - b * spec.block)
    return _draw(spec, 100 + b, m)


def generate_queries(spec: DatasetSpec, index: int) -> np.ndarray:
    """Query set `index` of a spec: 0 is the dataset's own batch, index > 0
    draws spec.nq further queries from the same distribution with a stream
    of their own (distinct batches for the ranks of a multi-GPU run)."""
    return _draw(spec, 2 if index == 0 else 1000 + index, spec.nq)


def _draw(spec: DatasetSpec, stream: int, m: int) -> np.ndarray:
    """m vectors of the spec's distribution from RNG stream `stream`
    (stream 0 holds the distribution's parameters, 1 the base, 2 the queries)."""
    if spec.kind == "int_gmm":
        cr = _rng(spec.seed, 0)
        centres = cr.uniform(spec.lo, spec.hi, size=(spec.n_comp, spec.dim))

        def draw(stream: int, m: int) -> np.ndarray:
            r = _rng(spec.seed, stream)
            lab = r.integers(0, spec.n_comp, size=m)
            out = np.empty((m, spec.dim), dtype=np.float32)
            step = 1 << 18
            for s in range(0, m, step):
                e = min(m, s + step)
                noise = r.standard_normal((e - s, spec.dim), dtype=np.float32) * np.float32(spec.sigma)
                v = centres[lab[s:e]].astype(np.float32) + noise
                np.rint(v, out=v)
                np.clip(v, spec.lo, spec.hi, out=v)
                out[s:e] = v
            return out

        return draw(stream, m)
    if spec.kind == "norm_aniso":
        cr = _rng(spec.seed, 0)
        centres = cr.standard_normal((spec.n_comp, spec.dim))
        scales = np.exp(cr.uniform(np.log(0.05), np.log(0.5), size=(spec.n_comp, spec.dim)))

        def draw(stream: int, m: int) -> np.ndarray:
            r = _rng(spec.seed, stream)
            lab = r.integers(0, spec.n_comp, size=m)
            out = np.empty((m, spec.dim), dtype=np.float32)
            step = 1 << 18  # rows per chunk (the stream's values do not depend on the chunking)
            for s0 in range(0, m, step):
                e = min(m, s0 + step)
                v = centres[lab[s0:e]] + r.standard_normal((e - s0, spec.dim)) * scales[lab[s0:e]]
                v /= np.linalg.norm(v, axis=1, keepdims=True)
                out[s0:e] = v
            return out

        return draw(stream, m)
    if spec.kind == "int_gmm_dup":
        # every base vector repeated 4 times (consecutive ids): long runs of
        # equal distances, for the merges' tie paths
        uniq = dataclasses.replace(spec, n=(spec.n + 3) // 4, kind="int_gmm")
        if stream != 1:
            return _draw(uniq, stream, m)
        return np.repeat(_draw(uniq, 1, uniq.n), 4, axis=0)[:m].copy()
    if spec.kind == "lowrank":
        # rank-64 latent x a fixed 64 x dim map + N(0, 0.02^2), L2-normalised
        cr = _rng(spec.seed, 0)
        rank = 64
        basis = cr.standard_normal((rank, spec.dim)).astype(np.float32) / np.float32(np.sqrt(rank))

        def draw(stream: int, m: int) -> np.ndarray:
            r = _rng(spec.seed, stream)
            out = np.empty((m, spec.dim), dtype=np.float32)
            step = 1 << 16
            for s0 in range(0, m, step):
                e = min(m, s0 + step)
                z = r.standard_normal((e - s0, rank), dtype=np.float32)
                v = z @ basis + r.standard_normal((e - s0, spec.dim), dtype=np.float32) * np.float32(0.02)
                v /= np.linalg.norm(v, axis=1, keepdims=True)
                out[s0:e] = v
            return out

        return draw(stream, m)
    raise ValueError(f"unknown dataset kind {spec.kind}")


def make_signs(D: int, seed: int) -> np.ndarray:
    r = _rng(seed, 7)
    return np.where(r.integers(0, 2, size=D) == 1, 1.0, -1.0).astype(np.float32)


# --------------------------------------------------------------------------
# exact nearest neighbours (offline, torch)
# --------------------------------------------------------------------------
def _device(device: Optional[str]) -> torch.device:
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    return torch.device(device)


def _is_integer_data(x: np.ndarray) -> bool:
    if x.size == 0:
        return True
    sample = x[: min(len(x), 4096)]
    return bool(np.all(sample == np.rint(sample))) and float(np.abs(x).max()) <= 255.0


def brute_force_knn(base: np.ndarray, queries: Optional[np.ndarray], k: int, device=None,
                    exclude_self: bool = False, chunk: int = 0, tf32: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """Exact k nearest neighbours by squared L2, ties broken by smaller id.

    Integer-valued data (|x| <= 255, the BASELINE integer configs) is searched
    with exact integer distances; float data with fp32 distances (tf32: the
    selection's products in TF32 on tensor cores -- graph construction only,
    the selected rows are still ranked by float64 distances).
    Returns (ids int64 [m, k], d2 float64 [m, k]) sorted ascending.
    """
    dev = _device(device)
    exact = _is_integer_data(base) and (queries is None or _is_integer_data(queries))
    xb = torch.from_numpy(np.ascontiguousarray(base)).to(dev)
    xq = xb if queries is None else torch.from_numpy(np.ascontiguousarray(queries)).to(dev)
    n, m = xb.shape[0], xq.shape[0]
    nb = xb.pow(2).sum(1)
    nqv = xq.pow(2).sum(1)
    shift = max(1, int(math.ceil(math.log2(max(n, 2)))))
    if chunk <= 0:
        budget = (6 << 30) if dev.type == "cuda" else (1 << 29)
        chunk = max(16, min(m, budget // max(1, n * 12)))
    idx_all = torch.arange(n, device=dev, dtype=torch.int64)
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = bool(tf32 and not exact)
    try:
        return _brute_chunks(xb, xq, nb, nqv, idx_all, k, m, n, chunk, exact, exclude_self, shift, dev)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32


def _brute_chunks(xb, xq, nb, nqv, idx_all, k, m, n, chunk, exact, exclude_self, shift, dev):
    ids_out = np.empty((m, k), dtype=np.int64)
    d_out = np.empty((m, k), dtype=np.float64)
    for s in range(0, m, chunk):
        e = min(m, s + chunk)
        d = nqv[s:e, None] + nb[None, :] - 2.0 * (xq[s:e] @ xb.T)
        d.clamp_(min=0)
        if exclude_self:
            r = torch.arange(s, e, device=dev)
            d[r - s, r] = float("inf")
        if exact:
            key = torch.round(d).to(torch.int64)
            if exclude_self:
                key[r - s, r] = (1 << 62) >> shift
            key = (key << shift) | idx_all[None, :]
            kv, ki = torch.topk(key, k, dim=1, largest=False, sorted=True)
            ids = kv & ((1 << shift) - 1)
        else:
            dv, ids = torch.topk(d, k, dim=1, largest=False, sorted=True)
        del d
        # recompute in float64 from the vectors and order by (distance, id)
        qv = xq[s:e].double()
        dd = (xb[ids].double() - qv[:, None, :]).pow(2).sum(-1)
        order = torch.argsort(ids, dim=1, stable=True)
        ids = torch.gather(ids, 1, order)
        dd = torch.gather(dd, 1, order)
        order = torch.argsort(dd, dim=1, stable=True)
        ids_out[s:e] = torch.gather(ids, 1, order).cpu().numpy()
        d_out[s:e] = torch.gather(dd, 1, order).cpu().numpy()
    return ids_out, d_out


def _nearest_centroid(x: torch.Tensor, cent: torch.Tensor, chunk: int = 1 << 18) -> torch.Tensor:
    """Index of the nearest centroid (squared L2) of every row of x."""
    cn = (cent * cent).sum(1)
    out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    for s in range(0, x.shape[0], chunk):
        xs = x[s:s + chunk]
        out[s:s + chunk] = torch.argmin(cn[None, :] - 2.0 * (xs @ cent.T), dim=1)
    return out


def partitioned_knn(x: np.ndarray, k: int, seed: int, device=None, cluster_size: int = 2048, probe: int = 8,
                    kmeans_iters: int = 10, verbose: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """Approximate k nearest neighbours of every row of x (itself excluded),
    for bases too large for the exact search: k-means (on a seeded sample,
    centroid sums formed on the host so the result is deterministic) splits
    the rows into clusters of about `cluster_size`; the neighbours of a row
    are the exact k nearest among the members of the `probe` clusters whose
    centroids lie nearest its own cluster's centroid (its own included).
    Returns (ids int64 [n, k], d2 float64 [n, k]) ascending, -1 / inf where a
    row's clusters hold fewer than k other rows."""
    import time
    t0 = time.time()
    dev = _device(device)
    n, dim = x.shape
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev)
    norms = (xt * xt).sum(1)
    C = max(1, n // cluster_size)
    rg = _rng(seed, 11)
    m = min(n, 64 * C)
    sample_idx = np.sort(rg.choice(n, size=m, replace=False))
    sample_h = np.ascontiguousarray(x[sample_idx], dtype=np.float32)
    sample = torch.from_numpy(sample_h).to(dev)
    cent_h = sample_h[rg.choice(m, size=C, replace=False)].astype(np.float64)
    for _ in range(kmeans_iters):
        lab = _nearest_centroid(sample, torch.from_numpy(cent_h.astype(np.float32)).to(dev)).cpu().numpy()
        order = np.argsort(lab, kind="stable")
        lab_s = lab[order]
        cuts = np.flatnonzero(np.diff(lab_s)) + 1
        first = np.concatenate([[0], cuts])
        sums = np.add.reduceat(sample_h[order].astype(np.float64), first, axis=0)
        cnt = np.diff(np.concatenate([first, [m]]))
        cent_h[lab_s[first]] = sums / cnt[:, None]
    cent = torch.from_numpy(cent_h.astype(np.float32)).to(dev)
    labels = _nearest_centroid(xt, cent)
    members = torch.argsort(labels, stable=True)
    counts = torch.bincount(labels, minlength=C)
    starts = torch.cumsum(counts, 0) - counts
    cc = (cent * cent).sum(1)
    cd = cc[:, None] + cc[None, :] - 2.0 * (cent @ cent.T)
    cd.fill_diagonal_(-1.0)  # a cluster always probes itself first
    nbr = torch.topk(cd, min(probe, C), dim=1, largest=False).indices.cpu().numpy()
    counts_h, starts_h = counts.cpu().numpy(), starts.cpu().numpy()
    if verbose:
        print(f"[builder] partitioned k-NN: {C} clusters (sizes {counts_h.min()}..{counts_h.max()}), "
              f"{time.time() - t0:.1f}s", flush=True)
    out_i = torch.full((n, k), -1, dtype=torch.int64, device=dev)
    out_d = torch.full((n, k), float("inf"), dtype=torch.float32, device=dev)
    for c in range(C):
        if counts_h[c] == 0:
            continue
        q = members[starts_h[c]:starts_h[c] + counts_h[c]]
        pool = torch.cat([members[starts_h[j]:starts_h[j] + counts_h[j]] for j in nbr[c]])
        d = norms[q][:, None] + norms[pool][None, :] - 2.0 * (xt[q] @ xt[pool].T)
        d.masked_fill_(q[:, None] == pool[None, :], float("inf"))
        kk = min(k, pool.numel() - 1)
        if kk <= 0:
            continue
        dv, di = torch.topk(d, kk, dim=1, largest=False, sorted=True)
        nb = pool[di]
        # distances recomputed as sums of squared differences: symmetric bit
        # for bit, so a pair's forward and reverse edges carry one value
        dx = ((xt[q][:, None, :] - xt[nb]) ** 2).sum(-1)
        dx, o = torch.sort(dx, dim=1, stable=True)
        nb = torch.gather(nb, 1, o)
        out_i[q, :kk] = torch.where(torch.isinf(torch.gather(dv, 1, o)), torch.full_like(nb, -1), nb)
        out_d[q, :kk] = dx
    if verbose:
        print(f"[builder] partitioned k-NN done, {time.time() - t0:.1f}s", flush=True)
    return out_i.cpu().numpy(), out_d.double().cpu().numpy()


# --------------------------------------------------------------------------
# graph construction
# --------------------------------------------------------------------------
def _merge_reverse(ids: np.ndarray, d: np.ndarray, cap: int, device) -> Tuple[np.ndarray, np.ndarray]:
    """Union of forward and reverse k-NN lists, nearest `cap` per node."""
    dev = _device(device)
    n, k = ids.shape
    src = torch.arange(n, device=dev).repeat_interleave(k)
    dst = torch.from_numpy(ids.reshape(-1)).to(dev)
    dd = torch.from_numpy(d.reshape(-1)).to(dev)
    node = torch.cat([src, dst])
    cand = torch.cat([dst, src])
    dist = torch.cat([dd, dd])
    o = torch.argsort(cand, stable=True)
    node, cand, dist = node[o], cand[o], dist[o]
    o = torch.argsort(dist, stable=True)
    node, cand, dist = node[o], cand[o], dist[o]
    o = torch.argsort(node, stable=True)
    node, cand, dist = node[o], cand[o], dist[o]
    keep = torch.ones_like(node, dtype=torch.bool)
    keep[1:] = (node[1:] != node[:-1]) | (cand[1:] != cand[:-1])
    # (node, cand) duplicates share a distance, so they are adjacent after the sort
    node, cand, dist = node[keep], cand[keep], dist[keep]
    counts = torch.bincount(node, minlength=n)
    starts = torch.cumsum(counts, 0) - counts
    rank = torch.arange(node.numel(), device=dev) - starts[node]
    sel = rank < cap
    out_i = torch.full((n, cap), -1, dtype=torch.int64, device=dev)
    out_d = torch.full((n, cap), float("inf"), dtype=torch.float64, device=dev)
    out_i[node[sel], rank[sel]] = cand[sel]
    out_d[node[sel], rank[sel]] = dist[sel]
    return out_i.cpu().numpy(), out_d.cpu().numpy()


def _merge_reverse_large(ids: np.ndarray, d: np.ndarray, cap: int, device) -> Tuple[np.ndarray, np.ndarray]:
    """_merge_reverse for bases of millions of rows: the same lists (nearest
    `cap` of the forward and reverse k-NN edges per node, ordered by
    (distance, id)), with 32-bit node ids and float32 distances on the
    device and two stable sorts instead of three, which keeps ten million
    nodes' 1.3 billion edges within a few tens of GB.  Needs symmetric
    distances (d(u, v) == d(v, u) bit for bit)."""
    dev = _device(device)
    n, k = ids.shape
    src = torch.arange(n, device=dev, dtype=torch.int32).repeat_interleave(k)
    dst = torch.from_numpy(ids.reshape(-1)).to(dev)
    dd = torch.from_numpy(d.reshape(-1).astype(np.float32)).to(dev)
    ok = dst >= 0
    src, dst, dd = src[ok], dst[ok].to(torch.int32), dd[ok]
    node = torch.cat([src, dst])
    cand = torch.cat([dst, src])
    dist = torch.cat([dd, dd])
    del src, dst, dd, ok
    o = torch.argsort(cand, stable=True)
    node, cand, dist = node[o], cand[o], dist[o]
    del o
    # (node, distance) as one 64-bit key: distances are >= 0, so their float
    # bits order like the values
    key = (node.to(torch.int64) << 32) | (dist.view(torch.int32).to(torch.int64) & 0xFFFFFFFF)
    o = torch.argsort(key, stable=True)
    del key
    node, cand, dist = node[o], cand[o], dist[o]
    del o
    keep = torch.ones_like(node, dtype=torch.bool)
    keep[1:] = (node[1:] != node[:-1]) | (cand[1:] != cand[:-1])
    node, cand, dist = node[keep], cand[keep], dist[keep]
    del keep
    counts = torch.bincount(node, minlength=n)
    starts = torch.cumsum(counts, 0) - counts
    rank = torch.arange(node.numel(), device=dev) - starts[node.long()]
    sel = rank < cap
    out_i = torch.full((n, cap), -1, dtype=torch.int64, device=dev)
    out_d = torch.full((n, cap), float("inf"), dtype=torch.float64, device=dev)
    nl = node[sel].long()
    out_i[nl, rank[sel]] = cand[sel].long()
    out_d[nl, rank[sel]] = dist[sel].double()
    return out_i.cpu().numpy(), out_d.cpu().numpy()


def rng_prune(x: np.ndarray, cand: np.ndarray, cand_d: np.ndarray, R: int, alpha: float = 1.0,
              device=None, batch: int = 0) -> np.ndarray:
    """Relative-neighbourhood pruning of sorted candidate lists.

    Candidate c of node p is dropped when a kept neighbour k has
    alpha^2 * d(k, c) <= d(p, c) (squared distances); the list is then filled
    to R with the nearest dropped candidates.  Returns int64 [n, R], -1 = empty.
    """
    dev = _device(device)
    n, C = cand.shape
    if batch <= 0:
        batch = 8192 if dev.type == "cuda" else 1024
        if dev.type == "cuda" and n > 2_000_000:
            # large bases: ~4 GB of gathered rows and pair distances per batch
            batch = int(min(32768, max(1024, (4 << 30) // (C * (x.shape[1] + C) * 8))))
    xt = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    out = np.full((n, R), -1, dtype=np.int64)
    a2 = alpha * alpha
    for s in range(0, n, batch):
        e = min(n, s + batch)
        ci = torch.from_numpy(cand[s:e]).to(dev)
        cd = torch.from_numpy(cand_d[s:e]).to(dev)
        valid = ci >= 0
        v = xt[ci.clamp(min=0)].double()
        g = v @ v.transpose(1, 2)
        sq = torch.diagonal(g, dim1=1, dim2=2)
        pair = (sq[:, :, None] + sq[:, None, :] - 2.0 * g).clamp_(min=0)
        B = e - s
        kept = torch.zeros((B, C), dtype=torch.bool, device=dev)
        count = torch.zeros(B, dtype=torch.int64, device=dev)
        for j in range(C):
            occl = (kept & (pair[:, :, j] * a2 <= cd[:, j:j + 1])).any(1)
            take = valid[:, j] & ~occl & (count < R)
            kept[:, j] = take
            count += take.to(torch.int64)
        # order: kept (by distance) then dropped (by distance)
        pos = torch.arange(C, device=dev)[None, :].expand(B, C)
        key = torch.where(kept, pos, pos + C)
        key = torch.where(valid, key, torch.full_like(key, 3 * C))
        order = torch.argsort(key, dim=1)[:, :R]
        chosen = torch.gather(ci, 1, order)
        chosen_valid = torch.gather(valid, 1, order)
        chosen = torch.where(chosen_valid, chosen, torch.full_like(chosen, -1))
        out[s:e, : chosen.shape[1]] = chosen.cpu().numpy()
    return out


def build_graph(x: np.ndarray, degree: int, seed: int, knn_k: int = 64, device=None,
                random_links: Optional[int] = None, knn: str = "exact",
                verbose: bool = False) -> Tuple[np.ndarray, int]:
    """Degree-`degree` neighbour lists (int64, -1 = empty) and an entry point.

    Every node keeps `degree - r` relative-neighbourhood-pruned local edges and
    `r` seeded uniformly random long edges (r = max(2, degree // 8)); the
    entry point (the node nearest the centroid) spends half of its slots on
    random long edges.  Without long edges a single entry point never leaves
    its own component of a well-separated mixture.  knn = "exact" takes the
    candidates from the brute-force k-NN, "partitioned" from
    partitioned_knn (bases of millions of rows), "exact_tf32" from the
    brute force with TF32 products (high-dimensional bases).
    """
    n = x.shape[0]
    k = min(knn_k, n - 1)
    r = max(2, degree // 8) if random_links is None else random_links
    r = min(r, degree - 1)
    if knn in ("exact", "exact_tf32"):
        ids, d = brute_force_knn(x, None, k, device=device, exclude_self=True, tf32=knn == "exact_tf32")
    elif knn == "partitioned":
        ids, d = partitioned_knn(x, k, seed, device=device, verbose=verbose)
    else:
        raise ValueError(f"unknown k-NN method {knn!r}")
    if verbose:
        print(f"[builder] k-NN ({knn}) done", flush=True)
    merge = _merge_reverse if knn == "exact" or n <= 2_000_000 else _merge_reverse_large
    cand, cand_d = merge(ids, d, cap=min(n - 1, max(96, int(1.5 * k))), device=device)
    if verbose:
        print("[builder] reverse edges merged", flush=True)
    local = rng_prune(x, cand, cand_d, degree - r, device=device)
    if verbose:
        print("[builder] pruned", flush=True)
    rg = _rng(seed, 5)
    if r:
        rand = (np.arange(n)[:, None] + 1 + rg.integers(0, max(1, n - 1), size=(n, r))) % n
        nbrs = np.concatenate([local, rand], axis=1)
    else:
        nbrs = local.copy()
    # a random target that repeats an earlier slot becomes an empty slot
    srt = np.sort(nbrs, axis=1)
    if np.any(srt[:, 1:] == srt[:, :-1]):
        for i in np.nonzero(np.any((srt[:, 1:] == srt[:, :-1]) & (srt[:, 1:] >= 0), axis=1))[0]:
            seen = set()
            for j in range(degree):
                v = int(nbrs[i, j])
                if v >= 0 and v in seen:
                    nbrs[i, j] = -1
                seen.add(v)
    centroid = x.astype(np.float64).mean(0)
    d2 = np.empty(n)
    step = 1 << 16
    for s in range(0, n, step):
        d2[s:s + step] = ((x[s:s + step].astype(np.float64) - centroid) ** 2).sum(1)
    entry = int(np.argmin(d2))
    half = degree // 2
    extra = (entry + 1 + rg.integers(0, max(1, n - 1), size=half)) % n
    row = [int(v) for v in local[entry] if v >= 0][: degree - half]
    for v in extra:
        if int(v) not in row and int(v) != entry:
            row.append(int(v))
    nbrs[entry] = -1
    nbrs[entry, : len(row)] = row[:degree]
    return nbrs, entry


# --------------------------------------------------------------------------
# device-resident construction (bases of millions of rows)
# --------------------------------------------------------------------------
# The same graph recipe as build_graph with knn="partitioned" and the same
# codes as encode_rows, with every intermediate kept on one GPU (32-bit ids,
# float32 distances), so that a shard of 12.5M rows needs no host copy of its
# k-NN lists, candidate lists or codebook.
def _kmeans_centroids(xt: torch.Tensor, C: int, seed: int, iters: int = 10) -> torch.Tensor:
    """k-means centroids of a seeded sample of the rows (sums on the host:
    deterministic)."""
    n = xt.shape[0]
    rg = _rng(seed, 11)
    m = min(n, 64 * C)
    idx = torch.from_numpy(np.sort(rg.choice(n, size=m, replace=False))).to(xt.device)
    sample_h = xt[idx].cpu().numpy().astype(np.float32)
    sample = torch.from_numpy(sample_h).to(xt.device)
    cent_h = sample_h[rg.choice(m, size=C, replace=False)].astype(np.float64)
    for _ in range(iters):
        lab = _nearest_centroid(sample, torch.from_numpy(cent_h.astype(np.float32)).to(xt.device)).cpu().numpy()
        order = np.argsort(lab, kind="stable")
        lab_s = lab[order]
        first = np.concatenate([[0], np.flatnonzero(np.diff(lab_s)) + 1])
        sums = np.add.reduceat(sample_h[order].astype(np.float64), first, axis=0)
        cnt = np.diff(np.concatenate([first, [m]]))
        cent_h[lab_s[first]] = sums / cnt[:, None]
    return torch.from_numpy(cent_h.astype(np.float32)).to(xt.device)


def knn_partitioned_device(xt: torch.Tensor, k: int, seed: int, cluster_size: int = 2048, probe: int = 8,
                           verbose: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """partitioned_knn on a device tensor: (ids int32 [n, k], d2 float32
    [n, k]) on the same device, ascending, -1 / inf where short."""
    import time
    t0 = time.time()
    dev = xt.device
    n = xt.shape[0]
    norms = (xt * xt).sum(1)
    C = max(1, n // cluster_size)
    cent = _kmeans_centroids(xt, C, seed)
    labels = _nearest_centroid(xt, cent)
    members = torch.argsort(labels, stable=True)
    counts = torch.bincount(labels, minlength=C)
    starts = torch.cumsum(counts, 0) - counts
    del labels
    cc = (cent * cent).sum(1)
    cd = cc[:, None] + cc[None, :] - 2.0 * (cent @ cent.T)
    cd.fill_diagonal_(-1.0)
    nbr = torch.topk(cd, min(probe, C), dim=1, largest=False).indices.cpu().numpy()
    counts_h, starts_h = counts.cpu().numpy(), starts.cpu().numpy()
    if verbose:
        print(f"[builder] partitioned k-NN: {C} clusters (sizes {counts_h.min()}..{counts_h.max()}), "
              f"{time.time() - t0:.1f}s", flush=True)
    out_i = torch.full((n, k), -1, dtype=torch.int32, device=dev)
    out_d = torch.full((n, k), float("inf"), dtype=torch.float32, device=dev)
    for c in range(C):
        if counts_h[c] == 0:
            continue
        q = members[starts_h[c]:starts_h[c] + counts_h[c]]
        pool = torch.cat([members[starts_h[j]:starts_h[j] + counts_h[j]] for j in nbr[c]])
        d = norms[q][:, None] + norms[pool][None, :] - 2.0 * (xt[q] @ xt[pool].T)
        d.masked_fill_(q[:, None] == pool[None, :], float("inf"))
        kk = min(k, pool.numel() - 1)
        if kk <= 0:
            continue
        dv, di = torch.topk(d, kk, dim=1, largest=False, sorted=True)
        nb = pool[di]
        dx = ((xt[q][:, None, :] - xt[nb]) ** 2).sum(-1)
        dx, o = torch.sort(dx, dim=1, stable=True)
        nb = torch.gather(nb, 1, o)
        out_i[q, :kk] = torch.where(torch.isinf(torch.gather(dv, 1, o)), torch.full_like(nb, -1), nb).to(torch.int32)
        out_d[q, :kk] = dx
    if verbose:
        print(f"[builder] partitioned k-NN done, {time.time() - t0:.1f}s", flush=True)
    return out_i, out_d


def merge_reverse_device(ids: torch.Tensor, d: torch.Tensor, cap: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """_merge_reverse_large on device tensors: (cand int32 [n, cap], cand_d
    float32 [n, cap]), -1 / inf where short."""
    dev = ids.device
    n, k = ids.shape
    src = torch.arange(n, device=dev, dtype=torch.int32).repeat_interleave(k)
    dst = ids.reshape(-1)
    dd = d.reshape(-1)
    ok = dst >= 0
    src, dst, dd = src[ok], dst[ok], dd[ok]
    node = torch.cat([src, dst])
    cand = torch.cat([dst, src])
    dist = torch.cat([dd, dd])
    del src, dst, dd, ok
    o = torch.argsort(cand, stable=True)
    node, cand, dist = node[o], cand[o], dist[o]
    del o
    key = (node.to(torch.int64) << 32) | (dist.view(torch.int32).to(torch.int64) & 0xFFFFFFFF)
    o = torch.argsort(key, stable=True)
    del key
    node, cand, dist = node[o], cand[o], dist[o]
    del o
    keep = torch.ones_like(node, dtype=torch.bool)
    keep[1:] = (node[1:] != node[:-1]) | (cand[1:] != cand[:-1])
    node, cand, dist = node[keep], cand[keep], dist[keep]
    del keep
    nl = node.long()
    del node
    counts = torch.bincount(nl, minlength=n)
    starts = torch.cumsum(counts, 0) - counts
    rank = torch.arange(nl.numel(), device=dev) - starts[nl]
    sel = rank < cap
    out_i = torch.full((n, cap), -1, dtype=torch.int32, device=dev)
    out_d = torch.full((n, cap), float("inf"), dtype=torch.float32, device=dev)
    out_i[nl[sel], rank[sel]] = cand[sel]
    out_d[nl[sel], rank[sel]] = dist[sel]
    return out_i, out_d


def rng_prune_device(xt: torch.Tensor, cand: torch.Tensor, cand_d: torch.Tensor, R: int,
                     alpha: float = 1.0) -> torch.Tensor:
    """rng_prune on device tensors (float32 pair distances): int32 [n, R]."""
    dev = xt.device
    n, C = cand.shape
    batch = int(min(65536, max(1024, (4 << 30) // (C * (xt.shape[1] + C) * 4))))
    out = torch.full((n, R), -1, dtype=torch.int32, device=dev)
    a2 = alpha * alpha
    pos = torch.arange(C, device=dev)[None, :]
    for s in range(0, n, batch):
        e = min(n, s + batch)
        ci = cand[s:e].long()
        cd = cand_d[s:e]
        valid = ci >= 0
        v = xt[ci.clamp(min=0)]
        g = v @ v.transpose(1, 2)
        sq = torch.diagonal(g, dim1=1, dim2=2)
        pair = (sq[:, :, None] + sq[:, None, :] - 2.0 * g).clamp_(min=0)
        del v, g
        B = e - s
        kept = torch.zeros((B, C), dtype=torch.bool, device=dev)
        count = torch.zeros(B, dtype=torch.int32, device=dev)
        for j in range(C):
            occl = (kept & (pair[:, :, j] * a2 <= cd[:, j:j + 1])).any(1)
            take = valid[:, j] & ~occl & (count < R)
            kept[:, j] = take
            count += take.to(torch.int32)
        key = torch.where(kept, pos, pos + C)
        key = torch.where(valid, key, torch.full_like(key, 3 * C))
        order = torch.argsort(key, dim=1)[:, :R]
        chosen = torch.gather(ci, 1, order)
        chosen_valid = torch.gather(valid, 1, order)
        out[s:e, :chosen.shape[1]] = torch.where(chosen_valid, chosen, torch.full_like(chosen, -1)).to(torch.int32)
    return out


def build_graph_device(xt: torch.Tensor, degree: int, seed: int, knn_k: int = 64,
                       verbose: bool = False, random_links: Optional[int] = None) -> Tuple[torch.Tensor, int]:
    """build_graph (partitioned k-NN) on a device tensor of the rows:
    (neighbour lists int32 [n, degree] on the device, -1 = empty; entry)."""
    import time
    t0 = time.time()
    dev = xt.device
    n = xt.shape[0]
    k = min(knn_k, n - 1)
    r = max(2, degree // 8) if random_links is None or random_links < 0 else random_links
    r = min(r, degree - 1)
    ids, d = knn_partitioned_device(xt, k, seed, verbose=verbose)
    cand, cand_d = merge_reverse_device(ids, d, cap=min(n - 1, max(96, int(1.5 * k))))
    del ids, d
    if verbose:
        print(f"[builder] reverse edges merged, {time.time() - t0:.1f}s", flush=True)
    local = rng_prune_device(xt, cand, cand_d, degree - r)
    del cand, cand_d
    if verbose:
        print(f"[builder] pruned, {time.time() - t0:.1f}s", flush=True)
    rg = _rng(seed, 5)
    if r:
        rand = torch.from_numpy(((np.arange(n)[:, None] + 1 + rg.integers(0, max(1, n - 1), size=(n, r))) % n)
                                .astype(np.int32)).to(dev)
        nbrs = torch.cat([local, rand], dim=1)
        del local, rand
    else:
        nbrs = local
    # a neighbour that repeats an earlier slot of its row becomes an empty slot
    tri = torch.ones((degree, degree), dtype=torch.bool, device=dev).tril(-1)  # [j, j']: j' < j
    step = 1 << 20
    for s0 in range(0, n, step):
        blk = nbrs[s0:s0 + step]
        dup = ((blk[:, :, None] == blk[:, None, :]) & tri[None] & (blk[:, None, :] >= 0)).any(2)
        blk.masked_fill_(dup, -1)
    # entry: the row nearest the centroid, half of its slots random long edges
    cen = xt.double().mean(0)
    best, best_d = 0, float("inf")
    for s0 in range(0, n, step):
        dd = ((xt[s0:s0 + step].double() - cen) ** 2).sum(1)
        v, i = torch.min(dd, 0)
        if float(v) < best_d:
            best_d, best = float(v), s0 + int(i)
    entry = best
    half = degree // 2
    extra = (entry + 1 + rg.integers(0, max(1, n - 1), size=half)) % n
    row = [int(v) for v in nbrs[entry, :degree - r].cpu().tolist() if v >= 0][: degree - half]
    for v in extra:
        if int(v) not in row and int(v) != entry:
            row.append(int(v))
    row = row[:degree] + [-1] * (degree - min(degree, len(row)))
    nbrs[entry] = torch.tensor(row, dtype=torch.int32, device=dev)
    if verbose:
        print(f"[builder] graph done, {time.time() - t0:.1f}s", flush=True)
    return nbrs, entry


def encode_rows_device(xt: torch.Tensor, nbrs: torch.Tensor, signs: np.ndarray, metric: str = "l2") -> torch.Tensor:
    """encode_rows on device tensors: the codebook rows float32 [n, row] on
    the device (the same bytes encode_rows writes)."""
    dev = xt.device
    n, dim = xt.shape
    R = nbrs.shape[1]
    L = layout(dim, R)
    D = L.padded_dim
    rows = torch.zeros((n, L.row), dtype=torch.float32, device=dev)
    rows[:, :dim] = xt
    rows_u8 = rows.view(torch.uint8)
    rows_i32 = rows.view(torch.int32)
    st = torch.zeros(D, dtype=torch.float64, device=dev)
    st[:dim] = torch.from_numpy(signs[:dim]).to(dev).double()
    scale = 2.0 if metric == "l2" else 1.0
    batch = max(1, (1 << 27) // (R * D))
    bitw = torch.tensor([8, 4, 2, 1], dtype=torch.int64, device=dev)
    FMAX = float(FLT_MAX)
    for s in range(0, n, batch):
        e = min(n, s + batch)
        nb = nbrs[s:e].long()
        valid = nb >= 0
        c = xt[s:e].double()
        o = xt[nb.clamp(min=0)].double()
        diff = o - c[:, None, :]
        u = torch.zeros((e - s, R, D), dtype=torch.float64, device=dev)
        u[..., :dim] = diff * st[:dim]
        u = fwht(u)
        bits = (u > 0)
        ip_xu = u.abs().sum(-1)
        norm_u = u.pow(2).sum(-1)
        fdq = torch.where(ip_xu > 0, -scale * norm_u / (D * ip_xu), torch.zeros_like(ip_xu))
        fvq = fdq * (2.0 * bits.sum(-1).double() - D)
        if metric == "l2":
            tx = diff.pow(2).sum(-1) + 2.0 * (diff * c[:, None, :]).sum(-1)
        else:
            tx = torch.zeros_like(fdq)
        nib = (bits.view(e - s, R, D // 4, 4).to(torch.int64) * bitw).sum(-1)
        byte = (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)
        tx = torch.where(valid, tx, torch.full_like(tx, FMAX))
        fdq = torch.where(valid, fdq, torch.zeros_like(fdq))
        fvq = torch.where(valid, fvq, torch.zeros_like(fvq))
        byte = torch.where(valid[..., None], byte, torch.zeros_like(byte))
        rows_u8[s:e, L.code_off * 4: L.code_off * 4 + R * (D // 8)] = byte.reshape(e - s, R * (D // 8))
        rows[s:e, L.factor_off: L.factor_off + R] = tx.float()
        rows[s:e, L.factor_off + R: L.factor_off + 2 * R] = fdq.float()
        rows[s:e, L.factor_off + 2 * R: L.factor_off + 3 * R] = fvq.float()
        rows_i32[s:e, L.nbr_off: L.nbr_off + R] = torch.where(valid, nb, torch.full_like(nb, -1)).to(torch.int32)
    return rows


def write_codebook_device(path: str, entry: int, rows: torch.Tensor, signs: np.ndarray,
                          chunk_rows: int = 1 << 20) -> None:
    """write_codebook from device rows, one chunk of rows at a time."""
    with open(path, "wb") as f:
        f.write(struct.pack("<I", entry & 0xFFFFFFFF))
        for s in range(0, rows.shape[0], chunk_rows):
            f.write(rows[s:s + chunk_rows].cpu().numpy().tobytes())
        f.write(np.ascontiguousarray(signs, dtype=np.float32).tobytes())


# --------------------------------------------------------------------------
# RaBitQ encoding
# --------------------------------------------------------------------------
def fwht(v: torch.Tensor) -> torch.Tensor:
    """Unnormalised Walsh-Hadamard transform over the last dim (power of two)."""
    D = v.shape[-1]
    shape = v.shape
    h = 1
    v = v.clone()
    while h < D:
        v = v.view(*shape[:-1], D // (2 * h), 2, h)
        a = v[..., 0, :].clone()
        b = v[..., 1, :]
        v[..., 0, :] = a + b
        v[..., 1, :] = a - b
        v = v.view(shape)
        h <<= 1
    return v


def encode_rows(x: np.ndarray, nbrs: np.ndarray, signs: np.ndarray, metric: str = "l2",
                device=None, batch: int = 0) -> np.ndarray:
    """Codebook rows (float32 [n, row]) in the qg_codebook layout."""
    dev = _device(device)
    n, dim = x.shape
    R = nbrs.shape[1]
    L = layout(dim, R)
    D = L.padded_dim
    rows = np.zeros((n, L.row), dtype=np.float32)
    rows[:, :dim] = x
    rows_u8 = rows.view(np.uint8)
    rows_u32 = rows.view(np.uint32)
    xt = torch.from_numpy(np.ascontiguousarray(x)).to(dev).double()
    st = torch.zeros(D, dtype=torch.float64, device=dev)
    st[:dim] = torch.from_numpy(signs[:dim]).to(dev).double()
    scale = 2.0 if metric == "l2" else 1.0
    if batch <= 0:
        batch = max(1, (1 << 27) // (R * D)) if dev.type == "cuda" else max(1, (1 << 22) // (R * D))
    bitw = torch.tensor([8, 4, 2, 1], dtype=torch.int64, device=dev)
    for s in range(0, n, batch):
        e = min(n, s + batch)
        nb = torch.from_numpy(nbrs[s:e]).to(dev)
        valid = nb >= 0
        c = xt[s:e]                                   # [B, dim]
        o = xt[nb.clamp(min=0)]                       # [B, R, dim]
        diff = o - c[:, None, :]
        u = torch.zeros((e - s, R, D), dtype=torch.float64, device=dev)
        u[..., :dim] = diff * st[:dim]
        u = fwht(u)
        bits = (u > 0)
        ip_xu = u.abs().sum(-1)
        norm_u = u.pow(2).sum(-1)
        fdq = torch.where(ip_xu > 0, -scale * norm_u / (D * ip_xu), torch.zeros_like(ip_xu))
        fvq = fdq * (2.0 * bits.sum(-1).double() - D)
        if metric == "l2":
            tx = diff.pow(2).sum(-1) + 2.0 * (diff * c[:, None, :]).sum(-1)
        else:
            tx = torch.zeros_like(fdq)
        # nibble for chunk cb: dims 4cb..4cb+3 -> bits 8,4,2,1 (include/utils.cuh:911-917)
        nib = (bits.view(e - s, R, D // 4, 4).to(torch.int64) * bitw).sum(-1)
        byte = (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)  # [B, R, D/8]
        tx = torch.where(valid, tx, torch.full_like(tx, float(FLT_MAX)))
        fdq = torch.where(valid, fdq, torch.zeros_like(fdq))
        fvq = torch.where(valid, fvq, torch.zeros_like(fvq))
        byte = torch.where(valid[..., None], byte, torch.zeros_like(byte))
        cb = byte.reshape(e - s, R * (D // 8)).cpu().numpy()
        rows_u8[s:e, L.code_off * 4: L.code_off * 4 + R * (D // 8)] = cb
        rows[s:e, L.factor_off: L.factor_off + R] = tx.float().cpu().numpy()
        rows[s:e, L.factor_off + R: L.factor_off + 2 * R] = fdq.float().cpu().numpy()
        rows[s:e, L.factor_off + 2 * R: L.factor_off + 3 * R] = fvq.float().cpu().numpy()
        ids32 = np.where(nbrs[s:e] >= 0, nbrs[s:e], 0xFFFFFFFF).astype(np.uint32)
        rows_u32[s:e, L.nbr_off: L.nbr_off + R] = ids32
    return rows


def write_codebook(path: str, entry: int, rows: np.ndarray, signs: np.ndarray) -> None:
    with open(path, "wb") as f:
        f.write(struct.pack("<I", entry & 0xFFFFFFFF))
        f.write(np.ascontiguousarray(rows, dtype=np.float32).tobytes())
        f.write(np.ascontiguousarray(signs, dtype=np.float32).tobytes())


def read_codebook(path: str, n: int, dim: int, degree: int) -> Tuple[int, np.ndarray, np.ndarray]:
    """(entry point, rows [n, row] float32, signs [D]); the rows are a
    read-only memory map of the file (codebooks of tens of GB)."""
    L = layout(dim, degree)
    with open(path, "rb") as f:
        entry = struct.unpack("<I", f.read(4))[0]
        f.seek(4 + n * L.row * 4)
        signs = np.fromfile(f, dtype=np.float32, count=L.padded_dim)
    rows = np.memmap(path, dtype=np.float32, mode="r", offset=4, shape=(n, L.row))
    return entry, rows, signs


# --------------------------------------------------------------------------
# fvecs / ivecs (include/data_io.hpp:18-77)
# --------------------------------------------------------------------------
def write_vecs(path: str, a: np.ndarray) -> None:
    a = np.ascontiguousarray(a)
    m, d = a.shape
    out = np.empty((m, d + 1), dtype=np.int32)
    out[:, 0] = d
    out[:, 1:] = a.view(np.int32) if a.dtype in (np.float32, np.int32) else a.astype(np.int32)
    out.tofile(path)


def read_vecs(path: str, dtype=np.float32) -> np.ndarray:
    raw = np.fromfile(path, dtype=np.int32)
    if raw.size == 0:
        return np.zeros((0, 0), dtype=dtype)
    d = int(raw[0])
    m = raw.size // (d + 1)
    return raw[: m * (d + 1)].reshape(m, d + 1)[:, 1:].copy().view(dtype)


# --------------------------------------------------------------------------
# one-call dataset materialisation with an on-disk cache
# --------------------------------------------------------------------------
@dataclasses.dataclass
class Dataset:
    spec: DatasetSpec
    base: np.ndarray
    queries: np.ndarray
    gt: np.ndarray          # int32 [nq, gt_k]
    rows: np.ndarray        # float32 [n, row]
    signs: np.ndarray
    entry: int
    layout: Layout
    codebook_path: str
    dir: str

    def digest(self) -> str:
        h = hashlib.sha256()
        h.update(struct.pack("<I", self.entry))
        h.update(self.rows.tobytes())
        h.update(self.signs.tobytes())
        return h.hexdigest()


def default_cache_dir() -> str:
    return os.environ.get("FLASHGANN_DATA", os.path.join(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__))), "_data"))


def materialize(name_or_spec, cache_dir: Optional[str] = None, device=None,
                verbose: bool = False) -> Dataset:
    spec = SPECS[name_or_spec] if isinstance(name_or_spec, str) else name_or_spec
    cache_dir = cache_dir or default_cache_dir()
    d = os.path.join(cache_dir, spec.name)
    os.makedirs(d, exist_ok=True)
    L = layout(spec.dim, spec.degree)
    paths = {k: os.path.join(d, v) for k, v in dict(
        base="base.fvecs", query="query.fvecs", gt="gt.ivecs", cb="qg_codebook.index").items()}
    if all(os.path.exists(p) for p in paths.values()):
        base = read_vecs(paths["base"])
        queries = read_vecs(paths["query"])
        gt = read_vecs(paths["gt"], np.int32)
        entry, rows, signs = read_codebook(paths["cb"], spec.n, spec.dim, spec.degree)
        return Dataset(spec, base, queries, gt, rows, signs, entry, L, paths["cb"], d)
    import time
    t0 = time.time()
    if spec.knn == "partitioned" and spec.n > 2_000_000:
        return _materialize_on_device(spec, paths, d, L, device, verbose)
    base, queries = generate_vectors(spec)
    if verbose:
        print(f"[builder] {spec.name}: vectors {time.time() - t0:.1f}s", flush=True)
    nbrs, entry = build_graph(base, spec.degree, spec.seed, knn_k=spec.knn_k, device=device, knn=spec.knn,
                              verbose=verbose, random_links=spec.random_links if spec.random_links >= 0 else None)
    if verbose:
        print(f"[builder] {spec.name}: graph {time.time() - t0:.1f}s", flush=True)
    signs = make_signs(L.padded_dim, spec.seed)
    rows = encode_rows(base, nbrs, signs, device=device)
    if verbose:
        print(f"[builder] {spec.name}: codes {time.time() - t0:.1f}s", flush=True)
    gt_ids, _ = brute_force_knn(base, queries, min(spec.gt_k, spec.n), device=device)
    gt = gt_ids.astype(np.int32)
    tmp = paths["cb"] + ".tmp"
    write_codebook(tmp, entry, rows, signs)
    write_vecs(paths["base"], base)
    write_vecs(paths["query"], queries)
    write_vecs(paths["gt"], gt)
    os.replace(tmp, paths["cb"])
    if verbose:
        print(f"[builder] {spec.name}: done {time.time() - t0:.1f}s", flush=True)
    return Dataset(spec, base, queries, gt, rows, signs, entry, L, paths["cb"], d)


def _materialize_on_device(spec: DatasetSpec, paths, d, L, device, verbose) -> Dataset:
    """materialize for bases of millions of rows: graph and codes built on the
    GPU (build_graph_device, encode_rows_device), codebook written from the
    device in chunks, rows returned memory-mapped."""
    import time
    t0 = time.time()
    dev = _device(device)
    if dev.type != "cuda":
        raise RuntimeError(f"{spec.name}: {spec.n} rows are built on a GPU only")
    base, queries = generate_vectors(spec)
    if verbose:
        print(f"[builder] {spec.name}: vectors {time.time() - t0:.1f}s", flush=True)
    xt = torch.from_numpy(base).to(dev)
    nbrs, entry = build_graph_device(xt, spec.degree, spec.seed, knn_k=spec.knn_k, verbose=verbose,
                                     random_links=spec.random_links)
    signs = make_signs(L.padded_dim, spec.seed)
    rows = encode_rows_device(xt, nbrs, signs)
    del nbrs, xt
    tmp = paths["cb"] + ".tmp"
    write_codebook_device(tmp, entry, rows, signs)
    del rows
    torch.cuda.empty_cache()
    if verbose:
        print(f"[builder] {spec.name}: codes {time.time() - t0:.1f}s", flush=True)
    gt_ids, _ = brute_force_knn(base, queries, min(spec.gt_k, spec.n), device=device)
    gt = gt_ids.astype(np.int32)
    write_vecs(paths["base"], base)
    write_vecs(paths["query"], queries)
    write_vecs(paths["gt"], gt)
    os.replace(tmp, paths["cb"])
    entry, rows, signs = read_codebook(paths["cb"], spec.n, spec.dim, spec.degree)
    if verbose:
        print(f"[builder] {spec.name}: done {time.time() - t0:.1f}s", flush=True)
    return Dataset(spec, base, queries, gt, rows, signs, entry, L, paths["cb"], d)


def query_set(ds: Dataset, index: int, device=None, cache_dir: Optional[str] = None,
              verbose: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """Query batch `index` of a materialised dataset with its exact ground
    truth (int32 [nq, gt_k]): 0 is the dataset's own batch; index > 0 is a
    further batch of the same distribution (generate_queries), its ground
    truth computed like the dataset's and cached beside it."""
    if index == 0:
        return ds.queries, ds.gt
    spec = ds.spec
    d = os.path.join(cache_dir or default_cache_dir(), spec.name)
    qp, gp = os.path.join(d, f"query_set{index}.fvecs"), os.path.join(d, f"gt_set{index}.ivecs")
    if os.path.exists(qp) and os.path.exists(gp):
        return read_vecs(qp), read_vecs(gp, np.int32)
    queries = generate_queries(spec, index)
    gt_ids, _ = brute_force_knn(ds.base, queries, min(spec.gt_k, spec.n), device=device)
    gt = gt_ids.astype(np.int32)
    write_vecs(gp + ".tmp", gt)
    write_vecs(qp + ".tmp", queries)
    os.replace(gp + ".tmp", gp)
    os.replace(qp + ".tmp", qp)
    if verbose:
        print(f"[builder] {spec.name}: query set {index} ({len(queries)} queries)", flush=True)
    return queries, gt


# --------------------------------------------------------------------------
# index shards (every GPU holds one shard with its
# own graph and entry point; global id = shard offset + local id)
# --------------------------------------------------------------------------
@dataclasses.dataclass
class Shard:
    spec: DatasetSpec
    index: int
    count: int
    offset: int           # global id of local node 0
    n: int
    queries: np.ndarray   # the full query batch
    gt: np.ndarray        # global exact neighbours of the full base
    rows: np.ndarray
    signs: np.ndarray
    entry: int
    layout: Layout
    codebook_path: str


def shard_range(n: int, count: int, index: int) -> Tuple[int, int]:
    base, extra = divmod(n, count)
    start = index * base + min(index, extra)
    return start, start + base + (1 if index < extra else 0)


def materialize_shard(name_or_spec, index: int, count: int, cache_dir: Optional[str] = None, device=None,
                      verbose: bool = False) -> Shard:
    """Shard `index` of `count` contiguous slices of a dataset's base vectors,
    with its own graph (built on the slice only), entry point and codebook;
    the signs are the dataset's.  The full dataset is materialised first (it
    provides the vectors and the global ground truth)."""
    spec = SPECS[name_or_spec] if isinstance(name_or_spec, str) else name_or_spec
    full = materialize(spec, cache_dir=cache_dir, device=device, verbose=verbose)
    s, e = shard_range(spec.n, count, index)
    L = full.layout
    d = os.path.join(cache_dir or default_cache_dir(), f"{spec.name}_shard{index}of{count}")
    os.makedirs(d, exist_ok=True)
    cb = os.path.join(d, "qg_codebook.index")
    if os.path.exists(cb):
        entry, rows, signs = read_codebook(cb, e - s, spec.dim, spec.degree)
    else:
        part = full.base[s:e]
        nbrs, entry = build_graph(part, spec.degree, spec.seed * 1000 + index, knn_k=spec.knn_k, device=device)
        signs = full.signs
        rows = encode_rows(part, nbrs, signs, device=device)
        write_codebook(cb + ".tmp", entry, rows, signs)
        os.replace(cb + ".tmp", cb)
        if verbose:
            print(f"[builder] {spec.name} shard {index}/{count}: {e - s} nodes", flush=True)
    return Shard(spec, index, count, s, e - s, full.queries, full.gt, rows, signs, entry, L, cb)


@dataclasses.dataclass
class DeviceShard:
    """One shard of a blocked spec built on its own GPU (materialize_shard_device)."""
    spec: DatasetSpec
    index: int
    count: int
    offset: int            # global id of local node 0
    n: int
    queries: np.ndarray    # the full query batch
    rows: torch.Tensor     # float32 [n, row] on the device
    signs: np.ndarray
    entry: int
    layout: Layout
    gt_ids: np.ndarray     # int64 [nq, gt_k]: this shard's exact nearest rows (global ids)
    gt_d: np.ndarray       # float64 [nq, gt_k]: their squared distances


def materialize_shard_device(name_or_spec, index: int, count: int, device, verbose: bool = False) -> DeviceShard:
    """Shard `index` of `count` of a blocked spec:
    its rows (whole blocks, drawn here), its own graph, entry point and codes,
    built and kept on `device`, plus its exact top-gt_k for every query.  No
    host ever holds the whole base: the global ground truth is the merge of
    every shard's lists (merge_shard_ground_truth)."""
    import time
    t0 = time.time()
    spec = SPECS[name_or_spec] if isinstance(name_or_spec, str) else name_or_spec
    s, e = shard_range(spec.n, count, index)
    if spec.block <= 0 or s % spec.block or (e % spec.block and e != spec.n):
        raise ValueError(f"{spec.name}: shard {index} of {count} does not cover whole blocks of {spec.block}")
    dev = _device(device)
    base = np.concatenate([generate_block(spec, b) for b in range(s // spec.block, (e + spec.block - 1) // spec.block)])
    queries = _draw(spec, 2, spec.nq)
    if verbose:
        print(f"[builder] {spec.name} shard {index}/{count}: {e - s} rows drawn, {time.time() - t0:.1f}s", flush=True)
    xt = torch.from_numpy(base).to(dev)
    nbrs, entry = build_graph_device(xt, spec.degree, spec.seed * 1000 + index, knn_k=spec.knn_k, verbose=verbose,
                                     random_links=spec.random_links)
    L = layout(spec.dim, spec.degree)
    signs = make_signs(L.padded_dim, spec.seed)
    rows = encode_rows_device(xt, nbrs, signs)
    del nbrs, xt
    torch.cuda.empty_cache()
    gi, gd = brute_force_knn(base, queries, min(spec.gt_k, e - s), device=device)
    if verbose:
        print(f"[builder] {spec.name} shard {index}/{count}: built, {time.time() - t0:.1f}s", flush=True)
    return DeviceShard(spec, index, count, s, e - s, queries, rows, signs, entry, L, gi + s, gd)


def merge_shard_ground_truth(ids: np.ndarray, d: np.ndarray, k: int) -> np.ndarray:
    """Global exact top-k from every shard's exact top lists (ids [S, nq, k']
    global, d [S, nq, k'] squared distances): ordered by (distance, id), as
    brute_force_knn orders the whole base.  Returns int32 [nq, k]."""
    S, nq, kk = ids.shape
    i = ids.transpose(1, 0, 2).reshape(nq, S * kk)
    dd = d.transpose(1, 0, 2).reshape(nq, S * kk)
    order = np.lexsort((i, dd), axis=1)[:, :k]
    return np.take_along_axis(i, order, 1).astype(np.int32)
