"""Shared helpers of the test suite."""

from __future__ import annotations

import functools
import json
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def dataset(name: str, device: str = ""):
    """A seeded dataset from flashgann_b200.builder, cached under _data/
    (built on the GPU when there is one; the result is the same bytes)."""
    if not device:
        import torch
        device = "cuda" if torch.cuda.is_available() else "cpu"
    return _dataset(name, device)


@functools.lru_cache(maxsize=None)
def _dataset(name: str, device: str):
    from flashgann_b200 import builder
    return builder.materialize(name, device=device)


@functools.lru_cache(maxsize=None)
def oracle_index(name: str):
    import oracle
    ds = dataset(name)
    return oracle.OracleIndex(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree)


def golden_manifest() -> dict:
    p = os.path.join(GOLDEN, "manifest.json")
    if not os.path.exists(p):
        return {}
    with open(p) as f:
        return json.load(f)


def golden(name: str):
    p = os.path.join(GOLDEN, name)
    return np.load(p) if os.path.exists(p) else None


def tie_order_only(ids, want, base, query, ip=False):
    """True when two result rows hold the same ids and every position where
    they differ lies inside a run of equal exact distances (squared L2, or
    the negated dot product for the inner-product metric)."""
    if set(ids.tolist()) != set(want.tolist()):
        return False

    def dist(rows):
        x = base[rows.astype(np.int64)].astype(np.float64)
        return -(x @ query) if ip else ((x - query) ** 2).sum(1)

    return np.array_equal(dist(ids), dist(want))


def compare_with_reference(ds, ids, want, ip=False):
    """Queries whose ids differ from the reference beyond tie order, and the
    number that differ only in the order of equal-distance results."""
    rows = np.nonzero((ids != want).any(axis=1))[0]
    ties = [int(i) for i in rows
            if tie_order_only(ids[i], want[i], ds.base, ds.queries[i].astype(np.float64), ip)]
    return [int(i) for i in rows if i not in ties], len(ties)


def merge_shard_topk_ref(ids, dists, offsets, K):
    """Plain-torch statement of the sharded index's per-query merge (what
    fg_shard_merge_device computes): ids [S, nq, k] int32 local ids (uint32
    bits), dists [S, nq, k] ascending per list; global id = local + offsets[s];
    the stable merge by (distance, shard, position).  Returns (ids int32 [nq, K]
    holding uint32 global ids, dists f32 [nq, K]) on the inputs' device."""
    import torch
    S, nq, k = dists.shape
    off = torch.tensor([int(o) for o in offsets], dtype=torch.int64, device=ids.device)
    g = (ids.to(torch.int64) & 0xFFFFFFFF) + off[:, None, None]
    d = dists.permute(1, 0, 2).reshape(nq, S * k)
    i = g.permute(1, 0, 2).reshape(nq, S * k)
    order = torch.argsort(d, dim=1, stable=True)[:, :K]
    gi = torch.gather(i, 1, order)
    gi = torch.where(gi >= 2 ** 31, gi - 2 ** 32, gi).to(torch.int32)
    return gi, torch.gather(d, 1, order)
