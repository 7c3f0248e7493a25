"""Shared helpers of the test suite."""

from __future__ import annotations

import functools
import json
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


@functools.lru_cache(maxsize=None)
def dataset(name: str, device: str = "cpu"):
    """A seeded dataset from flashgann_b200.builder, cached under _data/."""
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
