"""The seeded dataset / codebook builder: byte layout of the qg_codebook
(include/qg.hpp:17-42,66-73), determinism, and that the RaBitQ codes and
factors make the kernel's estimator (include/utils.cuh:989-993) estimate the
squared distance."""

from __future__ import annotations

import numpy as np
import pytest

from tests.common import dataset


@pytest.mark.parametrize("dim,degree,row", [(128, 32, 384), (128, 16, 256), (96, 32, 352), (100, 32, 356),
                                            (1536, 32, 3712)])
def test_layout_matches_reference_formula(dim, degree, row):
    from flashgann_b200 import builder
    import oracle
    L = builder.layout(dim, degree)
    assert L.row == row
    D = 1 << int(np.ceil(np.log2(dim)))
    assert L.padded_dim == D
    assert L.code_off == dim
    assert L.factor_off == dim + (D // 64) * 2 * degree
    assert L.nbr_off == L.factor_off + 3 * degree
    o = oracle.Layout()
    oracle.lib().og_compute_layout(dim, degree, oracle.ctypes.byref(o))
    assert (o.row, o.code_off, o.factor_off, o.nbr_off, o.padded_dim) == (L.row, L.code_off, L.factor_off,
                                                                         L.nbr_off, L.padded_dim)


def test_codebook_file_roundtrip(tmp_path):
    from flashgann_b200 import builder
    ds = dataset("t_2k")
    p = str(tmp_path / "cb.index")
    builder.write_codebook(p, ds.entry, ds.rows, ds.signs)
    raw = open(p, "rb").read()
    L = ds.layout
    assert len(raw) == 4 + ds.spec.n * L.row * 4 + L.padded_dim * 4
    e, rows, signs = builder.read_codebook(p, ds.spec.n, ds.spec.dim, ds.spec.degree)
    assert e == ds.entry and np.array_equal(signs, ds.signs)
    assert np.array_equal(rows.view(np.uint32), ds.rows.view(np.uint32))  # ids are NaN as floats


def test_rows_hold_vectors_ids_and_invalid_slots():
    ds = dataset("t_2k")
    L = ds.layout
    assert np.array_equal(ds.rows[:, : ds.spec.dim], ds.base)
    ids = ds.rows.view(np.uint32)[:, L.nbr_off: L.nbr_off + L.degree]
    tx = ds.rows[:, L.factor_off: L.factor_off + L.degree]
    valid = ids != 0xFFFFFFFF
    assert valid.mean() > 0.99
    assert np.all(ids[valid] < ds.spec.n)
    assert np.all(tx[~valid] == np.float32(3.4028234663852886e38))
    # no duplicate neighbours and no self loops
    for i in range(0, ds.spec.n, 97):
        v = ids[i][valid[i]]
        assert len(set(v.tolist())) == len(v) and i not in v.tolist()
    assert np.all(np.abs(ds.signs) == 1.0)


def test_estimator_tracks_true_distance():
    """The kernel's estimate (oracle restatement) vs exact squared L2."""
    import oracle
    ds = dataset("t_2k")
    L = ds.layout
    rng = np.random.default_rng(3)
    errs, trues = [], []
    for qi in range(16):
        q = ds.queries[qi]
        qp = oracle.query_prepare(q, ds.signs, ds.spec.dim, L.padded_dim)
        qf = oracle.QFactors(qp["low"], qp["high"], qp["width"], qp["sum_q"])
        for p in rng.integers(0, ds.spec.n, size=8):
            row = ds.rows[p]
            pd = float(((q - row[: ds.spec.dim]) ** 2).sum())
            codes = np.ascontiguousarray(row.view(np.uint8)[L.code_off * 4: L.code_off * 4 + L.degree * L.padded_dim // 8])
            ids = row.view(np.uint32)[L.nbr_off: L.nbr_off + L.degree]
            fac = row[L.factor_off: L.factor_off + 3 * L.degree]
            for j in range(L.degree):
                if ids[j] == 0xFFFFFFFF:
                    continue
                est = oracle.lib().og_estimate(qp["lut"].ctypes.data_as(oracle.c_u8p), oracle.ctypes.byref(qf),
                                               codes.ctypes.data_as(oracle.c_u8p), j, L.padded_dim,
                                               float(fac[j]), float(fac[L.degree + j]), float(fac[2 * L.degree + j]),
                                               pd, 0)
                true = float(((q - ds.base[ids[j]]) ** 2).sum())
                errs.append(est - true)
                trues.append(true)
    errs, trues = np.array(errs), np.array(trues)
    corr = np.corrcoef(errs + trues, trues)[0, 1]
    assert corr > 0.9, corr
    assert abs(np.median(errs / trues)) < 0.1


def test_generation_is_deterministic():
    from flashgann_b200 import builder
    spec = builder.SPECS["t_2k"]
    a, qa = builder.generate_vectors(spec)
    b, qb = builder.generate_vectors(spec)
    assert np.array_equal(a, b) and np.array_equal(qa, qb)
    assert a.min() >= 0 and a.max() <= 255 and np.all(a == np.rint(a))


def test_ground_truth_is_exact():
    ds = dataset("t_2k")
    d = ((ds.queries[:8, None, :].astype(np.float64) - ds.base[None].astype(np.float64)) ** 2).sum(-1)
    for i in range(8):
        order = np.lexsort((np.arange(ds.spec.n), d[i]))[: ds.gt.shape[1]]
        assert np.array_equal(order, ds.gt[i])


def test_shards_partition_the_base_with_local_graphs(tmp_path):
    from flashgann_b200 import builder
    spec = builder.SPECS["t_2k"]
    full = builder.materialize(spec, cache_dir=str(tmp_path))
    L = full.layout
    seen = 0
    for i in range(3):
        sh = builder.materialize_shard(spec, i, 3, cache_dir=str(tmp_path))
        s, e = builder.shard_range(spec.n, 3, i)
        assert (sh.offset, sh.n) == (s, e - s) and s == seen
        seen = e
        assert np.array_equal(sh.rows[:, :spec.dim], full.base[s:e])
        ids = sh.rows.view(np.uint32)[:, L.nbr_off:L.nbr_off + L.degree]
        assert ((ids < sh.n) | (ids == 0xFFFFFFFF)).all()
        assert 0 <= sh.entry < sh.n
        assert np.array_equal(sh.signs, full.signs)
        assert np.array_equal(sh.gt, full.gt)
    assert seen == spec.n
