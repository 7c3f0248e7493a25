"""Pins the CPU oracle to the reference's own sm_100a build.

tests/golden/ holds inputs and outputs of the reference's device functions
and of QuantizationGraph::gpu_search_adaptive, produced on a B200 by
tests/golden/make_golden.py (oracle/ref_harness.cu + the unmodified reference
sources).  Every comparison here is bit-exact unless stated."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from tests.common import compare_with_reference, dataset, golden, golden_manifest

UNIT = golden("ref_unit.npz")
needs_unit = pytest.mark.skipif(UNIT is None, reason="tests/golden/ref_unit.npz not generated yet")


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@needs_unit
@pytest.mark.parametrize("tag", ["i128", "f96", "f256", "i100", "f1536"])
def test_query_prepare(tag):
    import oracle
    from flashgann_b200 import builder
    q = UNIT[f"qp_{tag}_queries"]
    signs = UNIT[f"qp_{tag}_signs"]
    dim = q.shape[1]
    D = builder.padded_dim(dim)
    for i in range(q.shape[0]):
        o = oracle.query_prepare(q[i], signs, dim, D)
        assert np.array_equal(_bits(o["rotated"]), _bits(UNIT[f"qp_{tag}_rot"][i])), (tag, i, "rotated")
        assert np.array_equal(o["lut"], UNIT[f"qp_{tag}_lut"][i]), (tag, i, "lut")
        f = UNIT[f"qp_{tag}_fac"][i]
        assert np.array_equal(_bits([o["low"], o["high"], o["width"]]), _bits(f)), (tag, i, "factors")
        assert o["sum_q"] == int(UNIT[f"qp_{tag}_sumq"][i]), (tag, i, "sum_q")


@needs_unit
@pytest.mark.parametrize("tag,dim,deg", [("i128d32", 128, 32), ("f96d32", 96, 32), ("i128d16", 128, 16)])
def test_estimates_and_distances(tag, dim, deg):
    import oracle
    from flashgann_b200 import builder
    L = builder.layout(dim, deg)
    rows = UNIT[f"sc_{tag}_rows"]
    signs = UNIT[f"sc_{tag}_signs"]
    qv = UNIT[f"sc_{tag}_queries"]
    preps = [oracle.query_prepare(qv[i], signs, dim, L.padded_dim) for i in range(qv.shape[0])]
    lanes8, seq = UNIT[f"sc_{tag}_lanes8"], UNIT[f"sc_{tag}_seq"]
    for k, (qi, p, pd) in enumerate(zip(UNIT[f"sc_{tag}_pairs_q"], UNIT[f"sc_{tag}_parents"],
                                        UNIT[f"sc_{tag}_pdists"])):
        qp = preps[qi]
        qf = oracle.QFactors(qp["low"], qp["high"], qp["width"], qp["sum_q"])
        row = rows[p]
        codes = np.ascontiguousarray(row.view(np.uint8)[L.code_off * 4:])
        fac = row[L.factor_off:]
        for j in range(deg):
            args = (qp["lut"].ctypes.data_as(oracle.c_u8p), ctypes.byref(qf), codes.ctypes.data_as(oracle.c_u8p),
                    j, L.padded_dim, float(fac[j]), float(fac[deg + j]), float(fac[2 * deg + j]), float(pd))
            e1 = np.float32(oracle.lib().og_estimate(*args, 1))
            e0 = np.float32(oracle.lib().og_estimate(*args, 0))
            assert _bits([e1])[0] == _bits([lanes8[k, j]])[0], (tag, k, j, e1, lanes8[k, j])
            assert _bits([e0])[0] == _bits([seq[k, j]])[0], (tag, k, j, e0, seq[k, j])
    for use_ip, key in ((False, "l2"), (True, "ip")):
        want = UNIT[f"l2_{tag}_{key}"]
        for k, (qi, node) in enumerate(zip(UNIT[f"l2_{tag}_qidx"], UNIT[f"l2_{tag}_nodes"])):
            got = np.float32(oracle.warp_distance(qv[qi], rows[node][:dim], use_ip))
            assert _bits([got])[0] == _bits([want[k]])[0], (tag, key, k, got, want[k])


def _merge_keys():
    if UNIT is None:
        return []
    return sorted({k[: -len("_idx_in")] for k in UNIT.files if k.startswith("mg_") and k.endswith("_idx_in")})


@needs_unit
@pytest.mark.parametrize("key", _merge_keys())
def test_beam_merge(key):
    import oracle
    _, itopk, cbs, first = key.split("_")
    itopk, cbs, first = int(itopk), int(cbs), int(first)
    idx, dist = UNIT[key + "_idx_in"], UNIT[key + "_dist_in"]
    wi, wd = UNIT[key + "_idx_out"], UNIT[key + "_dist_out"]
    for c in range(idx.shape[0]):
        oi, od = oracle.beam_merge(idx[c], dist[c], cbs, itopk, bool(first))
        assert np.array_equal(oi[:itopk], wi[c]) and np.array_equal(_bits(od[:itopk]), _bits(wd[c])), (key, c)


@needs_unit
def test_controller_rho_and_keep():
    import oracle
    kn = oracle.default_knobs()
    ro = ctypes.c_float()
    ko = ctypes.c_int()
    for i in range(len(UNIT["ct_rho_prev"])):
        oracle.lib().og_rho_update(float(UNIT["ct_rho_prev"][i]), int(UNIT["ct_policy"][i]), float(UNIT["ct_rate"][i]),
                                   float(UNIT["ct_p2rho"][i]), int(UNIT["ct_active"][i]), int(UNIT["ct_cut"][i]),
                                   int(UNIT["ct_near"][i]), ctypes.byref(kn), ctypes.byref(ro), ctypes.byref(ko))
        assert _bits([ro.value])[0] == _bits([UNIT["ct_rho_out"][i]])[0], i
        assert ko.value == int(UNIT["ct_keep_out"][i]), i


# c1_100k is BASELINE.json configs[0] at full size (100K nodes, all 1000 queries x 6 beams)
SEARCH_SETS = ["t_2k", "t_8k16", "t_20k", "t_2k_ip", "c1_100k"]


@pytest.mark.parametrize("name", SEARCH_SETS)
def test_search_matches_reference(name):
    """Result ids of every query and beam equal the reference build's.

    One documented exception: in the speculative (theta > 1) expansion the
    reference's warps race to insert a child kept by two parents of the same
    iteration; which warp wins moves later candidates by one slot, and the
    bitonic sort may then order two candidates of equal distance the other
    way.  This build resolves the race deterministically (first parent wins),
    so a result row may differ from the reference only in the order of
    equal-distance entries -- allowed for at most 1% of queries."""
    man = golden_manifest().get(name)
    g = golden(f"ref_search_{name}.npz")
    if man is None or g is None:
        pytest.skip("search goldens not generated yet")
    import oracle
    ds = dataset(man.get("dataset", name))
    assert ds.digest() == man["digest"], "regenerated dataset differs from the golden one"
    oi = oracle.OracleIndex(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree,
                            use_ip=man.get("metric") == "ip")
    for beam in man["beams"]:
        ids, _ = oi.search(ds.queries, man["K"], beam)
        want = g[f"ids_{beam}"]
        bad, ties = compare_with_reference(ds, ids, want, man.get("metric") == "ip")
        assert not bad, f"{name} beam {beam}: queries {bad[:10]} differ from the reference"
        assert ties <= max(1, len(ids) // 100), f"{name} beam {beam}: {ties} tie-order differences"
        assert oracle.compute_recall(ids, ds.gt, man["K"]) == oracle.compute_recall(want, ds.gt, man["K"])


def test_duplicate_heavy_search_agrees_as_much_as_the_reference_with_itself():
    """t_2kdup stores every vector four times.  There the reference's race
    (several warps inserting a child kept by two parents, see above) fires in
    most iterations, and two runs of the reference build return the same ids
    for only 9-19 of the 64 queries and the same sorted distance list for
    58-60 of them (tests/golden/manifest.json, run_to_run_*).  Exact pinning
    is impossible, so this checks that the oracle's sorted distances equal
    those of one of the two reference runs about as often as the runs agree
    with each other, and that recall matches within 0.01."""
    man = golden_manifest().get("t_2kdup")
    g = golden("ref_search_t_2kdup.npz")
    if man is None or g is None:
        pytest.skip("search goldens not generated yet")
    import oracle
    ds = dataset("t_2kdup")
    assert ds.digest() == man["digest"]
    oi = oracle.OracleIndex(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree)

    def sorted_dists(ids, q):
        return np.sort(((ds.base[ids.astype(np.int64)].astype(np.float64) - q) ** 2).sum(1))

    for beam in man["beams"]:
        ids, _ = oi.search(ds.queries, man["K"], beam)
        a, b = g[f"ids_{beam}"], g[f"ids2_{beam}"]
        ours = runs = 0
        for i in range(len(ids)):
            q = ds.queries[i].astype(np.float64)
            da, db, do = sorted_dists(a[i], q), sorted_dists(b[i], q), sorted_dists(ids[i], q)
            ours += np.array_equal(do, da) or np.array_equal(do, db)
            runs += np.array_equal(da, db)
        assert ours >= runs - len(ids) // 16, f"beam {beam}: {ours} vs the reference's own {runs} of {len(ids)}"
        r = oracle.compute_recall(ids, ds.gt, man["K"])
        assert abs(r - oracle.compute_recall(a, ds.gt, man["K"])) <= 0.01
