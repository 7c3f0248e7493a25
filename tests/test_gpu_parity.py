"""CUDA search path vs the CPU oracle: bit-exact result ids, distances,
traversal traces and counters on seeded datasets (every call goes through
the C ABI of libflashgann.so)."""

from __future__ import annotations

import numpy as np
import pytest

from tests.common import dataset, oracle_index

pytestmark = pytest.mark.gpu

CASES = [
    ("t_2k", (32, 100, 128, 200, 256)),
    ("t_8k16", (16, 32, 64, 96, 128, 256, 512)),
    ("t_20k", (100, 128, 256, 384, 512, 1024)),
    # every vector four times: long runs of equal distances through both merges' tie paths
    ("t_2kdup", (100, 128, 200, 256, 512)),
    # padded dimension 512 and 2048: the one-CTA-per-query kernel
    ("t_2k300", (100, 256)),
    ("t_1k1536", (32, 128)),
    # ragged dimensions: padded 64 (W = 2) and 130 -> 256 with unaligned code rows (scalar loads)
    ("t_2k50", (64, 128, 256)),
    ("t_2k130", (64, 128, 256)),
]


def _gpu_index(name):
    import flashgann_b200 as fg
    ds = dataset(name)
    return ds, fg.QuantizationGraph.from_arrays(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree)


def _run_gpu(qg, queries, K, beam, trace_cap=0):
    import torch
    import flashgann_b200 as fg
    q = torch.from_numpy(np.ascontiguousarray(queries)).cuda()
    nq = q.shape[0]
    ids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    dists = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    stats = torch.zeros((nq, 4), dtype=torch.int32, device="cuda")
    tr = tc = None
    if trace_cap:
        tr = torch.full((nq, trace_cap, 8), -1, dtype=torch.int32, device="cuda")
        tc = torch.full((nq, trace_cap), -1, dtype=torch.int32, device="cuda")
    qg.search_device(q, K, beam, d_out=ids, d_dists=dists, d_stats=stats, d_trace=tr, d_trace_count=tc,
                     trace_cap=trace_cap)
    torch.cuda.synchronize()
    out = dict(ids=ids.cpu().numpy().view(np.uint32), dists=dists.cpu().numpy(), stats=stats.cpu().numpy())
    if trace_cap:
        out["trace"] = tr.cpu().numpy().view(np.uint32)
        out["trace_count"] = tc.cpu().numpy()
    return out


@pytest.fixture(params=["warp", "staged", "pair", "cta"])
def kernel(request, monkeypatch):
    """Every search kernel: the warp kernel, its staged variant (parent blocks
    copied to shared memory with cp.async), its pair mode (two warps per
    query) and the CTA kernel (the planner picks by batch size; FG_KERNEL
    forces one)."""
    monkeypatch.setenv("FG_KERNEL", request.param)
    return request.param


@pytest.mark.parametrize("name,beams", CASES)
def test_search_matches_oracle(name, beams, kernel):
    ds, qg = _gpu_index(name)
    oi = oracle_index(name)
    K = ds.spec.K
    nq = min(len(ds.queries), 200)
    for beam in beams:
        g = _run_gpu(qg, ds.queries[:nq], K, beam, trace_cap=160)
        bad = []
        for i in range(nq):
            o = oi.search_one(ds.queries[i], K, beam, trace_cap=160)
            if not np.array_equal(o["ids"], g["ids"][i]):
                bad.append((i, "ids"))
                continue
            if not np.array_equal(o["dists"].view(np.uint32), g["dists"][i].view(np.uint32)):
                bad.append((i, "dists"))
                continue
            n = len(o["trace_count"])
            if not (np.array_equal(o["trace_count"], g["trace_count"][i, :n]) and
                    np.array_equal(o["trace"], g["trace"][i, :n])):
                bad.append((i, "trace"))
                continue
            st = o["stats"]
            got = tuple(int(v) for v in g["stats"][i])
            want = (st.iterations, st.expansions, st.evaluations, st.estimates)
            if got != want:
                bad.append((i, f"stats {got} != {want}"))
        assert not bad, f"{name} beam {beam}: {len(bad)} queries differ, first {bad[:5]}"
    qg.close()


@pytest.mark.parametrize("name,beams", [("t_4k96f", (64, 100, 256)), ("t_2k", (128, 200))])
def test_inner_product_search_matches_oracle(name, beams, kernel):
    """METRIC_IP (the reference's Text2Image path, negated dot products) on a
    normalised 96-d set (padded to D = 128) and an integer 128-d set."""
    import oracle
    import flashgann_b200 as fg
    ds = dataset(name)
    qg = fg.QuantizationGraph.from_arrays(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree,
                                          metric=fg.METRIC_IP)
    oi = oracle.OracleIndex(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree, use_ip=True)
    K = ds.spec.K
    nq = min(len(ds.queries), 100)
    for beam in beams:
        g = _run_gpu(qg, ds.queries[:nq], K, beam, trace_cap=160)
        bad = []
        for i in range(nq):
            o = oi.search_one(ds.queries[i], K, beam, trace_cap=160)
            same = (np.array_equal(o["ids"], g["ids"][i]) and
                    np.array_equal(o["dists"].view(np.uint32), g["dists"][i].view(np.uint32)))
            n = len(o["trace_count"])
            same = same and np.array_equal(o["trace"], g["trace"][i, :n])
            if not same:
                bad.append(i)
        assert not bad, f"{name} IP beam {beam}: {len(bad)} queries differ, first {bad[:5]}"
    qg.close()


def test_host_buffer_api_matches_device_api():
    import flashgann_b200 as fg
    ds, qg = _gpu_index("t_2k")
    K = ds.spec.K
    out = np.empty((len(ds.queries), K), dtype=np.uint32)
    el = qg.gpu_search_adaptive(len(ds.queries), ds.queries, K, out, 128)
    assert el > 0
    g = _run_gpu(qg, ds.queries, K, 128)
    assert np.array_equal(out, g["ids"])
    qg.close()


def test_query_prepare_matches_oracle():
    import torch
    import oracle
    import flashgann_b200 as fg
    from flashgann_b200 import builder
    rng = np.random.default_rng(5)
    for dim in (128, 96, 100, 256, 1536):
        D = builder.padded_dim(dim)
        signs = builder.make_signs(D, dim)
        q = np.rint(rng.uniform(-128, 255, size=(64, dim))).astype(np.float32)
        q[32:] = rng.standard_normal((32, dim)).astype(np.float32)
        q[0] = 0.0
        dq = torch.from_numpy(q).cuda()
        ds_ = torch.from_numpy(signs).cuda()
        rot = torch.empty((64, D), dtype=torch.float32, device="cuda")
        quant = torch.empty((64, D), dtype=torch.uint8, device="cuda")
        lut = torch.empty((64, 4 * D), dtype=torch.uint8, device="cuda")
        fac = torch.empty((64, 3), dtype=torch.float32, device="cuda")
        sq = torch.empty(64, dtype=torch.int32, device="cuda")
        rc = fg.lib().fg_query_prepare_device(dq.data_ptr(), 64, dim, ds_.data_ptr(), rot.data_ptr(), quant.data_ptr(),
                                              lut.data_ptr(), fac.data_ptr(), sq.data_ptr(), None)
        assert rc == 0
        torch.cuda.synchronize()
        for i in range(64):
            o = oracle.query_prepare(q[i], signs, dim, D)
            assert np.array_equal(rot[i].cpu().numpy().view(np.uint32), o["rotated"].view(np.uint32)), (dim, i)
            assert np.array_equal(quant[i].cpu().numpy(), o["quant"]), (dim, i)
            assert np.array_equal(lut[i].cpu().numpy(), o["lut"]), (dim, i)
            f = fac[i].cpu().numpy()
            assert np.array_equal(f.view(np.uint32), np.array([o["low"], o["high"], o["width"]], np.float32).view(np.uint32)), (dim, i)
            assert int(sq[i]) == o["sum_q"], (dim, i)


@pytest.mark.parametrize("itopk", [32, 64, 128, 160, 200, 256, 384, 512, 1000, 1024])
def test_beam_merge_matches_oracle(itopk):
    import torch
    import oracle
    import flashgann_b200 as fg
    rng = np.random.default_rng(itopk)
    for cbs in (32, 16, 8):
        for first in ((0, 1) if itopk <= 128 else (0,)):
            ncase = 128
            total = itopk + cbs
            idx = np.full((ncase, total), 0xFFFFFFFF, dtype=np.uint32)
            dist = np.full((ncase, total), np.float32(3.4028234663852886e38), dtype=np.float32)
            for c in range(ncase):
                span = int(rng.choice([3, 16, 64, 1 << 20]))
                fill = 0 if first else int(rng.integers(1, itopk + 1))
                dist[c, :fill] = np.sort(rng.integers(0, span, size=fill)).astype(np.float32)
                idx[c, :fill] = rng.choice(1 << 20, size=fill, replace=False).astype(np.uint32) | \
                    ((rng.random(fill) < 0.5).astype(np.uint32) << np.uint32(31))
                nc = int(rng.integers(0, cbs + 1))
                pos = rng.choice(cbs, size=nc, replace=False)
                dist[c, itopk + pos] = rng.integers(0, span + 2, size=nc).astype(np.float32)
                idx[c, itopk + pos] = (1 << 21) + rng.choice(1 << 20, size=nc, replace=False).astype(np.uint32)
            di = torch.from_numpy(idx.view(np.int32).copy()).cuda()
            dd = torch.from_numpy(dist.copy()).cuda()
            rc = fg.lib().fg_beam_merge_device(di.data_ptr(), dd.data_ptr(), ncase, itopk, cbs, first, None)
            assert rc == 0
            torch.cuda.synchronize()
            gi = di.cpu().numpy().view(np.uint32)
            gd = dd.cpu().numpy()
            for c in range(ncase):
                oi, od = oracle.beam_merge(idx[c], dist[c], cbs, itopk, bool(first))
                assert np.array_equal(gi[c, :itopk], oi[:itopk]) and np.array_equal(gd[c, :itopk], od[:itopk]), \
                    (itopk, cbs, first, c)
