"""The C ABI library: loads, exports every declared entry point, and its
host-side paths (argument checks, file checks, CLI helpers) behave like the
reference's without needing a GPU."""

from __future__ import annotations

import ctypes
import os
import re
import struct

import numpy as np
import pytest

from tests.common import ROOT, dataset


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "flashgann.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fg_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    import flashgann_b200 as fg
    L = fg.lib()
    names = _declared_symbols()
    assert len(names) >= 18
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # and the Python declarations cover the same set
    from flashgann_b200 import _capi
    assert sorted(n for n, _, _ in _capi.SIGNATURES) == names


def test_status_strings():
    import flashgann_b200 as fg
    L = fg.lib()
    for code in range(8):
        assert L.fg_status_string(code).decode() != "unknown status"
    assert L.fg_status_string(99).decode() == "unknown status"


def test_index_load_errors(tmp_path):
    import flashgann_b200 as fg
    L = fg.lib()
    h = ctypes.c_void_p()
    assert L.fg_index_load(b"/definitely/missing", 10, 128, 32, 0, 0, ctypes.byref(h)) == fg.FG_ERR_IO
    assert b"cannot open codebook" in L.fg_last_error()
    # a file shorter than the layout needs
    p = tmp_path / "short.index"
    p.write_bytes(struct.pack("<I", 0) + b"\0" * 100)
    assert L.fg_index_load(os.fsencode(str(p)), 10, 128, 32, 0, 0, ctypes.byref(h)) == fg.FG_ERR_FORMAT
    # unsupported shapes are refused before any device work
    assert L.fg_index_load(os.fsencode(str(p)), 10, 128, 64, 0, 0, ctypes.byref(h)) == fg.FG_ERR_UNSUPPORTED
    assert L.fg_index_load(os.fsencode(str(p)), 10, 8, 16, 0, 0, ctypes.byref(h)) == fg.FG_ERR_UNSUPPORTED
    assert L.fg_index_load(os.fsencode(str(p)), 10, 128, 16, 7, 0, ctypes.byref(h)) == fg.FG_ERR_ARG
    assert L.fg_index_load(os.fsencode(str(p)), 0, 128, 16, 0, 0, ctypes.byref(h)) == fg.FG_ERR_ARG
    assert h.value is None


def test_index_load_without_gpu_reports_no_device(tmp_path):
    from tests.conftest import HAS_GPU
    if HAS_GPU:
        pytest.skip("a GPU is present")
    import flashgann_b200 as fg
    from flashgann_b200 import builder
    L = builder.layout(128, 16)
    p = tmp_path / "ok.index"
    builder.write_codebook(str(p), 0, np.zeros((4, L.row), np.float32), np.ones(L.padded_dim, np.float32))
    h = ctypes.c_void_p()
    assert fg.lib().fg_index_load(os.fsencode(str(p)), 4, 128, 16, 0, 0, ctypes.byref(h)) == fg.FG_ERR_NO_DEVICE


def test_null_arguments():
    import flashgann_b200 as fg
    L = fg.lib()
    assert L.fg_search(None, 1, None, 10, None, 128, None) == fg.FG_ERR_ARG
    assert L.fg_search_device(None, 1, None, 10, None, None, 128, None) == fg.FG_ERR_ARG
    assert L.fg_index_free(None) == fg.FG_OK
    assert L.fg_index_layout(None, None) == fg.FG_ERR_ARG
    assert L.fg_beam_merge_device(None, None, 1, 100, 32, 0, None) == fg.FG_ERR_ARG  # 100 is no sort width


def test_effective_sort_beam_size_matches_reference_rule():
    import flashgann_b200 as fg
    import oracle
    for b in list(range(1, 300)) + [384, 512, 640, 768, 896, 1000, 1024]:
        assert fg.effective_sort_beam_size(b) == oracle.lib().og_effective_sort_beam(b), b


def test_recall_counts_duplicates_like_reference():
    import flashgann_b200 as fg
    import oracle
    rng = np.random.default_rng(0)
    pred = rng.integers(0, 50, size=(64, 10)).astype(np.uint32)
    pred[:, 5:] = pred[:, 4:5]  # back-filled duplicates
    gt = rng.integers(0, 50, size=(64, 20)).astype(np.int32)
    for k in (10,):
        a = fg.compute_recall(pred, gt, k)
        b = oracle.compute_recall(pred, gt, k)
        assert a == b
        # direct restatement of include/common.hpp:49-66
        c = sum(1 for i in range(64) for j in range(k) if int(pred[i, j]) in gt[i, :min(k, 20)].tolist()) / (64 * k)
        assert abs(a - c) < 1e-6


def test_csv_schema(tmp_path):
    import flashgann_b200 as fg
    p = str(tmp_path / "r.csv")
    fg.append_run_stats_to_csv(p, 100, 128, 0.0123, 0.00123, 812345.678, 96.5)
    fg.append_run_stats_to_csv(p, 100, 256, 1.5, 0.15, 6666.6666, 99.25)
    lines = open(p).read().splitlines()
    assert lines[0] == "TopK,Beam_size,Runtime,Latency,Throughput,Recall"
    # std::ostream default formatting (6 significant digits), as the reference writes it
    assert lines[1] == "100,128,0.0123,0.00123,812346,96.5"
    assert lines[2] == "100,256,1.5,0.15,6666.67,99.25"


def test_metric_inference():
    import flashgann_b200 as fg
    assert fg.infer_metric_from_dataset_path("/d/Text2Image1M/base.fbin") == fg.METRIC_IP
    assert fg.infer_metric_from_dataset_path("/d/text2image1m_base.fvecs") == fg.METRIC_IP
    assert fg.infer_metric_from_dataset_path("/d/sift/base.fvecs") == fg.METRIC_L2


def test_vecs_roundtrip_and_errors(tmp_path):
    import flashgann_b200 as fg
    from flashgann_b200 import builder
    a = np.arange(5 * 7, dtype=np.float32).reshape(5, 7)
    p = str(tmp_path / "a.fvecs")
    builder.write_vecs(p, a)
    assert np.array_equal(fg.load_fvecs(p), a)
    g = np.arange(12, dtype=np.int32).reshape(3, 4)
    q = str(tmp_path / "g.ivecs")
    builder.write_vecs(q, g)
    assert np.array_equal(fg.load_ivecs(q), g)
    # a row whose leading dim disagrees (the reference asserts)
    raw = np.fromfile(p, dtype=np.int32)
    raw[8] = 6
    raw.tofile(p)
    with pytest.raises(fg.FlashGANNError) as e:
        fg.load_fvecs(p)
    assert e.value.status == fg.FG_ERR_FORMAT
    with pytest.raises(fg.FlashGANNError):
        fg.load_fvecs(str(tmp_path / "missing.fvecs"))


def test_cli_argument_errors():
    import subprocess
    exe = os.path.join(ROOT, "bin", "gpu_flashgann")
    if not os.path.exists(exe):
        pytest.skip("CLI not built")
    r = subprocess.run([exe], capture_output=True, text=True)
    assert r.returncode == 1 and "Usage:" in r.stderr
    r = subprocess.run([exe, "a", "b", "c", "d", "10", "-bogus"], capture_output=True, text=True)
    assert r.returncode == 1 and "Unknown argument: -bogus" in r.stderr
    r = subprocess.run([exe, "/missing/a", "b", "c", "d"], capture_output=True, text=True)
    assert r.returncode == 1 and "cannot open" in r.stderr


def test_entry_point_centroid_matches_oracle():
    """fg_entry_point_centroid (the UINT32_MAX entry-point fallback of
    include/common.hpp:26-47) equals the oracle's restatement on seeded data,
    reads only the first dim floats of each row, and keeps the first node on ties."""
    import ctypes
    import numpy as np
    import flashgann_b200 as fg
    import oracle
    L = fg.lib()
    O = oracle.lib()
    f32p = ctypes.POINTER(ctypes.c_float)

    def both(rows, dim, metric):
        rows = np.ascontiguousarray(rows, dtype=np.float32)
        n, row = rows.shape
        got = L.fg_entry_point_centroid(rows.ctypes.data_as(ctypes.c_void_p), n, dim, row, metric)
        want = O.og_entry_point_centroid(rows.ctypes.data_as(f32p), n, dim, row, metric)
        return int(got), int(want)

    rng = np.random.default_rng(7)
    ds = dataset("t_2k")
    for metric in (fg.FG_METRIC_L2, fg.FG_METRIC_IP):
        got, want = both(ds.rows, ds.spec.dim, metric)
        assert got == want
    # float data, rows wider than dim with noise after the raw vector
    x = rng.standard_normal((3000, 40)).astype(np.float32)
    x[:, 33:] = rng.uniform(-1e6, 1e6, (3000, 7))
    for metric in (fg.FG_METRIC_L2, fg.FG_METRIC_IP):
        got, want = both(x, 33, metric)
        assert got == want
    # the L2 choice is the float64 argmin on well separated data
    y = rng.integers(0, 256, (500, 64)).astype(np.float32)
    c = y.astype(np.float64).mean(0)
    d = ((y - c) ** 2).sum(1)
    if np.partition(d, 1)[1] - d.min() > 1.0:
        assert both(y, 64, fg.FG_METRIC_L2)[0] == int(np.argmin(d))
    # identical rows: the first node
    assert both(np.ones((50, 36), dtype=np.float32), 36, fg.FG_METRIC_L2) == (0, 0)
    # invalid arguments
    assert L.fg_entry_point_centroid(None, 10, 8, 8, 0) == 0xFFFFFFFF
    z = np.zeros((4, 8), dtype=np.float32)
    assert L.fg_entry_point_centroid(z.ctypes.data_as(ctypes.c_void_p), 4, 8, 7, 0) == 0xFFFFFFFF
    assert L.fg_entry_point_centroid(z.ctypes.data_as(ctypes.c_void_p), 0, 8, 8, 0) == 0xFFFFFFFF
