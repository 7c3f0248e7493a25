"""The gpu_flashgann command line as a drop-in for the reference's
bin/gpu_flashgann (main.cu:11-109): the same positional arguments read from
fvecs/ivecs files and a qg_codebook, the same result lines on stdout, and the
CSV appended in the reference's schema (include/common.hpp:68-94, header only
when the file is new).  The printed recall equals the oracle's on the same
files, and -- where the reference's own sm_100a build of the CLI is present
(oracle/_ref/gpu_flashgann_ref) -- the reference CLI's recall line."""

from __future__ import annotations

import csv
import os
import re
import subprocess

import numpy as np
import pytest

from tests.common import ROOT, dataset, oracle_index

pytestmark = pytest.mark.gpu

EXE = os.path.join(ROOT, "bin", "gpu_flashgann")
REF_EXE = os.path.join(ROOT, "oracle", "_ref", "gpu_flashgann_ref")

RESULT_LINES = (r"Total time: [0-9.]+ ms", r"Throughput: [0-9.]+ queries/sec", r"Avg latency: [0-9.]+ ms/query",
                r"Recall@\d+: [0-9.]+")


def _files(ds):
    d = os.path.dirname(ds.codebook_path)
    return [os.path.join(d, f) for f in ("base.fvecs", "query.fvecs", "gt.ivecs")] + [ds.codebook_path]


def _run(exe, ds, K, beam, csv_path=None):
    args = [exe] + _files(ds) + [str(K), str(beam), str(ds.spec.degree)]
    if csv_path:
        args += ["-csv", csv_path]
    r = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    for pat in RESULT_LINES:
        assert re.search("^" + pat + "$", r.stdout, re.M), f"{os.path.basename(exe)}: no line matching {pat!r}"
    return float(re.search(r"^Recall@%d: ([0-9.]+)$" % K, r.stdout, re.M).group(1))


@pytest.mark.parametrize("name", ["t_2k", "t_8k16"])
def test_cli_recall_and_csv(name, tmp_path):
    import flashgann_b200 as fg
    if not os.path.exists(EXE):
        pytest.fail("bin/gpu_flashgann is not built (make gpu_flashgann)")
    ds = dataset(name)
    K = ds.spec.K
    oi = oracle_index(name)
    out_csv = str(tmp_path / "runs.csv")
    beams = (64, 128)
    for beam in beams:
        got = _run(EXE, ds, K, beam, out_csv)
        ids, _ = oi.search(ds.queries, K, beam)
        want = 100.0 * fg.compute_recall(ids, ds.gt, K)
        # the CLI prints %.6f of a float32 percentage
        assert abs(got - want) < 1e-3, f"beam {beam}: CLI recall {got} vs oracle {want}"
        if os.path.exists(REF_EXE):
            ref = _run(REF_EXE, ds, K, beam)
            # the reference's speculative-expansion race may reorder ties; one
            # differing hit is 100 / (nq K) percent
            assert abs(got - ref) <= 100.0 / (len(ds.queries) * K) + 1e-3, f"beam {beam}: {got} vs reference {ref}"
    with open(out_csv) as f:
        rows = list(csv.reader(f))
    assert rows[0] == ["TopK", "Beam_size", "Runtime", "Latency", "Throughput", "Recall"]
    assert len(rows) == 1 + len(beams)
    for row, beam in zip(rows[1:], beams):
        assert int(row[0]) == K and int(row[1]) == beam
        runtime, latency, qps = (float(x) for x in row[2:5])
        assert runtime > 0 and qps > 0
        assert np.isclose(latency, runtime * 1e3 / len(ds.queries), rtol=1e-4)


COMPAT_EXE = os.path.join(ROOT, "oracle", "_ref", "gpu_flashgann_compat")


@pytest.mark.parametrize("name", ["t_2k", "t_8k16"])
def test_reference_main_against_the_class_drop_in(name):
    """The reference's own main.cu, compiled unmodified against
    include/qg_compat.hpp and linked to libflashgann.so (oracle/Makefile,
    target _ref/gpu_flashgann_compat): its result lines parse, and its recall
    equals this build's CLI's and is within one hit of the reference CLI's."""
    if not os.path.exists(COMPAT_EXE):
        pytest.skip("the class drop-in check is built only where the reference sources are mounted")
    ds = dataset(name)
    K = ds.spec.K
    for beam in (64, 128):
        got = _run(COMPAT_EXE, ds, K, beam)
        assert got == _run(EXE, ds, K, beam), f"beam {beam}: class drop-in and CLI recall differ"
        if os.path.exists(REF_EXE):
            ref = _run(REF_EXE, ds, K, beam)
            assert abs(got - ref) <= 100.0 / (len(ds.queries) * K) + 1e-3, f"beam {beam}: {got} vs reference {ref}"


def test_cli_on_two_gpus_matches_one():
    """bin/gpu_flashgann -gpus 2 (the codebook on devices 0 and 1, the batch
    split between them) prints the one-GPU recall."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    ds = dataset("t_8k16")
    K, beam = ds.spec.K, 64
    args = [EXE] + _files(ds) + [str(K), str(beam), str(ds.spec.degree)]
    one = subprocess.run(args, capture_output=True, text=True, timeout=300)
    two = subprocess.run(args + ["-gpus", "2"], capture_output=True, text=True, timeout=300)
    assert one.returncode == 0 and two.returncode == 0, two.stderr[-2000:]
    pat = r"^Recall@%d: ([0-9.]+)$" % K
    assert re.search(pat, one.stdout, re.M).group(1) == re.search(pat, two.stdout, re.M).group(1)
