"""bench.py's host-side helpers: the QPS interpolated to the target recall
along the beam sweep, and the metric label (no GPU needed)."""

from __future__ import annotations

import importlib.util
import os

import pytest

from tests.common import ROOT


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_interpolation_is_linear_in_recall_between_the_bracketing_beams():
    b = _bench()
    table = [(256, 0.80), (512, 0.93), (640, 0.97)]
    qps = {512: 1.2e6, 640: 1.0e6}
    out = b._interpolate(table, 640, lambda beam: qps[beam])
    assert out["beams"] == [512, 640]
    w = (0.95 - 0.93) / (0.97 - 0.93)
    assert out["qps"] == pytest.approx(1.2e6 + w * (1.0e6 - 1.2e6))
    assert out["recall"] == 0.95


def test_no_interpolation_when_the_first_beam_already_reaches_the_target():
    b = _bench()
    assert b._interpolate([(128, 0.96)], 128, lambda beam: 1.0) is None
    # the previous beam must lie below the target and the calibrated one reach it
    assert b._interpolate([(128, 0.96), (256, 0.97)], 256, lambda beam: 1.0) is None


def test_metric_label_names_the_config():
    b = _bench()
    from flashgann_b200 import builder
    assert b._metric_name(builder.SPECS["c2_1m"]) == "QPS @ recall@100=0.95 (1M x 128, deg 32)"
    assert b._metric_name(builder.SPECS["c1_100k"]) == "QPS @ recall@10=0.95 (100K x 128, deg 16)"


def test_calibration_measures_every_beam_and_picks_the_first_reaching_the_target():
    b = _bench()
    recalls = {100: 0.5, 256: 0.9, 512: 0.95, 1024: 0.99}
    calls = []

    def run(beam):
        calls.append(beam)
        return beam

    beam, r, table = b._calibrate(run, None, 10, (100, 256, 512, 1024), lambda ids, gt, k: recalls[ids])
    assert calls == [100, 256, 512, 1024]  # the whole curve, every rank the same calls
    assert beam == 512 and r == 0.95
    assert table == [(100, 0.5), (256, 0.9), (512, 0.95), (1024, 0.99)]
    beam, r, _ = b._calibrate(run, None, 10, (100, 256), lambda ids, gt, k: 0.1)
    assert beam == 256  # the last beam when none reaches the target


def test_workload_config_names_the_split():
    b = _bench()
    from flashgann_b200 import builder
    spec = builder.SPECS["c2_1m"]
    weak = b._workload_config(spec, 80000, 640, 8, "weak")
    strong = b._workload_config(spec, 10000, 640, 8, "strong")
    assert weak["queries_total"] == 80000 and "distinct 10000-query batch per GPU" in weak["parallelism"]
    assert strong["queries_total"] == 10000 and "split over 8 GPU" in strong["parallelism"]
    assert set(weak) == set(strong) and "recall" not in " ".join(weak)
