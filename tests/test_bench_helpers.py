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
