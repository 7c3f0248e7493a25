"""The planner's goal (fg_index_set_plan_goal, fg_search_plan through the C
ABI): which kernel a batch gets under the latency and the throughput goal,
and identical results whichever kernel runs."""

from __future__ import annotations

import numpy as np
import pytest

from tests.common import dataset

pytestmark = pytest.mark.gpu


@pytest.fixture
def graph(monkeypatch):
    import flashgann_b200 as fg
    monkeypatch.delenv("FG_KERNEL", raising=False)  # the environment overrides either goal
    ds = dataset("t_8k16")
    g = fg.QuantizationGraph.from_arrays(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree, device=0)
    yield ds, g
    g.close()


def test_kernel_choice_by_goal(graph):
    import torch
    ds, g = graph
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    K, beam = ds.spec.K, 64
    # latency (the default): CTA kernel up to 4 queries per SM, the pair mode
    # while the batch is resident at once, one warp per query above
    assert g.search_plan(4 * sms, K, beam)[0] == "cta"
    kern, pair_resident = g.search_plan(4 * sms + 1, K, beam)
    assert kern == "pair" and pair_resident > 4 * sms
    assert g.search_plan(pair_resident, K, beam)[0] == "pair"
    assert g.search_plan(pair_resident + 1, K, beam)[0] == "warp"
    # throughput: the pair mode while two batches are resident at once
    g.set_plan_goal("throughput")
    assert g.search_plan(1, K, beam) == ("pair", pair_resident)
    assert g.search_plan(pair_resident // 2, K, beam)[0] == "pair"
    assert g.search_plan(pair_resident // 2 + 1, K, beam)[0] == "warp"
    g.set_plan_goal("latency")
    assert g.search_plan(4 * sms, K, beam)[0] == "cta"


def test_forced_kernel_overrides_the_goal(graph, monkeypatch):
    ds, g = graph
    g.set_plan_goal("throughput")
    monkeypatch.setenv("FG_KERNEL", "cta")
    assert g.search_plan(10, ds.spec.K, 64)[0] == "cta"


def test_results_do_not_depend_on_the_goal(graph):
    import torch
    ds, g = graph
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    K, beam = ds.spec.K, 64
    _, pair_resident = g.search_plan(4 * sms + 1, K, beam)
    # batch sizes where the two goals pick different kernels (cta / pair, pair / warp)
    for nq in (3 * sms, pair_resident // 2 + 7):
        reps = -(-nq // len(ds.queries))
        q = np.ascontiguousarray(np.tile(ds.queries, (reps, 1))[:nq])
        out = {}
        for goal in ("latency", "throughput"):
            g.set_plan_goal(goal)
            ids = np.empty((nq, K), dtype=np.uint32)
            g.gpu_search_adaptive(nq, q, K, ids, beam)
            out[goal] = (ids, g.search_plan(nq, K, beam)[0])
        assert out["latency"][1] != out["throughput"][1]
        assert np.array_equal(out["latency"][0], out["throughput"][0])


def test_unknown_goal_is_rejected(graph):
    from flashgann_b200._capi import FG_ERR_ARG, lib
    _, g = graph
    with pytest.raises(ValueError):
        g.set_plan_goal("fast")
    assert lib().fg_index_set_plan_goal(g._h, 7) == FG_ERR_ARG
    assert b"goal" in lib().fg_last_error()
