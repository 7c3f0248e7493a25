"""fg_search_async (the streamed host-buffer search) and the pipelined
search_stream built on it, through the C ABI: every batch's ids equal
fg_search's, with batches of different sizes in flight in different slots
and streams, and a slot outside the range is rejected."""

from __future__ import annotations

import numpy as np
import pytest

from tests.common import dataset

pytestmark = pytest.mark.gpu


def _graph(name):
    import flashgann_b200 as fg
    ds = dataset(name)
    return ds, fg.QuantizationGraph.from_arrays(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree)


@pytest.mark.parametrize("depth", [1, 2, 4])
def test_stream_of_batches_matches_fg_search(depth):
    ds, qg = _graph("t_8k16")
    try:
        K, beam = ds.spec.K, 64
        q = ds.queries
        cuts = [0, 1, 37, 38, 120, 200]
        batches = [q[a:b] for a, b in zip(cuts[:-1], cuts[1:])] * 2
        got = list(qg.search_stream(batches, K, beam, depth=depth))
        assert len(got) == len(batches)
        for b, ids in zip(batches, got):
            assert np.array_equal(ids, qg.search(b, K, beam))
    finally:
        qg.close()


def test_async_slots_in_flight_together():
    import torch
    ds, qg = _graph("t_2k")
    try:
        K, beam = ds.spec.K, 128
        streams = [torch.cuda.Stream() for _ in range(3)]
        parts = [ds.queries[:20], ds.queries[20:51], ds.queries[51:]]
        outs = [torch.empty((len(p), K), dtype=torch.int32).pin_memory().numpy().view(np.uint32) for p in parts]
        hq = [torch.from_numpy(np.ascontiguousarray(p)).pin_memory().numpy() for p in parts]
        for i in range(3):
            qg.search_async(i, len(parts[i]), hq[i], K, outs[i], beam, streams[i])
        for st in streams:
            st.synchronize()
        for p, o in zip(parts, outs):
            assert np.array_equal(o, qg.search(p, K, beam))
    finally:
        qg.close()


def test_async_rejects_a_slot_out_of_range():
    import torch
    import flashgann_b200 as fg
    ds, qg = _graph("t_2k")
    try:
        q = np.ascontiguousarray(ds.queries[:4])
        out = np.zeros((4, ds.spec.K), dtype=np.uint32)
        with pytest.raises(fg.FlashGANNError):
            qg.search_async(fg._capi.FG_ASYNC_SLOTS, 4, q, ds.spec.K, out, 64, torch.cuda.current_stream())
    finally:
        qg.close()
