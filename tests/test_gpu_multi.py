"""fg_search_multi (one batch over index replicas on several devices, through
the C ABI) against the single-device search: same ids and distances, slices
stitched back in query order, mismatched handles rejected."""

from __future__ import annotations

import numpy as np
import pytest

from tests.common import dataset

pytestmark = pytest.mark.gpu


def _graph(name, device=0):
    import flashgann_b200 as fg
    ds = dataset(name)
    return fg.QuantizationGraph.from_arrays(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree, device=device)


@pytest.mark.parametrize("count", [1, 2, 3])
def test_multi_matches_single_device(count):
    import torch
    import flashgann_b200 as fg
    ds = dataset("t_8k16")
    ndev = torch.cuda.device_count()
    graphs = [_graph("t_8k16", device=i % ndev) for i in range(count)]
    try:
        K, beam = ds.spec.K, 64
        q = ds.queries[:101]  # not a multiple of the slice count
        ids, dists, el = fg.search_multi(graphs, q, K, beam, with_dists=True)
        assert el > 0
        dq = torch.from_numpy(np.ascontiguousarray(q)).cuda()
        want = torch.empty((len(q), K), dtype=torch.int32, device="cuda")
        wd = torch.empty((len(q), K), dtype=torch.float32, device="cuda")
        graphs[0].search_device(dq, K, beam, d_out=want, d_dists=wd)
        torch.cuda.synchronize()
        assert np.array_equal(ids, want.cpu().numpy().view(np.uint32))
        assert np.array_equal(dists.view(np.uint32), wd.cpu().numpy().view(np.uint32))
    finally:
        for g in graphs:
            g.close()


def test_multi_rejects_different_indexes():
    import flashgann_b200 as fg
    a, b = _graph("t_8k16"), _graph("t_2k")
    try:
        with pytest.raises(fg.FlashGANNError):
            fg.search_multi([a, b], dataset("t_2k").queries[:4], 10, 32)
    finally:
        a.close()
        b.close()


def test_multi_spans_distinct_devices_when_there_are_several():
    """With two or more GPUs visible, the replicas really live on different
    devices and the stitched result still equals one device's."""
    import torch
    import flashgann_b200 as fg
    ndev = torch.cuda.device_count()
    if ndev < 2:
        pytest.skip("one GPU visible")
    ds = dataset("t_20k")
    graphs = [_graph("t_20k", device=i) for i in range(ndev)]
    try:
        assert sorted(g.device for g in graphs) == list(range(ndev))
        K, beam = ds.spec.K, 256
        ids, _, _ = fg.search_multi(graphs, ds.queries, K, beam)
        assert np.array_equal(ids, graphs[0].search(ds.queries, K, beam))
    finally:
        for g in graphs:
            g.close()
