"""Indexes built on the GPU: fg_index_create_device (a codebook already in
device memory) searches exactly like fg_index_create on the same bytes, and
the shards of a blocked spec, each drawn and built on the device
(builder.materialize_shard_device), give the exact global ground truth when
their lists are merged and a merged search result through the
fg_shard_merge_device kernel that matches a host merge of the shards' own
results."""

from __future__ import annotations

import numpy as np
import pytest

from tests.common import dataset, merge_shard_topk_ref

pytestmark = pytest.mark.gpu


def test_index_from_device_buffers_matches_host_created():
    import torch
    import flashgann_b200 as fg
    ds = dataset("t_2k")
    K = ds.spec.K
    a = fg.QuantizationGraph.from_arrays(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree)
    rows = torch.from_numpy(np.ascontiguousarray(ds.rows)).cuda()
    signs = torch.from_numpy(np.ascontiguousarray(ds.signs)).cuda()
    b = fg.QuantizationGraph.from_device(rows, signs, ds.entry, ds.spec.dim, ds.spec.degree)
    del rows, signs
    try:
        for beam in (100, 256):
            assert np.array_equal(a.search(ds.queries, K, beam), b.search(ds.queries, K, beam))
    finally:
        a.close()
        b.close()


def test_device_built_shards_merge_to_the_global_answer():
    import torch
    import flashgann_b200 as fg
    from flashgann_b200 import builder
    from flashgann_b200.distributed import merge_shard_topk_device
    spec = builder.SPECS["t_blk40k"]
    base = np.concatenate([builder.generate_block(spec, b) for b in range(spec.n // spec.block)])
    queries = builder._draw(spec, 2, spec.nq)
    want_gt, _ = builder.brute_force_knn(base, queries, spec.gt_k, device="cuda")
    S, K, beam = 2, spec.K, 256
    shards = [builder.materialize_shard_device(spec, r, S, device="cuda") for r in range(S)]
    gt = builder.merge_shard_ground_truth(np.stack([sh.gt_ids for sh in shards]), np.stack([sh.gt_d for sh in shards]),
                                          spec.gt_k)
    assert np.array_equal(gt, want_gt.astype(np.int32))
    ids, dists = [], []
    for sh in shards:
        qg = fg.QuantizationGraph.from_device(sh.rows, torch.from_numpy(sh.signs).cuda(), sh.entry, spec.dim, spec.degree)
        q = torch.from_numpy(np.ascontiguousarray(sh.queries)).cuda()
        i = torch.empty((len(sh.queries), K), dtype=torch.int32, device="cuda")
        d = torch.empty((len(sh.queries), K), dtype=torch.float32, device="cuda")
        qg.search_device(q, K, beam, d_out=i, d_dists=d)
        torch.cuda.synchronize()
        ids.append(i)
        dists.append(d)
        qg.close()
    offsets = [sh.offset for sh in shards]
    mi, md = merge_shard_topk_device(torch.stack(ids), torch.stack(dists), offsets, K)
    ri, rd = merge_shard_topk_ref(torch.stack(ids).cpu(), torch.stack(dists).cpu(), offsets, K)
    assert np.array_equal(mi.cpu().numpy(), ri.numpy()) and np.array_equal(md.cpu().numpy(), rd.numpy())
    recall = fg.compute_recall(mi.cpu().numpy().view(np.uint32), gt, K)
    assert recall > 0.9, recall
