"""Multi-GPU host logic on CPU: world-size-2 and -3 gloo process groups run
the partitioned and the sharded search with an injected brute-force search
and, for the sharded index, the plain-torch restatement of the per-query
merge that fg_shard_merge_device computes on the GPU (the kernel itself is
checked against it in tests/test_gpu_shard_merge.py)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from flashgann_b200.distributed import partition
from tests.common import merge_shard_topk_ref


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _brute(base: np.ndarray, K: int):
    def search(q: np.ndarray):
        d = ((q[:, None, :].astype(np.float64) - base[None].astype(np.float64)) ** 2).sum(-1)
        order = np.lexsort((np.broadcast_to(np.arange(base.shape[0]), d.shape), d), axis=1)[:, :K]
        return order.astype(np.uint32), np.take_along_axis(d, order, 1).astype(np.float32)
    return search


def _worker(rank, world, port, mode, out_path):
    import torch.distributed as dist
    from flashgann_b200 import distributed as fgd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(0)
    base = np.rint(rng.uniform(0, 255, size=(600, 16))).astype(np.float32)
    queries = np.rint(rng.uniform(0, 255, size=(37, 16))).astype(np.float32)
    K = 10
    if mode == "partitioned":
        ids, d = fgd.search_partitioned(_brute(base, K), queries, K)
    else:
        s, e = fgd.partition(base.shape[0], world, rank)
        ids, d = fgd.search_sharded(_brute(base[s:e], K), queries, K, shard_offset=s, merge=merge_shard_topk_ref)
    t = fgd.max_over_ranks(float(rank + 1))
    if rank == 0:
        np.savez(out_path, ids=ids, d=d, t=t)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["partitioned", "sharded"])
def test_two_rank_search_equals_single_process(mode, tmp_path):
    out = str(tmp_path / "r.npz")
    mp.spawn(_worker, args=(2, _free_port(), mode, out), nprocs=2, join=True)
    r = np.load(out)
    rng = np.random.default_rng(0)
    base = np.rint(rng.uniform(0, 255, size=(600, 16))).astype(np.float32)
    queries = np.rint(rng.uniform(0, 255, size=(37, 16))).astype(np.float32)
    ids, d = _brute(base, 10)(queries)
    assert np.array_equal(r["d"], d)
    # equal distances may come from either shard: compare as (distance, id) sets per query
    for i in range(len(ids)):
        assert sorted(zip(r["d"][i].tolist(), r["ids"][i].tolist())) == sorted(zip(d[i].tolist(), ids[i].tolist()))
    assert float(r["t"]) == 2.0


def _gather_worker(rank, world, port, out_path):
    import torch
    import torch.distributed as dist
    from flashgann_b200 import distributed as fgd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(1)
    base = np.rint(rng.uniform(0, 255, size=(500, 8))).astype(np.float32)
    queries = np.rint(rng.uniform(0, 255, size=(21, 8))).astype(np.float32)
    s, e = fgd.partition(base.shape[0], world, rank)
    ids, d = _brute(base[s:e], 7)(queries)
    offsets = [fgd.partition(base.shape[0], world, r)[0] for r in range(world)]
    gi, gd = fgd.gather_shard_topk(torch.from_numpy(ids.view(np.int32)), torch.from_numpy(d), 7, offsets,
                                   merge=merge_shard_topk_ref)
    if rank == 0:
        np.savez(out_path, ids=gi.numpy().view(np.uint32), d=gd.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_device_shard_merge_equals_single_index(tmp_path):
    out = str(tmp_path / "g.npz")
    mp.spawn(_gather_worker, args=(3, _free_port(), out), nprocs=3, join=True)
    r = np.load(out)
    rng = np.random.default_rng(1)
    base = np.rint(rng.uniform(0, 255, size=(500, 8))).astype(np.float32)
    queries = np.rint(rng.uniform(0, 255, size=(21, 8))).astype(np.float32)
    ids, d = _brute(base, 7)(queries)
    assert np.array_equal(r["d"], d)
    for i in range(len(ids)):
        assert sorted(zip(r["d"][i].tolist(), r["ids"][i].tolist())) == sorted(zip(d[i].tolist(), ids[i].tolist()))


def test_partition_covers_everything():
    for n in (0, 1, 7, 10000):
        for w in (1, 2, 3, 8):
            parts = [partition(n, w, r) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))
            sizes = [e - s for s, e in parts]
            assert max(sizes) - min(sizes) <= 1


def test_merge_reference_ties_by_shard_then_position():
    import torch
    d = torch.tensor([[[1.0, 2.0, 5.0]], [[1.0, 3.0, 4.0]]])
    i = torch.tensor([[[0, 1, 2]], [[0, 1, 2]]], dtype=torch.int32)
    mi, md = merge_shard_topk_ref(i, d, [10, 20], 4)
    assert mi.tolist() == [[10, 20, 11, 21]] and md.tolist() == [[1.0, 1.0, 2.0, 3.0]]
