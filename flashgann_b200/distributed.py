"""Multi-GPU search: one process per GPU over torch.distributed.

The reference has no multi-GPU code (its search uses the current device
only, gpu_search_adaptive.cu:30-34).  Two modes are provided:

* replicated index, partitioned queries (configs 1-4): every rank holds the
  whole codebook, searches a contiguous slice of the query batch, and the
  slices are gathered -- the only collective is that gather of results;
* sharded index (the 100M config): every rank holds one shard with its own
  graph, searches *all* queries on it, and the per-shard top-K lists
  (distance, global id) are all-gathered and merged per query.

Both work with any torch.distributed backend (NCCL on GPUs, gloo on CPU for
the tests); the search itself is injected, so the host logic is testable
without a GPU.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist


def partition(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, end) slice of n items for `rank`."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _device_for(group) -> torch.device:
    backend = dist.get_backend(group)
    return torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")


def search_partitioned(search: Callable[[np.ndarray], Tuple[np.ndarray, np.ndarray]], queries: np.ndarray, K: int,
                       group=None) -> Tuple[np.ndarray, np.ndarray]:
    """Replicated index: this rank searches its slice of `queries` with
    `search(q) -> (ids uint32 [m, K], dists float32 [m, K])`; every rank
    returns the full (ids, dists) in query order."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    nq = queries.shape[0]
    s, e = partition(nq, world, rank)
    ids, dists = search(queries[s:e])
    dev = _device_for(group)
    maxm = nq // world + (1 if nq % world else 0)
    buf_i = torch.full((maxm, K), -1, dtype=torch.int64, device=dev)
    buf_d = torch.full((maxm, K), float("inf"), dtype=torch.float32, device=dev)
    buf_i[: e - s] = torch.from_numpy(ids.astype(np.int64)).to(dev)
    buf_d[: e - s] = torch.from_numpy(np.ascontiguousarray(dists, dtype=np.float32)).to(dev)
    all_i = [torch.empty_like(buf_i) for _ in range(world)]
    all_d = [torch.empty_like(buf_d) for _ in range(world)]
    dist.all_gather(all_i, buf_i, group=group)
    dist.all_gather(all_d, buf_d, group=group)
    out_i = np.empty((nq, K), dtype=np.uint32)
    out_d = np.empty((nq, K), dtype=np.float32)
    for r in range(world):
        rs, re = partition(nq, world, r)
        out_i[rs:re] = all_i[r][: re - rs].cpu().numpy().astype(np.uint32)
        out_d[rs:re] = all_d[r][: re - rs].cpu().numpy()
    return out_i, out_d


def merge_shard_topk(dists: torch.Tensor, ids: torch.Tensor, K: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Merge per-shard sorted top-K lists into one top-K per query.

    dists/ids: [S, nq, K] (shard-major, each list ascending, global ids).
    Ties are ordered by shard, then by position in the shard's list, so the
    result is deterministic.  Returns (ids [nq, K], dists [nq, K])."""
    S, nq, k = dists.shape
    d = dists.permute(1, 0, 2).reshape(nq, S * k)
    i = ids.permute(1, 0, 2).reshape(nq, S * k)
    order = torch.argsort(d, dim=1, stable=True)[:, :K]
    return torch.gather(i, 1, order), torch.gather(d, 1, order)


def search_sharded(search: Callable[[np.ndarray], Tuple[np.ndarray, np.ndarray]], queries: np.ndarray, K: int,
                   shard_offset: int, group=None) -> Tuple[np.ndarray, np.ndarray]:
    """Sharded index: this rank searches all queries on its shard (local ids
    + shard_offset = global ids); the per-shard lists are all-gathered and
    merged.  Every rank returns the merged (ids, dists)."""
    world = dist.get_world_size(group)
    ids, dists = search(queries)
    dev = _device_for(group)
    gi = torch.from_numpy(ids.astype(np.int64) + int(shard_offset)).to(dev)
    gd = torch.from_numpy(np.ascontiguousarray(dists, dtype=np.float32)).to(dev)
    all_i = [torch.empty_like(gi) for _ in range(world)]
    all_d = [torch.empty_like(gd) for _ in range(world)]
    dist.all_gather(all_i, gi, group=group)
    dist.all_gather(all_d, gd, group=group)
    mi, md = merge_shard_topk(torch.stack(all_d), torch.stack(all_i), K)
    return mi.cpu().numpy().astype(np.uint32), md.cpu().numpy()


def gather_shard_topk(ids: torch.Tensor, dists: torch.Tensor, K: int, shard_offset: int,
                      group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Device-side merge for a sharded index: this rank's per-query top-K
    (local ids [nq, K] int32 / uint32 bits, dists [nq, K] f32, on this rank's
    device) are offset to global ids, all-gathered (NCCL over NVLink on GPUs)
    and merged into the global top-K on every rank.  Returns (ids int64,
    dists f32), both [nq, K] on the input device."""
    world = dist.get_world_size(group)
    gi = (ids.to(torch.int64) & 0xFFFFFFFF) + int(shard_offset)
    gd = dists.contiguous()
    nq, k = gi.shape
    all_i = torch.empty((world * nq, k), dtype=gi.dtype, device=gi.device)
    all_d = torch.empty((world * nq, k), dtype=gd.dtype, device=gd.device)
    dist.all_gather_into_tensor(all_i, gi, group=group)
    dist.all_gather_into_tensor(all_d, gd, group=group)
    return merge_shard_topk(all_d.view(world, nq, k), all_i.view(world, nq, k), K)


def max_over_ranks(x: float, group=None) -> float:
    """Device-timed step time: the slowest rank's."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=_device_for(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
