"""Multi-GPU search: one process per GPU over torch.distributed.

The reference has no multi-GPU code (its search uses the current device
only, gpu_search_adaptive.cu:30-34).  Two modes are provided:

* replicated index, partitioned queries (configs 1-4): every rank holds the
  whole codebook, searches a contiguous slice of the query batch, and the
  slices are gathered -- the only collective is that gather of results;
* sharded index (the 100M config): every rank holds one shard with its own
  graph, searches *all* queries on it, and the per-shard top-K lists
  (distance, local id) are all-gathered and merged per query by a CUDA
  kernel (fg_shard_merge_device) into global ids.

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


def merge_shard_topk_device(ids: torch.Tensor, dists: torch.Tensor, offsets, K: int,
                            out_ids: Optional[torch.Tensor] = None,
                            out_dists: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Global top-K from per-shard sorted lists, on the GPU (the
    fg_shard_merge_device kernel of libflashgann.so).

    ids [S, nq, k] int32 (local ids as the search returns them, uint32 bits),
    dists [S, nq, k] f32, both CUDA tensors, shard-major, each list
    ascending; offsets: the S global ids of each shard's node 0.  The merge is
    the lists' stable merge by (distance, shard, position).  Returns
    (ids int32 [nq, K] holding uint32 global ids, dists f32 [nq, K]) on the
    stream torch currently uses."""
    import ctypes
    from . import _capi
    S, nq, k = dists.shape
    if out_ids is None:
        out_ids = torch.empty((nq, K), dtype=torch.int32, device=dists.device)
    if out_dists is None:
        out_dists = torch.empty((nq, K), dtype=torch.float32, device=dists.device)
    off = (ctypes.c_uint32 * S)(*[int(o) for o in offsets])
    L = _capi.lib()
    rc = L.fg_shard_merge_device(_capi.device_ptr(ids.contiguous()), _capi.device_ptr(dists.contiguous()), off, S,
                                 nq, k, K, _capi.device_ptr(out_ids), _capi.device_ptr(out_dists),
                                 ctypes.c_void_p(torch.cuda.current_stream(dists.device).cuda_stream))
    if rc != _capi.FG_OK:
        raise _capi.FlashGANNError(rc, f"fg_shard_merge_device: {L.fg_last_error().decode()}")
    return out_ids, out_dists


def search_sharded(search: Callable[[np.ndarray], Tuple[np.ndarray, np.ndarray]], queries: np.ndarray, K: int,
                   shard_offset: int, merge: Callable, group=None) -> Tuple[np.ndarray, np.ndarray]:
    """Sharded index: this rank searches all queries on its shard (local ids
    + shard_offset = global ids); the per-shard lists (local ids) and every
    rank's shard offset are all-gathered and merged by
    `merge(ids [S, nq, k], dists [S, nq, k], offsets, K) -> (ids, dists)`
    (merge_shard_topk_device on GPUs).  Every rank returns the merged
    (ids uint32, dists f32)."""
    world = dist.get_world_size(group)
    ids, dists = search(queries)
    dev = _device_for(group)
    li = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.uint32).view(np.int32)).to(dev)
    gd = torch.from_numpy(np.ascontiguousarray(dists, dtype=np.float32)).to(dev)
    offs = torch.tensor([int(shard_offset)], dtype=torch.int64, device=dev)
    all_i = [torch.empty_like(li) for _ in range(world)]
    all_d = [torch.empty_like(gd) for _ in range(world)]
    all_o = [torch.empty_like(offs) for _ in range(world)]
    dist.all_gather(all_i, li, group=group)
    dist.all_gather(all_d, gd, group=group)
    dist.all_gather(all_o, offs, group=group)
    mi, md = merge(torch.stack(all_i), torch.stack(all_d), [int(o.item()) for o in all_o], K)
    return mi.cpu().numpy().view(np.uint32).copy(), md.cpu().numpy()


def gather_shard_topk(ids: torch.Tensor, dists: torch.Tensor, K: int, offsets, group=None,
                      merge: Callable = merge_shard_topk_device) -> Tuple[torch.Tensor, torch.Tensor]:
    """Device-side step of a sharded index: this rank's per-query top-k
    (local ids [nq, k] int32 holding uint32 bits, dists [nq, k] f32, on this
    rank's GPU) are all-gathered (NCCL over NVLink) and merged by the
    fg_shard_merge_device kernel (or an injected `merge` of the same
    signature) into the global top-K on every rank; `offsets` lists every
    rank's shard offset (global id of its node 0).  Returns (ids int32
    [nq, K] holding uint32 global ids, dists f32 [nq, K])."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    li = ids.contiguous()
    gd = dists.contiguous()
    nq, k = li.shape
    if world == 1:  # one shard (a single process): the merge only maps to global ids
        return merge(li.view(1, nq, k), gd.view(1, nq, k), offsets, K)
    all_i = torch.empty((world * nq, k), dtype=li.dtype, device=li.device)
    all_d = torch.empty((world * nq, k), dtype=gd.dtype, device=gd.device)
    dist.all_gather_into_tensor(all_i, li, group=group)
    dist.all_gather_into_tensor(all_d, gd, group=group)
    return merge(all_i.view(world, nq, k), all_d.view(world, nq, k), offsets, K)


def max_over_ranks(x: float, group=None) -> float:
    """Device-timed step time: the slowest rank's."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=_device_for(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
