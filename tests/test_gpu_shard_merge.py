"""fg_shard_merge_device (the sharded index's per-query merge, on the GPU)
against its plain-torch statement: random ascending lists with many equal
distances across and within shards, several shard counts, k below, equal to
and above K, and shard offsets that push global ids past 2^31."""

from __future__ import annotations

import numpy as np
import pytest

from tests.common import merge_shard_topk_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("S,nq,k,K", [(2, 37, 10, 10), (8, 513, 100, 100), (3, 64, 64, 100), (8, 200, 128, 100),
                                      (1, 9, 50, 20), (16, 33, 32, 256)])
def test_device_merge_equals_reference(S, nq, k, K):
    import torch
    from flashgann_b200.distributed import merge_shard_topk_device
    rng = np.random.default_rng(S * 1000 + k)
    # few distinct values: ties everywhere
    d = np.sort(rng.integers(0, 40, size=(S, nq, k)).astype(np.float32), axis=2)
    ids = rng.integers(0, 1 << 20, size=(S, nq, k)).astype(np.uint32)
    offsets = [s * (1 << 28) for s in range(S)]  # up to 15 * 2^28: global ids above 2^31
    ti = torch.from_numpy(ids.view(np.int32))
    td = torch.from_numpy(d)
    want_i, want_d = merge_shard_topk_ref(ti, td, offsets, K)
    gi, gd = merge_shard_topk_device(ti.cuda(), td.cuda(), offsets, K)
    torch.cuda.synchronize()
    assert np.array_equal(gi.cpu().numpy(), want_i.numpy())
    assert np.array_equal(gd.cpu().numpy(), want_d.numpy())


def test_device_merge_rejects_lists_too_short_for_k():
    import torch
    from flashgann_b200._capi import FlashGANNError
    from flashgann_b200.distributed import merge_shard_topk_device
    ti = torch.zeros((2, 4, 10), dtype=torch.int32, device="cuda")
    td = torch.zeros((2, 4, 10), dtype=torch.float32, device="cuda")
    with pytest.raises(FlashGANNError):
        merge_shard_topk_device(ti, td, [0, 10], 21)
