"""fg_search_noalloc (the search entry point that allocates no device memory)
against fg_search on the same index: identical result ids on two calls in a
row, and a clear error when a batch does not fit the fixed scratch.  Every
call goes through the C ABI of libflashgann.so.  The file is named so that it
is collected last, after the other GPU tests have used the library."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from tests.common import dataset

pytestmark = pytest.mark.gpu

FG_ERR_ARG = 3
SCRATCH_BYTES = 8388608  # FG_NOALLOC_SCRATCH_BYTES in include/flashgann.h


def _index(name):
    from flashgann_b200._capi import lib
    ds = dataset(name)
    h = ctypes.c_void_p()
    rows = np.ascontiguousarray(ds.rows, dtype=np.float32)
    signs = np.ascontiguousarray(ds.signs, dtype=np.float32)
    rc = lib().fg_index_create(rows.ctypes.data_as(ctypes.c_void_p), signs.ctypes.data_as(ctypes.c_void_p),
                               ds.entry, rows.shape[0], ds.spec.dim, ds.spec.degree, 0, 0, ctypes.byref(h))
    assert rc == 0, lib().fg_last_error()
    return ds, h


def _call(fn, h, queries, K, beam):
    from flashgann_b200._capi import lib
    q = np.ascontiguousarray(queries, dtype=np.float32)
    out = np.full((q.shape[0], K), 0xDEADBEEF, dtype=np.uint32)
    el = ctypes.c_double(-1.0)
    rc = getattr(lib(), fn)(h, q.shape[0], q.ctypes.data_as(ctypes.c_void_p), K,
                            out.ctypes.data_as(ctypes.c_void_p), beam, ctypes.byref(el))
    assert rc == 0, f"{fn}: {lib().fg_last_error().decode()}"
    assert el.value > 0
    return out


@pytest.mark.parametrize("name,beam", [("t_2k", 128), ("t_8k16", 64)])
def test_noalloc_matches_fg_search_on_two_calls(name, beam):
    from flashgann_b200._capi import lib
    ds, h = _index(name)
    try:
        K = ds.spec.K
        nq = len(ds.queries)
        # two different batches in a row: the second call must not see the first one's staged data
        for queries in (ds.queries, ds.queries[nq // 3:]):
            want = _call("fg_search", h, queries, K, beam)
            got = _call("fg_search_noalloc", h, queries, K, beam)
            assert np.array_equal(got, want)
    finally:
        lib().fg_index_free(h)


def test_noalloc_rejects_a_batch_beyond_the_scratch():
    from flashgann_b200._capi import lib
    ds, h = _index("t_2k")
    try:
        K = ds.spec.K
        dim = ds.spec.dim
        per_query = dim * 4 + K * 4
        nq = SCRATCH_BYTES // per_query + 8
        q = np.zeros((nq, dim), dtype=np.float32)
        out = np.zeros((nq, K), dtype=np.uint32)
        rc = lib().fg_search_noalloc(h, nq, q.ctypes.data_as(ctypes.c_void_p), K,
                                     out.ctypes.data_as(ctypes.c_void_p), 128, None)
        assert rc == FG_ERR_ARG
        assert b"scratch" in lib().fg_last_error()
        # after the rejection a batch that fits still runs and matches fg_search
        small = ds.queries[:7]
        assert np.array_equal(_call("fg_search_noalloc", h, small, K, 128), _call("fg_search", h, small, K, 128))
    finally:
        lib().fg_index_free(h)


def test_noalloc_on_a_fresh_index_leaves_device_memory_unchanged():
    """On an index that fg_search has never used (so it owns no query or
    result buffers), repeated fg_search_noalloc calls leave the device's free
    memory exactly as it was, and their results still match fg_search's.  The
    130-d set has rows that are not 16-byte aligned and a query length that
    is not a multiple of 4 floats, so the staged result ids start right after
    an odd-sized query block."""
    import torch
    from flashgann_b200._capi import lib
    ds, h = _index("t_2k130")
    try:
        K = ds.spec.K
        q = ds.queries[:33]
        first = _call("fg_search_noalloc", h, q, K, 128)  # looks up the scratch's address on this device
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        outs = [_call("fg_search_noalloc", h, q, K, 128) for _ in range(3)]
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
        for o in outs:
            assert np.array_equal(o, first)
        assert np.array_equal(first, _call("fg_search", h, q, K, 128))
    finally:
        lib().fg_index_free(h)
