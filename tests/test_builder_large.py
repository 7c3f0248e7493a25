"""The builder's paths for bases of millions of rows, checked on small cases
on the CPU: the partitioned k-NN against the exact one, the device-resident
graph and codes against the host functions they restate, blocked drawing of a
base, and the merge of per-shard ground truths into the global one."""

from __future__ import annotations

import dataclasses

import numpy as np
import torch

from flashgann_b200 import builder


def _spec(n=6000, **kw):
    # 20 components of ~300 rows: the rows-per-component regime of the 10M config
    return dataclasses.replace(builder.SPECS["c3_10m"], name="cpu_small", n=n, nq=50, n_comp=20, **kw)


def test_partitioned_knn_finds_nearly_all_exact_neighbours():
    spec = _spec()
    x, _ = builder.generate_vectors(spec)
    ids, d = builder.partitioned_knn(x, 32, 3, device="cpu", cluster_size=256)
    ei, _ = builder.brute_force_knn(x, None, 32, device="cpu", exclude_self=True)
    recall = np.mean([len(set(ids[i]) & set(ei[i])) / 32 for i in range(len(x))])
    assert recall > 0.97, recall
    assert np.all(np.diff(d, axis=1) >= 0)  # ascending
    assert not np.any(ids == np.arange(len(x))[:, None])  # itself excluded


def test_device_knn_equals_host_partitioned_knn():
    spec = _spec()
    x, _ = builder.generate_vectors(spec)
    hi, hd = builder.partitioned_knn(x, 24, 5, device="cpu", cluster_size=300)
    di, dd = builder.knn_partitioned_device(torch.from_numpy(x), 24, 5, cluster_size=300)
    assert np.array_equal(hi, di.numpy().astype(np.int64))
    assert np.array_equal(hd.astype(np.float32), dd.numpy())


def test_device_reverse_merge_equals_host_merge():
    spec = _spec()
    x, _ = builder.generate_vectors(spec)
    ids, d = builder.partitioned_knn(x, 16, 5, device="cpu", cluster_size=300)
    hi, hd = builder._merge_reverse_large(ids, d, 24, "cpu")
    di, dd = builder.merge_reverse_device(torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(d.astype(np.float32)), 24)
    assert np.array_equal(hi, di.numpy().astype(np.int64))
    assert np.array_equal(hd.astype(np.float32), dd.numpy())


def test_device_codes_equal_host_codes():
    spec = _spec(n=3000)
    x, _ = builder.generate_vectors(spec)
    nb, entry = builder.build_graph_device(torch.from_numpy(x), 32, 3)
    assert 0 <= entry < len(x)
    L = builder.layout(spec.dim, 32)
    signs = builder.make_signs(L.padded_dim, 3)
    rows_d = builder.encode_rows_device(torch.from_numpy(x), nb, signs).numpy()
    rows_h = builder.encode_rows(x, nb.numpy().astype(np.int64), signs, device="cpu")
    assert np.array_equal(rows_d.view(np.uint32), rows_h.view(np.uint32))


def test_device_graph_rows_have_no_repeated_neighbours():
    spec = _spec(n=3000)
    x, _ = builder.generate_vectors(spec)
    nb, _ = builder.build_graph_device(torch.from_numpy(x), 32, 3, random_links=12)
    nb = nb.numpy()
    for row in nb:
        v = row[row >= 0]
        assert len(v) == len(set(v.tolist()))


def test_blocked_base_is_the_concatenation_of_its_blocks():
    spec = dataclasses.replace(builder.SPECS["t_blk40k"], n=30_000, block=7_500)
    a = np.concatenate([builder.generate_block(spec, b) for b in range(4)])
    b = builder.generate_block(spec, 2)
    assert np.array_equal(a[15_000:22_500], b)
    assert a.min() >= -128 and a.max() <= 127 and np.all(a == np.rint(a))


def test_shard_ground_truths_merge_to_the_global_one():
    spec = dataclasses.replace(builder.SPECS["t_blk40k"], n=8_000, block=1_000, nq=40, n_comp=20)
    base = np.concatenate([builder.generate_block(spec, b) for b in range(8)])
    q = builder._draw(spec, 2, spec.nq)
    want, _ = builder.brute_force_knn(base, q, 100, device="cpu")
    parts = []
    for r in range(4):
        s, e = builder.shard_range(spec.n, 4, r)
        i, d = builder.brute_force_knn(base[s:e], q, 100, device="cpu")
        parts.append((i + s, d))
    got = builder.merge_shard_ground_truth(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]), 100)
    assert np.array_equal(got, want.astype(np.int32))
