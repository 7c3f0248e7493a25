"""Generate golden vectors from the reference's own sm_100a build.

Runs on a machine with a B200 and the prebuilt oracle/_ref/libfgref.so
(oracle/Makefile `ref` target, compiled from the reference sources).
Writes, under --out:

  ref_unit.npz       inputs and outputs of the reference device functions:
                     query rotation/quantisation/LUT, both RaBitQ estimate
                     variants, the warp exact distance (L2 and IP), the beam
                     merge (register bitonic and merge path, tie-heavy), the
                     adaptive rho / keep-count update
  ref_search_<ds>.npz  result ids of QuantizationGraph::gpu_search_adaptive
                     for every beam of a seeded dataset, two runs each
                     (<ds>_ip: with the inner-product metric, set_metric(IP))
  manifest.json      dataset digests and shapes

Usage:  python tests/golden/make_golden.py --out golden_out
        python tests/golden/make_golden.py --out golden_out --no-unit \
            --sets t_2kdup,t_2k:ip --manifest-in tests/golden/manifest.json
(then copy the new files from --out into tests/golden/)
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from flashgann_b200 import builder  # noqa: E402
from oracle import ref  # noqa: E402

SEARCH_SETS = ["t_2k", "t_8k16", "t_20k", "c1_100k", "t_2kdup", "t_2k:ip"]


def unit_goldens(rng: np.random.Generator):
    out = {}
    # ---------------- query preparation: integer and float data, edge cases
    for tag, dim in (("i128", 128), ("f96", 96), ("f256", 256), ("i100", 100), ("f1536", 1536)):
        D = builder.padded_dim(dim)
        signs = builder.make_signs(D, 100 + dim)
        n = 48
        if tag.startswith("i"):
            q = np.rint(rng.uniform(0, 255, size=(n, dim))).astype(np.float32)
            if dim == 100:
                q = np.rint(rng.uniform(-128, 127, size=(n, dim))).astype(np.float32)
        else:
            q = rng.standard_normal((n, dim)).astype(np.float32)
            q /= np.linalg.norm(q, axis=1, keepdims=True)
        # edge cases: constant rotation (width 0), and chunks whose four codes are all 64
        q[0] = 0.0
        q[1] = 0.0
        q[1, 0] = 7.0 * signs[0]
        q[2] = 0.0
        q[2, 0] = 3.0 * signs[0]
        q[2, 4] = 3.0 * signs[4]
        q[3] = 0.0
        q[3, 0] = 5.0 * signs[0]
        q[3, 1] = 5.0 * signs[1]
        q[3, 4] = 5.0 * signs[4]
        q[3, 5] = 5.0 * signs[5]
        rot, lut, fac, sq = ref.query_prep(q, signs, dim, D)
        out[f"qp_{tag}_queries"] = q
        out[f"qp_{tag}_signs"] = signs
        out[f"qp_{tag}_rot"] = rot
        out[f"qp_{tag}_lut"] = lut
        out[f"qp_{tag}_fac"] = fac
        out[f"qp_{tag}_sumq"] = sq

    # ---------------- estimates and exact distances on synthetic codebook rows
    for tag, dim, deg, integer in (("i128d32", 128, 32, True), ("f96d32", 96, 32, False), ("i128d16", 128, 16, True)):
        L = builder.layout(dim, deg)
        n = 256
        if integer:
            x = np.rint(rng.uniform(0, 255, size=(n, dim))).astype(np.float32)
        else:
            x = rng.standard_normal((n, dim)).astype(np.float32)
            x /= np.linalg.norm(x, axis=1, keepdims=True)
        nbrs = np.stack([rng.choice(n, size=deg, replace=False) for _ in range(n)]).astype(np.int64)
        nbrs[rng.random((n, deg)) < 0.05] = -1  # invalid slots
        signs = builder.make_signs(L.padded_dim, 200 + dim)
        rows = builder.encode_rows(x, nbrs, signs, device="cpu")
        # a few valid ids whose triple_x is FLT_MAX (inconsistent codebook quirk)
        rows[:4, L.factor_off + 1] = builder.FLT_MAX
        nq = 16
        qv = (np.rint(rng.uniform(0, 255, size=(nq, dim))) if integer else rng.standard_normal((nq, dim))).astype(np.float32)
        rot, lut, fac, sq = ref.query_prep(qv, signs, dim, L.padded_dim)
        pairs_q = rng.integers(0, nq, size=64)
        parents = rng.integers(0, n, size=64)
        parents[:4] = np.arange(4)
        pd = rng.uniform(0, 1e5 if integer else 2.0, size=64).astype(np.float32)
        l8, seq = ref.scan(rows, L, parents, pd, lut[pairs_q], fac[pairs_q], sq[pairs_q])
        out[f"sc_{tag}_rows"] = rows
        out[f"sc_{tag}_signs"] = signs
        out[f"sc_{tag}_queries"] = qv
        out[f"sc_{tag}_pairs_q"] = pairs_q
        out[f"sc_{tag}_parents"] = parents
        out[f"sc_{tag}_pdists"] = pd
        out[f"sc_{tag}_lanes8"] = l8
        out[f"sc_{tag}_seq"] = seq
        qi = rng.integers(0, nq, size=512)
        nodes = rng.integers(0, n, size=512)
        out[f"l2_{tag}_qidx"] = qi
        out[f"l2_{tag}_nodes"] = nodes
        out[f"l2_{tag}_l2"] = ref.l2(qv, rows, L.row, qi, nodes, False)
        out[f"l2_{tag}_ip"] = ref.l2(qv, rows, L.row, qi, nodes, True)

    # ---------------- beam merges (tie-heavy small-integer distances)
    for itopk in (32, 64, 128, 160, 200, 256, 384, 512, 1000, 1024):
        for cbs in (32, 16):
            for first in ((0, 1) if itopk <= 128 else (0,)):
                ncase = 96
                total = itopk + cbs
                idx = np.empty((ncase, total), dtype=np.uint32)
                dist = np.empty((ncase, total), dtype=np.float32)
                for c in range(ncase):
                    span = int(rng.choice([4, 16, 64, 100000]))
                    fill = int(rng.integers(1, itopk + 1))
                    b = np.sort(rng.integers(0, span, size=fill)).astype(np.float32)
                    bd = np.full(itopk, builder.FLT_MAX, dtype=np.float32)
                    bd[:fill] = b
                    bi = np.full(itopk, 0xFFFFFFFF, dtype=np.uint32)
                    bi[:fill] = rng.choice(1 << 20, size=fill, replace=False).astype(np.uint32)
                    bi[:fill] |= (rng.random(fill) < 0.5).astype(np.uint32) << np.uint32(31)
                    nc = int(rng.integers(0, cbs + 1))
                    cd = np.full(cbs, builder.FLT_MAX, dtype=np.float32)
                    ci = np.full(cbs, 0xFFFFFFFF, dtype=np.uint32)
                    pos = rng.choice(cbs, size=nc, replace=False)
                    cd[pos] = rng.integers(0, span + span // 4 + 1, size=nc).astype(np.float32)
                    ci[pos] = (1 << 21) + rng.choice(1 << 20, size=nc, replace=False).astype(np.uint32)
                    if first:
                        bd[:] = builder.FLT_MAX
                        bi[:] = 0xFFFFFFFF
                    idx[c, :itopk], dist[c, :itopk] = bi, bd
                    idx[c, itopk:], dist[c, itopk:] = ci, cd
                oi, od = ref.merge(idx, dist, itopk, cbs, bool(first))
                key = f"mg_{itopk}_{cbs}_{first}"
                out[key + "_idx_in"], out[key + "_dist_in"] = idx, dist
                out[key + "_idx_out"], out[key + "_dist_out"] = oi[:, :itopk], od[:, :itopk]

    # ---------------- controller rho update and keep counts
    n = 4096
    rho_prev = rng.uniform(0, 0.9, size=n).astype(np.float32)
    policy = rng.choice([0, 1, 5], size=n).astype(np.int32)
    rate = rng.uniform(0, 1, size=n).astype(np.float32)
    rate[:64] = 0.0
    rate[64:128] = 1.0
    # rates that land rho on keep-count rounding boundaries for degree 32 / 16
    k = rng.integers(1, 32, size=512)
    rate[128:640] = ((1.0 - k / 32.0 - 0.25) / 0.625).clip(0, 1).astype(np.float32)
    p2 = rng.choice(np.array([1 - 4 / 32, 1 - 4 / 16, 0.0], dtype=np.float32), size=n)
    active = rng.integers(1, 33, size=n).astype(np.uint32)
    cut = rng.integers(0, 2, size=n).astype(np.int32)
    near = rng.integers(0, 33, size=n).astype(np.uint32)
    ro, ko = ref.ctrl(rho_prev, policy, rate, p2, active, cut, near)
    out.update(ct_rho_prev=rho_prev, ct_policy=policy, ct_rate=rate, ct_p2rho=p2, ct_active=active, ct_cut=cut,
               ct_near=near, ct_rho_out=ro, ct_keep_out=ko)
    return out


def search_goldens(entry: str, manifest: dict, out_dir: str, device: str) -> None:
    t0 = time.time()
    name, _, metric = entry.partition(":")
    ip = metric == "ip"
    key = f"{name}_ip" if ip else name
    ds = builder.materialize(name, device=device)
    spec = ds.spec
    manifest[key] = dict(digest=ds.digest(), n=spec.n, dim=spec.dim, degree=spec.degree, K=spec.K,
                         beams=list(spec.beams), nq=spec.nq, entry=int(ds.entry), dataset=name,
                         metric="ip" if ip else "l2")
    g = ref.RefGraph(ds.codebook_path, spec.n, spec.dim, spec.degree, use_ip=ip)
    res = {}
    for beam in spec.beams:
        a, _ = g.search(ds.queries, spec.K, beam)
        b, _ = g.search(ds.queries, spec.K, beam)
        res[f"ids_{beam}"] = a
        res[f"ids2_{beam}"] = b
        diff = int((a != b).any(axis=1).sum())
        manifest[key][f"run_to_run_queries_differing_{beam}"] = diff
    g.close()
    np.savez_compressed(os.path.join(out_dir, f"ref_search_{key}.npz"), **res)
    print(f"[golden] {key}: {time.time() - t0:.1f}s", flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(ROOT, "golden_out"))
    ap.add_argument("--sets", default=",".join(SEARCH_SETS))
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--no-unit", action="store_true", help="skip the device-function goldens")
    ap.add_argument("--manifest-in", default="", help="existing manifest to add the new search sets to")
    args = ap.parse_args()
    os.makedirs(args.out, exist_ok=True)
    if not args.no_unit:
        rng = np.random.default_rng(20260101)
        t0 = time.time()
        unit = unit_goldens(rng)
        np.savez_compressed(os.path.join(args.out, "ref_unit.npz"), **unit)
        print(f"[golden] unit: {time.time() - t0:.1f}s", flush=True)
    manifest = {}
    if args.manifest_in:
        with open(args.manifest_in) as f:
            manifest = json.load(f)
    manifest["reference_internal_topk"] = int(ref.lib().ref_internal_topk())
    for name in [s for s in args.sets.split(",") if s]:
        search_goldens(name, manifest, args.out, args.device)
    with open(os.path.join(args.out, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
