"""FlashGANN-B200 benchmark: QPS at recall@100 >= 0.95 on the 1M x 128,
degree-32 seeded synthetic config.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flashgann|reference]
                    [--config NAME] [--scaling weak|strong] [--mode replicated|sharded]

One step = one search of a query batch at the smallest beam of the config's
beam list whose recall reaches 0.95 (the whole recall-vs-beam curve is
measured first, untimed, and printed).  The index is replicated on every GPU
and the queries are partitioned, with no collective on the data path:
--scaling weak (default) gives every rank a distinct batch of the config's
size (rank 0's is the config's own batch); --scaling strong splits the
config's one batch into N slices.  Rank 0 prints one JSON line.

--impl reference runs the reference's algorithm on the host cores (the C
oracle port with OpenMP; the reference itself has no CPU path) on a bounded
sample, and additionally times the reference's own sm_100a build
(oracle/_ref, QuantizationGraph::gpu_search_adaptive) on the same batch.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TARGET_RECALL = 0.95


def _dist():
    import torch
    import torch.distributed as dist
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=900))
    return ws, rank, local


def _barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    few milliseconds while the timed region runs (read-only queries), so that
    even a short region gets samples; nvidia-smi is the fallback."""

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.cuda_index = cuda_index
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._handle = None

    def _open(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.cuda_index)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            h = pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        return pynvml, h

    def _run(self):
        nv, h = self._nv, self._handle
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap,
                "hw_power_brake_slowdown": nv.nvmlClocksEventReasonHwPowerBrakeSlowdown}
        while True:
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for n, bit in bits.items():
                    if r & bit:
                        self.reasons.add(n)
            except Exception:
                break
            if self._stop.wait(self.period):
                break

    def __enter__(self):
        try:
            self._nv, self._handle = self._open()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml"}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def _traffic_per_query():
    """DRAM bytes per query from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "search_kernel_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return None


def _data_name(spec):
    kinds = {"int_gmm": f"{spec.n_comp}-component integer Gaussian mixture",
             "norm_aniso": f"{spec.n_comp}-component L2-normalised anisotropic mixture",
             "lowrank": "L2-normalised rank-64 latent x fixed map + noise"}
    return f"synthetic (seeded {kinds.get(spec.kind, spec.kind)}, config {spec.name})"


def _metric_name(spec, extra=""):
    n = spec.n
    ns = f"{n // 1_000_000}M" if n % 1_000_000 == 0 else (f"{n // 1000}K" if n % 1000 == 0 else str(n))
    return f"QPS @ recall@{spec.K}={TARGET_RECALL:.2f} ({ns} x {spec.dim}, deg {spec.degree}){extra}"


def _interpolate(table, beam, qps_at):
    """QPS at exactly the target recall, linear in recall between the last
    beam below the target and the calibrated beam (the metric's 'interpolate
    along the beam sweep'); None if the first beam already reaches it."""
    rs = dict(table)
    beams = [b for b, _ in table]
    if beam not in rs or beams.index(beam) == 0:
        return None
    b0 = beams[beams.index(beam) - 1]
    r0, r1 = rs[b0], rs[beam]
    if not (r0 < TARGET_RECALL <= r1):
        return None
    q0, q1 = qps_at(b0), qps_at(beam)
    w = (TARGET_RECALL - r0) / (r1 - r0)
    return {"recall": TARGET_RECALL, "qps": q0 + w * (q1 - q0), "beams": [b0, beam], "qps_at_beams": [q0, q1]}


def _calibrate(run, gt, K, beams, recall_fn):
    """The recall-vs-beam curve over every beam of the config's list, and the
    smallest beam whose recall reaches the target (the last beam if none
    does).  Every beam runs, so every rank makes the same calls (recall_fn
    may be a collective)."""
    table = [(beam, recall_fn(run(beam), gt, K)) for beam in beams]
    hit = [b for b, r in table if r >= TARGET_RECALL]
    beam = hit[0] if hit else beams[-1]
    return beam, dict(table)[beam], table


def cpu_baseline(ds, beam, budget_s=12.0, threads=0):
    """The oracle port (C, OpenMP over queries) on a bounded sample."""
    import oracle
    oi = oracle.OracleIndex(ds.rows, ds.signs, ds.entry, ds.spec.dim, ds.spec.degree)
    cores = threads or os.cpu_count() or 1
    probe = min(len(ds.queries), max(8, cores))
    t0 = time.perf_counter()
    oi.search(ds.queries[:probe], ds.spec.K, beam, threads=cores)
    dt = time.perf_counter() - t0
    n = int(min(len(ds.queries), max(probe, budget_s / max(dt, 1e-6) * probe)))
    t0 = time.perf_counter()
    ids, _ = oi.search(ds.queries[:n], ds.spec.K, beam, threads=cores)
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"first {n} of {len(ds.queries)} queries at beam {beam}, {dt:.1f} s on {cores} threads"}, ids


def _workload_config(spec, total_q, beam, ws, scaling):
    """The `config` object of both arms: the workload only (results go elsewhere)."""
    from flashgann_b200 import builder
    L = builder.layout(spec.dim, spec.degree)
    if scaling == "strong":
        par = f"queries partitioned: one {total_q}-query batch split over {ws} GPU(s), index replicated"
    else:
        par = f"queries partitioned: a distinct {total_q // ws}-query batch per GPU, index replicated x{ws}"
    return {"workload": spec.name, "n": spec.n, "dim": spec.dim, "degree": spec.degree, "K": spec.K,
            "queries_total": total_q, "beam": beam, "parallelism": par,
            "l2": "inputs larger than L2 (codebook %.2f GB > 126 MB)" % (spec.n * L.row * 4 / 1e9)}


def _sum_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def run_flashgann(args, ws, rank, local):
    """Replicated index, queries partitioned over the ranks.  weak: every
    rank searches a batch of its own (query set `rank` of the config, each
    spec.nq queries; rank 0's is the config's own batch), so per-GPU work is
    fixed as N grows; strong: the config's one batch is split into N
    contiguous slices.  Recall is over all ranks' queries."""
    import torch
    import flashgann_b200 as fg
    from flashgann_b200 import builder
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    # rank 0 materialises the dataset (cached under _data/); the others read it
    if rank == 0:
        ds = builder.materialize(args.config, device=dev, verbose=True)
    _barrier(ws)
    if rank != 0:
        ds = builder.materialize(args.config, device=dev)
    spec = ds.spec
    strong = args.scaling == "strong"
    if strong:
        queries, gt = ds.queries, ds.gt
        if args.queries:
            queries, gt = queries[:args.queries], gt[:args.queries]
        lo, hi = builder.shard_range(len(queries), ws, rank)
        queries, gt = queries[lo:hi], gt[lo:hi]
    else:
        queries, gt = builder.query_set(ds, rank, device=dev, verbose=True)
        if args.queries:
            queries, gt = queries[:args.queries], gt[:args.queries]
    K, nq = spec.K, len(queries)
    total_q = _sum_over_ranks(float(nq), ws)
    qg = fg.QuantizationGraph(spec.n, spec.dim, spec.degree, ds.codebook_path, device=local)
    dq = torch.from_numpy(np.ascontiguousarray(queries)).to(dev)
    dout = torch.empty((nq, K), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()

    def run_dev(beam):
        qg.search_device(dq, K, beam, d_out=dout, stream=stream)
        torch.cuda.synchronize()
        return dout.cpu().numpy().view(np.uint32)

    def recall_all(ids, g, k):
        # hits over every rank's queries
        return _sum_over_ranks(fg.compute_recall(ids, g, k) * len(ids) * k, ws) / (total_q * k)

    if args.beam:
        beam, table = args.beam, []
        recall = recall_all(run_dev(beam), gt, K)
    else:
        beam, recall, table = _calibrate(run_dev, gt, K, spec.beams, recall_all)
    # counters of one pass (traversal is deterministic) for the roofline
    dstats = torch.zeros((nq, 4), dtype=torch.int32, device=dev)
    qg.search_device(dq, K, beam, d_out=dout, stream=stream, d_stats=dstats)
    torch.cuda.synchronize()
    st = dstats.cpu().numpy().astype(np.int64)
    evals, expans = int(st[:, 2].sum()), int(st[:, 1].sum())
    L = builder.layout(spec.dim, spec.degree)
    graded_bytes = evals * (spec.dim * 4 + spec.degree * L.padded_dim // 8 + spec.degree * 4)
    refined_bytes = evals * spec.dim * 4 + expans * spec.degree * (L.padded_dim // 8 + 4 + 12)

    # Steps alternate between two streams (each with its own output buffer
    # and work counter), so a step's first wave fills the SMs the previous
    # step's last wave leaves idle; the events bracket all of them on the
    # launching stream.  The planner aims for throughput (batches in flight
    # on two streams); results do not depend on the kernel it picks.
    qg.set_plan_goal("throughput")
    plan = dict(zip(("kernel", "resident_queries"), qg.search_plan(nq, K, beam)))
    side = [torch.cuda.Stream() for _ in range(2)]
    douts = [dout, torch.empty_like(dout)]

    def timed_steps(n, b):
        """Device ms per step of n steps at beam b."""
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for st_ in side:
            st_.wait_stream(stream)
        for i in range(n):
            qg.search_device(dq, K, b, d_out=douts[i % 2], stream=side[i % 2])
        for st_ in side:
            stream.wait_stream(st_)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    timed_steps(args.warmup, beam)
    _barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms = timed_steps(args.steps, beam)
    _barrier(ws)
    torch.cuda.synchronize()
    ms_max = _max_over_ranks(ms, ws)
    clocks = clk.summary()
    steps_ok = bool(torch.equal(douts[0], douts[1])) if args.steps > 1 else None

    def qps_at(b):
        if b == beam:
            return total_q / (ms_max / 1e3)
        timed_steps(2, b)
        _barrier(ws)
        return total_q / (_max_over_ranks(timed_steps(4, b), ws) / 1e3)

    interp = _interpolate(table, beam, qps_at)

    # end to end through the public host-buffer API: every step uploads its
    # queries from pinned host memory and downloads its ids into pinned host
    # memory.  Streamed (fg_search_async over two slots and streams: one
    # step's copies overlap the previous step's search) and, for comparison,
    # synchronous (fg_search, the reference's call shape).
    hq = torch.from_numpy(np.ascontiguousarray(queries)).pin_memory().numpy()
    hres = [torch.empty((nq, K), dtype=torch.int32).pin_memory().numpy().view(np.uint32) for _ in range(2)]
    streams = [torch.cuda.Stream() for _ in range(2)]

    def streamed(n):
        for i in range(n):
            sl = i % 2
            streams[sl].synchronize()
            qg.search_async(sl, nq, hq, K, hres[sl], beam, streams[sl])
        for st_ in streams:
            st_.synchronize()

    def synchronous(n):
        # one call at a time, as the reference is called: the latency plan
        qg.set_plan_goal("latency")
        for _ in range(n):
            qg.gpu_search_adaptive(nq, hq, K, hres[0], beam)
        qg.set_plan_goal("throughput")

    e2e = {}
    for name, fn in (("streamed", streamed), ("synchronous", synchronous)):
        fn(max(2, args.warmup // 2))
        _barrier(ws)
        t0 = time.perf_counter()
        fn(args.steps)
        e2e[name] = _max_over_ranks((time.perf_counter() - t0) / args.steps, ws)
    e2e_ok = bool(np.array_equal(hres[0], hres[1]))
    qg.set_plan_goal("latency")
    sync_plan = dict(zip(("kernel", "resident_queries"), qg.search_plan(nq, K, beam)))
    qg.close()

    value = total_q / (ms_max / 1e3)
    peak, peak_kind = _peaks()
    achieved = graded_bytes / (ms / 1e3) / 1e9
    traffic = _traffic_per_query()
    if traffic and not str(traffic.get("workload", "")).startswith(spec.name + " "):
        traffic = None  # the committed capture is of another workload
    out = {
        "metric": _metric_name(spec),
        "value": value, "unit": "queries/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max, "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f32", "data": _data_name(spec),
        "config": _workload_config(spec, int(total_q), beam, ws, args.scaling),
        "recall": {"at_beam": recall, "curve": table, "qps_interpolated_to_target_recall": interp},
        "e2e": {"value": total_q / e2e["streamed"], "unit": "queries/s",
                "h2d_bytes_per_step": nq * spec.dim * 4, "d2h_bytes_per_step": nq * K * 4,
                "api": "fg_search_async, two slots and streams, pinned host buffers",
                "synchronous_value": total_q / e2e["synchronous"], "synchronous_api": "fg_search",
                "results_match": e2e_ok},
        "gpu_launches": args.steps,
        "timing": "device events around all steps; steps alternate between two streams (consecutive "
                  "steps overlap); outputs of both streams identical: %s" % steps_ok,
        "plan": {"steps_and_streamed_e2e": dict(plan, goal="throughput"),
                 "synchronous_e2e": dict(sync_plan, goal="latency")},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": (traffic["dram_bytes_per_query"] * nq if traffic else None),
                     "algorithmic_bytes_per_step": graded_bytes, "refined_bytes_per_step": refined_bytes,
                     "visited_per_query": evals / nq, "expanded_per_query": expans / nq},
        "clocks": clocks,
    }
    if rank == 0 and not args.no_cpu:
        out["cpu_baseline"], _ = cpu_baseline(ds, beam, budget_s=args.cpu_seconds)
    return out


def run_sharded(args, ws, rank, local):
    """The index split into one shard per rank, each with its own graph
    (BASELINE.json configs[4] at the config's scale): every rank searches the
    whole query batch on its shard, the per-shard top-K lists are all-gathered
    over NCCL and merged on the device.  One step = search + all-gather +
    merge of the batch; value = queries answered per second by the job."""
    import torch
    import flashgann_b200 as fg
    from flashgann_b200 import builder
    from flashgann_b200 import distributed as fgd
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    spec0 = builder.SPECS[args.config]
    build_s = None
    if spec0.block:
        # a blocked spec: every rank draws and builds its own
        # shard on its own GPU; the global ground truth is the merge of every
        # shard's exact lists
        import torch.distributed as dist
        t0 = time.perf_counter()
        sh = builder.materialize_shard_device(args.config, rank, ws, device=dev, verbose=(rank == 0))
        qg = fg.QuantizationGraph.from_device(sh.rows, torch.from_numpy(sh.signs).to(dev), sh.entry, spec0.dim,
                                              spec0.degree)
        sh.rows = None
        torch.cuda.empty_cache()
        gi = torch.from_numpy(sh.gt_ids).to(dev)
        gd = torch.from_numpy(sh.gt_d).to(dev)
        if ws > 1:
            all_i = [torch.empty_like(gi) for _ in range(ws)]
            all_d = [torch.empty_like(gd) for _ in range(ws)]
            dist.all_gather(all_i, gi)
            dist.all_gather(all_d, gd)
        else:
            all_i, all_d = [gi], [gd]
        gt = builder.merge_shard_ground_truth(np.stack([t.cpu().numpy() for t in all_i]),
                                              np.stack([t.cpu().numpy() for t in all_d]), spec0.gt_k)
        build_s = _max_over_ranks(time.perf_counter() - t0, ws)
        queries = sh.queries
    else:
        if rank == 0:
            builder.materialize(args.config, device=dev, verbose=True)
        _barrier(ws)
        sh = builder.materialize_shard(args.config, rank, ws, device=dev, verbose=(rank == 0))
        qg = fg.QuantizationGraph(sh.n, spec0.dim, spec0.degree, sh.codebook_path, device=local)
        queries, gt = sh.queries, sh.gt
    _barrier(ws)
    spec = sh.spec
    K = spec.K
    if args.queries:
        queries, gt = queries[:args.queries], gt[:args.queries]
    nq = len(queries)
    dq = torch.from_numpy(queries).to(dev)
    dout = torch.empty((nq, K), dtype=torch.int32, device=dev)
    dd = torch.empty((nq, K), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    offsets = [builder.shard_range(spec.n, ws, r)[0] for r in range(ws)]
    assert offsets[rank] == sh.offset

    def step(beam, q=dq):
        qg.search_device(q, K, beam, d_out=dout, d_dists=dd, stream=stream)
        return fgd.gather_shard_topk(dout, dd, K, offsets)

    def run(beam):
        ids, _ = step(beam)
        torch.cuda.synchronize()
        return ids.cpu().numpy().view(np.uint32)

    if args.beam:
        beam, table = args.beam, []
        recall = fg.compute_recall(run(beam), gt, K)
    else:
        beam, recall, table = _calibrate(run, gt, K, spec.beams, fg.compute_recall)
    for _ in range(args.warmup):
        step(beam)
    torch.cuda.synchronize()
    _barrier(ws)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step(beam)
        ev1.record(stream)
        torch.cuda.synchronize()
    _barrier(ws)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = _max_over_ranks(ms, ws)
    # the search alone (no all-gather, no merge), for the collective's share of a step
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        qg.search_device(dq, K, beam, d_out=dout, d_dists=dd, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    search_ms = _max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)
    _barrier(ws)
    # end to end: pinned host queries in, merged ids out, every step
    hq = torch.from_numpy(queries).pin_memory()
    hres = torch.empty((nq, K), dtype=torch.int32).pin_memory()
    _barrier(ws)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dq.copy_(hq, non_blocking=True)
        ids, _ = step(beam)
        hres.copy_(ids, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = _max_over_ranks((time.perf_counter() - t0) / args.steps, ws)
    qg.close()
    return {
        "metric": _metric_name(spec, ", index sharded over the GPUs"),
        "value": nq / (ms_max / 1e3), "unit": "queries/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": _data_name(spec),
        "config": {"workload": f"{spec.name} in {ws} shards", "n": spec.n, "shard_nodes": sh.n, "dim": spec.dim,
                   "degree": spec.degree, "K": K, "queries_total": nq, "beam": beam,
                   "parallelism": f"index sharded x{ws} (per-shard graphs), all-gather of per-shard top-{K} + "
                                  "merge kernel (fg_shard_merge_device)",
                   "l2": "inputs larger than L2 (shard codebook %.2f GB > 126 MB)" % (sh.n * sh.layout.row * 4 / 1e9)},
        "recall": {"at_beam": recall, "curve": table},
        "shard_build_s": build_s,
        "step_breakdown_ms": {"search": search_ms, "all_gather_and_merge": ms_max - search_ms,
                              "all_gather_bytes_per_rank": nq * K * 8},
        "e2e": {"value": nq / e2e_s, "unit": "queries/s", "h2d_bytes_per_step": nq * spec.dim * 4,
                "d2h_bytes_per_step": nq * K * 4},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }


def run_reference(args, ws, rank, local):
    """The reference arm.  Its value is the reference's algorithm on the host
    cores (the reference itself has no CPU path, so the C oracle port with
    OpenMP) on a bounded sample; beside it, key reference_gpu, the
    reference's own sm_100a build (oracle/_ref, QuantizationGraph::
    gpu_search_adaptive, index upload excluded as the reference times it) on
    the same batch, with its recall-vs-beam curve.  Recall is scored by the
    oracle, so this arm loads no library of this build."""
    import oracle
    from flashgann_b200 import builder
    if rank != 0:
        return None
    import torch
    dev = f"cuda:{local}" if torch.cuda.is_available() else "cpu"
    ds = builder.materialize(args.config, device=dev, verbose=True)
    spec = ds.spec
    K, nq = spec.K, len(ds.queries)
    extra = {}
    beam = args.beam
    try:
        from oracle import ref
        if ref.available() and torch.cuda.is_available():
            g = ref.RefGraph(ds.codebook_path, spec.n, spec.dim, spec.degree)
            ref_table = []
            if not beam:
                beam, _, ref_table = _calibrate(lambda b: g.search(ds.queries, K, b)[0], ds.gt, K, spec.beams,
                                                oracle.compute_recall)
            ids, _ = g.search(ds.queries, K, beam)
            times = []
            for _ in range(max(1, args.steps)):
                t0 = time.perf_counter()
                ids, el = g.search(ds.queries, K, beam)
                times.append((el, time.perf_counter() - t0))
            el = statistics.median(t[0] for t in times)
            call = statistics.median(t[1] for t in times)

            def ref_qps(b):
                if b == beam:
                    return nq / el
                return nq / statistics.median(g.search(ds.queries, K, b)[1] for _ in range(3))

            ref_interp = _interpolate(ref_table, beam, ref_qps) if ref_table else None
            g.close()
            extra["reference_gpu"] = {
                "what": "reference sm_100a build, QuantizationGraph::gpu_search_adaptive, 1 GPU",
                "value": nq / el, "unit": "queries/s", "beam": beam,
                "recall_at_k": oracle.compute_recall(ids, ds.gt, K), "recall_table": ref_table,
                "elapsed_s": el, "call_s_including_index_upload": call,
                "qps_interpolated_to_target_recall": ref_interp}
    except Exception as e:  # the CPU leg below is the contract's reference arm
        extra["reference_gpu"] = {"unavailable": f"{type(e).__name__}: {e}"}
    if not beam:
        beam = spec.beams[-1]
    steps = []
    for _ in range(max(1, args.steps)):
        cb, _ = cpu_baseline(ds, beam, budget_s=args.cpu_seconds / max(1, args.steps))
        steps.append(cb)
    value = statistics.median(s["value"] for s in steps)
    cb = dict(steps[0])
    cb["value"] = value
    out = {
        "impl": "reference", "metric": _metric_name(spec), "value": value,
        "unit": "queries/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "data": _data_name(spec),
        "config": _workload_config(spec, nq, beam, 1, args.scaling),
        "cpu_baseline": cb, "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0,
                                    "d2h_bytes_per_step": 0},
    }
    out.update(extra)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="flashgann", choices=["flashgann", "reference"])
    ap.add_argument("--config", default="c2_1m")
    ap.add_argument("--beam", type=int, default=0, help="fixed beam (default: calibrate to recall 0.95)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--mode", default="replicated", choices=["replicated", "sharded"],
                    help="replicated: index on every GPU, queries partitioned (default); "
                         "sharded: one index shard per GPU, top-K gathered and merged")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="replicated mode over N GPUs: weak = a distinct batch per GPU (default), "
                         "strong = the config's one batch split over the GPUs")
    ap.add_argument("--queries", type=int, default=0,
                    help="search only the first N queries of the batch (small cases for profiler captures)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    ws, rank, local = _dist()
    if args.impl == "reference":
        out = run_reference(args, ws, rank, local)
    elif args.mode == "sharded":
        out = run_sharded(args, ws, rank, local)
    else:
        out = run_flashgann(args, ws, rank, local)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
