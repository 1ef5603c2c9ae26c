#!/usr/bin/env python
"""Benchmark of the hot path. Default: exact FlatIndex cosine search, 10,000-query batches, k=10.

Workload: 1,183,514 x 100 float32 vectors from a 1,000-component Gaussian mixture,
L2-normalized; 10,000 queries drawn the same way (seeded synthetic data standing in for
GloVe-1.2M). On N GPUs (one process per GPU) every GPU holds the whole database (0.74 GB) and
answers its 1/N slice of every query batch, with no exchange (``--shard queries``, the default);
``--shard rows`` instead splits the database by id range, gives every GPU the whole batch and
merges the per-GPU top-k with one NCCL all-gather plus a device k-way merge. A step is one search
of the whole 10k batch. Total work is fixed, so N>1 is strong scaling.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c2|c3] [--nprobe P] [--filter] [--shard queries|rows]

``--workload c2`` / ``c3`` measure IVF-PQ search instead (L2 nlist 2048 m 32 over 1M skewed-int
rows; cosine nlist 2048 m 25 refine 8 over the 1.18M mixture rows): the trained,
empty index the reference saved (tests/golden/ivf_c{2,3}_trained.qvr) is loaded on every GPU,
each rank adds its id range of the database on its GPU, and a step is one search of the 10k
batch at ``--nprobe`` (c3: refine_factor 8; ``--filter``: a seeded random 1 % allowed-id set).

Rank 0 prints one JSON line. ``value`` is whole-job QPS with queries already on the GPUs;
``e2e`` is the same metric through the public Python API with the queries in pinned host memory
and the results copied back every step. ``--impl reference`` times the reference library's own
CPU FlatIndex::search_batch (compiled from the reference sources into oracle/_ref) on the host
cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "QPS (10k-query batch, k=10) at 1/2/4/8 B200; % of HBM/tensor roofline"
WORKLOAD = "FlatIndex cosine k=10, 1,183,514 x 100 Gaussian-mixture rows, 10,000 queries"
N_DB, N_Q, DIM, K = 1_183_514, 10_000, 100, 10


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=N_DB,
                    help="database rows (default: the workload's 1,183,514; smaller for "
                         "profiling)")
    ap.add_argument("--queries", type=int, default=N_Q, help="queries per batch (default 10,000)")
    ap.add_argument("--workload", choices=["c1", "c2", "c3", "c4"], default="c1")
    ap.add_argument("--nprobe", type=int, default=64, help="IVF-PQ workloads: lists probed")
    ap.add_argument("--filter", action="store_true", help="IVF-PQ workloads: 1%% allowed ids")
    ap.add_argument("--shard", choices=["rows", "queries"], default="queries",
                    help="Flat on N GPUs: id-range row shards + all-gather merge, or the rows "
                         "replicated and each batch's queries split by rank (no exchange)")
    return ap.parse_args()


IVF_WORKLOADS = {
    # name: (trained file, metric, dim, refine_factor, rows, description)
    "c2": ("ivf_c2_trained.qvr", "l2", 128, 0, 1_000_000,
           "IvfPqIndex L2 nlist 2048 m 32, 1,000,000 x 128 skewed-int rows, 10,000 queries"),
    "c3": ("ivf_c3_trained.qvr", "cosine", 100, 8, 1_183_514,
           "IvfPqIndex cosine nlist 2048 m 25 refine 8, 1,183,514 x 100 Gaussian-mixture rows, "
           "10,000 queries"),
}


def ivf_data(workload: str):
    from quiver_b200.synthetic import config2, config3
    return config2() if workload == "c2" else config3()


def ivf_allowed(n: int) -> np.ndarray:
    """The filtered run's allowed ids: a seeded random 1 % of [0, n)."""
    rng = np.random.default_rng(7)
    return np.sort(rng.choice(n, n // 100, replace=False)).astype(np.uint64)


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            p = json.load(fh)
        return p.get("hbm_gbs", 6650.0), p.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed region.

    Reads NVML every few milliseconds from a thread (the timed region can be well under a second),
    on the NVML device matched to the CUDA device by PCI bus id; falls back to `nvidia-smi -lms`.
    Reading only: no clock or other GPU setting is changed."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, cuda_device: int):
        self.cuda_device = cuda_device
        self.sm, self.smax, self.reasons = [], [], set()
        self.stop_evt = threading.Event()
        self.thread = None
        self.proc = None
        self.source = "none"

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.cuda_device)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def start(self):
        try:
            nv, h = self._nvml_handle()
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            masks = [(name, getattr(nv, attr)) for name, attr in self.REASONS]

            def poll():
                while not self.stop_evt.is_set():
                    try:
                        self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                        self.smax.append(float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)))
                        bits = get_reasons(h)
                        self.reasons.update(n for n, m in masks if bits & m)
                    except Exception:  # noqa: BLE001 - a failed read only loses one sample
                        pass
                    self.stop_evt.wait(0.005)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            self.source = "nvml"
        except Exception:  # noqa: BLE001 - NVML missing or device not matched
            self._start_smi()

    def _start_smi(self):
        fields = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.cuda_device), f"--query-gpu={fields}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi"
        except (OSError, ValueError):
            self.proc = None
            return

        def read():
            for line in self.proc.stdout:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    self.sm.append(float(parts[1]))
                    self.smax.append(float(parts[2]))
                except ValueError:
                    continue
                for (n, _), v in zip(self.REASONS, parts[5:9]):
                    if v.lower() == "active":
                        self.reasons.add(n)

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def stop(self):
        self.stop_evt.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock samples"],
                    "samples": 0, "source": self.source}
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": max(self.smax),
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": self.source}


def flat_config(args) -> dict:
    """The Flat workload's description (identical in both arms' JSON lines)."""
    n_db, n_q = args.rows, args.queries
    full = (n_db, n_q) == (N_DB, N_Q)
    return {"workload": WORKLOAD if full else
            f"FlatIndex cosine k=10, {n_db:,} x 100 Gaussian-mixture rows (reduced), "
            f"{n_q:,} queries",
            "global_batch": n_q, "k": K, "database_rows": n_db, "dim": DIM, "metric": "cosine",
            "l2": "inputs larger than L2 (473 MB database read per pass)"}


def ivf_config(args) -> dict:
    """The IVF-PQ workload's description (identical in both arms' JSON lines)."""
    fname, metric, dim, refine, rows, desc = IVF_WORKLOADS[args.workload]
    return {"workload": desc, "nprobe": args.nprobe, "refine_factor": refine,
            "filter": "1% ids" if args.filter else None, "global_batch": min(args.queries, N_Q),
            "k": K, "database_rows": rows, "dim": dim, "metric": metric,
            "l2": "codes (32 MB / 30 MB) are L2-resident; no flush between steps"}


def cpu_reference_qps(db, queries, seconds: float, threads: int = 0):
    """Times the reference's own FlatIndex::search_batch (oracle/_ref) on host cores for about
    `seconds`. Returns (qps, cores, sample description, kind) or None if unavailable."""
    from oracle.oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        return None
    try:
        ref = Reference()
    except OSError:
        return None
    f = ref.flat(DIM, "cosine")
    f.add(db)
    cores = threads or ref.threads
    f.search(queries[:32], K, threads=threads)  # warm-up
    t0 = time.perf_counter()
    f.search(queries[:64], K, threads=threads)
    per_q = (time.perf_counter() - t0) / 64
    n = int(min(len(queries), max(64, seconds / max(per_q, 1e-9))))
    t0 = time.perf_counter()
    f.search(queries[:n], K, threads=threads)
    dt = time.perf_counter() - t0
    sample = (f"{n} of the {len(queries)} queries against the full {len(db):,}-row database, "
              f"FlatIndex::search_batch with {cores} threads, ISA {ref.isa}")
    return n / dt, cores, sample, "reference"


def cpu_port_qps(db, queries, seconds: float):
    from oracle.oracle import Oracle
    o = Oracle()
    stored = db  # already normalized by the generator; the oracle scans the stored rows as-is
    labels = np.arange(len(db), dtype=np.uint64)
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < seconds and n < len(queries):
        o.flat_search(stored, labels, "cosine", queries[n:n + 1], K)
        n += 1
    dt = time.perf_counter() - t0
    return n / dt, 1, f"{n} queries, single-threaded C restatement (oracle/qv_oracle.c)", "port"


def ref_ivf_index(ref, workload: str, db):
    """The reference's own IvfPqIndex: its trained file plus the database added on the CPU."""
    ix = ref.ivf_load(os.path.join(ROOT, "tests", "golden", IVF_WORKLOADS[workload][0]))
    ix.add(db)
    return ix


def cpu_reference_ivf_qps(ref, ix, queries, nprobe, refine, allowed, seconds: float):
    ix.search(queries[:64], K, nprobe, refine, allowed)  # warm-up
    t0 = time.perf_counter()
    ix.search(queries[:256], K, nprobe, refine, allowed)
    per_q = (time.perf_counter() - t0) / 256
    n = int(min(len(queries), max(256, seconds / max(per_q, 1e-9))))
    t0 = time.perf_counter()
    ix.search(queries[:n], K, nprobe, refine, allowed)
    return n / (time.perf_counter() - t0), n


REF_STEP_SECONDS = 3.0  # CPU time of one reference step: a bounded sample of the batch


def run_reference_arm(args, rank, world):
    """The reference's own CPU search (oracle/_ref, compiled from the reference sources) on the
    host cores, same workload and metric. Each step searches a bounded sample of the batch
    (about REF_STEP_SECONDS of CPU) against the whole database; the line reports the sample size
    and the measured time per step."""
    if rank != 0:
        return
    from oracle.oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        print(json.dumps({"impl": "reference",
                          "unavailable": "reference library oracle/_ref was not built"}))
        return
    try:
        ref = Reference()
    except OSError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"oracle/_ref not loadable: {e}"}))
        return
    scale = 1.0  # the reference scans a row sample; QPS scales linearly to the whole collection
    if args.workload == "c1":
        from quiver_b200.synthetic import config1
        db, q = config1(args.rows, args.queries)
        config = flat_config(args)
        f = ref.flat(DIM, "cosine")
        f.add(db)
        search = lambda qs: f.search(qs, K)  # noqa: E731
        what = "FlatIndex::search_batch"
    elif args.workload == "c4":
        from quiver_b200.synthetic import C4_ROWS, config4_chunk
        rows = C4_ROWS if args.rows == N_DB else args.rows
        sample_rows = min(200_000, rows)
        db = config4_chunk(sample_rows, 0)
        q = config4_chunk(4096, 63)
        config = c4_config(args, rows)
        f = ref.flat(768, "ip")
        f.add(db)
        search = lambda qs: f.search(qs, C4_K)  # noqa: E731
        scale = sample_rows / rows
        what = (f"FlatIndex::search_batch over a {sample_rows:,}-row sample of the {rows:,} rows, "
                f"QPS scaled by the row ratio")
    else:
        db, q = ivf_data(args.workload)
        q = q[:args.queries]
        config = ivf_config(args)
        ix = ref_ivf_index(ref, args.workload, db)
        allowed = ivf_allowed(len(db)) if args.filter else None
        refine = IVF_WORKLOADS[args.workload][3]
        search = lambda qs: ix.search(qs, K, args.nprobe, refine, allowed)  # noqa: E731
        what = (f"IvfPqIndex::search_batch nprobe {args.nprobe} refine {refine}"
                f"{' filtered 1%' if args.filter else ''}")
    n_q = len(q)
    t0 = time.perf_counter()
    search(q[:64])
    per_q = (time.perf_counter() - t0) / 64
    per_step = int(min(n_q, max(64, REF_STEP_SECONDS / max(per_q, 1e-9))))
    for _ in range(args.warmup):
        search(q[:per_step])
    times = []
    for i in range(args.steps):
        lo = (i * per_step) % max(1, n_q - per_step + 1)
        t0 = time.perf_counter()
        search(q[lo:lo + per_step])
        times.append(time.perf_counter() - t0)
    step_s = statistics.mean(times)
    qps = per_step / step_s * scale
    sample = (f"{per_step} of the {n_q:,} queries per step against the full {len(db):,}-row "
              f"database, {what}, {ref.threads} threads, ISA {ref.isa}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "QPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * step_s, "queries_per_step": per_step,
        "rows_per_step": len(db), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config, "parallelism": f"{ref.threads} host threads (reference thread pool)",
        "cpu_baseline": {"value": qps, "unit": "QPS", "cores": ref.threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": qps, "unit": "QPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


C4_Q, C4_K = 16_384, 100
C4_DESC = ("FlatIndex inner product k=100, 40,000,000 x 768 Gaussian-mixture rows "
           "(4,096 components), 16,384-query batches")


def c4_config(args, rows) -> dict:
    return {"workload": C4_DESC if rows == 40_000_000 else
            f"FlatIndex inner product k=100, {rows:,} x 768 Gaussian-mixture rows (reduced), "
            f"{C4_Q:,}-query batches",
            "global_batch": C4_Q, "k": C4_K, "database_rows": rows, "dim": 768, "metric": "ip",
            "l2": "inputs larger than L2 (the fp16 rows of a shard are read once per pass)"}


def run_c4(args, rank, world, local):
    """The 40M x 768 inner-product collection, id-range sharded (rank r holds rows
    [r*N/W, (r+1)*N/W), generated on its GPU), every rank searching the whole 16,384-query batch
    with the tensor-core screen, one packed NCCL all-gather and a device merge per step."""
    import torch
    import torch.distributed as dist
    import quiver_b200 as qv
    from quiver_b200 import _native
    from quiver_b200.distributed import ShardedFlatIndex, shard_range
    from quiver_b200.synthetic import C4_ROWS, config4_device

    rows = C4_ROWS if args.rows == N_DB else args.rows
    lo, hi = shard_range(rows, rank, world)
    dev = torch.device(f"cuda:{local}")
    index = ShardedFlatIndex(768, "ip", device=local)
    index.local.reserve(hi - lo)
    for first, x in config4_device(lo, hi, dev):
        index.add_range_device(x, first)
        del x
    q = next(config4_device(0, C4_Q, dev, queries=True))[1]
    torch.cuda.empty_cache()
    q_host = q.cpu().pin_memory().numpy()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        index.search_device(q, C4_K)
    torch.cuda.synchronize()
    _native.set_timing(True)
    qv.last_search_stats()
    sampler = ClockSampler(local)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        index.search_device(q, C4_K)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    st = qv.last_search_stats()
    _native.set_timing(False)
    elapsed = e0.elapsed_time(e1)
    launches, rescans = st["kernel_launches"], st["rescanned_queries"]
    if world > 1:
        t = torch.tensor([elapsed], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
        c = torch.tensor([launches, rescans], device=dev, dtype=torch.float64)
        dist.all_reduce(c, op=dist.ReduceOp.SUM)
        launches, rescans = int(c[0].item()), int(c[1].item())
    value = C4_Q * args.steps / (elapsed / 1000.0)

    for _ in range(max(1, args.warmup)):
        index.search(q_host, C4_K)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        index.search(q_host, C4_K)
    e2e_s = time.perf_counter() - t0
    barrier()
    if world > 1:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    hbm, tflops, peak_kind = load_peaks()
    avg_ms = st["dominant_kernel_ms"] / max(1, args.steps)
    work = st["dominant_kernel_work"] / max(1, args.steps)
    achieved = work / (avg_ms / 1000.0) / 1e12 if avg_ms else 0.0
    line = {
        "metric": METRIC, "value": value, "unit": "QPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": c4_config(args, rows), "parallelism": f"id-range shards x{world}",
        "gpu_launches": launches, "rescanned_queries": rescans,
        "roofline": {"bound": "tensor", "kernel": st["dominant_kernel"], "achieved": achieved,
                     "peak": tflops, "unit": "TFLOP/s", "frac": achieved / tflops,
                     "peak_source": f"{peak_kind} bf16 dense (burst)", "traffic": None,
                     "avg_launch_ms": avg_ms, "work_per_launch": work},
        "clocks": clocks,
        "e2e": {"value": C4_Q * args.steps / e2e_s, "unit": "QPS",
                "h2d_bytes_per_step": world * C4_Q * 768 * 4,
                "d2h_bytes_per_step": world * C4_Q * C4_K * (8 + 4)},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # The reference on a bounded sample: 64 queries against the first 1,000,000 rows, scaled
        # linearly to the whole collection (its scan is linear in rows).
        from oracle.oracle import REF_SO, Reference
        if os.path.exists(REF_SO):
            ref = Reference()
            sample_rows = min(1_000_000, hi - lo)
            x0 = index.local.rows(0, sample_rows)[0]  # rank 0's first rows, copied out
            f = ref.flat(768, "ip")
            f.add(x0)
            f.search(q_host[:8], C4_K)
            t0 = time.perf_counter()
            f.search(q_host[:64], C4_K)
            dt = time.perf_counter() - t0
            line["cpu_baseline"] = {
                "value": 64 / dt * sample_rows / rows, "unit": "QPS", "cores": ref.threads,
                "kind": "reference",
                "sample": f"64 queries against the first {sample_rows:,} rows with "
                          f"FlatIndex::search_batch ({ref.threads} threads, ISA {ref.isa}), "
                          f"scaled by {sample_rows:,} / {rows:,} rows"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_ivf(args, rank, world, local):
    """IVF-PQ workloads (configs 2 and 3): value, e2e, roofline (HBM) and CPU baseline."""
    import torch
    import torch.distributed as dist
    import quiver_b200 as qv
    from quiver_b200 import _native
    from quiver_b200.distributed import ShardedIvfPqIndex

    fname, metric, dim, refine, rows, desc = IVF_WORKLOADS[args.workload]
    db, q = ivf_data(args.workload)
    q = q[:args.queries]
    nq = len(q)
    n = len(db)
    lo, hi = rank * n // world, (rank + 1) * n // world
    index = ShardedIvfPqIndex.from_trained(os.path.join(ROOT, "tests", "golden", fname),
                                           db[lo:hi], np.arange(lo, hi, dtype=np.uint64),
                                           total=n, device=local)
    allowed = ivf_allowed(n) if args.filter else None
    bitmap = index.filter_bitmap(allowed)
    dq = torch.from_numpy(q).cuda()
    q_host = torch.from_numpy(q).pin_memory().numpy()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        index.search_device(dq, K, args.nprobe, refine, bitmap)
    torch.cuda.synchronize()
    _native.set_timing(True)
    sampler = ClockSampler(local)
    sampler.start()
    qv.last_search_stats()  # start the accumulation here
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        index.search_device(dq, K, args.nprobe, refine, bitmap)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    # With timing on, the library recorded CUDA events around each step's scan on its stream and
    # counted launches; reading the stats resolves them (after the timed region).
    st = qv.last_search_stats()
    launches, kernel_ms, kernel_bytes = (st["kernel_launches"], st["dominant_kernel_ms"],
                                         st["dominant_kernel_work"])
    _native.set_timing(False)
    elapsed = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([elapsed], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
        c = torch.tensor([launches], device="cuda", dtype=torch.float64)
        dist.all_reduce(c, op=dist.ReduceOp.SUM)
        launches = int(c[0].item())
    value = nq * args.steps / (elapsed / 1000.0)

    def e2e_call():
        if world == 1:
            return index.local.search(q_host, K, args.nprobe, refine, filter=allowed)
        return index.search(q_host, K, args.nprobe, refine, filter=allowed)

    for _ in range(max(1, args.warmup)):
        e2e_call()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_call()
    e2e_s = time.perf_counter() - t0
    barrier()
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    hbm, _, peak_kind = load_peaks()
    avg_ms = kernel_ms / max(1, args.steps)
    per_launch = kernel_bytes / max(1, args.steps)
    achieved = per_launch / (avg_ms / 1000.0) / 1e9 if avg_ms else 0.0
    line = {
        "metric": METRIC, "value": value, "unit": "QPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": ivf_config(args), "parallelism": f"id-range shards x{world}",
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "ivf_scan_kernel", "achieved": achieved,
                     "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": f"{peak_kind} HBM copy", "traffic": None,
                     "avg_launch_ms": avg_ms, "work_per_launch": per_launch},
        "clocks": clocks,
        "e2e": {"value": nq * args.steps / e2e_s, "unit": "QPS",
                "h2d_bytes_per_step": world * nq * dim * 4,
                "d2h_bytes_per_step": world * nq * K * (8 + 4)},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.oracle import REF_SO, Reference
        if os.path.exists(REF_SO):
            ref = Reference()
            ix = ref_ivf_index(ref, args.workload, db)
            qps, nsamp = cpu_reference_ivf_qps(ref, ix, q, args.nprobe, refine, allowed, 15.0)
            line["cpu_baseline"] = {
                "value": qps, "unit": "QPS", "cores": ref.threads, "kind": "reference",
                "sample": f"{nsamp} of the {nq} queries, IvfPqIndex::search_batch, "
                          f"{ref.threads} threads, ISA {ref.isa}"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank, world, local = env_rank()
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    if args.workload == "c4":
        run_c4(args, rank, world, local)
        if world > 1:
            dist.destroy_process_group()
        return
    if args.workload != "c1":
        run_ivf(args, rank, world, local)
        if world > 1:
            dist.destroy_process_group()
        return
    import quiver_b200 as qv
    from quiver_b200 import _native
    from quiver_b200.distributed import ReplicatedFlatIndex, ShardedFlatIndex
    from quiver_b200.synthetic import config1

    n_db, n_q = args.rows, args.queries
    db, q = config1(n_db, n_q)
    by_queries = args.shard == "queries" and world > 1
    if by_queries:
        index = ReplicatedFlatIndex(DIM, "cosine", device=local)
        index.add(db)
    else:
        lo, hi = rank * n_db // world, (rank + 1) * n_db // world
        index = ShardedFlatIndex(DIM, "cosine", device=local)
        index.add_shard(db[lo:hi], np.arange(lo, hi, dtype=np.uint64), np.arange(lo, hi))
    dq = torch.from_numpy(q).cuda()
    q_pinned = torch.from_numpy(q).pin_memory()
    q_host = q_pinned.numpy()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- value: inputs resident in HBM ----
    for _ in range(args.warmup):
        index.search_device(dq, K)
    torch.cuda.synchronize()
    _native.set_timing(True)
    sampler = ClockSampler(local)
    sampler.start()
    qv.last_search_stats()  # start the accumulation here
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        index.search_device(dq, K)  # enqueues only: no host round trip per step
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    # With timing on, the library recorded CUDA events around each step's screen on its stream,
    # counted launches and rescans; reading the stats resolves them (after the timed region).
    st = qv.last_search_stats()
    launches, kernel_ms, kernel_work = (st["kernel_launches"], st["dominant_kernel_ms"],
                                        st["dominant_kernel_work"])
    kernel_name, rescans = st["dominant_kernel"], st["rescanned_queries"]
    _native.set_timing(False)
    elapsed = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([elapsed], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
        c = torch.tensor([launches, rescans], device="cuda", dtype=torch.float64)
        dist.all_reduce(c, op=dist.ReduceOp.SUM)
        launches, rescans = int(c[0].item()), int(c[1].item())
    ms_per_step = elapsed / args.steps
    value = n_q * args.steps / (elapsed / 1000.0)

    # ---- e2e: public API, pinned host queries in, host results out ----
    def e2e_call():
        if world == 1:
            return index.local.search(q_host, K)
        return index.search(q_host, K)

    for _ in range(max(1, args.warmup)):
        e2e_call()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        labels, dists = e2e_call()
    e2e_s = time.perf_counter() - t0
    barrier()
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    copies = 1 if by_queries else world  # query slices, or the whole batch on every rank
    e2e = {"value": n_q * args.steps / e2e_s, "unit": "QPS",
           "h2d_bytes_per_step": copies * n_q * DIM * 4,
           "d2h_bytes_per_step": copies * n_q * K * (8 + 4)}

    hbm, tflops, peak_kind = load_peaks()
    launches_timed = max(1, args.steps)
    avg_kernel_ms = kernel_ms / launches_timed
    achieved = (kernel_work / launches_timed) / (avg_kernel_ms / 1000.0) / 1e12 if avg_kernel_ms else 0.0
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if world == 1 and (n_db, n_q) == (N_DB, N_Q) and os.path.exists(tpath):
        with open(tpath) as fh:
            traffic = json.load(fh).get(kernel_name, {}).get("bytes_per_launch_c1_shard_1gpu")
    line = {
        "metric": METRIC, "value": value, "unit": "QPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": flat_config(args),
        "parallelism": (f"query slices x{world}, rows replicated" if by_queries
                        else f"id-range shards x{world}"),
        "gpu_launches": launches, "rescanned_queries": rescans,
        "roofline": {"bound": "tensor", "kernel": kernel_name, "achieved": achieved,
                     "peak": tflops, "unit": "TFLOP/s", "frac": achieved / tflops,
                     "peak_source": f"{peak_kind} bf16 dense (burst)", "traffic": traffic,
                     "avg_launch_ms": avg_kernel_ms,
                     "work_per_launch": kernel_work / launches_timed},
        "clocks": clocks, "e2e": e2e,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_reference_qps(db, q, seconds=15.0) or cpu_port_qps(db, q, seconds=10.0)
        qps, cores, sample, kind = base
        line["cpu_baseline"] = {"value": qps, "unit": "QPS", "cores": cores, "kind": kind,
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
