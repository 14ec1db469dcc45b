"""Benchmark: batched fp16 top-k (k=50) on B200, one JSON line per run.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one process per GPU)

Workload: configuration C3 of BASELINE.json, 1024 segments x 151936 fp16 values, k=50,
256 fp16 levels with +0/-0 (heavy ties), seeded synthetic data.  This is the configuration
the north-star target names (>= 70 % of HBM on effective input bytes on one GPU).  With N
ranks each rank owns its own 1024 segments (weak scaling, no collective on the data path;
segments shard naturally).  The input (311 MB) is larger than L2 (126 MB), so no flush is
needed between steps.

value      segments/s over all ranks, inputs resident in HBM, device-timed (CUDA events,
           max over ranks).
e2e        the same metric through the public API from pinned host memory: per step the
           H2D copy of the input and the D2H copy of the values and indices are inside the
           timed region.
roofline   the streaming kernel (bt::f16::topk_kernel<false>, k <= 128) over the device
           time per step of the timed region (the kernel plus the unoverlapped part of the
           set-up kernel launched behind it: an upper bound on the kernel's duration);
           kernel_ms_isolated is the kernel alone, from events the library's profiling hook
           records around it in a second pass (they also expose its launch latency);
           algorithmic bytes = 2 B per input value (the output, 6 B per selected entry, is
           0.2 % of it and left out).
cpu_baseline  the reference's own CPU top-k (cpu_reference_topk, oracle/_ref) on this host's
           cores, on a bounded sample of the same workload (rank 0, N=1 only).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "segments/s and effective input GB/s (% of HBM peak), k=50, at 1/2/4/8 B200"


class Workload:
    """One bench workload: how each rank builds its input and calls the library.

    C3 (default, the metric's configuration): 1024 rows x 151936 fp16 per rank, k=50, weak
        scaling (rank r owns rows [1024 r, 1024 (r+1)) of the seeded C3 generator).
    C5: 1024 rows x 262144 fp16 per rank, k=1024, weak scaling; at 8 ranks the ranks hold the
        whole 8192-row C5 batch (4 GiB), rank r rows [1024 r, 1024 (r+1)).
    C4: the 4096-segment CSR batch (lengths U{1..262144}), k from --k, strong scaling: the
        segments are split into contiguous element-balanced ranges, one per rank."""

    def __init__(self, name: str, k: int | None, rank: int, world: int):
        from batch_topk_b200 import workloads as wl
        from batch_topk_b200.shard import csr_local, csr_ranges

        self.name, self.rank, self.world = name, rank, world
        if name in ("C3", "C5"):
            self.kind = "fixed"
            self.seg_len = 151936 if name == "C3" else 262144
            self.k = k or (50 if name == "C3" else 1024)
            self.rows = range(rank * 1024, (rank + 1) * 1024)
            self.seg_num = 1024
            self.seg_total = 1024 * world
            self.elements = 1024 * self.seg_len
            self.elements_total = self.elements * world
            self.scaling = "weak"
        elif name == "C4":
            self.kind = "csr"
            self.k = k or 50
            off = wl.c4_offsets()
            self.s0, self.s1 = csr_ranges(off, world)[rank]
            self.local_off, self.e0, self.e1 = csr_local(off, self.s0, self.s1)
            self.seg_num = self.s1 - self.s0
            self.seg_total = len(off) - 1
            self.elements = self.e1 - self.e0
            self.elements_total = int(off[-1] - off[0])
            self.scaling = "strong"
        else:
            raise ValueError(f"unknown workload {name}")

    def describe(self) -> str:
        if self.name == "C3":
            return "C3: 1024 x 151936 fp16 per GPU, k=50, heavy ties"
        if self.name == "C5":
            return (f"C5: 1024 x 262144 fp16 per GPU (rows of the 8192-row batch), k={self.k}, "
                    "constant / sorted / U[1,2) rows")
        return (f"C4: 4096 CSR segments (lengths U{{1..262144}}, {self.elements_total} values) "
                f"split by elements over {self.world} GPU(s), k={self.k}")

    def device_input(self, dev):
        """This rank's input, generated in place on its device (bit-identical to the host
        generators, batch_topk_b200.workloads)."""
        from batch_topk_b200 import gen

        import torch

        if self.name == "C3":
            return gen.gen_c3(rows=self.rows, device=dev), None
        if self.name == "C5":
            return gen.gen_c5(rows=self.rows, device=dev), None
        x = gen.gen_c4_range(self.s0, self.s1, device=dev)
        return x, torch.from_numpy(self.local_off).to(dev)

    def call(self, bt, x, d_off, ov, oi, ws, nbytes, stream):
        if self.kind == "fixed":
            return bt.batch_topk_half(x.data_ptr(), self.seg_num, self.seg_len, self.k,
                                      ov.data_ptr(), oi.data_ptr(), ws.data_ptr(), nbytes, stream)
        return bt.batch_topk_half_segmented(x.data_ptr(), d_off.data_ptr(), self.seg_num,
                                            self.elements, self.k, ov.data_ptr(), oi.data_ptr(),
                                            ws.data_ptr(), nbytes, stream)

    def workspace_bytes(self, bt):
        if self.kind == "fixed":
            return bt.batch_topk_half_workspace_size(self.seg_num, self.seg_len, self.k)
        return bt.batch_topk_half_segmented_workspace_size(self.seg_num, self.elements, self.k)

    def check(self, orc, x_host, ov, oi, n: int = 8) -> bool:
        """The first n segments of this rank against the checker."""
        if self.kind == "fixed":
            exp_v, exp_i = orc.topk(x_host.reshape(self.seg_num, self.seg_len)[:n], self.k)
        else:
            off = self.local_off.astype(np.int64)[: n + 1]
            exp_v, exp_i = orc.topk_csr(x_host[: int(off[-1])], off, self.k)
        return bool(np.array_equal(oi[:n], exp_i) and np.array_equal(ov[:n], exp_v))

    def sample(self, x_host, n: int):
        """(values, offsets or None, segments) of the first n segments, for the CPU baseline."""
        if self.kind == "fixed":
            return x_host.reshape(self.seg_num, self.seg_len)[:n], None, n
        off = self.local_off.astype(np.int64)[: n + 1]
        return x_host[: int(off[-1])], off, n


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_launch(workload: str, k: int, elements: int):
    """DRAM bytes per launch of the streaming kernel from the committed ncu summary of this
    workload (scaled by elements when the capture held a smaller case of it), or None."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            d = json.load(f)
        for e in d.values():
            if e.get("workload") == workload and int(e.get("k", k)) == k:
                per_elem = float(e["dram_bytes_per_launch"]) / float(e["elements"])
                return per_elem * elements
    except Exception:
        pass
    return None


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_baseline(work: Workload, sample_fn, target_core_s: float = 15.0, method: str = "reference"):
    """The reference's cpu_reference_topk (oracle/_ref; its stable_sort of the index
    permutation) or, with method="partial_sort" or when oracle/_ref is absent, the C
    restatement (a partial sort with the same comparator), on all host threads over a bounded
    sample of the workload's segments; sample_fn(n) gives (values, offsets or None, n)."""
    import oracle

    threads = os.cpu_count() or 1
    ref = oracle.load_ref() if method == "reference" else None
    k = work.k
    vals, off, n0 = sample_fn(2)
    if ref is not None:
        kind = "reference"
        _, _, el = ref.topk(vals, k, offsets=off, threads=1)
        per_seg = el / n0
    else:
        kind = "port"
        o = oracle.load()
        t0 = time.perf_counter()
        if off is None:
            o.topk(vals, k, method=oracle.METHOD_SORT, threads=1)
        else:
            o.topk_csr(vals, off, k, method=oracle.METHOD_SORT, threads=1)
        per_seg = (time.perf_counter() - t0) / n0
    n = int(min(work.seg_num, max(threads, target_core_s / max(per_seg, 1e-6))))
    n = max(threads, n - n % threads) if n >= threads else n
    n = min(n, work.seg_num)
    vals, off, n = sample_fn(n)
    if kind == "reference":
        _, _, el = ref.topk(vals, k, offsets=off, threads=threads)
    else:
        t0 = time.perf_counter()
        if off is None:
            oracle.load().topk(vals, k, method=oracle.METHOD_SORT, threads=threads)
        else:
            oracle.load().topk_csr(vals, off, k, method=oracle.METHOD_SORT, threads=threads)
        el = time.perf_counter() - t0
    elems = int(vals.size)
    what = ("the reference's cpu_reference_topk (stable_sort of the index permutation)"
            if kind == "reference" else "std::partial_sort-style C restatement, same comparator")
    return {"value": n / el, "unit": "segments/s", "cores": threads, "kind": kind,
            "cpu_model": cpu_model(),
            "sample": f"first {n} of this GPU's {work.seg_num} {work.name} segments "
                      f"({elems} fp16 values), k={k}, {threads} threads; {what}; fp16->float "
                      "conversion outside the timed region",
            "effective_input_gbs": elems * 2 / el / 1e9}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU top-k on this host's cores (rank 0 only)."""
    if rank != 0:
        return
    work = Workload(args.workload, args.k, 0, 1)
    from batch_topk_b200 import workloads as wl

    cache = {}

    def sample_fn(n):  # the sample segments, generated once on the host
        if n not in cache:
            if work.name == "C3":
                cache[n] = (wl.gen_c3(rows=np.arange(n)), None, n)
            elif work.name == "C5":
                cache[n] = (wl.gen_c5(rows=np.arange(n)), None, n)
            else:
                off = work.local_off.astype(np.int64)[: n + 1]
                cache[n] = (wl.gen_c4_range(0, n), off, n)
        return cache[n]

    vals = []
    base = None
    for i in range(args.warmup + args.steps):
        b = cpu_baseline(work, sample_fn, target_core_s=args.ref_core_seconds)
        if i >= args.warmup:
            vals.append(b["value"])
            base = b
    v = float(np.median(vals))
    line = {
        "metric": METRIC, "value": v, "unit": "segments/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": work.seg_num / v * 1e3, "higher_is_better": True,
        "scaling": work.scaling, "vs_baseline": None, "dtype": "f16",
        "data": f"synthetic (seeded {work.name} generator)",
        "config": {"workload": work.describe(), "seg_num": work.seg_num, "k": work.k,
                   "parallelism": f"reference CPU path on host cores (rank 0 of {world})"},
        "effective_input_gbs": base["effective_input_gbs"],
        "cpu_baseline": {k2: base[k2] for k2 in ("value", "unit", "cores", "kind", "sample",
                                                  "cpu_model")},
        "e2e": {"value": v, "unit": "segments/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch

    import batch_topk_b200 as bt

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
    work = Workload(args.workload, args.k, rank, world)
    k = work.k
    x, d_off = work.device_input(dev)
    x_host = x.cpu().numpy().view(np.uint16).reshape(-1)  # checker, end-to-end and CPU legs
    nbytes = work.workspace_bytes(bt)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    ov = torch.empty((work.seg_num, k), dtype=torch.int16, device=dev)
    oi = torch.empty((work.seg_num, k), dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(dev)
    sp = stream.cuda_stream

    def step():
        rc = work.call(bt, x, d_off, ov, oi, ws, nbytes, sp)
        if rc != 0:
            raise bt.BatchTopkError(rc, "top-k")

    def barrier():
        if dist is not None:
            dist.barrier()

    def gather(v: float) -> list:
        if dist is None:
            return [v]
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return [float(p.item()) for p in parts]

    # correctness gate before timing: this rank's first 8 segments vs the checker
    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    import oracle

    orc = oracle.load()
    ok = work.check(orc, x_host, ov.cpu().numpy().view(np.uint16), oi.cpu().numpy())
    if not all(v > 0 for v in gather(1.0 if ok else 0.0)):
        raise SystemExit("bench: GPU result differs from the oracle; refusing to time it")

    for _ in range(args.warmup):
        step()
    stream.synchronize()

    # device-resident timed region: `steps` steps back to back, as a caller runs them,
    # repeated `repeats` times; each repetition is timed on the launching stream and its
    # max over ranks taken; the median repetition is reported
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    reps_local, reps_max = [], []
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.repeats):
            barrier()
            torch.cuda.synchronize(dev)
            e0.record(stream)
            for _ in range(args.steps):
                step()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            barrier()
            t = e0.elapsed_time(e1) / args.steps
            reps_local.append(t)
            reps_max.append(max(gather(t)))
    order = np.argsort(reps_max)
    mid = int(order[len(order) // 2])
    ms_per_step = reps_max[mid]
    per_rank_ms = gather(reps_local[mid])
    # the streaming kernel alone: the same steps again, with the library's profiling hook
    # recording events around the kernel on its stream (the events sit between the two
    # launches and break their overlap, so this loop is not the one `value` is taken from)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for e in starts + stops:
        e.record(stream)  # materialise the events before handing their handles over
    torch.cuda.synchronize(dev)
    for i in range(args.steps):
        bt.set_profile_events(starts[i].cuda_event, stops[i].cuda_event)
        step()
    bt.set_profile_events(None, None)
    torch.cuda.synchronize(dev)
    kern_ms = float(np.mean([a.elapsed_time(b) for a, b in zip(starts, stops)]))
    per_rank_kern = gather(kern_ms)
    value = work.seg_total / (ms_per_step / 1e3)
    in_bytes = work.elements * 2

    # end to end through the public API: pinned host input -> H2D -> top-k -> D2H results
    from batch_topk_b200 import torch_api

    xh = torch.from_numpy(x_host.view(np.int16)).pin_memory()
    hv = torch.empty((work.seg_num, k), dtype=torch.int16).pin_memory()
    hi = torch.empty((work.seg_num, k), dtype=torch.int32).pin_memory()
    if work.kind == "csr":
        oh = torch.from_numpy(work.local_off).pin_memory()
        dbuf = torch.empty(work.elements, dtype=torch.float16, device=dev)
        doff = torch.empty(work.seg_num + 1, dtype=torch.int32, device=dev)

    def e2e_step():
        if work.kind == "fixed":
            torch_api.topk_from_host(xh.view(work.seg_num, work.seg_len), k, out_host=(hv, hi),
                                     stream=stream)
            return
        with torch.cuda.stream(stream):
            dbuf.view(torch.int16).copy_(xh, non_blocking=True)
            doff.copy_(oh, non_blocking=True)
            v, i = torch_api.topk_segmented(dbuf, doff, k, max_total_len=work.elements,
                                            stream=stream)
            hv.copy_(v.view(torch.int16), non_blocking=True)
            hi.copy_(i, non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_step()
    stream.synchronize()
    e2e_steps = max(3, min(args.steps, 10))
    barrier()
    torch.cuda.synchronize(dev)
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    a1.record(stream)
    stream.synchronize()
    e2e_ms = max(gather(a0.elapsed_time(a1))) / e2e_steps
    ok = work.check(orc, x_host, hv.numpy().view(np.uint16), hi.numpy())
    if not all(v > 0 for v in gather(1.0 if ok else 0.0)):
        raise SystemExit("bench: end-to-end result differs from the oracle")

    peak, peak_kind = peaks()
    # The roofline divides by the device time per step over the timed region: the streaming
    # kernel plus whatever part of the set-up kernel it does not overlap (an upper bound on
    # the kernel's own duration).  kern_ms, from events recorded between the two launches,
    # also holds the kernel's launch latency, which those events expose.
    achieved = in_bytes / (ms_per_step / 1e3) / 1e9
    kernel = f"bt::f16::topk_kernel<{'true' if k > 128 else 'false'}>"
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "segments/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": work.scaling,
        "vs_baseline": None,
        "dtype": "f16",
        "data": f"synthetic (seeded {work.name} generator, run on the device)",
        "config": {
            "workload": work.describe(),
            "seg_num_per_gpu": work.seg_num, "k": k,
            "global_segments": work.seg_total,
            "parallelism": f"segment-sharded x{world}, no collective on the data path",
            "l2": "inputs larger than L2 (126 MB) on every rank; no flush",
            "timed_repeats": args.repeats,
            "timing": f"{args.repeats} timed loops of {args.steps} steps; per loop the max "
                      "over ranks; the median loop is reported",
        },
        "effective_input_gbs": work.elements_total * 2 / (ms_per_step / 1e3) / 1e9,
        "pct_hbm_per_gpu": achieved / peak,
        "gpu_launches": 2 * args.steps,  # set-up kernel + streaming kernel per step
        "roofline": {
            "bound": "hbm", "kernel": kernel,
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
            "algorithmic_bytes_per_launch": in_bytes,
            "duration_ms": ms_per_step,
            "duration_source": "device time per step over the timed region (CUDA events on "
                               "the launching stream): streaming kernel + unoverlapped set-up",
            "kernel_ms_isolated": kern_ms,
            "traffic": traffic_per_launch(work.name, k, work.elements),
        },
        "per_rank": {
            "ms_per_step": per_rank_ms,
            "kernel_ms_isolated": per_rank_kern,
            "slowest_rank": int(np.argmax(per_rank_ms)),
            "repeats_ms_per_step_max_over_ranks": reps_max,
        },
        "e2e": {"value": work.seg_total / (e2e_ms / 1e3), "unit": "segments/s",
                "h2d_bytes_per_step": in_bytes + (4 * (work.seg_num + 1) if work.kind == "csr" else 0),
                "d2h_bytes_per_step": work.seg_num * k * 6,
                "ms_per_step": e2e_ms,
                "limiter": "the host-to-device copy of the input from pinned memory"},
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(work, lambda n: work.sample(x_host, n),
                                            target_core_s=args.ref_core_seconds)
        if args.partial_sort_baseline:
            line["cpu_baseline_partial_sort"] = cpu_baseline(
                work, lambda n: work.sample(x_host, n), target_core_s=args.ref_core_seconds,
                method="partial_sort")
    if rank == 0:
        print(json.dumps(line), flush=True)


# The reference's own benchmark table (include/batch_topk_benchmark.cuh:14-20 of the
# reference): seg_num, seg_len, k and its published target latency in us.
REF_GPU_SHAPES = [(128, 10000, 50, 11.0), (1500, 10000, 50, 82.0), (3000, 10000, 50, 161.0),
                  (4500, 10000, 50, 241.0), (6000, 10000, 50, 319.0)]


def ref_bench_input(seg_num: int, seg_len: int) -> np.ndarray:
    """The reference benchmark's input (bench/bench_batch_topk.cu:10-16 of the reference):
    value i = ((i * 17 + 13) mod 2048 - 1024) / 16 as fp16 bits (2048 levels, heavy ties)."""
    i = np.arange(seg_num * seg_len, dtype=np.uint64)
    raw = ((i * np.uint64(17) + np.uint64(13)) % np.uint64(2048)).astype(np.int64) - 1024
    return (raw.astype(np.float32) / 16.0).astype(np.float16).view(np.uint16).reshape(
        seg_num, seg_len)


def run_reference_gpu_race(args):
    """--suite reference-gpu: the reference's own GPU path (its src/batch_topk.cu built for
    sm_100a into oracle/_ref/libref_gpu.so) against bt_topk_half on the reference's five
    benchmark shapes, on the same GPU and stream, one JSON line per shape.

    hot:     the reference harness's method (bench/bench_batch_topk.cu:56-132): 5 warm-up
             calls, then CUDA events around 20 calls back to back; median of 5 such loops.
             Its inputs (<= 120 MB) fit in L2, so repeated calls read them from L2.
    flushed: one call between two events after writing a 512 MiB buffer (L2 is 126 MB);
             median of 15.
    Both outputs are checked against the oracle on every row."""
    import torch

    import batch_topk_b200 as bt
    import oracle

    ref = oracle.load_ref_gpu()
    if ref is None:
        print(json.dumps({"suite": "reference-gpu",
                          "unavailable": "oracle/_ref/libref_gpu.so was not built (reference "
                                         "tree absent at build time)"}), flush=True)
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s = torch.cuda.Stream(dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    orc = oracle.load()
    for seg_num, seg_len, k, target in REF_GPU_SHAPES:
        bits = ref_bench_input(seg_num, seg_len)
        x = torch.from_numpy(bits.view(np.int16)).to(dev)
        exp_v, exp_i = orc.topk(bits, k)
        arms = {}
        for name in ("ours", "reference"):
            if name == "ours":
                nb = bt.batch_topk_half_workspace_size(seg_num, seg_len, k)
                fn = bt.batch_topk_half
            else:
                nb = ref.workspace_size(seg_num, seg_len, k)
                fn = ref.topk_half
            ws = torch.empty(nb, dtype=torch.uint8, device=dev)
            ov = torch.empty((seg_num, k), dtype=torch.int16, device=dev)
            oi = torch.empty((seg_num, k), dtype=torch.int32, device=dev)

            def call():
                rc = fn(x.data_ptr(), seg_num, seg_len, k, ov.data_ptr(), oi.data_ptr(),
                        ws.data_ptr(), nb, s.cuda_stream)
                if rc != 0:
                    raise RuntimeError(f"{name} returned {rc} on {seg_num}x{seg_len}")

            for _ in range(5):
                call()
            s.synchronize()
            exact = bool(np.array_equal(oi.cpu().numpy(), exp_i) and
                         np.array_equal(ov.cpu().numpy().view(np.uint16), exp_v))
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            hot = []
            for _ in range(5):
                e0.record(s)
                for _ in range(20):
                    call()
                e1.record(s)
                e1.synchronize()
                hot.append(e0.elapsed_time(e1) * 1e3 / 20)
            cold = []
            for _ in range(15):
                with torch.cuda.stream(s):
                    flush.fill_(len(cold) & 0xFF)
                e0.record(s)
                call()
                e1.record(s)
                e1.synchronize()
                cold.append(e0.elapsed_time(e1) * 1e3)
            arms[name] = {"hot_us": float(np.median(hot)), "flushed_us": float(np.median(cold)),
                          "exact": exact}
        o, r = arms["ours"], arms["reference"]
        print(json.dumps({
            "suite": "reference-gpu", "seg_num": seg_num, "seg_len": seg_len, "k": k,
            "input": "reference bench fill ((i*17+13) mod 2048 - 1024)/16",
            "ours_hot_us": round(o["hot_us"], 2), "ref_hot_us": round(r["hot_us"], 2),
            "speedup_hot": round(r["hot_us"] / o["hot_us"], 3),
            "ours_flushed_us": round(o["flushed_us"], 2),
            "ref_flushed_us": round(r["flushed_us"], 2),
            "speedup_flushed": round(r["flushed_us"] / o["flushed_us"], 3),
            "ref_target_us_4080": target, "ours_exact": o["exact"], "ref_exact": r["exact"],
        }), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--suite", choices=["reference-gpu"],
                    help="instead of the bench line: the reference's own GPU path against this "
                         "library on the reference's benchmark shapes (one GPU)")
    ap.add_argument("--ref-core-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["C3", "C5", "C4"], default="C3",
                    help="C3 (default): the metric's configuration; C5 / C4: the large-k and "
                         "variable-length configurations")
    ap.add_argument("--k", type=int, help="k (default: the workload's own)")
    ap.add_argument("--repeats", type=int, default=5,
                    help="timed loops of --steps steps each; the median loop is reported")
    ap.add_argument("--partial-sort-baseline", action="store_true",
                    help="also time the partial-sort CPU restatement next to the reference's")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.suite == "reference-gpu":
        run_reference_gpu_race(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
