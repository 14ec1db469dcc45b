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

WORKLOAD = "C3"
SEG_NUM, SEG_LEN, K = 1024, 151936, 50
METRIC = "segments/s and effective input GB/s (% of HBM peak), k=50, at 1/2/4/8 B200"


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_launch():
    """DRAM bytes per launch of the streaming kernel from the committed ncu summary."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            d = json.load(f)
        e = d["topk_kernel"]
        if e.get("workload") == WORKLOAD:
            return float(e["dram_bytes_per_launch"])
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


def make_input_device(rank: int, device):
    """This rank's C3 rows, generated in place on its device (bit-identical to the host
    generator: batch_topk_b200.gen)."""
    from batch_topk_b200 import gen

    return gen.gen_c3(rows=range(rank * SEG_NUM, (rank + 1) * SEG_NUM), device=device)


def host_rows(rank: int, n: int) -> np.ndarray:
    """The first n of this rank's C3 rows from the host generator."""
    from batch_topk_b200 import workloads as wl

    return wl.gen_c3(rows=np.arange(rank * SEG_NUM, rank * SEG_NUM + n))


def cpu_baseline(rows_fn, target_core_s: float = 15.0):
    """The reference's cpu_reference_topk (oracle/_ref) or, if absent, the C restatement of
    it (sort method), on all host threads over a bounded sample of segments; rows_fn(n)
    gives the first n rows of the workload."""
    import oracle

    threads = os.cpu_count() or 1
    ref = oracle.load_ref()
    probe = rows_fn(2)
    if ref is not None:
        kind = "reference"
        _, _, el = ref.topk(probe, K, threads=1)
        per_seg = el / probe.shape[0]
    else:
        kind = "port"
        o = oracle.load()
        t0 = time.perf_counter()
        o.topk(probe, K, method=0, threads=1)
        per_seg = (time.perf_counter() - t0) / probe.shape[0]
    n = int(min(SEG_NUM, max(threads, target_core_s / max(per_seg, 1e-6))))
    n = max(threads, n - n % threads) if n >= threads else n
    sample = rows_fn(n)
    if kind == "reference":
        _, _, el = ref.topk(sample, K, threads=threads)
    else:
        t0 = time.perf_counter()
        oracle.load().topk(sample, K, method=0, threads=threads)
        el = time.perf_counter() - t0
    return {"value": n / el, "unit": "segments/s", "cores": threads, "kind": kind,
            "sample": f"first {n} of {SEG_NUM} C3 segments (151936 fp16 each), k=50, "
                      f"{threads} threads, fp16->float conversion outside the timed region",
            "effective_input_gbs": n * SEG_LEN * 2 / el / 1e9}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU top-k on this host's cores (rank 0 only)."""
    if rank != 0:
        return
    cache = {}

    def rows_fn(n):  # the sample rows, generated once
        if n not in cache:
            cache[n] = host_rows(0, n)
        return cache[n]

    vals = []
    base = None
    for i in range(args.warmup + args.steps):
        b = cpu_baseline(rows_fn, target_core_s=args.ref_core_seconds)
        if i >= args.warmup:
            vals.append(b["value"])
            base = b
    v = float(np.median(vals))
    line = {
        "metric": METRIC, "value": v, "unit": "segments/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": SEG_NUM / v * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded C3 generator)",
        "config": {"workload": "C3: 1024 x 151936 fp16 per GPU, k=50, 256 levels incl. +0/-0",
                   "seg_num": SEG_NUM, "seg_len": SEG_LEN, "k": K,
                   "parallelism": f"reference CPU path on host cores (rank 0 of {world})"},
        "effective_input_gbs": v * SEG_LEN * 2 / 1e9,
        "cpu_baseline": {k2: base[k2] for k2 in ("value", "unit", "cores", "kind", "sample")},
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
    x = make_input_device(rank, dev)
    x_host = x.cpu().numpy().view(np.uint16)  # for the checker, the end-to-end leg, the CPU leg
    nbytes = bt.batch_topk_half_workspace_size(SEG_NUM, SEG_LEN, K)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    ov = torch.empty((SEG_NUM, K), dtype=torch.int16, device=dev)
    oi = torch.empty((SEG_NUM, K), dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(dev)
    sp = stream.cuda_stream

    def step():
        rc = bt.batch_topk_half(x.data_ptr(), SEG_NUM, SEG_LEN, K, ov.data_ptr(), oi.data_ptr(),
                                ws.data_ptr(), nbytes, sp)
        if rc != 0:
            raise bt.BatchTopkError(rc, "bt_topk_half")

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # correctness gate before timing: rank's first 8 segments vs the checker
    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    import oracle

    exp_v, exp_i = oracle.load().topk(x_host[:8], K)
    if not (np.array_equal(oi[:8].cpu().numpy(), exp_i)
            and np.array_equal(ov[:8].cpu().numpy().view(np.uint16), exp_v)):
        raise SystemExit("bench: GPU result differs from the oracle; refusing to time it")

    for _ in range(args.warmup):
        step()
    stream.synchronize()

    # device-resident timed region: the steps back to back, as a caller runs them
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms_local = e0.elapsed_time(e1)
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
    ms = max_over_ranks(ms_local)
    ms_per_step = ms / args.steps
    seg_total = SEG_NUM * world
    value = seg_total / (ms_per_step / 1e3)
    in_bytes = SEG_NUM * SEG_LEN * 2

    # end to end through the public API: pinned host input -> H2D -> top-k -> D2H results
    from batch_topk_b200.torch_api import topk_from_host

    xh = torch.from_numpy(x_host.view(np.int16)).pin_memory()
    hv = torch.empty((SEG_NUM, K), dtype=torch.int16).pin_memory()
    hi = torch.empty((SEG_NUM, K), dtype=torch.int32).pin_memory()
    for _ in range(2):
        topk_from_host(xh, K, out_host=(hv, hi), stream=stream)
    stream.synchronize()
    e2e_steps = max(3, min(args.steps, 10))
    barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(e2e_steps):
        topk_from_host(xh, K, out_host=(hv, hi), stream=stream)
    a1.record(stream)
    stream.synchronize()
    e2e_ms = max_over_ranks(a0.elapsed_time(a1)) / e2e_steps
    _ = time.perf_counter() - t0
    if not (np.array_equal(hi[:8].numpy(), exp_i) and np.array_equal(hv[:8].numpy().view(np.uint16), exp_v)):
        raise SystemExit("bench: end-to-end result differs from the oracle")

    peak, peak_kind = peaks()
    # The roofline divides by the device time per step over the timed region: the streaming
    # kernel plus whatever part of the set-up kernel it does not overlap (an upper bound on
    # the kernel's own duration).  kern_ms, from events recorded between the two launches,
    # also holds the kernel's launch latency, which those events expose.
    achieved = in_bytes / (ms_per_step / 1e3) / 1e9
    traffic = traffic_per_launch()
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "segments/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded C3 generator, run on the device: 256 fp16 levels U[-4,4] with +0/-0)",
        "config": {
            "workload": "C3: 1024 x 151936 fp16 per GPU, k=50, heavy ties",
            "seg_num_per_gpu": SEG_NUM, "seg_len": SEG_LEN, "k": K,
            "global_segments": seg_total,
            "parallelism": f"segment-sharded x{world}, no collective on the data path",
            "l2": "inputs larger than L2 (311 MB > 126 MB); no flush",
        },
        "effective_input_gbs": seg_total * SEG_LEN * 2 / (ms_per_step / 1e3) / 1e9,
        "pct_hbm_per_gpu": in_bytes / (ms_per_step / 1e3) / 1e9 / peak,
        "gpu_launches": 2 * args.steps,  # init_kernel + topk_kernel per step
        "roofline": {
            "bound": "hbm", "kernel": "bt::f16::topk_kernel<false>",
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
            "algorithmic_bytes_per_launch": in_bytes,
            "duration_ms": ms_per_step,
            "duration_source": "device time per step over the timed region (CUDA events on "
                               "the launching stream): streaming kernel + unoverlapped set-up",
            "kernel_ms_isolated": kern_ms,
            "traffic": traffic,
        },
        "e2e": {"value": seg_total / (e2e_ms / 1e3), "unit": "segments/s",
                "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": SEG_NUM * K * 6,
                "ms_per_step": e2e_ms},
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(lambda n: x_host[:n], target_core_s=args.ref_core_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ref-core-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
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
