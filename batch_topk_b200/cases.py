"""Time the library on the five benchmark configurations (or one of them), one JSON line each.

    python -m batch_topk_b200.cases [--config C1|C2|C3|C4|C5|N01] [--k K] [--iters N] [--rows R]
                                    [--dtype f16|bf16|f32]

Inputs are generated on the device (batch_topk_b200.gen).  Each line gives the median time of
the streaming kernel alone (CUDA events recorded around it on its stream by the library's
profiling hook) and of the whole call, and the effective input bandwidth against the
measured HBM copy peak.  With --dtype bf16 each generated fp16 value is converted to the
nearest bfloat16 and the bf16 entry points run; with --dtype f32 it is widened (exactly) to
float32 and the fp32 entry points run (4 bytes a value).  The same command is the target of the ncu
summaries under profiles/.
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np
import torch

from . import batch_topk_bf16, batch_topk_bf16_segmented, batch_topk_bf16_segmented_workspace_size
from . import batch_topk_f32, batch_topk_f32_segmented, batch_topk_f32_segmented_workspace_size
from . import batch_topk_f32_workspace_size
from . import batch_topk_bf16_workspace_size, batch_topk_half, batch_topk_half_segmented
from . import batch_topk_half_segmented_workspace_size, batch_topk_half_workspace_size
from . import set_profile_events, workspace_status
from . import gen
from . import workloads as wl

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def hbm_peak() -> float:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def make(config: str, rows: int | None):
    """(device int16 values, host int64 offsets or None, default k, row count)."""
    if config == "C4":
        off = wl.c4_offsets()
        n = rows or (len(off) - 1)
        return gen.gen_c4_range(0, n), off[: n + 1], 50, n
    if config == "N01":  # i.i.d. N(0,1) rows of C3's shape: a tie-free stream
        n = rows or 1024
        x = torch.empty((n, 151936), dtype=torch.int16, device="cuda")
        gen.normal_(x.view(-1), 0, 11, 0, 1.0)
        return x, None, 50, n
    cfg = wl.CONFIGS[config]
    n = rows or cfg.seg_num
    fn = {"C1": gen.gen_c1, "C2": gen.gen_c2, "C3": gen.gen_c3, "C5": gen.gen_c5}[config]
    return fn(rows=range(n)), None, cfg.k, n


def run(config: str, k: int | None, iters: int, rows: int | None, outputs: bool = False,
        dtype: str = "f16"):
    """One JSON-ready line; with outputs=True also (input, offsets, values, indices) on the device."""
    x, off, k0, n = make(config, rows)
    bf16 = dtype == "bf16"
    f32 = dtype == "f32"
    esize = 4 if f32 else 2
    if bf16:
        x = x.view(torch.float16).to(torch.bfloat16).view(torch.int16)
    if f32:
        x = x.view(torch.float16).float().view(torch.int32)
    fixed, fixed_ws = (batch_topk_bf16, batch_topk_bf16_workspace_size) if bf16 else (
        (batch_topk_f32, batch_topk_f32_workspace_size) if f32 else
        (batch_topk_half, batch_topk_half_workspace_size))
    csr, csr_ws = (batch_topk_bf16_segmented, batch_topk_bf16_segmented_workspace_size) if bf16 else (
        (batch_topk_f32_segmented, batch_topk_f32_segmented_workspace_size) if f32 else
        (batch_topk_half_segmented, batch_topk_half_segmented_workspace_size))
    k = k or k0
    dev = x.device
    s = torch.cuda.current_stream(dev)
    if off is None:
        seg_len = x.shape[1]
        nbytes = fixed_ws(n, seg_len, k)
        total = n * seg_len
    else:
        total = int(off[-1])
        nbytes = csr_ws(n, total, k)
        d_off = torch.from_numpy(off.astype(np.int32)).to(dev)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    ov = torch.empty((n, k), dtype=torch.int32 if f32 else torch.int16, device=dev)
    oi = torch.empty((n, k), dtype=torch.int32, device=dev)

    def call():
        if off is None:
            rc = fixed(x.data_ptr(), n, seg_len, k, ov.data_ptr(), oi.data_ptr(), ws.data_ptr(),
                       nbytes, s.cuda_stream)
        else:
            rc = csr(x.data_ptr(), d_off.data_ptr(), n, total, k, ov.data_ptr(), oi.data_ptr(),
                     ws.data_ptr(), nbytes, s.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"top-k call returned {rc}")

    for _ in range(3):
        call()
    k0e, k1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0e, c1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0e.record(s)
    k1e.record(s)
    torch.cuda.synchronize(dev)
    set_profile_events(k0e.cuda_event, k1e.cuda_event)
    kern, whole = [], []
    try:
        for _ in range(iters):
            c0e.record(s)
            call()
            c1e.record(s)
            torch.cuda.synchronize(dev)
            kern.append(k0e.elapsed_time(k1e))
            whole.append(c0e.elapsed_time(c1e))
    finally:
        set_profile_events(None, None)
    flags, _ = workspace_status(ws.data_ptr(), n, s.cuda_stream)
    kt, wt = float(np.median(kern)), float(np.median(whole))
    gbs = total * esize / kt / 1e6
    line = {"config": config, "dtype": dtype, "segments": n, "k": k, "values": total, "kernel_us": round(kt * 1e3, 2),
            "call_us": round(wt * 1e3, 2), "input_gbs": round(gbs, 1),
            "pct_hbm": round(gbs / hbm_peak(), 4), "status": flags}
    return (line, (x, off, ov, oi)) if outputs else line


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--config", choices=["C1", "C2", "C3", "C4", "C5", "N01"], action="append")
    ap.add_argument("--k", type=int, action="append", help="k values (C4: default 1, 8, 50, 256)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--rows", type=int, help="first R segments only (C5 defaults to 384)")
    ap.add_argument("--dtype", choices=["f16", "bf16", "f32"], default="f16")
    a = ap.parse_args()
    for config in a.config or ["C1", "C2", "C3", "N01", "C4", "C5"]:
        ks = a.k or (list(wl.C4_K_VALUES) if config == "C4" else [None])
        rows = a.rows or (384 if config == "C5" else None)
        for k in ks:
            print(json.dumps(run(config, k, a.iters, rows, dtype=a.dtype)), flush=True)


if __name__ == "__main__":
    main()
