"""Builds the sm_100a shared library (batch_topk_b200/lib/libbatch_topk_b200.so) with nvcc.

Run as ``python -m batch_topk_b200.build``.  The library is built in-tree so that it
travels with the repository; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "batch_topk.cu")
GEN_SRC = os.path.join(HERE, "csrc", "gen.cu")  # device-side input generation
LOGITS_SRC = os.path.join(HERE, "csrc", "bt_logits.cu")  # logits producer, fused top-k epilogue
HEADERS = [os.path.join(HERE, "csrc", f) for f in ("bt_device.cuh", "bt_kernels.cuh", "bt_body.cuh",
                                                   "bt_elem.cuh", "bt_small.cuh",
                                                   "bt_large.cuh", "bt_common.cuh", "bt_f32.cuh")] + [
    os.path.join(REPO, "include", "batch_topk_b200.h"),
    os.path.join(REPO, "include", "batch_topk_b200_gen.h"),
]
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libbatch_topk_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in [SRC, GEN_SRC, LOGITS_SRC, *HEADERS])


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-o", tmp, SRC, GEN_SRC, LOGITS_SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
