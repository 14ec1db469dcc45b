"""The C++ drop-in headers: a host caller built with g++ against include/ and linked with the
library runs the reference's CPU-unit checks and the error contract (no GPU needed); where
the reference tree is present, its own benchmark driver (bench/bench_batch_topk.cu) compiles
and links against these headers unchanged."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

import batch_topk_b200 as bt

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(REPO, "include")
CUDA_INC = "/usr/local/cuda/include"
LIBDIR = os.path.dirname(bt.library_path())


def _link_flags():
    return [f"-L{LIBDIR}", "-lbatch_topk_b200", f"-Wl,-rpath,{LIBDIR}"]


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_host_caller_builds_and_passes(tmp_path):
    exe = tmp_path / "shim_check"
    src = os.path.join(REPO, "tests", "cpp", "shim_check.cpp")
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{INCLUDE}", f"-I{CUDA_INC}", src,
                    *_link_flags(), "-o", str(exe)], check=True, capture_output=True, text=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "FAIL" not in res.stdout and res.stdout.count("ok ") >= 14


def _ref_bench():
    import oracle

    d = oracle.reference_dir()  # BT_REFERENCE_DIR, or a reference tree beside the repository
    return os.path.join(d, "bench", "bench_batch_topk.cu") if d else ""


REF_BENCH = _ref_bench()


@pytest.mark.skipif(not REF_BENCH or not os.path.exists(REF_BENCH),
                    reason="reference tree not present (set BT_REFERENCE_DIR)")
def test_reference_benchmark_driver_builds_against_headers(tmp_path):
    exe = tmp_path / "bench_dropin"
    nvcc = "/usr/local/cuda/bin/nvcc"
    res = subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                          f"-I{INCLUDE}", REF_BENCH, f"-L{LIBDIR}", "-lbatch_topk_b200",
                          "-Xlinker", f"-rpath,{LIBDIR}", "-o", str(exe)],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    nm = subprocess.run(["nm", "-D", "--undefined-only", str(exe)], capture_output=True,
                        text=True, check=True).stdout
    assert "bt_topk_half" in nm and "bt_topk_half_workspace_size" in nm
