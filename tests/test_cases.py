"""The timing command `python -m batch_topk_b200.cases`: options parse on the CPU; on a GPU each
configuration's line is produced by the library and the outputs of its first segments equal
the C checker's."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cases_help():
    r = subprocess.run([sys.executable, "-m", "batch_topk_b200.cases", "--help"], cwd=REPO,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "--config" in r.stdout and "--rows" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("config,k,rows", [("C1", None, 4), ("C2", None, 8), ("C3", None, 16),
                                           ("N01", None, 8), ("C4", 256, 12), ("C5", None, 6)])
@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_cases_line_and_parity(orc, config, k, rows, dtype):
    from batch_topk_b200 import cases

    line, (x, off, ov, oi) = cases.run(config, k, 2, rows, outputs=True, dtype=dtype)
    bf16 = dtype == "bf16"
    json.dumps(line)
    assert line["segments"] == rows and line["status"] == 0
    assert line["kernel_us"] > 0 and line["call_us"] >= line["kernel_us"] * 0.5
    if dtype == "f32":
        xh = x.cpu().numpy().view(np.uint32)
        if off is None:
            ev, ei = orc.topk_f32(xh, line["k"])
        else:
            ev, ei = orc.topk_csr_f32(xh.reshape(-1), off, line["k"])
        assert np.array_equal(oi.cpu().numpy(), ei)
        assert np.array_equal(ov.cpu().numpy().view(np.uint32), ev)
        return
    xh = x.cpu().numpy().view(np.uint16)
    if off is None:
        ev, ei = orc.topk(xh, line["k"], bf16=bf16)
    else:
        ev, ei = orc.topk_csr(xh, off, line["k"], bf16=bf16)
    assert np.array_equal(oi.cpu().numpy(), ei)
    assert np.array_equal(ov.cpu().numpy().view(np.uint16), ev)
