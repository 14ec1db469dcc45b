"""Device-side input generation (batch_topk_b200.gen, include/batch_topk_b200_gen.h):
bit-identical to the host generators of workloads.py on every configuration."""
from __future__ import annotations

import os
import re

import numpy as np
import pytest

import batch_topk_b200 as bt
from batch_topk_b200 import _lib
from batch_topk_b200 import workloads as wl

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_generator_symbols_exported():
    text = open(os.path.join(REPO, "include", "batch_topk_b200_gen.h")).read()
    names = set(re.findall(r"^int (bt_gen_\w+)\(", text, flags=re.M))
    assert names == {"bt_gen_normal", "bt_gen_uniform", "bt_gen_levels", "bt_gen_mask"}
    lib = _lib.load()
    for n in names:
        assert hasattr(lib, n)


def test_generator_rejects_null_output():
    from batch_topk_b200 import gen

    lib = gen._gen_lib()
    assert lib.bt_gen_normal(None, 10, 0, 1, 0, 1.0, None) == bt.CUDA_ERROR_INVALID_VALUE
    assert lib.bt_gen_levels(1 << 20, 10, 0, 1, 0, None, None) == bt.CUDA_ERROR_INVALID_VALUE


def _bits(t):
    return t.cpu().numpy().view(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("cfg,rows", [("C1", None), ("C2", [0, 1, 5, 63]), ("C3", [0, 1, 2, 1000]),
                                      ("C5", [0, 1, 2, 4, 3])])
def test_device_rows_equal_host(cfg, rows):
    from batch_topk_b200 import gen

    dev = {"C1": gen.gen_c1, "C2": gen.gen_c2, "C3": gen.gen_c3, "C5": gen.gen_c5}[cfg](rows=rows)
    host = {"C1": wl.gen_c1, "C2": wl.gen_c2, "C3": wl.gen_c3, "C5": wl.gen_c5}[cfg](rows=rows)
    assert np.array_equal(_bits(dev), host)


@pytest.mark.gpu
def test_device_c4_equals_host():
    from batch_topk_b200 import gen

    assert np.array_equal(_bits(gen.gen_c4_range(0, 64)), wl.gen_c4_range(0, 64))
    assert np.array_equal(_bits(gen.gen_c4_range(4000, 4096)), wl.gen_c4_range(4000, 4096))


@pytest.mark.gpu
def test_device_normal_tails_and_rounding():
    """A long normal stream exercises the series' whole range and fp16 subnormal rounding."""
    import torch

    from batch_topk_b200 import gen

    n = 1 << 22
    out = gen.normal_(torch.empty(n, dtype=torch.int16, device="cuda"), 123456789, 77, 5, 1.0)
    idx = np.arange(123456789, 123456789 + n, dtype=np.int64)
    assert np.array_equal(_bits(out), wl.to_half_bits(wl.normal(77, 5, idx)))
    tiny = gen.normal_(torch.empty(n, dtype=torch.int16, device="cuda"), 0, 9, 1, 1e-4)
    assert np.array_equal(_bits(tiny), wl.to_half_bits(wl.normal(9, 1, np.arange(n), sigma=1e-4)))
