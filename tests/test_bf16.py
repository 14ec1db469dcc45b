"""bfloat16 inputs (bt_topk_bf16, bt_topk_bf16_segmented).

The reference is fp16 only, so bf16 parity is anchored on the checker's bf16 path, and that
path is pinned on the CPU two independent ways:
- an order built with numpy alone: NaN last, then larger value first, then lower index, on
  the exact float32 value of each bf16 pattern;
- torch.topk's values.
The GPU tests compare the CUDA path with it bit for bit: value bits and int32 indices.
"""
from __future__ import annotations

import numpy as np
import pytest

from util import assert_exact, gpu_topk, gpu_topk_csr

NEG_INF_BF16 = 0xFF80


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round to nearest even (NaN kept as a quiet NaN)."""
    u = np.asarray(x, np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r).astype(np.uint16)


def numpy_topk_bf16(bits: np.ndarray, k: int):
    """Independent reference order, per row."""
    rows, n = bits.shape
    kk = min(k, n)
    idx = np.full((rows, k), -1, np.int32)
    val = np.full((rows, k), NEG_INF_BF16, np.uint16)
    for r in range(rows):
        f32 = bf16_to_f32(bits[r])
        nan = np.isnan(f32)
        with np.errstate(invalid="ignore"):  # signalling-NaN payloads
            f = f32.astype(np.float64)
        neg = np.where(nan, 0.0, -f)  # -0.0 == 0.0: ties between zeros go by index
        order = np.lexsort((np.arange(n), neg, nan))[:kk]
        idx[r, :kk] = order
        val[r, :kk] = bits[r, order]
    return val, idx


def make_rows(kind: str, rows: int, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "normal":
        return f32_to_bf16(rng.standard_normal((rows, n)).astype(np.float32))
    if kind == "bits":  # every pattern: NaNs, infinities, subnormals, zeros of both signs
        return rng.integers(0, 1 << 16, (rows, n), dtype=np.uint32).astype(np.uint16)
    if kind == "levels":  # heavy ties: 64 levels with +0 and -0
        lv = f32_to_bf16(rng.uniform(-4, 4, 64).astype(np.float32))
        lv[0], lv[1] = 0x0000, 0x8000
        return lv[rng.integers(0, 64, (rows, n))]
    if kind == "specials":
        pool = np.array([0x7FC0, 0xFFC1, 0x7F80, 0xFF80, 0x0000, 0x8000, 0x3F80, 0xBF80, 0x0001,
                         0x8001, 0x7F7F, 0xFF7F], np.uint16)
        return pool[rng.integers(0, pool.size, (rows, n))]
    raise ValueError(kind)


# ---- CPU: the checker's bf16 path ------------------------------------------------------------

@pytest.mark.parametrize("kind", ["normal", "bits", "levels", "specials"])
@pytest.mark.parametrize("k", [1, 13, 128, 700])
def test_oracle_bf16_matches_independent_order(orc, kind, k):
    x = make_rows(kind, 5, 3001, seed=k * 7 + len(kind))
    ev, ei = numpy_topk_bf16(x, k)
    for method in (0, 1):
        gv, gi = orc.topk(x, k, method=method, bf16=True)
        assert_exact(gv, gi, ev, ei, f"{kind} k={k} method={method}")


def test_oracle_bf16_values_match_torch_topk(orc):
    import torch

    x = make_rows("normal", 4, 5000, seed=3)
    t = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16)
    tv = torch.topk(t.float(), 50, dim=1).values.numpy()
    gv, _ = orc.topk(x, 50, bf16=True)
    np.testing.assert_array_equal(bf16_to_f32(gv), tv)


def test_oracle_bf16_csr_pads_with_bf16_neg_inf(orc):
    x = make_rows("normal", 1, 40, seed=5).reshape(-1)
    off = np.array([0, 0, 3, 40], np.int64)
    gv, gi = orc.topk_csr(x, off, 5, bf16=True)
    assert (gi[0] == -1).all() and (gv[0] == NEG_INF_BF16).all()
    assert (gi[1, 3:] == -1).all() and (gv[1, 3:] == NEG_INF_BF16).all()
    ev, ei = numpy_topk_bf16(x[3:40][None, :], 5)
    assert_exact(gv[2:3], gi[2:3], ev, ei, "csr row 2")


def test_bf16_entry_points_keep_the_argument_contract():
    """Shapes and sizes as the fp16 entry points; bad arguments rejected on the host."""
    import batch_topk_b200 as bt

    for shape in [(4, 151936, 50), (1, 10, 10), (1024, 262144, 1024)]:
        assert bt.batch_topk_bf16_workspace_size(*shape) == bt.batch_topk_half_workspace_size(*shape)
    assert bt.batch_topk_bf16_workspace_size(1, 10, 11) == 0
    assert bt.batch_topk_bf16_segmented_workspace_size(8, 1000, 50) == \
        bt.batch_topk_half_segmented_workspace_size(8, 1000, 50)
    fake = 1 << 20
    inv = bt.CUDA_ERROR_INVALID_VALUE
    assert bt.batch_topk_bf16(fake, 0, 100, 5, fake, fake, fake, 1 << 30) == inv   # seg_num
    assert bt.batch_topk_bf16(fake, 1, 100, 101, fake, fake, fake, 1 << 30) == inv  # k > len
    assert bt.batch_topk_bf16(0, 1, 100, 5, fake, fake, fake, 1 << 30) == inv      # null input
    assert bt.batch_topk_bf16(fake, 1, 100, 5, fake, fake, fake, 16) == inv        # workspace
    assert bt.batch_topk_bf16_segmented(fake, 0, 2, 100, 5, fake, fake, fake, 1 << 30) == inv


# ---- GPU: the CUDA path against the checker ------------------------------------------------

SHAPES = [(4, 1000), (16, 32000), (3, 151936), (2, 300001)]
CASES = [(s, k) for s in SHAPES for k in (1, 50, 128, 129, 1024) if k <= s[1]]


@pytest.mark.gpu
@pytest.mark.parametrize("shape,k", CASES, ids=[f"{r}x{n}-k{k}" for (r, n), k in CASES])
@pytest.mark.parametrize("misalign", [0, 3])
def test_bf16_normal_rows(orc, shape, k, misalign):
    rows, n = shape
    x = make_rows("normal", rows, n, seed=rows * 31 + k)
    ev, ei = orc.topk(x, k, bf16=True)
    gv, gi = gpu_topk(x, k, misalign=misalign, bf16=True)
    assert_exact(gv, gi, ev, ei, f"bf16 {shape} k={k} misalign={misalign}")


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["bits", "levels", "specials"])
@pytest.mark.parametrize("k", [1, 50, 300])
def test_bf16_special_rows(orc, kind, k):
    x = make_rows(kind, 6, 40000, seed=k + 11)
    ev, ei = orc.topk(x, k, bf16=True)
    gv, gi = gpu_topk(x, k, misalign=5, bf16=True)
    assert_exact(gv, gi, ev, ei, f"bf16 {kind} k={k}")


@pytest.mark.gpu
@pytest.mark.parametrize("rows", ["all_nan", "all_equal", "ascending", "descending", "zeros"])
def test_bf16_degenerate_rows(orc, rows):
    n = 20000
    if rows == "all_nan":
        x = np.full((2, n), 0x7FC0, np.uint16)
    elif rows == "all_equal":
        x = np.full((2, n), 0x4040, np.uint16)
    elif rows == "zeros":
        x = np.where(np.arange(n) % 2 == 0, 0x0000, 0x8000).astype(np.uint16)[None, :].repeat(2, 0)
    else:
        v = np.sort(np.random.default_rng(1).standard_normal(n).astype(np.float32))
        if rows == "descending":
            v = v[::-1].copy()
        x = f32_to_bf16(v)[None, :].repeat(2, 0)
    for k in (1, 50, 1000):
        ev, ei = orc.topk(x, k, bf16=True)
        gv, gi = gpu_topk(x, k, bf16=True)
        assert_exact(gv, gi, ev, ei, f"bf16 {rows} k={k}")


@pytest.mark.gpu
@pytest.mark.parametrize("k", [8, 50, 256])
def test_bf16_csr(orc, k):
    rng = np.random.default_rng(k)
    lens = np.concatenate([[0, 1, k - 1, k], rng.integers(1, 70000, 60)])
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    x = f32_to_bf16(rng.uniform(-1, 1, int(off[-1])).astype(np.float32))
    ev, ei = orc.topk_csr(x, off, k, bf16=True)
    gv, gi = gpu_topk_csr(x, off, k, misalign=1, bf16=True)
    assert_exact(gv, gi, ev, ei, f"bf16 csr k={k}")
    assert (gv[0] == NEG_INF_BF16).all() and (gi[0] == -1).all()


@pytest.mark.gpu
def test_bf16_tie_heavy_block(orc):
    """C3's shape and tie structure in bf16: 256 levels with +-0, k=50, 64 rows."""
    x = make_rows("levels", 64, 151936, seed=9)
    ev, ei = orc.topk(x, 50, bf16=True)
    gv, gi = gpu_topk(x, 50, bf16=True)
    assert_exact(gv, gi, ev, ei, "bf16 tie-heavy")


@pytest.mark.gpu
def test_bf16_torch_op_matches_torch_topk_values():
    import torch

    import batch_topk_b200.torch_api  # noqa: F401  (registers the operators)

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn((32, 100000), device="cuda", generator=g).to(torch.bfloat16)
    v, i = torch.ops.batch_topk_b200.topk(x, 64)
    assert v.dtype == torch.bfloat16 and i.dtype == torch.int32
    tv = torch.topk(x.float(), 64, dim=1).values
    assert torch.equal(v.float(), tv)
    assert torch.equal(x.gather(1, i.long()), v)
