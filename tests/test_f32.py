"""float32 inputs (bt_topk_f32, bt_topk_f32_segmented).

The reference is fp16 only (other input types are a listed non-goal), so fp32 parity is anchored
on the checker's fp32 path (oracle/topk_oracle.c, *_f32: the reference's comparator on the float
values themselves, and a 32-bit descending key for the O(n) method).  That path is pinned on the
CPU two independent ways:
- an order built with numpy alone: NaN last, then larger value first (-0 == +0), then lower
  index;
- torch.topk's values.
The GPU tests compare the CUDA path with it bit for bit: the value bit patterns and the int32
indices, on random patterns (NaN payloads, infinities, subnormals, zeros of both signs), normal
values, tie-heavy levels, sorted and constant rows, misaligned inputs, k from 1 to 1024, and CSR
batches with empty and shorter-than-k segments.
"""
from __future__ import annotations

import numpy as np
import pytest

import batch_topk_b200 as bt

from util import _dev_copy32, assert_exact32

NEG_INF_F32 = 0xFF800000


def numpy_topk_f32(bits: np.ndarray, k: int):
    """Independent reference order, per row of uint32 bit patterns."""
    rows, n = bits.shape
    kk = min(k, n)
    idx = np.full((rows, k), -1, np.int32)
    val = np.full((rows, k), NEG_INF_F32, np.uint32)
    for r in range(rows):
        f = bits[r].view(np.float32)
        nan = np.isnan(f)
        with np.errstate(invalid="ignore"):
            neg = np.where(nan, 0.0, -f.astype(np.float64))
        order = np.lexsort((np.arange(n), neg, nan))[:kk]
        idx[r, :kk] = order
        val[r, :kk] = bits[r, order]
    return val, idx


def make_rows(kind: str, rows: int, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "normal":
        return rng.standard_normal((rows, n)).astype(np.float32).view(np.uint32)
    if kind == "bits":  # every kind of pattern: NaN payloads, infinities, subnormals, +-0
        return rng.integers(0, 1 << 32, (rows, n), dtype=np.uint64).astype(np.uint32)
    if kind == "levels":  # heavy ties: 64 levels with +0 and -0
        lv = rng.uniform(-4, 4, 64).astype(np.float32).view(np.uint32)
        lv[0], lv[1] = 0x00000000, 0x80000000
        return lv[rng.integers(0, 64, (rows, n))]
    if kind == "specials":
        pool = np.array([0x7FC00000, 0xFFC00001, 0x7F800000, 0xFF800000, 0x00000000, 0x80000000,
                         0x3F800000, 0xBF800000, 0x00000001, 0x80000001, 0x7F7FFFFF, 0xFF7FFFFF],
                        np.uint32)
        return pool[rng.integers(0, pool.size, (rows, n))]
    if kind == "sorted":
        x = np.sort(rng.standard_normal((rows, n)).astype(np.float32), axis=1)
        return x.view(np.uint32)
    if kind == "constant":
        return np.full((rows, n), np.float32(1.25).view(np.uint32), np.uint32)
    if kind == "uniform12":  # one exponent: the high key digits are constant
        return rng.uniform(1, 2, (rows, n)).astype(np.float32).view(np.uint32)
    raise ValueError(kind)


KINDS = ["normal", "bits", "levels", "specials", "sorted", "constant", "uniform12"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("k", [1, 5, 64, 300])
def test_checker_f32_matches_numpy(orc, kind, k):
    bits = make_rows(kind, 6, 2000, seed=len(kind) * 31 + k)
    exp_v, exp_i = numpy_topk_f32(bits, k)
    for method in (0, 1):
        v, i = orc.topk_f32(bits, k, method=method)
        assert np.array_equal(i, exp_i), (kind, k, method)
        assert np.array_equal(v, exp_v), (kind, k, method)


def test_checker_f32_matches_torch_topk_values(orc):
    import torch

    x = np.random.default_rng(3).standard_normal((8, 5000)).astype(np.float32)
    v, _ = orc.topk_f32(x.view(np.uint32), 40)
    tv, _ = torch.topk(torch.from_numpy(x), 40, dim=1)
    assert np.array_equal(v.view(np.float32), tv.numpy())


def test_f32_workspace_and_argument_contract():
    assert bt.batch_topk_f32_workspace_size(0, 100, 5) == 0
    assert bt.batch_topk_f32_workspace_size(4, 100, 101) == 0
    assert bt.batch_topk_f32_workspace_size(4, 100, bt.MAX_K + 1) == 0
    n16 = bt.batch_topk_half_workspace_size(1024, 151936, 50)
    n32 = bt.batch_topk_f32_workspace_size(1024, 151936, 50)
    assert n32 >= n16 > 0 and n32 % 256 == 0  # 4 values a 16-byte vector: more chunk slots
    fake = 1 << 20
    # misaligned (2-byte) input or output values are refused before any launch
    assert bt.batch_topk_f32(fake + 2, 4, 100, 5, fake, fake, fake, n32, 0) == bt.CUDA_ERROR_INVALID_VALUE
    assert bt.batch_topk_f32(fake, 4, 100, 5, fake + 2, fake, fake, n32, 0) == bt.CUDA_ERROR_INVALID_VALUE
    assert bt.batch_topk_f32_segmented_workspace_size(3, 1000, 50) > 0


SHAPES = [(8, 40000, 50), (3, 70001, 1), (300, 1000, 128), (16, 5000, 1024), (2, 262144, 1024),
          (64, 128256, 50), (1, 8, 8), (5, 33333, 256), (1024, 4096, 7)]


@pytest.mark.gpu
@pytest.mark.parametrize("seg_num,seg_len,k", SHAPES)
@pytest.mark.parametrize("kind", ["normal", "levels", "bits"])
def test_gpu_f32_shapes(orc, seg_num, seg_len, k, kind):
    bits = make_rows(kind, seg_num, seg_len, seed=seg_num * 13 + seg_len + k)
    got_v, got_i = gpu_topk32(bits, k, misalign=(seg_len % 3))
    exp_v, exp_i = orc.topk_f32(bits, k)
    assert_exact32(got_v, got_i, exp_v, exp_i, f"{kind} {seg_num}x{seg_len} k={k}")


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["specials", "sorted", "constant", "uniform12"])
@pytest.mark.parametrize("k", [1, 50, 129, 1024])
def test_gpu_f32_adversarial_rows(orc, kind, k):
    bits = make_rows(kind, 12, 70000, seed=k + len(kind))
    got_v, got_i = gpu_topk32(bits, k, misalign=1)
    exp_v, exp_i = orc.topk_f32(bits, k)
    assert_exact32(got_v, got_i, exp_v, exp_i, f"{kind} k={k}")


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 50, 300])
def test_gpu_f32_csr(orc, k):
    import torch

    rng = np.random.default_rng(k)
    lens = np.array([0, 1, 5, k - 1 if k > 1 else 0, k, k + 1, 9000, 0, 40000, 3, 16384, 16385],
                    np.int64)
    off = np.zeros(lens.size + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    vals = rng.standard_normal(int(off[-1])).astype(np.float32).view(np.uint32)
    vals[off[8]:off[8] + 100] = 0x7FC00000  # NaNs inside the long segment
    dev = torch.device("cuda:0")
    _buf, x = _dev_copy32(torch, vals, 3, dev)
    d_off = torch.from_numpy(off.astype(np.int32)).to(dev)
    seg_num, total = lens.size, int(off[-1])
    nbytes = bt.batch_topk_f32_segmented_workspace_size(seg_num, total, k)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev).fill_(0xA5)
    ov = torch.full((seg_num, k), 0x1234, dtype=torch.int32, device=dev)
    oi = torch.full((seg_num, k), -7, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev)
    rc = bt.batch_topk_f32_segmented(x.data_ptr(), d_off.data_ptr(), seg_num, total, k,
                                     ov.data_ptr(), oi.data_ptr(), ws.data_ptr(), nbytes,
                                     s.cuda_stream)
    assert rc == 0
    s.synchronize()
    assert bt.workspace_status(ws.data_ptr(), seg_num, s.cuda_stream)[0] == 0
    exp_v, exp_i = orc.topk_csr_f32(vals, off, k)
    assert_exact32(ov.cpu().numpy().view(np.uint32), oi.cpu().numpy(), exp_v, exp_i, f"csr k={k}")


@pytest.mark.gpu
def test_gpu_f32_torch_op_matches_torch_topk(orc):
    import torch

    import batch_topk_b200.torch_api  # noqa: F401  (registers the operators)

    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(64, 128256, device="cuda", generator=g)
    v, i = torch.ops.batch_topk_b200.topk(x, 50)
    tv, _ = torch.topk(x, 50, dim=1)
    assert v.dtype == torch.float32 and torch.equal(v, tv)
    exp_v, exp_i = orc.topk_f32(x.cpu().numpy().view(np.uint32), 50)
    assert np.array_equal(i.cpu().numpy(), exp_i)


def gpu_topk32(bits: np.ndarray, k: int, misalign: int = 0):
    """Fixed-length fp32 top-k on cuda:0 through bt_topk_f32; (value bits, indices)."""
    import torch

    dev = torch.device("cuda:0")
    seg_num, seg_len = bits.shape
    _buf, x = _dev_copy32(torch, bits, misalign, dev)
    nbytes = bt.batch_topk_f32_workspace_size(seg_num, seg_len, k)
    assert nbytes > 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev).fill_(0xA5)
    ov = torch.full((seg_num, k), 0x1234, dtype=torch.int32, device=dev)
    oi = torch.full((seg_num, k), -7, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev)
    rc = bt.batch_topk_f32(x.data_ptr(), seg_num, seg_len, k, ov.data_ptr(), oi.data_ptr(),
                           ws.data_ptr(), nbytes, s.cuda_stream)
    assert rc == 0, f"bt_topk_f32 returned {rc}"
    s.synchronize()
    flags, _ = bt.workspace_status(ws.data_ptr(), seg_num, s.cuda_stream)
    assert flags == 0, f"device status flags {flags}"
    return ov.cpu().numpy().view(np.uint32), oi.cpu().numpy()
