"""Bit-exact parity of the CUDA path (through the C ABI) against the reference's CPU top-k.

Expected outputs come from (a) golden fixtures computed by the reference's own
cpu_reference_topk (tests/golden/make_golden.py) and (b) the C restatement in oracle/,
which tests/test_oracle.py pins against the reference.  Values are compared as raw fp16
bits and indices as int32, so NaN payloads and -0/+0 are checked too.
"""
from __future__ import annotations

import numpy as np
import pytest

import ref_generators as rg
from batch_topk_b200 import workloads as wl
from util import assert_exact, expected_from_indices, gpu_topk, gpu_topk_csr, load_npz, sha

pytestmark = pytest.mark.gpu


# ---- the reference's own end-to-end test inputs, expected = reference cpu_reference_topk --

@pytest.mark.parametrize("name,build,k", rg.REFERENCE_CASES, ids=[c[0] for c in rg.REFERENCE_CASES])
@pytest.mark.parametrize("misalign", [0, 3])
def test_reference_cases(name, build, k, misalign):
    gold = load_npz("reference_cases.npz")
    x = build()
    assert sha(x) == str(gold[f"{name}/sha256"]), "regenerated input differs from the fixture"
    exp_i = gold[f"{name}/indices"]
    exp_v = expected_from_indices(x, exp_i)
    got_v, got_i = gpu_topk(x, k, misalign=misalign)
    assert_exact(got_v, got_i, exp_v, exp_i, name)


def _config_inputs(name):
    if name == "C1_full":
        return wl.gen_c1(), None
    if name == "C2_rows0-7":
        return wl.gen_c2(rows=slice(0, 8)), None
    if name == "C3_rows0-15":
        return wl.gen_c3(rows=slice(0, 16)), None
    if name.startswith("C4_"):
        vals, off = wl.gen_c4()
        sub = off[:65]
        return vals[: sub[-1]], sub
    if name == "C5_rows0-5":
        return wl.gen_c5(rows=slice(0, 6)), None
    raise KeyError(name)


CONFIG_CASES = ["C1_full", "C2_rows0-7", "C3_rows0-15", "C4_segs0-63_k1", "C4_segs0-63_k8",
                "C4_segs0-63_k50", "C4_segs0-63_k256", "C5_rows0-5"]


@pytest.mark.parametrize("name", CONFIG_CASES)
def test_config_golden(name):
    gold = load_npz("config_cases.npz")
    x, off = _config_inputs(name)
    assert sha(x) == str(gold[f"{name}/sha256"]), "regenerated input differs from the fixture"
    k = int(gold[f"{name}/k"])
    exp_i = gold[f"{name}/indices"]
    if off is None:
        exp_v = expected_from_indices(x, exp_i)
        got_v, got_i = gpu_topk(x, k)
    else:
        rows = [x[off[s]:off[s + 1]] for s in range(off.size - 1)]
        exp_v = expected_from_indices(rows, exp_i)
        got_v, got_i = gpu_topk_csr(x, off, k)
    assert_exact(got_v, got_i, exp_v, exp_i, name)


# ---- full-size configurations against the C restatement -------------------------------

@pytest.mark.parametrize("cfg", ["C1", "C2", "C3"])
def test_config_full(orc, cfg):
    x, _, k = wl.generate(cfg)
    exp_v, exp_i = orc.topk(x, k)
    got_v, got_i = gpu_topk(x, k)
    assert_exact(got_v, got_i, exp_v, exp_i, cfg)


@pytest.mark.parametrize("k", wl.C4_K_VALUES)
def test_config_c4_full(orc, k):
    vals, off = wl.gen_c4()
    exp_v, exp_i = orc.topk_csr(vals, off, k)
    got_v, got_i = gpu_topk_csr(vals, off, k)
    assert_exact(got_v, got_i, exp_v, exp_i, f"C4 k={k}")


def test_config_c5_rows(orc):
    x = wl.gen_c5(rows=slice(0, 48))
    exp_v, exp_i = orc.topk(x, 1024)
    got_v, got_i = gpu_topk(x, 1024)
    assert_exact(got_v, got_i, exp_v, exp_i, "C5 rows 0-47")


# ---- shapes, alignments and k across every dispatch branch ------------------------------

SHAPES = [
    (3, 1, 1), (5, 7, 3), (4, 8, 8), (4, 9, 5), (6, 100, 50), (3, 1000, 128), (2, 1000, 1000),
    (4, 16383, 50), (4, 16384, 64), (4, 16385, 65), (3, 32771, 129), (2, 100000, 256),
    (2, 100003, 257), (2, 70001, 1024), (9, 10000, 50), (1, 262144, 1024), (300, 2000, 16),
]


@pytest.mark.parametrize("seg_num,seg_len,k", SHAPES)
@pytest.mark.parametrize("misalign", [0, 1, 5])
def test_shapes_random(orc, seg_num, seg_len, k, misalign):
    rng = np.random.default_rng(seg_num * 1000003 + seg_len * 7 + k)
    x = rng.standard_normal((seg_num, seg_len)).astype(np.float16).view(np.uint16)
    exp_v, exp_i = orc.topk(x, k)
    got_v, got_i = gpu_topk(x, k, misalign=misalign)
    assert_exact(got_v, got_i, exp_v, exp_i, f"{seg_num}x{seg_len} k={k} +{misalign}")


def _special_rows(seg_len, rng):
    rows = []
    rows.append(np.full(seg_len, 0x3C00, np.uint16))                       # all equal (1.0)
    rows.append(np.full(seg_len, 0x7E00, np.uint16))                       # all NaN
    r = rng.standard_normal(seg_len).astype(np.float16).view(np.uint16)
    r[rng.random(seg_len) < 0.995] = 0x7FFF                                 # NaN-heavy
    rows.append(r)
    r = np.where(rng.random(seg_len) < 0.5, 0x0000, 0x8000).astype(np.uint16)  # +0/-0 only
    rows.append(r)
    r = rng.choice(np.array([0x7C00, 0xFC00, 0x3C00, 0xBC00, 0x0001, 0x8001], np.uint16), seg_len)
    rows.append(r)                                                          # +-inf, +-1, subnormals
    v = np.sort(rng.standard_normal(seg_len)).astype(np.float16).view(np.uint16)
    rows.append(v)                                                          # ascending
    rows.append(v[::-1].copy())                                             # descending
    rows.append(rng.integers(0, 4, seg_len).astype(np.float16).view(np.uint16))  # 4 levels
    r = rng.integers(0, 0x10000, seg_len, dtype=np.uint32).astype(np.uint16)  # every bit pattern
    rows.append(r)
    r = np.full(seg_len, 0xFC00, np.uint16)
    r[rng.integers(0, seg_len, 3)] = 0x7FFF                                 # -inf with a few NaN
    rows.append(r)
    return np.stack(rows)


@pytest.mark.parametrize("seg_len,k", [(64, 50), (1000, 50), (20000, 50), (50000, 1024),
                                       (40000, 200), (16384, 1), (300, 257)])
def test_special_values(orc, seg_len, k):
    rng = np.random.default_rng(seg_len + k)
    x = _special_rows(seg_len, rng)
    exp_v, exp_i = orc.topk(x, k)
    got_v, got_i = gpu_topk(x, k, misalign=1)
    assert_exact(got_v, got_i, exp_v, exp_i, f"special len={seg_len} k={k}")


# ---- CSR -------------------------------------------------------------------------------

@pytest.mark.parametrize("k", [1, 8, 50, 256, 1024])
def test_csr_ragged(orc, k):
    rng = np.random.default_rng(k)
    lens = np.concatenate([[0, 1, 2, 7, 8, 9, 0, 0, k - 1 if k > 1 else 0, k, k + 1, 16384, 16385,
                            40000, 0], rng.integers(0, 70000, 40)])
    off = np.zeros(lens.size + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    vals = rng.standard_normal(int(off[-1])).astype(np.float16).view(np.uint16)
    vals[rng.random(vals.size) < 0.01] = 0x7FFF
    exp_v, exp_i = orc.topk_csr(vals, off, k)
    for mis in (0, 3):
        got_v, got_i = gpu_topk_csr(vals, off, k, misalign=mis)
        assert_exact(got_v, got_i, exp_v, exp_i, f"csr k={k} +{mis}")


def test_csr_nonzero_first_offset(orc):
    rng = np.random.default_rng(5)
    vals = rng.standard_normal(50000).astype(np.float16).view(np.uint16)
    off = np.array([1000, 1000, 5000, 5001, 30000, 49999], np.int64)
    exp_v, exp_i = orc.topk_csr(vals, off, 50)
    got_v, got_i = gpu_topk_csr(vals, off, 50)
    assert_exact(got_v, got_i, exp_v, exp_i, "csr offset0=1000")


# ---- repeatability: the workspace carries nothing between calls --------------------------

def test_repeat_calls_same_workspace(orc):
    import torch

    import batch_topk_b200 as bt

    dev = torch.device("cuda:0")
    rng = np.random.default_rng(11)
    ws = None
    for seg_len, k in [(30000, 50), (30000, 1024), (500, 3), (30000, 50)]:
        x = rng.standard_normal((16, seg_len)).astype(np.float16).view(np.uint16)
        nbytes = bt.batch_topk_half_workspace_size(16, seg_len, k)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 1 << 22), dtype=torch.uint8, device=dev)
        xt = torch.from_numpy(x.view(np.int16)).to(dev)
        ov = torch.empty((16, k), dtype=torch.int16, device=dev)
        oi = torch.empty((16, k), dtype=torch.int32, device=dev)
        rc = bt.batch_topk_half(xt.data_ptr(), 16, seg_len, k, ov.data_ptr(), oi.data_ptr(),
                                ws.data_ptr(), ws.numel(), 0)
        assert rc == 0
        torch.cuda.synchronize()
        exp_v, exp_i = orc.topk(x, k)
        assert_exact(ov.cpu().numpy().view(np.uint16), oi.cpu().numpy(), exp_v, exp_i,
                     f"repeat {seg_len} {k}")


def test_torch_api_matches_torch_topk():
    """Values agree with torch.topk on NaN-free data (torch's tie order is unspecified)."""
    import torch

    from batch_topk_b200.torch_api import topk

    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(64, 128256, device="cuda", generator=g).half()
    v, i = topk(x, 50)
    tv, _ = torch.topk(x.float(), 50, dim=1)
    assert torch.equal(v.float(), tv)
    assert torch.equal(torch.gather(x, 1, i.long()), v)


def test_back_to_back_calls_without_sync(orc):
    """Calls queued back to back on one stream, sharing a workspace, with kernels that rewrite
    the input in between and no host synchronisation until the end.  Each call's set-up kernel
    is launched early behind the previous kernel and waits for it: every result must match the
    checker on the input as it was at that call (snapshots are taken in stream order)."""
    import torch

    import batch_topk_b200 as bt

    dev = torch.device("cuda:0")
    s = torch.cuda.current_stream(dev)
    rng = np.random.default_rng(21)
    seg_num, seg_len = 64, 40000
    xt = torch.from_numpy(rng.standard_normal((seg_num, seg_len)).astype(np.float16)).to(dev)
    off = np.linspace(0, seg_num * seg_len, 9).astype(np.int64)  # 8 CSR segments, same buffer
    d_off = torch.from_numpy(off.astype(np.int32)).to(dev)
    total = seg_num * seg_len
    plan = [("fixed", 50), ("neg", 0), ("fixed", 1024), ("csr", 50), ("scale", 0), ("fixed", 8),
            ("csr", 300), ("fixed", 50)]
    need = max(bt.batch_topk_half_workspace_size(seg_num, seg_len, 1024),
               bt.batch_topk_half_segmented_workspace_size(8, total, 300))
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    ws.fill_(0xA5)
    runs = []
    for op, k in plan:
        if op == "neg":
            xt.neg_()
            continue
        if op == "scale":
            xt.mul_(0.5)
            continue
        snap = xt.clone()
        rows = seg_num if op == "fixed" else 8
        ov = torch.empty((rows, k), dtype=torch.int16, device=dev)
        oi = torch.empty((rows, k), dtype=torch.int32, device=dev)
        if op == "fixed":
            rc = bt.batch_topk_half(xt.data_ptr(), seg_num, seg_len, k, ov.data_ptr(),
                                    oi.data_ptr(), ws.data_ptr(), ws.numel(), s.cuda_stream)
        else:
            rc = bt.batch_topk_half_segmented(xt.data_ptr(), d_off.data_ptr(), 8, total, k,
                                              ov.data_ptr(), oi.data_ptr(), ws.data_ptr(),
                                              ws.numel(), s.cuda_stream)
        assert rc == 0
        runs.append((op, k, snap, ov, oi))
    torch.cuda.synchronize(dev)
    for n, (op, k, snap, ov, oi) in enumerate(runs):
        bits = snap.cpu().numpy().view(np.uint16)
        if op == "fixed":
            exp_v, exp_i = orc.topk(bits, k)
        else:
            exp_v, exp_i = orc.topk_csr(bits.reshape(-1), off, k)
        assert_exact(ov.cpu().numpy().view(np.uint16), oi.cpu().numpy(), exp_v, exp_i,
                     f"call {n} ({op}, k={k})")


def _rising_rows(seg_num, seg_len, seed):
    """Rows whose values climb chunk after chunk (the k > 128 path probes such a segment's last
    chunk out of turn), cycling over several kinds, one seed per row."""
    rows = np.empty((seg_num, seg_len), np.uint16)
    for i in range(seg_num):
        rng = np.random.default_rng(seed + i)
        kind = i % 6
        if kind == 0:  # ascending N(0,1): fp16 ties near zero
            r = np.sort(rng.standard_normal(seg_len)).astype(np.float16)
        elif kind == 1:  # ascending plateaus: 64 levels
            r = np.sort(rng.integers(0, 64, seg_len)).astype(np.float16)
        elif kind == 2:  # ascending, then the last stretch falls: the probe's threshold is loose
            r = np.sort(rng.standard_normal(seg_len)).astype(np.float16)
            r[-(seg_len // 5):] = -r[-(seg_len // 5):]
        elif kind == 3:  # rising sawtooth: each 16384-value stretch ascends, every stretch higher
            t = (np.arange(seg_len) % 16384) / 16384.0 + np.arange(seg_len) // 16384
            r = t.astype(np.float16)
        elif kind == 4:  # ascending, the tail one repeated value (ties with the probe's certificate)
            r = np.sort(rng.standard_normal(seg_len)).astype(np.float16)
            r[-3000:] = r[-3000]
        else:  # ascending with NaNs and -inf sprinkled in
            r = np.sort(rng.standard_normal(seg_len)).astype(np.float16)
            r[rng.random(seg_len) < 0.01] = np.float16(np.nan)
            r[rng.random(seg_len) < 0.01] = np.float16(-np.inf)
        rows[i] = r.view(np.uint16)
    return rows


@pytest.mark.parametrize("seg_len,k", [(70001, 129), (70001, 300), (131072, 513), (262144, 1024)])
@pytest.mark.parametrize("misalign", [0, 3])
def test_rising_rows_large_k(orc, seg_len, k, misalign):
    # at least as many rows as resident blocks, so each block takes whole segments (the
    # out-of-turn probe of a rising segment's last chunk happens on whole segments only)
    x = _rising_rows(300, seg_len, 7 * seg_len + k)
    exp_v, exp_i = orc.topk(x, k)
    got_v, got_i = gpu_topk(x, k, misalign=misalign)
    assert_exact(got_v, got_i, exp_v, exp_i, f"rising 300x{seg_len} k={k} +{misalign}")


def _tail_rows(seg_num, seg_len, seed):
    """More rows than resident blocks (so blocks take whole rows and, once every row is
    claimed, idle blocks help the last ones), of uneven cost: heavy ties on a few levels (the
    helper's and the owner's lists hold ties at the cutoff that only the index order ranks),
    i.i.d. N(0,1), ascending rows, and constant rows."""
    rows = np.empty((seg_num, seg_len), np.uint16)
    for i in range(seg_num):
        rng = np.random.default_rng(seed + i)
        kind = i % 4
        if kind == 0:
            r = rng.integers(0, 16, seg_len).astype(np.float16)
        elif kind == 1:
            r = rng.standard_normal(seg_len).astype(np.float16)
        elif kind == 2:
            r = np.sort(rng.standard_normal(seg_len)).astype(np.float16)
        else:
            r = np.full(seg_len, 1.5, np.float16)
        rows[i] = r.view(np.uint16)
    return rows


@pytest.mark.parametrize("k", [50, 256, 1024])
@pytest.mark.parametrize("misalign", [0, 3])
def test_tail_helpers(orc, k, misalign):
    # 600 rows of 20 chunks (k > 128 helpers need 12 unclaimed): the last rows claimed are
    # shared with blocks that ran dry, whose chunks interleave with the owner's; the split merge
    # and the shared thresholds must give the single-block answer bit for bit
    seg_len = 20 * 16384 - 5
    x = _tail_rows(600, seg_len, 31 * k + misalign)
    exp_v, exp_i = orc.topk(x, k)
    got_v, got_i = gpu_topk(x, k, misalign=misalign)
    assert_exact(got_v, got_i, exp_v, exp_i, f"tail 600x{seg_len} k={k} +{misalign}")
