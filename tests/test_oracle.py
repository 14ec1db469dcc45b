"""The checker (oracle/) pinned against the reference's known answers, fixtures and own code.

Known answers restate the reference's CPU- and GPU-unit checks of
test/test_batch_topk.cu (fire-emblem/batch_topk):
  :19-25 ordering, :27-36 NaN ordering, :38-44 bounded length, :46-51 codec, :53-64 tie
  rule, :66-74 boundary state, :169-183 cutoff state, :187-201 sentinel state,
  :203-234 histogram bins.
Fixtures (tests/golden/*.npz) hold the reference cpu_reference_topk's own outputs.  Where
oracle/_ref (the reference's header compiled here) is present, the oracle is also compared
with it on seeded random cases.  No GPU needed.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import ref_generators as rg
from batch_topk_b200 import workloads as wl
from util import load_npz, sha


def h(vals) -> np.ndarray:
    return np.asarray(vals, np.float32).astype(np.float16).view(np.uint16)


def desc(x: float) -> int:
    return int(oracle.encode_desc(h([x]))[0])


# ---- codec: include/type_codec.cuh:13-38 ----------------------------------------------

def test_codec_known_keys(orc):
    cases = {np.inf: 0x03FF, -np.inf: 0xFC00, 1.0: 0x43FF, 1.999: 0x4000, 0.0: 0x7FFF,
             -0.0: 0x7FFF}
    for v, key in cases.items():
        assert desc(v) == key, v
        assert orc.lib.oracle_encode_desc(int(h([v])[0])) == key
    for nan_bits in (0x7C01, 0x7E00, 0x7FFF, 0xFC01, 0xFFFF):
        assert int(oracle.encode_desc(np.array([nan_bits], np.uint16))[0]) == 0xFFFF
        assert orc.lib.oracle_encode_desc(nan_bits) == 0xFFFF


def test_codec_special_order():
    """test/test_batch_topk.cu:46-51: desc(3) < desc(-1) < desc(NaN)."""
    assert desc(3.0) < desc(-1.0) < int(oracle.encode_desc(np.array([0x7E00], np.uint16))[0])


def test_codec_is_monotone_over_all_half_patterns(orc):
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    f = bits.view(np.float16).astype(np.float64)
    key = oracle.encode_desc(bits)
    num = ~np.isnan(f)
    order = np.argsort(-f[num], kind="stable")
    ks = key[num][order].astype(np.int64)
    assert np.all(np.diff(ks) >= 0)
    # equal numbers (only +0/-0 among distinct patterns) share a key; distinct ones do not
    fs = f[num][order]
    assert np.all((np.diff(ks) == 0) == (np.diff(fs) == 0))
    assert np.all(key[~num] == 0xFFFF) and ks.max() < 0xFFFF
    c_keys = np.array([orc.lib.oracle_encode_desc(int(b)) for b in bits[::97]], np.uint16)
    assert np.array_equal(c_keys, key[::97])


# ---- ordering: include/batch_topk_types.cuh:50-113 ---------------------------------------

@pytest.mark.parametrize("method", [oracle.METHOD_SORT, oracle.METHOD_COUNT])
def test_reference_ordering(orc, method):
    v, i = orc.topk(h([[5, 7, 7, 1]]), 2, method=method)
    assert i.tolist() == [[1, 2]] and v.tolist() == [h([7, 7]).tolist()]


@pytest.mark.parametrize("method", [oracle.METHOD_SORT, oracle.METHOD_COUNT])
def test_reference_nan_ordering(orc, method):
    x = h([[np.nan, 3, -1, np.nan]])
    v, i = orc.topk(x, 3, method=method)
    assert i.tolist() == [[1, 2, 0]]
    assert v[0, 2] == x[0, 0]  # the NaN's own bits come back


def test_reference_bounded_length_pads(orc):
    """:38-44: k > len returns min(k, len) entries; the CSR entry pads with -inf / -1."""
    v, i = orc.topk_csr(h([2, 1]), np.array([0, 2]), 4)
    assert i.tolist() == [[0, 1, -1, -1]]
    assert v.tolist() == [[int(h([2])[0]), int(h([1])[0]), 0xFC00, 0xFC00]]


def test_candidate_tie_rule(orc):
    """:53-64: equal values go to the lower index; -0 ties +0."""
    _, i = orc.topk(h([[1, 5, 5, 0]]), 1)
    assert i.tolist() == [[1]]
    x = np.array([[0x8000, 0x0000, 0x8000]], np.uint16)
    v, i = orc.topk(x, 3)
    assert i.tolist() == [[0, 1, 2]] and v.tolist() == x.tolist()


# ---- radix select state: src/radix_boundary_select.cuh, src/radix_histogram.cuh --------

NINE_TO_TWO = h([9, 8, 7, 6, 5, 4, 3, 2])


def test_boundary_state(orc):
    """:66-74 and :169-183: values 9..2, k=3."""
    st = orc.select_state(NINE_TO_TWO, 3)
    assert st["selected_count"] == 2 and st["live_count"] == 1
    assert st["boundary_digit"] == 56 and st["prefix"] == 0x3800 and st["prefix_mask"] == 0xFF00
    assert st["strictly_better_count"] == 2 and st["remaining_slots"] == 1
    assert st["cutoff_key"] == desc(7.0)


def test_boundary_state_sentinel(orc):
    """:187-201: k > len forces the sentinel state."""
    st = orc.select_state(NINE_TO_TWO, 9)
    assert (st["prefix"], st["prefix_mask"], st["cutoff_key"]) == (0xFFFF, 0xFFFF, 0xFFFF)
    assert st["live_count"] == 0 and st["boundary_digit"] == 255
    assert st["strictly_better_count"] == 8 and st["remaining_slots"] == 1


def test_histogram_pass(orc):
    """:203-234: high-digit bins, then the low digit filtered by the boundary prefix."""
    hist = orc.histogram_pass(NINE_TO_TWO, 8, 0, 0)
    expect = np.zeros(256, np.uint32)
    for b, c in {55: 2, 56: 1, 57: 1, 58: 1, 59: 1, 61: 1, 63: 1}.items():
        expect[b] = c
    assert np.array_equal(hist, expect)
    st = orc.select_state(NINE_TO_TWO, 3)
    low = orc.histogram_pass(NINE_TO_TWO, 0, st["prefix"], st["prefix_mask"])
    assert low[255] == 1 and low.sum() == 1


def test_select_state_matches_reference(ref_orc, orc):
    """simulate_radix_boundary (src/radix_select_state.cuh:9-51) fills the high-digit fields;
    the cutoff fields are pinned by the known answers above."""
    rng = np.random.default_rng(5)
    for trial in range(40):
        n = int(rng.integers(1, 400))
        x = rng.integers(0, 1 << 16, n, dtype=np.uint32).astype(np.uint16)
        if trial % 3 == 0:
            x = x[rng.integers(0, 8, n)]  # heavy ties
        k = int(rng.integers(1, n + 1))
        mine, theirs = orc.select_state(x, k), ref_orc.simulate_radix_boundary(x, k)
        for key in ("prefix", "prefix_mask", "selected_count", "live_count", "boundary_digit"):
            assert mine[key] == theirs[key], (trial, key)


# ---- fixtures computed by the reference's own cpu_reference_topk --------------------------

def _check_against(orc, x, k, exp_i, exp_fv, offsets=None):
    for method in (oracle.METHOD_SORT, oracle.METHOD_COUNT):
        if offsets is None:
            v, i = orc.topk(x, k, method=method)
        else:
            v, i = orc.topk_csr(x, offsets, k, method=method)
        assert np.array_equal(i, exp_i), f"indices differ (method {method})"
        got = v.view(np.float16).astype(np.float32)
        valid = exp_i >= 0
        same = (got == exp_fv) | (np.isnan(got) & np.isnan(exp_fv))
        assert np.all(same[valid]), f"values differ (method {method})"


@pytest.mark.parametrize("name,build,k", rg.REFERENCE_CASES, ids=[c[0] for c in rg.REFERENCE_CASES])
def test_oracle_matches_reference_fixture(orc, name, build, k):
    gold = load_npz("reference_cases.npz")
    x = build()
    assert sha(x) == str(gold[f"{name}/sha256"])
    _check_against(orc, x, k, gold[f"{name}/indices"], gold[f"{name}/values"])


@pytest.mark.parametrize("name", ["C1_full", "C2_rows0-7", "C3_rows0-15", "C4_segs0-63_k8",
                                  "C4_segs0-63_k256", "C5_rows0-5"])
def test_oracle_matches_config_fixture(orc, name):
    gold = load_npz("config_cases.npz")
    off = None
    if name == "C1_full":
        x = wl.gen_c1()
    elif name == "C2_rows0-7":
        x = wl.gen_c2(rows=slice(0, 8))
    elif name == "C3_rows0-15":
        x = wl.gen_c3(rows=slice(0, 16))
    elif name == "C5_rows0-5":
        x = wl.gen_c5(rows=slice(0, 6))
    else:
        off = gold[f"{name}/offsets"]
        assert np.array_equal(off, wl.c4_offsets()[:65])
        x = wl.gen_c4_range(0, 64)
    assert sha(x) == str(gold[f"{name}/sha256"])
    _check_against(orc, x, int(gold[f"{name}/k"]), gold[f"{name}/indices"],
                   gold[f"{name}/values"], offsets=off)


# ---- the oracle against the reference's own code, seeded random cases -----------------------

@pytest.mark.parametrize("seed", range(6))
def test_oracle_matches_reference_code(ref_orc, orc, seed):
    rng = np.random.default_rng(100 + seed)
    seg_num, seg_len = int(rng.integers(1, 9)), int(rng.integers(1, 3000))
    kind = seed % 3
    if kind == 0:  # every bit pattern, NaNs and infinities included
        x = rng.integers(0, 1 << 16, (seg_num, seg_len), dtype=np.uint32).astype(np.uint16)
    elif kind == 1:  # a handful of levels, +0 / -0 among them
        lv = np.array([0x0000, 0x8000, 0x3C00, 0xBC00, 0x7C00, 0xFC00, 0x7E00, 0x4000], np.uint16)
        x = lv[rng.integers(0, lv.size, (seg_num, seg_len))]
    else:
        x = rng.standard_normal((seg_num, seg_len)).astype(np.float16).view(np.uint16)
    k = int(rng.integers(1, min(seg_len, 1024) + 1))
    exp_i, exp_v, _ = ref_orc.topk(x, k)
    _check_against(orc, x, k, exp_i, exp_v)


def test_generators_match_reference_code(ref_orc):
    """ref_generators.py restates the reference test's generators bit for bit."""
    for seg_num, seg_len, seed in ((1, 10000, 7), (3, 256, 2026), (2, 777, 1234)):
        assert np.array_equal(rg.make_random_input(seg_num, seg_len, seed),
                              ref_orc.make_random_input(seg_num, seg_len, seed))
    assert np.array_equal(rg.make_duplicate_heavy_input(4, 10000),
                          ref_orc.make_duplicate_heavy_input(4, 10000))
    assert np.array_equal(rg.make_special_values_input(2, 10000),
                          ref_orc.make_special_values_input(2, 10000))
