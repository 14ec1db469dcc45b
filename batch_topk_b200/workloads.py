"""Seeded synthetic inputs for the five benchmark configurations.

Every value is a pure function of (seed, stream, element index), using a counter-based
splitmix64 generator, so any shard of rows can be generated on its own.  The normal draws
use Box-Muller in double precision, with ln and cos written as fixed polynomial sequences
of IEEE add/multiply/divide/sqrt.  That makes the bits identical on every host, with no
dependence on a libm.  Values are rounded to fp16 with round-to-nearest-even.

Configurations (fp16 bit patterns are returned as uint16):

  C1  4 x 32000, N(0,1), k=50.
  C2  64 x 128256, N(0, sigma=2); each entry -inf with p=0.05; then 20 distinct positions
      per row set to U(8,12), overriding the mask; k=50.
  C3  1024 x 151936; a table of 256 fp16 levels drawn from U[-4,4] holding both +0 and -0;
      every element picks a level uniformly; k=50.
  C4  4096 CSR segments with lengths U{1..262144}, int32 offsets, U(-1,1); k from
      {1, 8, 50, 256}.
  C5  8192 x 262144, k=1024; row r has type r % 3: (a) one constant per row; (b) N(0,1)
      sorted ascending; (c) U[1,2), where the high radix digit is constant.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

_GOLD = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_LN2 = 0.6931471805599453
_TWO_PI = 6.283185307179586


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def rand_u64(seed: int, stream: int, index: np.ndarray) -> np.ndarray:
    """splitmix64 of (seed, stream) keyed counter; index is an int64/uint64 array."""
    with np.errstate(over="ignore"):
        key = _mix64(np.array([(seed * 0x100000001B3 + stream * 0x9E3779B1 + 1) & (2**64 - 1)],
                              dtype=np.uint64))[0]
        z = key + (np.asarray(index, dtype=np.uint64) + np.uint64(1)) * _GOLD
        return _mix64(z)


def uniform01(u: np.ndarray) -> np.ndarray:
    """53-bit uniform double in [0, 1)."""
    return (u >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def _ln(x: np.ndarray) -> np.ndarray:
    """Natural log for x in (0, 1]: frexp, then the atanh series on [sqrt(.5), sqrt(2))."""
    m, e = np.frexp(x)
    small = m < 0.7071067811865476
    m = np.where(small, m * 2.0, m)
    e = np.where(small, e - 1, e).astype(np.float64)
    s = (m - 1.0) / (m + 1.0)
    s2 = s * s
    p = np.full_like(s, 1.0 / 23.0)
    for n in range(21, 0, -2):
        p = p * s2 + (1.0 / n)
    return 2.0 * s * p + e * _LN2


def _cos2pi(u: np.ndarray) -> np.ndarray:
    """cos(2*pi*u) for u in [0, 1) by octant reduction and Taylor series on [0, pi/4]."""
    t = u - np.floor(u + 0.5)  # [-0.5, 0.5)
    a = np.abs(t)
    neg = a > 0.25
    a = np.where(neg, 0.5 - a, a)  # cos(2pi a) with a in [0, 0.25], sign flipped if neg
    use_sin = a > 0.125
    x = np.where(use_sin, (0.25 - a) * _TWO_PI, a * _TWO_PI)  # [0, pi/4]
    x2 = x * x
    c = np.full_like(x, 1.0)
    for n in range(18, 0, -2):  # cos: 1 - x^2/2! + ...
        c = 1.0 - c * x2 / float(n * (n - 1))
    s = np.full_like(x, 1.0)
    for n in range(19, 1, -2):  # sin: x (1 - x^2/3! + ...)
        s = 1.0 - s * x2 / float(n * (n - 1))
    s = s * x
    r = np.where(use_sin, s, c)
    return np.where(neg, -r, r)


def normal(seed: int, stream: int, index: np.ndarray, sigma: float = 1.0) -> np.ndarray:
    """N(0, sigma^2) by Box-Muller from two counter draws per element."""
    i = np.asarray(index, dtype=np.uint64)
    u1 = 1.0 - uniform01(rand_u64(seed, stream, i * np.uint64(2)))  # (0, 1]
    u2 = uniform01(rand_u64(seed, stream, i * np.uint64(2) + np.uint64(1)))
    r = np.sqrt(-2.0 * _ln(u1))
    return sigma * r * _cos2pi(u2)


def to_half_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float64).astype(np.float16).view(np.uint16)


def uniform_half(seed: int, stream: int, index: np.ndarray, lo: float, hi: float) -> np.ndarray:
    return to_half_bits(lo + (hi - lo) * uniform01(rand_u64(seed, stream, index)))


# ---------------------------------------------------------------------------------------


@dataclass(frozen=True)
class Config:
    name: str
    seg_num: int
    seg_len: int  # 0 for CSR
    k: int
    seed: int
    description: str


CONFIGS = {
    "C1": Config("C1", 4, 32000, 50, 1, "4x32000 N(0,1) fp16, k=50"),
    "C2": Config("C2", 64, 128256, 50, 2,
                 "64x128256 logits-like: N(0,2), 5% -inf, 20 outliers U(8,12) per row, k=50"),
    "C3": Config("C3", 1024, 151936, 50, 3,
                 "1024x151936 heavy ties: 256 fp16 levels U[-4,4] with +0/-0, k=50"),
    "C4": Config("C4", 4096, 0, 50, 4,
                 "CSR 4096 segments, lengths U{1..262144}, U(-1,1), k in {1,8,50,256}"),
    "C5": Config("C5", 8192, 262144, 1024, 5,
                 "8192x262144 adversarial thirds (equal / sorted N(0,1) / U[1,2)), k=1024"),
}

C4_K_VALUES = (1, 8, 50, 256)
C4_MAX_LEN = 262144


def _rows(cfg: Config, rows) -> np.ndarray:
    if rows is None:
        return np.arange(cfg.seg_num, dtype=np.int64)
    if isinstance(rows, slice):
        return np.arange(cfg.seg_num, dtype=np.int64)[rows]
    return np.asarray(rows, dtype=np.int64)


def gen_c1(rows=None, seg_len=None, seed=None) -> np.ndarray:
    cfg = CONFIGS["C1"]
    L = seg_len or cfg.seg_len
    r = _rows(cfg, rows)
    idx = (r[:, None] * L + np.arange(L, dtype=np.int64)[None, :]).reshape(-1)
    return to_half_bits(normal(seed or cfg.seed, 0, idx)).reshape(r.size, L)


def c2_outliers(row: int, seg_len: int, seed: int):
    """C2's 20 planted outliers of one row: (distinct positions, fp16 bits of U(8,12))."""
    cand = (rand_u64(seed, 2, row * 64 + np.arange(64, dtype=np.int64)) % np.uint64(seg_len)).astype(np.int64)
    _, first = np.unique(cand, return_index=True)
    pos = cand[np.sort(first)][:20]  # the first 20 distinct draws, in draw order
    assert pos.size == 20
    return pos, uniform_half(seed, 3, row * 64 + np.arange(20, dtype=np.int64), 8.0, 12.0)


def gen_c2(rows=None, seg_len=None, seed=None) -> np.ndarray:
    cfg = CONFIGS["C2"]
    L = seg_len or cfg.seg_len
    s = seed or cfg.seed
    r = _rows(cfg, rows)
    out = np.empty((r.size, L), np.uint16)
    col = np.arange(L, dtype=np.int64)
    for j, row in enumerate(r):
        idx = row * L + col
        v = to_half_bits(normal(s, 0, idx, sigma=2.0))
        masked = uniform01(rand_u64(s, 1, idx)) < 0.05
        v[masked] = 0xFC00
        pos, vals = c2_outliers(int(row), L, s)
        v[pos] = vals
        out[j] = v
    return out


def c3_levels(seed=None) -> np.ndarray:
    """256 fp16 levels from U[-4,4], distinct, holding +0 (0x0000) and -0 (0x8000)."""
    s = seed or CONFIGS["C3"].seed
    levels = [0x0000, 0x8000]
    seen = {0x0000, 0x8000}
    i = 0
    while len(levels) < 256:
        b = int(uniform_half(s, 10, np.array([i], np.int64), -4.0, 4.0)[0])
        i += 1
        if (b & 0x7FFF) == 0 or b in seen:
            continue
        seen.add(b)
        levels.append(b)
    return np.array(levels, np.uint16)


def gen_c3(rows=None, seg_len=None, seed=None) -> np.ndarray:
    cfg = CONFIGS["C3"]
    L = seg_len or cfg.seg_len
    s = seed or cfg.seed
    lv = c3_levels(s)
    r = _rows(cfg, rows)
    out = np.empty((r.size, L), np.uint16)
    col = np.arange(L, dtype=np.int64)
    for j, row in enumerate(r):
        u = rand_u64(s, 0, row * L + col)
        out[j] = lv[(u >> np.uint64(56)).astype(np.int64)]
    return out


def c4_offsets(seg_num=None, max_len=C4_MAX_LEN, seed=None) -> np.ndarray:
    cfg = CONFIGS["C4"]
    n = seg_num or cfg.seg_num
    s = seed or cfg.seed
    lens = 1 + (rand_u64(s, 20, np.arange(n, dtype=np.int64)) % np.uint64(max_len)).astype(np.int64)
    off = np.zeros(n + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    assert off[-1] < 2**31
    return off


def gen_c4(seg_num=None, max_len=C4_MAX_LEN, seed=None):
    """Returns (values uint16 1-D, offsets int64 [seg_num+1])."""
    s = seed or CONFIGS["C4"].seed
    off = c4_offsets(seg_num, max_len, s)
    total = int(off[-1])
    vals = np.empty(total, np.uint16)
    step = 1 << 24
    for b in range(0, total, step):
        e = min(total, b + step)
        vals[b:e] = uniform_half(s, 0, np.arange(b, e, dtype=np.int64), -1.0, 1.0)
    return vals, off


def gen_c4_range(s0: int, s1: int, seed=None) -> np.ndarray:
    """Values of C4 segments [s0, s1) alone (the slice gen_c4 would hold there), so one shard
    or a small test case regenerates without the whole 1.07 GB batch."""
    s = seed or CONFIGS["C4"].seed
    off = c4_offsets(seed=s)
    b, e = int(off[s0]), int(off[s1])
    return uniform_half(s, 0, np.arange(b, e, dtype=np.int64), -1.0, 1.0)


def gen_c5(rows=None, seg_len=None, seed=None) -> np.ndarray:
    cfg = CONFIGS["C5"]
    L = seg_len or cfg.seg_len
    s = seed or cfg.seed
    r = _rows(cfg, rows)
    out = np.empty((r.size, L), np.uint16)
    col = np.arange(L, dtype=np.int64)
    for j, row in enumerate(r):
        kind = int(row) % 3
        idx = row * L + col
        if kind == 0:  # (a) all values equal
            out[j] = uniform_half(s, 30, np.array([row], np.int64), -4.0, 4.0)[0]
        elif kind == 1:  # (b) N(0,1) sorted ascending, ties ordered by bit pattern
            v = to_half_bits(normal(s, 0, idx))
            from_key = sort_ascending_bits(v)
            out[j] = from_key
        else:  # (c) U[1,2): the high radix digit is constant
            out[j] = uniform_half(s, 0, idx, 1.0, 2.0)
    return out


def sort_ascending_bits(v: np.ndarray) -> np.ndarray:
    """Sort fp16 bit patterns ascending by value; equal values (+0/-0) by raw bits."""
    v = np.asarray(v, np.uint16)
    nan = ((v & 0x7C00) == 0x7C00) & ((v & 0x03FF) != 0)
    zero = (v & 0x7FFF) == 0
    norm = np.where(nan, np.uint16(0xFFFF), np.where(zero, np.uint16(0), v)).astype(np.uint16)
    asc = np.where(norm & 0x8000, ~norm, norm ^ np.uint16(0x8000)).astype(np.uint32)
    comp = (asc << np.uint32(16)) | v.astype(np.uint32)
    return (np.sort(comp) & np.uint32(0xFFFF)).astype(np.uint16)


def generate(name: str, rows=None, seg_len=None, seed=None):
    """Uniform entry point: returns (values, offsets_or_None, k)."""
    cfg = CONFIGS[name]
    if name == "C4":
        vals, off = gen_c4(seed=seed)
        return vals, off, cfg.k
    fn = {"C1": gen_c1, "C2": gen_c2, "C3": gen_c3, "C5": gen_c5}[name]
    return fn(rows=rows, seg_len=seg_len, seed=seed), None, cfg.k
