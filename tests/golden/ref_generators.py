"""numpy restatement of the reference test's input generators.

fire-emblem/batch_topk test/test_batch_topk.cu:
  :446-454  make_random_input(seg_num, seg_len, seed): std::mt19937(seed),
            std::uniform_real_distribution<float>(-64, 64), rounded through half.
  :456-471  make_duplicate_heavy_input(seg_num, seg_len).
  :473-496  make_optimized_special_values_input(seg_num, seg_len): +-inf, NaN, planted maxima.
  :602-617  the 64-value final-sort case (42, 42, +inf, +inf, 17, 17, NaN, -inf, then -i).

The libstdc++ float path is: one 32-bit draw u, s = float(u) / 2^32 (clamped below 1),
value = s * (b - a) + a, all in float.
``tests/test_oracle.py::test_generators_match_reference_code`` checks these bit for bit against
the same generators compiled from C++ (oracle/_ref) when that build is present.
"""
from __future__ import annotations

import numpy as np

HALF_NAN = 0x7FFF  # cuda_fp16's host __float2half(NAN) bit pattern


def mt19937_raw(seed: int, n: int) -> np.ndarray:
    bg = np.random.MT19937(0)
    bg._legacy_seeding(seed)  # std::mt19937(seed) initialisation
    return bg.random_raw(n).astype(np.uint32)


def make_random_input(seg_num: int, seg_len: int, seed: int) -> np.ndarray:
    n = seg_num * seg_len
    s = mt19937_raw(seed, n).astype(np.float32) / np.float32(4294967296.0)
    s = np.where(s >= np.float32(1.0), np.nextafter(np.float32(1.0), np.float32(0.0)), s)
    v = (s * np.float32(128.0) + np.float32(-64.0)).astype(np.float32)
    return v.astype(np.float16).view(np.uint16).reshape(seg_num, seg_len)


def make_duplicate_heavy_input(seg_num: int, seg_len: int) -> np.ndarray:
    out = np.empty((seg_num, seg_len), np.float32)
    i = np.arange(seg_len)
    for seg in range(seg_num):
        row = (((i + seg) % 5) - 2).astype(np.float32)
        head = 200.0 - (seg * 64 + np.arange(min(64, seg_len)))
        row[: head.size] = head
        out[seg] = row
    return out.astype(np.float16).view(np.uint16)


def make_special_values_input(seg_num: int, seg_len: int) -> np.ndarray:
    out = np.empty((seg_num, seg_len), np.float32)
    i = np.arange(seg_len)
    for seg in range(seg_num):
        row = (-512.0 + ((i + seg) % 113)).astype(np.float32)
        row[3] = np.inf
        row[9] = np.inf
        row[15] = 2048.0 - seg
        row[21] = 2048.0 - seg
        row[27] = 1024.0 + seg
        row[33] = -np.inf
        out[seg] = row
    bits = out.astype(np.float16).view(np.uint16)
    bits[:, [39, 45]] = HALF_NAN  # __float2half(NAN) on the host
    return bits


def final_sort_case() -> np.ndarray:
    v = -np.arange(64, dtype=np.float32)
    v[0] = 42.0
    v[1] = 42.0
    v[2] = np.inf
    v[3] = np.inf
    v[4] = 17.0
    v[5] = 17.0
    v[7] = -np.inf
    bits = v.astype(np.float16).view(np.uint16).reshape(1, 64)
    bits[0, 6] = HALF_NAN
    return bits


def small_correctness_case() -> np.ndarray:
    """test/test_batch_topk.cu:332-340: 2 x 8, k = 3."""
    v = np.array([1, 9, 2, 8, 3, 7, 4, 6, 5, 4, 9, 1, 9, 2, 0, 8], np.float32)
    return v.astype(np.float16).view(np.uint16).reshape(2, 8)


# (name, builder, k) -- every end-to-end case the reference's test main() runs.
REFERENCE_CASES = [
    ("small_2x8_k3", lambda: small_correctness_case(), 3),
    ("random_1x10000_k50_s7", lambda: make_random_input(1, 10000, 7), 50),
    ("random_8x10000_k50_s17", lambda: make_random_input(8, 10000, 17), 50),
    ("random_32x10000_k50_s23", lambda: make_random_input(32, 10000, 23), 50),
    ("final_sort_64_k50", lambda: final_sort_case(), 50),
    ("special_2x10000_k50", lambda: make_special_values_input(2, 10000), 50),
    ("random_3x256_k128_s2026", lambda: make_random_input(3, 256, 2026), 128),
    ("duplicate_heavy_4x10000_k50", lambda: make_duplicate_heavy_input(4, 10000), 50),
    ("random_128x10000_k50_s1234", lambda: make_random_input(128, 10000, 1234), 50),
    ("zeros_1x10000_k50", lambda: np.zeros((1, 10000), np.uint16), 50),
]
