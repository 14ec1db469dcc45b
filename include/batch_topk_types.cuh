// batch_topk_types.cuh -- the reference's public type and ordering names, for source
// compatibility of callers written against fire-emblem/batch_topk.
//
// Same names, fields and semantics as the reference's include/batch_topk_types.cuh and
// include/type_codec.cuh; the implementations here are this library's own.  The library's
// kernels do not use this header (their codec lives in the CUDA sources); it is for host
// code that checks or post-processes results in the reference's terms.
//
// Ordering (the contract every entry point follows): NaN ranks below every number, -inf
// included; otherwise the larger value ranks first; -0 == +0; equal values go to the lower
// index.
#pragma once

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime_api.h>

#include "batch_topk_b200.h"

namespace radix_topk {

// Limits of this implementation (the reference's are 128 and 10000).
inline constexpr int kMaxSupportedK = BT_MAX_K;
inline constexpr int kMaxSupportedSegLen = BT_MAX_SEG_LEN;

struct Candidate {
  uint32_t encoded_key = 0;
  half value = __float2half(0.0f);
  int index = 0;
};

struct ReferenceTopKResult {
  std::vector<float> values;
  std::vector<int> indices;
};

// Per-segment radix-select state in the reference's two-digit (8+8 bit) formulation over the
// descending key: the high digit that holds the k-th key (boundary_digit, prefix/prefix_mask),
// how many keys rank strictly above that digit (selected_count) and inside it (live_count),
// the exact k-th key (cutoff_key), how many keys beat it (strictly_better_count) and how many
// cutoff-equal keys the top-k takes (remaining_slots).
struct SegmentSelectState {
  uint16_t prefix = 0;
  uint16_t prefix_mask = 0;
  uint16_t cutoff_key = 0xffffu;
  int selected_count = 0;
  int live_count = 0;
  int boundary_digit = 0;
  int strictly_better_count = 0;
  int remaining_slots = 0;
};

__host__ __device__ inline bool is_nan_value(float v) { return v != v; }

// Every NaN becomes 0xFFFF and -0 becomes +0, so each ordering class has one bit pattern.
__host__ __device__ inline uint16_t normalize_half_bits(uint16_t bits) {
  const bool nan = (bits & 0x7C00u) == 0x7C00u && (bits & 0x03FFu) != 0;
  if (nan) return 0xFFFFu;
  return (bits & 0x7FFFu) == 0 ? static_cast<uint16_t>(0) : bits;
}

__host__ __device__ inline uint16_t half_bits(half h) {
  uint16_t b;
  memcpy(&b, &h, sizeof(b));
  return b;
}

// Unsigned key that grows with the value: negative numbers have all bits inverted, others get
// the sign bit set.  NaN (normalised to 0xFFFF, a "negative" pattern) maps to 0x0000.
__host__ __device__ inline uint16_t encode_half_asc(half value) {
  const uint16_t b = normalize_half_bits(half_bits(value));
  return (b & 0x8000u) ? static_cast<uint16_t>(b ^ 0xFFFFu) : static_cast<uint16_t>(b | 0x8000u);
}

// Smaller key ranks first: the best value has the smallest key and NaN the largest (0xFFFF).
__host__ __device__ inline uint16_t encode_half_desc(half value) {
  return static_cast<uint16_t>(encode_half_asc(value) ^ 0xFFFFu);
}

__host__ __device__ inline bool candidate_better(const Candidate& lhs, const Candidate& rhs) {
  const float a = __half2float(lhs.value), b = __half2float(rhs.value);
  const bool an = is_nan_value(a), bn = is_nan_value(b);
  if (an || bn) return an == bn ? lhs.index < rhs.index : bn;
  if (a != b) return a > b;
  return lhs.index < rhs.index;
}

// The top min(k, len) of values[0 .. min(seg_len, values.size())) in the order above.  A host
// check for callers; empty for seg_len <= 0 or k <= 0.
inline ReferenceTopKResult cpu_reference_topk(const std::vector<float>& values, int seg_len,
                                              int k) {
  ReferenceTopKResult r;
  const long long len = std::min<long long>(seg_len, static_cast<long long>(values.size()));
  if (len <= 0 || k <= 0) return r;
  const long long take = std::min<long long>(k, len);
  std::vector<int> idx(static_cast<size_t>(len));
  std::iota(idx.begin(), idx.end(), 0);
  auto ranks_first = [&](int i, int j) {
    const float a = values[static_cast<size_t>(i)], b = values[static_cast<size_t>(j)];
    const bool an = std::isnan(a), bn = std::isnan(b);
    if (an || bn) return an == bn ? i < j : bn;
    return a != b ? a > b : i < j;
  };
  std::partial_sort(idx.begin(), idx.begin() + take, idx.end(), ranks_first);
  r.indices.assign(idx.begin(), idx.begin() + take);
  r.values.reserve(static_cast<size_t>(take));
  for (int i : r.indices) r.values.push_back(values[static_cast<size_t>(i)]);
  return r;
}

}  // namespace radix_topk
