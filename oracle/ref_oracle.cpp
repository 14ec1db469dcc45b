// ref_oracle.cpp -- exposes the reference's OWN CPU implementation through a C ABI.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile against the reference's headers
// where they lie (fire-emblem/batch_topk: include/batch_topk_types.cuh, include/type_codec.cuh,
// src/radix_select_state.cuh); the output goes to oracle/_ref/ and never into the product.
// Used to pin the C restatement in topk_oracle.c, to generate golden fixtures, and as the
// timed CPU baseline ("kind": "reference") in bench.py.
//
// The input generators below restate the reference test's generators
// (test/test_batch_topk.cu:446-454 make_random_input, :456-471 make_duplicate_heavy_input,
// :473-496 make_optimized_special_values_input) with the same standard-library engines, so
// the golden fixtures are computed on exactly the inputs the reference's tests use.
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

#include "batch_topk_types.cuh"
#include "radix_select_state.cuh"

namespace {

uint16_t half_bits(half h) {
  uint16_t b;
  std::memcpy(&b, &h, sizeof(b));
  return b;
}

half bits_half(uint16_t b) {
  half h;
  std::memcpy(&h, &b, sizeof(b));
  return h;
}

float q(float v) { return __half2float(__float2half(v)); }

}  // namespace

extern "C" {

// Runs radix_topk::cpu_reference_topk per segment.  Inputs are fp16 bit patterns; the
// fp16 -> float conversion happens before the timed region.  Writes min(k,len) indices per
// row (rest -1) and the reference's float values.  Returns wall seconds of the timed region
// in *elapsed_s.  offsets (CSR, seg_num+1 entries) may be NULL for fixed-length rows.
int ref_cpu_topk(const uint16_t* in, const int64_t* offsets, int64_t seg_num, int64_t seg_len,
                 int k, int32_t* out_idx, float* out_val, int threads, double* elapsed_s) {
  if (seg_num <= 0 || k <= 0) return -1;
  if (threads < 1) threads = 1;
  std::vector<std::vector<float>> rows(static_cast<size_t>(seg_num));
  for (int64_t s = 0; s < seg_num; ++s) {
    const int64_t start = offsets ? offsets[s] : s * seg_len;
    const int64_t len = offsets ? offsets[s + 1] - offsets[s] : seg_len;
    rows[s].resize(static_cast<size_t>(len));
    for (int64_t i = 0; i < len; ++i) rows[s][i] = __half2float(bits_half(in[start + i]));
  }
  auto work = [&](int64_t b, int64_t e) {
    for (int64_t s = b; s < e; ++s) {
      const int len = static_cast<int>(rows[s].size());
      const radix_topk::ReferenceTopKResult r = radix_topk::cpu_reference_topk(rows[s], len, k);
      for (int i = 0; i < k; ++i) {
        const bool have = i < static_cast<int>(r.indices.size());
        out_idx[s * k + i] = have ? r.indices[i] : -1;
        out_val[s * k + i] = have ? r.values[i] : -INFINITY;
      }
    }
  };
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back(work, seg_num * t / threads, seg_num * (t + 1) / threads);
  }
  for (auto& th : pool) th.join();
  const auto t1 = std::chrono::steady_clock::now();
  if (elapsed_s) *elapsed_s = std::chrono::duration<double>(t1 - t0).count();
  return 0;
}

// radix_topk::simulate_radix_boundary on fp16 inputs; out[6] = {prefix, prefix_mask,
// cutoff_key, selected_count, live_count, boundary_digit}.
void ref_simulate_radix_boundary(const uint16_t* in, int len, int k, int32_t* out) {
  std::vector<float> v(static_cast<size_t>(len));
  for (int i = 0; i < len; ++i) v[i] = __half2float(bits_half(in[i]));
  const radix_topk::SegmentSelectState st = radix_topk::simulate_radix_boundary(v, len, k);
  out[0] = st.prefix;
  out[1] = st.prefix_mask;
  out[2] = st.cutoff_key;
  out[3] = st.selected_count;
  out[4] = st.live_count;
  out[5] = st.boundary_digit;
}

uint16_t ref_encode_half_desc(uint16_t bits) { return radix_topk::encode_half_desc(bits_half(bits)); }

// candidate_better(lhs, rhs) on (fp16 bits, index) pairs.
int ref_candidate_better(uint16_t lv, int li, uint16_t rv, int ri) {
  radix_topk::Candidate a{}, b{};
  a.value = bits_half(lv);
  a.index = li;
  b.value = bits_half(rv);
  b.index = ri;
  return radix_topk::candidate_better(a, b) ? 1 : 0;
}

uint16_t ref_float_to_half_bits(float v) { return half_bits(__float2half(v)); }

// test/test_batch_topk.cu:446-454: mt19937(seed), U(-64,64) float, rounded through half.
void ref_make_random_input(int seg_num, int seg_len, uint32_t seed, uint16_t* out) {
  std::mt19937 rng(seed);
  std::uniform_real_distribution<float> dist(-64.0f, 64.0f);
  const size_t n = static_cast<size_t>(seg_num) * static_cast<size_t>(seg_len);
  for (size_t i = 0; i < n; ++i) out[i] = half_bits(__float2half(q(dist(rng))));
}

// test/test_batch_topk.cu:456-471.
void ref_make_duplicate_heavy_input(int seg_num, int seg_len, uint16_t* out) {
  for (int seg = 0; seg < seg_num; ++seg) {
    const size_t base = static_cast<size_t>(seg) * seg_len;
    for (int i = 0; i < seg_len; ++i) {
      const float v = i < 64 ? 200.0f - static_cast<float>(seg * 64 + i)
                             : static_cast<float>(((i + seg) % 5) - 2);
      out[base + i] = half_bits(__float2half(v));
    }
  }
}

// test/test_batch_topk.cu:477-496.
void ref_make_special_values_input(int seg_num, int seg_len, uint16_t* out) {
  for (int seg = 0; seg < seg_num; ++seg) {
    const size_t base = static_cast<size_t>(seg) * seg_len;
    std::vector<float> v(static_cast<size_t>(seg_len));
    for (int i = 0; i < seg_len; ++i) v[i] = q(-512.0f + static_cast<float>((i + seg) % 113));
    v[3] = q(INFINITY);
    v[9] = q(INFINITY);
    v[15] = q(2048.0f - static_cast<float>(seg));
    v[21] = q(2048.0f - static_cast<float>(seg));
    v[27] = q(1024.0f + static_cast<float>(seg));
    v[33] = q(-INFINITY);
    v[39] = q(NAN);
    v[45] = q(NAN);
    for (int i = 0; i < seg_len; ++i) out[base + i] = half_bits(__float2half(v[i]));
  }
}

}  // extern "C"
