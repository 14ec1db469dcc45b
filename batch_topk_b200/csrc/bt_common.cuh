// bt_common.cuh -- element-independent warp and block helpers shared by the top-k kernels of
// every element type: packed per-round scans of the strided counts, and the warp-register
// bitonic sort of 64-bit (key, index) composites.
#pragma once

#include <cstdint>

#include "bt_device.cuh"

namespace bt {

// 16-bit field j of four packed words (selects rather than indexing, so a run-time j keeps
// the words in registers).
__device__ __forceinline__ uint32_t field16(const uint32_t (&w)[4], int j) {
  const uint32_t x = j < 2 ? w[0] : (j < 4 ? w[1] : (j < 6 ? w[2] : w[3]));
  return (x >> ((j & 1) * 16)) & 0xFFFFu;
}

// Inclusive warp scan of four words of packed 16-bit counts.
__device__ __forceinline__ void warp_scan4(uint32_t (&w)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w[i], o);
      if (lane >= o) w[i] += y;
    }
  }
}

// Per-round block offsets from the warps' inclusive round totals in rw[w][half * 4 ...]:
// base_j = (survivors of rounds before j) + (round j survivors of lower warps) + (round j
// survivors of lower lanes).  Returns the grand total.
__device__ __forceinline__ uint32_t round_bases(const uint32_t (*rw)[8], int half,
                                                const uint32_t (&incl)[4],
                                                const uint32_t (&own)[4], uint32_t (&base)[4]) {
  const int warp = threadIdx.x >> 5;
  uint32_t tot[4] = {0, 0, 0, 0}, pre[4] = {0, 0, 0, 0};
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint4 v = lds128(&rw[w][half * 4]);
    const uint32_t x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      tot[i] += x[i];
      pre[i] += w < warp ? x[i] : 0u;
    }
  }
  uint32_t start = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t b = start + field16(pre, j) + field16(incl, j) - field16(own, j);
    if (j & 1) base[j >> 1] |= b << 16; else base[j >> 1] = b;
    start += field16(tot, j);
  }
  return start;
}

// ---- warp-register bitonic sort of 64-bit composites ------------------------------------
//
// A striped array of N = 32 R composites: element r * 32 + lane lives in x[r] of lane `lane`.

__device__ __forceinline__ unsigned long long shfl64(unsigned long long v, int src) {
  const uint32_t lo = __shfl_sync(0xFFFFFFFFu, static_cast<uint32_t>(v), src);
  const uint32_t hi = __shfl_sync(0xFFFFFFFFu, static_cast<uint32_t>(v >> 32), src);
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}

__device__ __forceinline__ unsigned long long shfl_xor64(unsigned long long v, int mask) {
  const uint32_t lo = __shfl_xor_sync(0xFFFFFFFFu, static_cast<uint32_t>(v), mask);
  const uint32_t hi = __shfl_xor_sync(0xFFFFFFFFu, static_cast<uint32_t>(v >> 32), mask);
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}

// One bitonic compare-exchange step (block `size`, distance `stride`) over the striped array;
// size == 0 means "ascending everywhere" (the final merge of a bitonic sequence).
template <int R>
__device__ __forceinline__ void bitonic_step(unsigned long long (&x)[R], int size, int stride) {
  const int lane = threadIdx.x & 31;
  if (stride >= 32) {
    const int rs = stride >> 5;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if ((r & rs) == 0) {
        const bool up = size == 0 || (((r << 5) + lane) & size) == 0;
        const unsigned long long a = x[r], b = x[r | rs];
        if ((a > b) == up) {
          x[r] = b;
          x[r | rs] = a;
        }
      }
    }
  } else {
    const bool lower = (lane & stride) == 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const bool up = size == 0 || (((r << 5) + lane) & size) == 0;
      const unsigned long long y = shfl_xor64(x[r], stride);
      const unsigned long long mn = x[r] < y ? x[r] : y;
      const unsigned long long mx = x[r] < y ? y : x[r];
      x[r] = (lower == up) ? mn : mx;
    }
  }
}

template <int R>
__device__ __forceinline__ void warp_sort_regs(unsigned long long (&x)[R]) {
#pragma unroll
  for (int size = 2; size <= 32 * R; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) bitonic_step<R>(x, size, stride);
  }
}

}  // namespace bt
