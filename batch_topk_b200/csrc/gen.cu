// gen.cu -- device-side generation of the benchmark inputs, bit-identical to the host
// generators of batch_topk_b200/workloads.py.
//
// Every value is a pure function of (seed, stream, element index): a splitmix64 counter, a
// 53-bit uniform double, Box-Muller with ln and cos written as fixed sequences of IEEE double
// add / multiply / divide / sqrt.  Each operation uses the correctly rounded intrinsic
// (__dadd_rn, __dmul_rn, __ddiv_rn, __dsqrt_rn), which is never fused into an FMA, so the
// device performs exactly the host's operations in the host's order.  The double -> fp16
// conversion is written out (round to nearest even, subnormals included).  The per-row
// tables the host builds (C3's 256 levels, C2's outliers, C5's row constants) and the sort of
// C5's ascending rows stay on the host side of the call.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/batch_topk_b200_gen.h"

namespace btgen {

constexpr double kLn2 = 0.6931471805599453;
constexpr double kTwoPi = 6.283185307179586;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// The key of (seed, stream): splitmix64 of seed * 0x100000001B3 + stream * 0x9E3779B1 + 1.
__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return mix64(seed * 0x100000001B3ull + stream * 0x9E3779B1ull + 1ull);
}

__device__ __forceinline__ uint64_t rand_u64(uint64_t key, uint64_t index) {
  return mix64(key + (index + 1ull) * 0x9E3779B97F4A7C15ull);
}

__device__ __forceinline__ double uniform01(uint64_t u) {
  return __dmul_rn(static_cast<double>(u >> 11), 1.0 / 9007199254740992.0);
}

// ln(x), x in (0, 1]: frexp, then the atanh series 2 s (1 + s^2/3 + ... + s^22/23) on
// [sqrt(1/2), sqrt(2)).
__device__ double ln01(double x) {
  int e;
  double m = frexp(x, &e);
  if (m < 0.7071067811865476) {
    m = __dmul_rn(m, 2.0);
    e -= 1;
  }
  const double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
  const double s2 = __dmul_rn(s, s);
  double p = 1.0 / 23.0;
#pragma unroll
  for (int n = 21; n > 0; n -= 2) p = __dadd_rn(__dmul_rn(p, s2), 1.0 / static_cast<double>(n));
  return __dadd_rn(__dmul_rn(__dmul_rn(2.0, s), p), __dmul_rn(static_cast<double>(e), kLn2));
}

// cos(2 pi u), u in [0, 1): octant reduction to [0, pi/4], then Taylor series of cos or sin.
__device__ double cos2pi(double u) {
  const double t = __dsub_rn(u, floor(__dadd_rn(u, 0.5)));
  double a = fabs(t);
  const bool neg = a > 0.25;
  if (neg) a = __dsub_rn(0.5, a);
  const bool use_sin = a > 0.125;
  const double x = use_sin ? __dmul_rn(__dsub_rn(0.25, a), kTwoPi) : __dmul_rn(a, kTwoPi);
  const double x2 = __dmul_rn(x, x);
  double r;
  if (use_sin) {
    double s = 1.0;
#pragma unroll
    for (int n = 19; n > 1; n -= 2) {
      s = __dsub_rn(1.0, __ddiv_rn(__dmul_rn(s, x2), static_cast<double>(n * (n - 1))));
    }
    r = __dmul_rn(s, x);
  } else {
    double c = 1.0;
#pragma unroll
    for (int n = 18; n > 0; n -= 2) {
      c = __dsub_rn(1.0, __ddiv_rn(__dmul_rn(c, x2), static_cast<double>(n * (n - 1))));
    }
    r = c;
  }
  return neg ? -r : r;
}

__device__ double normal(uint64_t key, uint64_t i, double sigma) {
  const double u1 = __dsub_rn(1.0, uniform01(rand_u64(key, i * 2ull)));  // (0, 1]
  const double u2 = uniform01(rand_u64(key, i * 2ull + 1ull));
  const double r = __dsqrt_rn(__dmul_rn(-2.0, ln01(u1)));
  return __dmul_rn(__dmul_rn(sigma, r), cos2pi(u2));
}

// double -> IEEE binary16, round to nearest even (subnormals, overflow to infinity).
__device__ uint16_t to_half_rne(double x) {
  const uint64_t b = static_cast<uint64_t>(__double_as_longlong(x));
  const uint16_t sign = static_cast<uint16_t>((b >> 48) & 0x8000u);
  const uint64_t ab = b & 0x7FFFFFFFFFFFFFFFull;
  if (ab >= 0x7FF0000000000000ull) {  // inf or NaN
    return sign | (ab > 0x7FF0000000000000ull ? 0x7E00u : 0x7C00u);
  }
  if (ab == 0) return sign;
  const int exp = static_cast<int>(ab >> 52) - 1023;
  const uint64_t frac = ab & 0x000FFFFFFFFFFFFFull;
  // significand with its leading one (double subnormals are far below fp16's range)
  const uint64_t mant = (ab >> 52) ? (frac | 0x0010000000000000ull) : frac;
  if (exp > 15) return sign | 0x7C00u;
  int shift = 42;                     // keep 11 significant bits (1 + 10 fraction bits)
  if (exp < -14) shift += -14 - exp;  // fp16 subnormal: fewer bits
  if (shift > 53) return sign;        // below half the smallest subnormal
  const uint64_t q = mant >> shift;
  const uint64_t rem = mant & ((1ull << shift) - 1ull);
  const uint64_t half = 1ull << (shift - 1);
  const uint64_t qr = q + ((rem > half || (rem == half && (q & 1ull))) ? 1ull : 0ull);
  uint32_t bits;
  if (exp < -14) {
    bits = static_cast<uint32_t>(qr);  // 0x400 after rounding up is the smallest normal
  } else {
    bits = (static_cast<uint32_t>(exp + 15) << 10) + static_cast<uint32_t>(qr - 1024ull);
    if (bits >= 0x7C00u) bits = 0x7C00u;
  }
  return sign | static_cast<uint16_t>(bits);
}

enum Kind { kNormal = 0, kUniform = 1, kLevels = 2, kMask = 3 };

struct GenArgs {
  uint16_t* out;
  long long n;
  unsigned long long idx0;  // flat index of out[0]
  unsigned long long key;
  double a, b;              // sigma | lo, hi | mask probability
  const uint16_t* table;    // 256 levels
  uint16_t fill;            // mask value
  int kind;
};

__global__ void gen_kernel(GenArgs g) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < g.n;
       i += stride) {
    const uint64_t idx = g.idx0 + static_cast<uint64_t>(i);
    switch (g.kind) {
      case kNormal:
        g.out[i] = to_half_rne(normal(g.key, idx, g.a));
        break;
      case kUniform: {
        const double u = uniform01(rand_u64(g.key, idx));
        g.out[i] = to_half_rne(__dadd_rn(g.a, __dmul_rn(__dsub_rn(g.b, g.a), u)));
        break;
      }
      case kLevels:
        g.out[i] = g.table[rand_u64(g.key, idx) >> 56];
        break;
      default:  // kMask: entries whose uniform draw is below a become `fill`
        if (uniform01(rand_u64(g.key, idx)) < g.a) g.out[i] = g.fill;
        break;
    }
  }
}

int launch(const GenArgs& g, void* stream) {
  if (!g.out || g.n < 0) return cudaErrorInvalidValue;
  if (g.n == 0) return cudaSuccess;
  long long blocks = (g.n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  gen_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(g);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace btgen

extern "C" {

int bt_gen_normal(void* d_out, long long n, unsigned long long idx0, unsigned long long seed,
                  unsigned long long stream_id, double sigma, void* stream) {
  btgen::GenArgs g{};
  g.out = static_cast<uint16_t*>(d_out);
  g.n = n;
  g.idx0 = idx0;
  g.key = btgen::stream_key(seed, stream_id);
  g.a = sigma;
  g.kind = btgen::kNormal;
  return btgen::launch(g, stream);
}

int bt_gen_uniform(void* d_out, long long n, unsigned long long idx0, unsigned long long seed,
                   unsigned long long stream_id, double lo, double hi, void* stream) {
  btgen::GenArgs g{};
  g.out = static_cast<uint16_t*>(d_out);
  g.n = n;
  g.idx0 = idx0;
  g.key = btgen::stream_key(seed, stream_id);
  g.a = lo;
  g.b = hi;
  g.kind = btgen::kUniform;
  return btgen::launch(g, stream);
}

int bt_gen_levels(void* d_out, long long n, unsigned long long idx0, unsigned long long seed,
                  unsigned long long stream_id, const void* d_levels256, void* stream) {
  if (!d_levels256) return cudaErrorInvalidValue;
  btgen::GenArgs g{};
  g.out = static_cast<uint16_t*>(d_out);
  g.n = n;
  g.idx0 = idx0;
  g.key = btgen::stream_key(seed, stream_id);
  g.table = static_cast<const uint16_t*>(d_levels256);
  g.kind = btgen::kLevels;
  return btgen::launch(g, stream);
}

int bt_gen_mask(void* d_inout, long long n, unsigned long long idx0, unsigned long long seed,
                unsigned long long stream_id, double p, unsigned short fill_bits, void* stream) {
  btgen::GenArgs g{};
  g.out = static_cast<uint16_t*>(d_inout);
  g.n = n;
  g.idx0 = idx0;
  g.key = btgen::stream_key(seed, stream_id);
  g.a = p;
  g.fill = fill_bits;
  g.kind = btgen::kMask;
  return btgen::launch(g, stream);
}

}  // extern "C"
