// bt_f32.cuh -- batched top-k of 32-bit floats (fp32) on sm_100a.
//
// The reference is fp16 only (other input types are a listed non-goal); this path gives fp32
// rows the same contract and order: values descending, equal values (-0 == +0) by lower index,
// every NaN last (NaNs by index), output values the input's own bit patterns.
//
// One streaming pass with the structure of the large-k path (bt_large.cuh), for every k:
//   * the producer warp (bt_kernels.cuh) streams 32 KiB chunks (8192 floats) of each work part
//     into two shared-memory stages with cp.async.bulk (no multicast);
//   * 8 consumer warps keep the part's candidates in a 2048-entry shared-memory cache of
//     (32-bit descending key, 32-bit index) composites, in index order, under a certified
//     threshold: the chunk's k-th best group maximum, or the cache's k-th key once k candidates
//     are known;
//   * when the cache lacks room it drops what the current chunk's top k beats and cuts itself
//     to its exact k best (four 8-bit digit passes over 32-bit keys);
//   * at the end of a part the cache's k best are sorted (warp-register bitonic runs, ranks by
//     binary search) and written; the value bits are read back from the input by index.
// Split segments publish exact per-part lists that the last block to finish merges.
//
// Thread t owns vectors t + 256 j (j = 0..7, "round j") of a chunk: round-major order is index
// order, and 16-byte shared loads of consecutive threads are conflict-free.
#pragma once

namespace bt {
namespace f32 {

constexpr int kEpvShift = 2;                 // 4 floats per 16-byte vector
constexpr int kCache = 2048;                 // candidate cache entries
constexpr uint32_t kNaNKey = 0xFFFFFFFFu;    // key of every NaN (ranks last)

// Descending key: smaller key ranks first.  Any NaN -> 0xFFFFFFFF; +-0 -> 0x7FFFFFFF; else
// bits ^ (sign ? 0 : 0x7FFFFFFF).  A bijection on values, with -0 == +0 and all NaNs equal.
__host__ __device__ __forceinline__ uint32_t desc_key32(uint32_t bits) {
  const uint32_t mag = bits & 0x7FFFFFFFu;
  const uint32_t key = (bits & 0x80000000u) ? bits : (bits ^ 0x7FFFFFFFu);
  return mag > 0x7F800000u ? kNaNKey : (mag == 0 ? 0x7FFFFFFFu : key);
}

// 4-bit mask of the elements of aligned vector gv that lie inside [a0, a1).
__device__ __forceinline__ uint32_t valid_mask4(long long gv, long long a0, long long a1) {
  const long long e0 = gv * 4;
  long long lo = a0 - e0, hi = a1 - e0;
  lo = lo < 0 ? 0 : (lo > 4 ? 4 : lo);
  hi = hi < 0 ? 0 : (hi > 4 ? 4 : hi);
  if (hi <= lo) return 0u;
  return (0xFu << lo) & (0xFu >> (4 - hi)) & 0xFu;
}

__device__ __forceinline__ uint32_t word_of(const uint4& w, int e) {
  return e == 0 ? w.x : (e == 1 ? w.y : (e == 2 ? w.z : w.w));
}

// The float whose key is `key` (+0 for the key of zero).  Keys of numbers run from 0x007FFFFF
// (+inf) to 0xFF800000 (-inf); above that (bucket bounds, the NaN key) the bits are a NaN.
__device__ __forceinline__ float key_value(uint32_t key) {
  return __uint_as_float(key < 0x80000000u ? (key ^ 0x7FFFFFFFu) : key);
}

// Is `key < T` the float compare `value > key_value(T)` (false for a NaN value)?  Yes while T
// is the key of a number.
__device__ __forceinline__ bool float_threshold(uint32_t T) { return T <= 0xFF800000u; }

__device__ __forceinline__ unsigned long long comp(uint32_t key, uint32_t idx) {
  return (static_cast<unsigned long long>(key) << 32) | idx;
}

struct alignas(16) FScratch {
  uint32_t hist[256];                       // digit histogram (zero between uses)
  unsigned long long cache[kCache];         // candidates, (key << 32 | index), index order
  alignas(16) uint32_t rw[2][kWarps][8];    // strided counts: per-warp round totals
  uint32_t tbase[kThreads];                 // split-segment merge: list lengths of 256 slots
  uint32_t warp_tot[kWarps];
  int bin;
  uint32_t before;
  uint32_t bcast[4];
  uint32_t fail;
};
static_assert(offsetof(FScratch, hist) % 16 == 0 && offsetof(FScratch, rw) % 16 == 0,
              "16-byte alignment of lds128 operands");

// Dynamic shared memory: [2 stages | FScratch | full[2] | empty[2] | StageInfo[2]].
struct FLayout {
  static constexpr int S = 2;
  static constexpr size_t off_scratch = static_cast<size_t>(S) * kStageBytes;
  static constexpr size_t off_full = off_scratch + sizeof(FScratch);
  static constexpr size_t off_empty = off_full + S * sizeof(uint64_t);
  static constexpr size_t off_info = off_empty + S * sizeof(uint64_t);
  static constexpr size_t bytes = off_info + S * sizeof(StageInfo);
  static_assert(sizeof(FScratch) % 16 == 0 && off_full % 8 == 0 && off_info % 8 == 0, "layout");
};
static_assert(FLayout::S == Cfg<true>::kStagesN, "the producer's stage count");

constexpr int kBlockThreads = kThreads + 32;  // 8 consumer warps + the producer warp

struct FState {
  int s = -1;
  int part = -2;
  uint32_t K = 0;          // strict threshold key: later candidates need key < K (when hasK)
  bool hasK = false;
  bool quiet = false;      // the previous chunk added nothing
  bool rising = false;     // the previous chunk beat the stale threshold
  uint32_t nbuf = 0;       // candidates in the cache
  uint32_t added = 0;      // candidates appended since K was last tightened from the cache
  int mycnt = 0;
  int nchunks = 0;
  long long part_slot = 0, seg_slot = 0, a0 = 0, a1 = 0;
};

// ---- block-wide digit select over 32-bit keys -------------------------------------------

// k-th smallest of the keys the block supplies (N per thread; key(i, &v) returns whether
// slot i holds a key), by four 8-bit digit passes, most significant first.  Returns it and,
// in *before, how many keys are smaller; when fewer than k keys exist, returns false.
// The histogram is zero on entry and left zero.
//
// With PASSES = 2 only the top 16 bits are resolved: the result is then the largest key of the
// 65536-key bucket that holds the k-th key (at least k keys are <= it, and no key of a lower
// bucket reaches it), a certified bound at half the cost, loose by at most that bucket (a
// relative 2^-7 of the value for normal floats).
template <int N, int PASSES = 4, class KeyFn>
__device__ __forceinline__ bool block_kth32(KeyFn&& key, uint32_t k, FScratch& sm,
                                            uint32_t* kth, uint32_t* before) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, base = 0;
#pragma unroll 1
  for (int d = 3; d >= 4 - PASSES; --d) {
    const int sh = 8 * d;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      uint32_t v;
      const bool ok = key(i, &v);
      // the digits above d equal the prefix's (64-bit shifts: sh + 8 may be 32)
      const bool match = (static_cast<uint64_t>(v) >> (sh + 8)) ==
                         (static_cast<uint64_t>(prefix) >> (sh + 8));
      if (ok && match) atomicAdd(&sm.hist[(v >> sh) & 0xFFu], 1u);
    }
    csync();
    if (tid < 32) warp_find_bin(sm.hist, base, k, &sm.bin, &sm.before);
    csync();
    const int b = sm.bin;
    const uint32_t bf = sm.before;
    sm.hist[tid] = 0;
    csync();
    if (b >= 256) return false;  // fewer than k keys (uniform)
    base = bf;
    prefix |= static_cast<uint32_t>(b) << sh;
  }
  *kth = PASSES == 4 ? prefix : (prefix | 0xFFFFu);
  *before = base;
  return true;
}

// ---- strided count and append ------------------------------------------------------------

enum CountMode { kAll = 0, kLt = 1, kLe = 2, kTies = 3 };

struct FCount {
  uint32_t M;         // survivors: bit 4 j + e = element e of the thread's round-j vector
  uint32_t E;         // kTies: the survivors whose key equals T (subset of M)
  uint32_t base[4];   // per round (16-bit fields): rank of the thread's first survivor (kTies:
                      // among key < T) in round-major index order
  uint32_t ebase[4];  // kTies, per round: survivors with key == T ahead of the thread's first
  uint32_t total;     // survivors (kTies: those with key < T)
  uint32_t total_eq;  // kTies: survivors with key == T
  bool fail;
};

// Counts the chunk's survivors: every valid value (kAll), key < T (kLt), key <= T (kLe), or
// key <= T with the ties at T counted apart (kTies).  One barrier.
template <int MODE>
__device__ __forceinline__ FCount fcount(const StageInfo& si, const uint8_t* buf, FScratch& sm,
                                         uint32_t T, int& par) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  FCount c;
  c.M = 0;
  c.E = 0;
  // a strict threshold below the NaN key is a float compare against its value
  const bool fcmp = MODE == kLt && float_threshold(T);
  const float V = key_value(T);
  uint32_t own[4] = {0, 0, 0, 0}, owne[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int vi = j * kThreads + tid;
    if (vi < si.nvc) {
      const uint4 w = lds128(buf + vi * 16);
      uint32_t m = 0, e = 0;
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        bool pass;
        if (MODE == kLt && fcmp) {  // key < T  <=>  value > V (false for a NaN value)
          pass = __uint_as_float(word_of(w, x)) > V;
        } else {
          const uint32_t key = desc_key32(word_of(w, x));
          const bool lt = key < T, eq = key == T;
          pass = MODE == kAll ? true : (MODE == kLt ? lt : (lt || eq));
          if (MODE == kTies) e |= static_cast<uint32_t>(eq) << x;
        }
        m |= static_cast<uint32_t>(pass) << x;
      }
      if (vi == si.vlo || vi == si.vhi) {
        const uint32_t vm = valid_mask4(si.cv0 + vi, si.a0, si.a1);
        m &= vm;
        e &= vm;
      }
      c.M |= m << (4 * j);
      c.E |= e << (4 * j);
      own[j >> 1] |= static_cast<uint32_t>(__popc(m & ~e)) << ((j & 1) * 16);
      if (MODE == kTies) owne[j >> 1] |= static_cast<uint32_t>(__popc(e)) << ((j & 1) * 16);
    }
  }
  uint32_t incl[4] = {own[0], own[1], own[2], own[3]};
  uint32_t incle[4] = {owne[0], owne[1], owne[2], owne[3]};
  if (__ballot_sync(0xFFFFFFFFu, c.M != 0)) {
    warp_scan4(incl);
    if (MODE == kTies) warp_scan4(incle);
  }
  if (lane == 31) {
    *reinterpret_cast<uint4*>(&sm.rw[par][warp][0]) = make_uint4(incl[0], incl[1], incl[2], incl[3]);
    if (MODE == kTies) {
      *reinterpret_cast<uint4*>(&sm.rw[par][warp][4]) =
          make_uint4(incle[0], incle[1], incle[2], incle[3]);
    }
  }
  csync();
  c.fail = sm.fail != 0;
  c.total = round_bases(sm.rw[par], 0, incl, own, c.base);
  c.total_eq = 0;
  if (MODE == kTies) c.total_eq = round_bases(sm.rw[par], 1, incle, owne, c.ebase);
  par ^= 1;
  return c;
}

// Appends the counted survivors at sm.cache[nbuf ...] in index order; with TIES every survivor
// with key < T and the first `need` with key == T.
template <bool TIES>
__device__ __forceinline__ void fappend(const StageInfo& si, const uint8_t* buf, const FCount& c,
                                        uint32_t need, FScratch& sm, uint32_t nbuf) {
  const int tid = threadIdx.x;
  unsigned long long* out = sm.cache + nbuf;
#pragma unroll 1
  for (int j = 0; j < kVecPerThread; ++j) {
    uint32_t m = (c.M >> (4 * j)) & 0xFu;
    const uint32_t em = (c.E >> (4 * j)) & 0xFu;
    const uint32_t lpos = field16(c.base, j);
    const uint32_t epos = TIES ? field16(c.ebase, j) : 0u;
    if (TIES && epos >= need) m &= ~em;  // every tie of this round is past the first `need`
    if (m == 0) continue;
    const int vi = j * kThreads + tid;
    const uint4 w = lds128(buf + vi * 16);
    const long long e0 = (si.cv0 + vi) * 4 - si.a0;  // segment index of element 0
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      if (!((m >> x) & 1u)) continue;
      const uint32_t below = (1u << x) - 1u;
      const uint32_t lt_before = static_cast<uint32_t>(__popc(m & ~em & below));
      const uint32_t eq_rank = epos + static_cast<uint32_t>(__popc(em & below));
      const unsigned long long cv =
          comp(desc_key32(word_of(w, x)), static_cast<uint32_t>(e0 + x));
      if (TIES && ((em >> x) & 1u)) {
        if (eq_rank < need) out[lpos + lt_before + eq_rank] = cv;
      } else {
        out[lpos + lt_before + (TIES ? (eq_rank < need ? eq_rank : need) : 0u)] = cv;
      }
    }
  }
  csync();
}

// ---- contiguous count and append (the steady state) ------------------------------------
//
// Thread t owns vectors 8t .. 8t+7 (visited rotated by t mod 8, so a quarter-warp's 16-byte
// loads cover all banks): one warp scan and one barrier give each thread its first output
// position, and each thread writes its own survivors.  Cheapest while survivors are few and
// spread; when one thread holds many, the strided form spreads the writes instead.
struct CCount32 {
  uint32_t M;  // survivors: bit 4 j + e = element e of the thread's vector 8t + j
  uint32_t base, total, maxcnt;
  bool fail;
};

// STRICT: key < K (value > V); otherwise key <= K (value >= V).  K is the key of a number.
template <bool STRICT>
__device__ __forceinline__ CCount32 fcount_contig(const StageInfo& si, const uint8_t* buf,
                                                  FScratch& sm, uint32_t K, int& par) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const float V = key_value(K);
  const int sw = tid & 7;
  CCount32 c;
  c.M = 0;
#pragma unroll
  for (int jj = 0; jj < kVecPerThread; ++jj) {
    const int j = jj ^ sw;
    const int vi = tid * kVecPerThread + j;
    if (vi < si.nvc) {
      const uint4 w = lds128(buf + vi * 16);
      const float a = __uint_as_float(w.x), b = __uint_as_float(w.y),
                  cc = __uint_as_float(w.z), d = __uint_as_float(w.w);
      uint32_t m = STRICT ? ((a > V ? 1u : 0u) | (b > V ? 2u : 0u) | (cc > V ? 4u : 0u) |
                             (d > V ? 8u : 0u))
                          : ((a >= V ? 1u : 0u) | (b >= V ? 2u : 0u) | (cc >= V ? 4u : 0u) |
                             (d >= V ? 8u : 0u));
      if (vi == si.vlo || vi == si.vhi) m &= valid_mask4(si.cv0 + vi, si.a0, si.a1);
      c.M |= m << (4 * j);
    }
  }
  const uint32_t cnt = static_cast<uint32_t>(__popc(c.M));
  uint32_t incl = 0, wmax = 0;
  if (__ballot_sync(0xFFFFFFFFu, cnt != 0)) {
    incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    wmax = __reduce_max_sync(0xFFFFFFFFu, cnt);
  }
  if (lane == 31) sm.rw[par][warp][0] = incl | (wmax << 16);  // total <= 8192, max <= 32
  csync();
  c.fail = sm.fail != 0;
  uint32_t total = 0, wpre = 0, mx = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t t = sm.rw[par][w][0];
    wpre += w < warp ? (t & 0xFFFFu) : 0u;
    total += t & 0xFFFFu;
    mx = (t >> 16) > mx ? (t >> 16) : mx;
  }
  c.total = total;
  c.maxcnt = mx;
  c.base = wpre + incl - cnt;
  par ^= 1;
  return c;
}

__device__ __forceinline__ void fappend_contig(const StageInfo& si, const uint8_t* buf,
                                               const CCount32& c, FScratch& sm, uint32_t nbuf) {
  const int tid = threadIdx.x;
  unsigned long long* out = sm.cache + nbuf + c.base;
  uint32_t r = 0;
#pragma unroll 1
  for (int j = 0; j < kVecPerThread; ++j) {
    uint32_t m = (c.M >> (4 * j)) & 0xFu;
    if (m == 0) continue;
    const int vi = tid * kVecPerThread + j;
    const uint4 w = lds128(buf + vi * 16);
    const long long e0 = (si.cv0 + vi) * 4 - si.a0;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      if ((m >> x) & 1u) out[r++] = comp(desc_key32(word_of(w, x)), static_cast<uint32_t>(e0 + x));
    }
  }
  csync();
}

// A thread holding more survivors than this writes too long alone: the strided form is used.
constexpr uint32_t kClusterMax = 16;

// ---- cache maintenance -----------------------------------------------------------------

// Keeps, in order, the cache entries with key < K and the first `need` with key == K; returns
// the new count.  Each thread holds its 8 entries in registers across the scan's barriers.
__device__ uint32_t fcompact(FScratch& sm, uint32_t n, uint32_t K, uint32_t need) {
  constexpr int kPer = kCache / kThreads;
  const uint32_t i0 = threadIdx.x * kPer;
  unsigned long long v[kPer];
  uint32_t lt = 0, eq = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t i = i0 + j;
    v[j] = i < n ? sm.cache[i] : ~0ull;
    const uint32_t key = static_cast<uint32_t>(v[j] >> 32);
    lt += (i < n && key < K) ? 1u : 0u;
    eq += (i < n && key == K) ? 1u : 0u;
  }
  uint32_t tot;
  const uint32_t pre = block_excl_scan<kThreads, true>(lt | (eq << 16), &tot, sm.warp_tot);
  uint32_t e = pre >> 16;
  uint32_t w = (pre & 0xFFFFu) + (e < need ? e : need);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t i = i0 + j;
    const uint32_t key = static_cast<uint32_t>(v[j] >> 32);
    if (i < n && key < K) {
      sm.cache[w++] = v[j];
    } else if (i < n && key == K) {
      if (e < need) sm.cache[w++] = v[j];
      ++e;
    }
  }
  csync();
  const uint32_t ties = tot >> 16;
  return (tot & 0xFFFFu) + (ties < need ? ties : need);
}

// Cuts the cache to its exact k best (it holds at least k) and makes the k-th key the strict
// threshold.
__device__ void fcut_to_k(FScratch& sm, FState& fs, uint32_t k) {
  constexpr int kPer = kCache / kThreads;
  const uint32_t i0 = threadIdx.x * kPer;
  const uint32_t n = fs.nbuf;
  uint32_t kk = 0, before = 0;
  block_kth32<kPer>(
      [&](int i, uint32_t* v) {
        const uint32_t x = i0 + static_cast<uint32_t>(i);
        *v = x < n ? static_cast<uint32_t>(sm.cache[x] >> 32) : 0u;
        return x < n;
      },
      k, sm, &kk, &before);
  fs.nbuf = fcompact(sm, n, kk, k - before);
  if (!fs.hasK || kk < fs.K) fs.K = kk;
  fs.hasK = true;
  fs.added = 0;
}

// The cache's exact k-th key (it holds at least k), without cutting.  Exact, not a bucket
// bound: on tie-heavy rows only the exact key as a strict threshold leaves later chunks quiet.
__device__ uint32_t fcache_kth(FScratch& sm, uint32_t n, uint32_t k) {
  constexpr int kPer = kCache / kThreads;
  const uint32_t i0 = threadIdx.x * kPer;
  uint32_t kk = 0, before = 0;
  block_kth32<kPer>(
      [&](int i, uint32_t* v) {
        const uint32_t x = i0 + static_cast<uint32_t>(i);
        *v = x < n ? static_cast<uint32_t>(sm.cache[x] >> 32) : 0u;
        return x < n;
      },
      k, sm, &kk, &before);
  return kk;
}

// ---- per-chunk thresholds --------------------------------------------------------------

// A certified chunk threshold from the group maxima (8 groups of 4 floats per thread, 2048 in
// all; each maximum is a distinct element): the 16-bit bucket bound of their k-th best key, so
// at least k elements have a key <= it.  False when fewer than k groups hold a number.
__device__ bool fgroup_kth(const StageInfo& si, const uint8_t* buf, FScratch& sm, uint32_t k,
                           uint32_t* kc) {
  const int tid = threadIdx.x;
  float mx[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) mx[g] = __int_as_float(0x7FC00000);  // NaN: an empty group
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int vi = j * kThreads + tid;
    if (vi < si.nvc) {
      uint4 w = lds128(buf + vi * 16);
      if (vi == si.vlo || vi == si.vhi) {
        const uint32_t vm = valid_mask4(si.cv0 + vi, si.a0, si.a1);
        if (!(vm & 1u)) w.x = 0x7FC00000u;
        if (!(vm & 2u)) w.y = 0x7FC00000u;
        if (!(vm & 4u)) w.z = 0x7FC00000u;
        if (!(vm & 8u)) w.w = 0x7FC00000u;
      }
      const int h = (j >> 2) * 4;  // rounds 0-3 and 4-7 form separate groups
      mx[h + 0] = fmaxf(mx[h + 0], __uint_as_float(w.x));  // fmaxf skips a NaN operand
      mx[h + 1] = fmaxf(mx[h + 1], __uint_as_float(w.y));
      mx[h + 2] = fmaxf(mx[h + 2], __uint_as_float(w.z));
      mx[h + 3] = fmaxf(mx[h + 3], __uint_as_float(w.w));
    }
  }
  uint32_t keys[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) keys[g] = desc_key32(__float_as_uint(mx[g]));
  uint32_t before;
  return block_kth32<8, 2>(
      [&](int i, uint32_t* v) {
        *v = keys[i];
        return keys[i] != kNaNKey;
      },
      k, sm, kc, &before);
}

// The exact k-th smallest key among the survivors counted in c (at least k of them).
__device__ uint32_t fsurvivor_kth(const uint8_t* buf, const FCount& c, FScratch& sm, uint32_t k) {
  const int tid = threadIdx.x;
  uint32_t kk = 0, before = 0;
  block_kth32<32>(
      [&](int i, uint32_t* v) {
        const int j = i >> 2, x = i & 3;
        const bool ok = (c.M >> i) & 1u;
        *v = ok ? desc_key32(word_of(lds128(buf + (j * kThreads + tid) * 16), x)) : 0u;
        return ok;
      },
      k, sm, &kk, &before);
  return kk;
}

// Appends this chunk's exact top k among the survivors counted in t (at least k, under a
// threshold certified for this chunk): the k-th smallest survivor key T2 (t's own threshold
// when t was tie-counted there and fewer than k survivors beat it), every survivor below T2
// and the first ties at T2 by index.  The cache first drops what these k entries beat and,
// if still short of room, is cut to its k best.  Returns false when a wait failed.
__device__ bool fappend_topk(const StageInfo& si, const uint8_t* buf, FCount& t, uint32_t T,
                             bool tie_counted, FScratch& sm, FState& fs, uint32_t k, int& par) {
  uint32_t T2 = T;
  if (!tie_counted || t.total >= k) {
    T2 = fsurvivor_kth(buf, t, sm, k);
    t = fcount<kTies>(si, buf, sm, T2, par);
    if (t.fail) return false;
  }
  const uint32_t need = k - t.total;
  if (k > kCache - fs.nbuf && fs.nbuf > 0 && T2 != kNaNKey) {
    fs.nbuf = fcompact(sm, fs.nbuf, T2 + 1u, 0u);  // entries with key > T2 are beaten
  }
  if (k > kCache - fs.nbuf) fcut_to_k(sm, fs, k);
  fappend<true>(si, buf, t, need, sm, fs.nbuf);
  fs.nbuf += k;
  fs.added = 0;
  fs.quiet = false;
  if (!fs.hasK || T2 < fs.K) fs.K = T2;
  fs.hasK = true;
  return true;
}

// One non-empty chunk.  Returns false when a wait failed.
__device__ bool fchunk(const StageInfo& si, const uint8_t* buf, FScratch& sm, FState& fs,
                       uint32_t k, int& par) {
  constexpr uint32_t C = kCache;
  const int tid = threadIdx.x;
  if (fs.quiet && fs.hasK && float_threshold(fs.K)) {  // after a quiet chunk: one OR-barrier
    // the maximum of the thread's values (fmaxf skips NaN) against the threshold's value
    float mx = __int_as_float(0x7FC00000);
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      const int vi = j * kThreads + tid;
      if (vi < si.nvc) {
        uint4 w = lds128(buf + vi * 16);
        if (vi == si.vlo || vi == si.vhi) {
          const uint32_t vm = valid_mask4(si.cv0 + vi, si.a0, si.a1);
          if (!(vm & 1u)) w.x = 0x7FC00000u;
          if (!(vm & 2u)) w.y = 0x7FC00000u;
          if (!(vm & 4u)) w.z = 0x7FC00000u;
          if (!(vm & 8u)) w.w = 0x7FC00000u;
        }
        mx = fmaxf(fmaxf(mx, fmaxf(__uint_as_float(w.x), __uint_as_float(w.y))),
                   fmaxf(__uint_as_float(w.z), __uint_as_float(w.w)));
      }
    }
    if (!group_or<kThreads>(mx > key_value(fs.K) || sm.fail != 0)) return true;
  }
  FCount c;
  bool counted = false;
  if (fs.hasK && !fs.rising) {
    uint32_t total;
    if (float_threshold(fs.K)) {
      const CCount32 cc = fcount_contig<true>(si, buf, sm, fs.K, par);
      if (cc.fail) return false;
      total = cc.total;
      if (total <= C - fs.nbuf) {
        if (cc.maxcnt <= kClusterMax) {
          fappend_contig(si, buf, cc, sm, fs.nbuf);
        } else {
          c = fcount<kLt>(si, buf, sm, fs.K, par);
          if (c.fail) return false;
          fappend<false>(si, buf, c, 0u, sm, fs.nbuf);
        }
      }
    } else {
      c = fcount<kLt>(si, buf, sm, fs.K, par);
      if (c.fail) return false;
      total = c.total;
      if (total <= C - fs.nbuf) fappend<false>(si, buf, c, 0u, sm, fs.nbuf);
    }
    if (total <= C - fs.nbuf) {
      fs.nbuf += total;
      fs.added += total;
      fs.quiet = total == 0;
      if (fs.added >= k && fs.nbuf >= k) {  // k more since the last tightening
        const uint32_t kk = fcache_kth(sm, fs.nbuf, k);
        if (kk < fs.K) fs.K = kk;
        fs.added = 0;
      }
      return true;
    }
    counted = true;
  }
  uint32_t kc = 0;
  const bool have_kc = fgroup_kth(si, buf, sm, k, &kc);
  if (sm.fail) return false;
  const bool own = have_kc && (!fs.hasK || kc < fs.K);
  fs.rising = (counted || fs.rising) && own;
  if (own && float_threshold(kc) && kCache - fs.nbuf >= k + k / 8) {
    // every value with key <= kc, when the cache has room for them (the usual first chunk)
    const CCount32 cc = fcount_contig<false>(si, buf, sm, kc, par);
    if (cc.fail) return false;
    if (cc.total <= C - fs.nbuf && cc.maxcnt <= kClusterMax) {
      fappend_contig(si, buf, cc, sm, fs.nbuf);
      fs.nbuf += cc.total;
      fs.added = 0;
      fs.quiet = false;
      fs.K = kc;  // certified: >= k values with key <= kc are in the cache now
      fs.hasK = true;
      return true;
    }
  }
  if (own) {
    FCount t = fcount<kTies>(si, buf, sm, kc, par);
    if (t.fail) return false;
    const uint32_t all = t.total + t.total_eq;
    if (all <= C - fs.nbuf && C - fs.nbuf >= k + k / 8) {  // every value with key <= kc fits
      fappend<true>(si, buf, t, t.total_eq, sm, fs.nbuf);
      fs.nbuf += all;
      fs.added = 0;
      fs.quiet = false;
      fs.K = kc;  // certified: >= k values with key <= kc are in the cache now
      fs.hasK = true;
      return true;
    }
    return fappend_topk(si, buf, t, kc, true, sm, fs, k, par);
  }
  // kc is no better than the segment's threshold (or there is neither)
  c = fs.hasK ? fcount<kLt>(si, buf, sm, fs.K, par) : fcount<kAll>(si, buf, sm, 0u, par);
  if (c.fail) return false;
  if (c.total > C - fs.nbuf && fs.nbuf > k) {
    const uint32_t K1 = fs.K;
    fcut_to_k(sm, fs, k);
    if (fs.K != K1) {
      c = fcount<kLt>(si, buf, sm, fs.K, par);
      if (c.fail) return false;
    }
  }
  if (c.total <= C - fs.nbuf) {
    fappend<false>(si, buf, c, 0u, sm, fs.nbuf);
    fs.nbuf += c.total;
    fs.quiet = c.total == 0;
    return true;
  }
  return fappend_topk(si, buf, c, fs.K, false, sm, fs, k, par);
}

// ---- row output ------------------------------------------------------------------------

// Writes row s from the n <= 1024 composites at sm.cache[0 .. n): the first k in ascending
// composite order, the value bits read back from the input by index; when n < k, slots
// n .. k-1 get -inf and index -1.
__device__ void fsort_emit(const TopkParams& p, FScratch& sm, uint32_t n, int s, long long a0,
                           long long len) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const uint32_t warp = static_cast<uint32_t>(tid >> 5);
  const uint32_t k = static_cast<uint32_t>(p.k);
  const uint32_t runs = (n + 127) / 128;
  unsigned long long x[4];
  if (warp < runs) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t i = warp * 128 + r * 32 + lane;
      x[r] = i < n ? sm.cache[i] : ~0ull;
    }
    warp_sort_regs<4>(x);
  }
  csync();
  if (warp < runs) {
#pragma unroll
    for (int r = 0; r < 4; ++r) sm.cache[warp * 128 + r * 32 + lane] = x[r];
  }
  csync();
  uint32_t* ov = p.out_values32 + static_cast<long long>(s) * k;
  int* oi = p.out_indices + static_cast<long long>(s) * k;
  const uint32_t* in32 = reinterpret_cast<const uint32_t*>(p.base);
  if (warp < runs) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const unsigned long long v = x[r];
      if (v == ~0ull) continue;
      uint32_t rank = static_cast<uint32_t>(r * 32 + lane);
      for (uint32_t q = 0; q < runs; ++q) {
        if (q == warp) continue;
        const unsigned long long* run = sm.cache + q * 128;
        uint32_t lo = 0;
#pragma unroll
        for (uint32_t step = 128; step > 0; step >>= 1) {
          if (lo + step <= 128 && run[lo + step - 1] < v) lo += step;
        }
        rank += lo;
      }
      if (rank < k) {
        const uint32_t idx = static_cast<uint32_t>(v & 0xFFFFFFFFu);
        ov[rank] = in32[a0 + idx];
        oi[rank] = static_cast<int>(idx);
      }
    }
  }
  for (uint32_t r = n + tid; r < k; r += kThreads) {
    ov[r] = p.pad_bits;
    oi[r] = -1;
  }
  if (tid == 0) {
    if (n < k && len >= static_cast<long long>(k)) atomicOr(&p.status[0], kStatusCertifyFailed);
    if (p.stats) atomicAdd(&p.status[4], 1u);
  }
  csync();
}

// End of this block's part of segment fs.s: write the row, or publish the part's top k and,
// if this block finishes the segment, merge all parts in index order.
__device__ void fclose(const TopkParams& p, FState& fs, FScratch& sm) {
  if (fs.mycnt == 0) return;
  const uint32_t k = static_cast<uint32_t>(p.k);
  const long long len = fs.a1 - fs.a0;
  if (fs.mycnt == fs.nchunks) {
    // the sort ranks up to 1024 entries and writes the first k: no cut below that
    if (fs.nbuf > 1024) fcut_to_k(sm, fs, k);
    fsort_emit(p, sm, fs.nbuf, fs.s, fs.a0, len);
    return;
  }
  if (fs.nbuf > k) fcut_to_k(sm, fs, k);
  const int tid = threadIdx.x;
  unsigned long long* dst = reinterpret_cast<unsigned long long*>(p.cand + fs.part_slot * p.cap);
  for (uint32_t i = tid; i < fs.nbuf; i += kThreads) dst[i] = sm.cache[i];
  __threadfence();
  csync();
  if (tid == 0) {
    p.chunk_count[fs.part_slot] = fs.nbuf;
    __threadfence();
    const uint32_t old = atomicAdd(&p.seg_done[fs.s], static_cast<uint32_t>(fs.mycnt));
    sm.bcast[0] = old + static_cast<uint32_t>(fs.mycnt) == static_cast<uint32_t>(fs.nchunks);
  }
  csync();
  if (!sm.bcast[0]) return;
  __threadfence();
  uint32_t n = 0;
  for (int c0 = 0; c0 < fs.nchunks; c0 += kThreads) {
    const int c = c0 + tid;
    sm.tbase[tid] = c < fs.nchunks ? __ldcg(&p.chunk_count[fs.seg_slot + c]) : 0u;
    csync();
    const int m = fs.nchunks - c0 < kThreads ? fs.nchunks - c0 : kThreads;
    for (int j = 0; j < m; ++j) {
      const uint32_t cj = sm.tbase[j];
      if (cj == 0) continue;
      if (n + cj > static_cast<uint32_t>(kCache)) {
        fs.nbuf = n;
        fcut_to_k(sm, fs, k);
        n = fs.nbuf;
      }
      const unsigned long long* src =
          reinterpret_cast<const unsigned long long*>(p.cand + (fs.seg_slot + c0 + j) * p.cap);
      for (uint32_t i = tid; i < cj; i += kThreads) sm.cache[n + i] = __ldcg(src + i);
      n += cj;
      csync();
    }
    csync();
  }
  fs.nbuf = n;
  if (fs.nbuf > 1024) fcut_to_k(sm, fs, k);
  fsort_emit(p, sm, fs.nbuf, fs.s, fs.a0, len);
}

__device__ void fconsumer_loop(const TopkParams& p, uint8_t* stages, uint64_t* full,
                               uint64_t* empty, const StageInfo* info, FScratch& sm) {
  constexpr int S = FLayout::S;
  const uint32_t k = static_cast<uint32_t>(p.k);
  FState fs;
  int st = 0, par = 0;
  uint32_t ph = 0;
  bool failed = false;
  for (;;) {
    // A failed wait is noticed by every consumer at the next barrier (sm.fail); stage info is
    // never garbage (initialised), so all keep taking the same branches.
    if (!mbar_wait(&full[st], ph)) sm.fail = 1u;
    const StageInfo& si = info[st];
    if (si.part != fs.part) {
      if (group_or<kThreads>(sm.fail != 0)) {
        failed = true;
        break;
      }
      fclose(p, fs, sm);
      if (si.part == kStopPart) break;
      fs = FState{};
      fs.s = si.s;
      fs.part = si.part;
      fs.nchunks = si.nchunks;
      fs.part_slot = si.slot;
      fs.seg_slot = si.slot - si.c;
      fs.a0 = si.a0;
      fs.a1 = si.a1;
    }
    if (si.nvc > 0) {
      const uint8_t* buf = stages + static_cast<size_t>(st) * kStageBytes;
      if (!fchunk(si, buf, sm, fs, k, par)) {
        failed = true;
        break;
      }
      ++fs.mycnt;
    }
    release_stage(&empty[st]);
    if (++st == S) {
      st = 0;
      ph ^= 1u;
    }
  }
  if (failed && threadIdx.x == 0) atomicOr(&p.status[0], kStatusWaitTimeout);
  if (failed) sm.fail = 1u;
}

// 96 registers: two 9-warp blocks per SM.
__global__ void __maxnreg__(96) topk_kernel(TopkParams p) {
  using L = FLayout;
  constexpr int S = L::S;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  FScratch& sm = *reinterpret_cast<FScratch*>(smem + L::off_scratch);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::off_full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L::off_empty);
  StageInfo* info = reinterpret_cast<StageInfo*>(smem + L::off_info);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int st = 0; st < S; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kWarps);
      StageInfo z{};
      z.s = -1;
      z.part = kStopPart;
      z.vlo = z.vhi = -1;
      info[st] = z;
    }
    fence_mbar_init();
    sm.fail = 0u;
  }
  if (tid < 256) sm.hist[tid] = 0;
  __syncthreads();
  grid_dep_wait();    // the set-up kernel's resets are complete and visible from here on
  grid_dep_launch();  // the next call's set-up kernel may launch (it waits for this grid)
  if (tid >= kThreads) {
    if (tid == kThreads) producer_loop<true>(p, stages, full, empty, info, &sm.fail);
    return;
  }
  fconsumer_loop(p, stages, full, empty, info, sm);
}

}  // namespace f32
}  // namespace bt
