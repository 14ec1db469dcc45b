// bt_body.cuh -- the kernels that read input values, compiled once per element type.
//
// Included by bt_kernels.cuh inside namespace bt::BT_ELEM_NS, once for fp16 (bt::f16) and
// once for bf16 (bt::bf16, with BT_ELEM_BF16 defined): no include guard.  Everything here
// reaches the values only through the element helpers of bt_elem.cuh (key codec, paired
// compares and maxima, NaN fill); the types, the producer and the key-only selection code
// they use live once in namespace bt.

namespace bt {
namespace BT_ELEM_NS {

#include "bt_elem.cuh"

// k-th smallest of the block's group keys, nw packed words (two 16-bit keys each) per thread
// held in kw (0xFFFF: a NaN maximum, never counted), or kNoThreshold when fewer than k keys are
// numeric: two 8-bit digit histograms over the block (per-thread runs aggregated before the
// shared atomics).  The histograms are zero on entry and left zero.
template <class SM>
__device__ __forceinline__ uint32_t block_kth_keys(const uint32_t (&kw)[4], int nw, uint32_t k,
                                                   SM& sm) {
  const int tid = threadIdx.x;
  RunHist rh;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (i < nw) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t key = (kw[i] >> (16 * h)) & 0xFFFFu;
        if (key != 0xFFFFu) rh.add(sm.hist1, key >> 8);
      }
    }
  }
  rh.flush(sm.hist1);
  csync();
  if (tid < 32) warp_find_bin(sm.hist1, 0, k, &sm.bin1, &sm.before1);
  csync();
  const int b1 = sm.bin1;
  uint32_t result = kNoThreshold;
  if (b1 < 256) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i < nw) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t key = (kw[i] >> (16 * h)) & 0xFFFFu;
          if (key != 0xFFFFu && (key >> 8) == static_cast<uint32_t>(b1)) {
            rh.add(sm.hist2, key & 0xFFu);
          }
        }
      }
    }
    rh.flush(sm.hist2);
    csync();
    if (tid < 32) warp_find_bin(sm.hist2, sm.before1, k, &sm.bin2, &sm.before2);
    csync();
    result = (static_cast<uint32_t>(b1) << 8) | static_cast<uint32_t>(sm.bin2);
  }
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  csync();
  return result;
}

// k-th best group maximum of the chunk (descending key), or kNoThreshold when the chunk has
// fewer than k non-NaN maxima.  Each maximum is a distinct element, so at least k elements
// of the chunk are >= it and every member of the segment's top-k is >= it.  k <= 128: two
// barriers (the group keys go to shared memory, warp 0 selects, and the result is broadcast);
// larger k: the block-wide digit select above over 1024 or 2048 group keys.
template <bool BIG>
__device__ uint32_t chunk_select(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                                 Scratch<BIG>& sm) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  uint32_t acc0 = kNaN2, acc1 = kNaN2, acc2 = kNaN2, acc3 = kNaN2;
  const int nvc = si.nvc, vlo = si.vlo, vhi = si.vhi;
  // Rolled: this pass runs once per segment, mostly with a cold instruction cache, where
  // the unrolled form cost about twice as many cycles.
#pragma unroll 1
  for (int j = 0; j < kVecPerThread; ++j) {
    const int vi = j * kThreads + tid;  // strided groups: values 2048 apart
    if (vi < nvc) {
      uint4 w = lds128(buf + vi * 16);
      if (vi == vlo || vi == vhi) w = nan_fill(w, valid_mask8(si.cv0 + vi, si.a0, si.a1));
      acc0 = h2_as_u32(__hmax2(u32_as_h2(acc0), u32_as_h2(w.x)));
      acc1 = h2_as_u32(__hmax2(u32_as_h2(acc1), u32_as_h2(w.y)));
      acc2 = h2_as_u32(__hmax2(u32_as_h2(acc2), u32_as_h2(w.z)));
      acc3 = h2_as_u32(__hmax2(u32_as_h2(acc3), u32_as_h2(w.w)));
    }
  }
  // group keys, packed two per 32-bit word: ng = 2 * nw keys per thread
  uint32_t kw[4];
  int nw;
  if (BIG && p.groups >= 8) {
    kw[0] = desc_key(acc0) | (desc_key(acc0 >> 16) << 16);
    kw[1] = desc_key(acc1) | (desc_key(acc1 >> 16) << 16);
    kw[2] = desc_key(acc2) | (desc_key(acc2 >> 16) << 16);
    kw[3] = desc_key(acc3) | (desc_key(acc3 >> 16) << 16);
    nw = 4;
  } else {
    const uint32_t m0 = h2_as_u32(__hmax2(u32_as_h2(acc0), u32_as_h2(acc2)));
    const uint32_t m1 = h2_as_u32(__hmax2(u32_as_h2(acc1), u32_as_h2(acc3)));
    if (BIG && p.groups == 4) {
      kw[0] = desc_key(m0) | (desc_key(m0 >> 16) << 16);
      kw[1] = desc_key(m1) | (desc_key(m1 >> 16) << 16);
      nw = 2;
    } else {
      const uint32_t m = h2_as_u32(__hmax2(u32_as_h2(m0), u32_as_h2(m1)));
      if (p.groups == 2) {
        kw[0] = desc_key(m) | (desc_key(m >> 16) << 16);
      } else {  // one maximum per thread; the pad key 0xFFFF never counts below a threshold
        kw[0] = desc_key(top_bits(m)) | 0xFFFF0000u;
      }
      nw = 1;
    }
  }
  if constexpr (BIG) {
    if (tid == 0 && p.stats) atomicAdd(&p.status[3], 1u);
    return block_kth_keys(kw, nw, static_cast<uint32_t>(p.k), sm);
  } else {
    for (int i = 0; i < nw; ++i) sm.gkeys[i * kThreads + tid] = kw[i];
    csync();
    if (tid < 32) {  // lane l owns words [l * per, (l + 1) * per) of the nw * kThreads words
      const int per = nw * kThreads / 32;
      const uint32_t K = per == 8 ? kth_keys16(sm.gkeys + lane * 8, static_cast<uint32_t>(p.k))
                                  : kth_packed_keys(sm.gkeys + lane * per, per,
                                                    static_cast<uint32_t>(p.k));
      if (lane == 0) sm.bcast[3] = K;
      if (lane == 0 && p.stats) atomicAdd(&p.status[3], 1u);
    }
    csync();
    return sm.bcast[3];  // 0xFFFF: no certified threshold (fewer than k non-NaN maxima)
  }
}

// Threshold test of one 16-byte vector: 8-bit element mask (bit e = element e) of values
// passing `key < K` (STRICT) or `key <= K`, i.e. value > V or value >= V (never NaN).
template <bool STRICT>
__device__ __forceinline__ uint32_t pass_mask8(const uint4& w, h2t v2) {
  return STRICT ? gt_mask8(w, v2) : ge_mask8(w, v2);
}

// Is any half of the vector passing?  (OR of the four compares, no compression.)
template <bool STRICT>
__device__ __forceinline__ bool pass_any(const uint4& w, h2t v2) {
  if (STRICT) {
    return (__hgt2_mask(u32_as_h2(w.x), v2) | __hgt2_mask(u32_as_h2(w.y), v2) |
            __hgt2_mask(u32_as_h2(w.z), v2) | __hgt2_mask(u32_as_h2(w.w), v2)) != 0;
  }
  return (__hge2_mask(u32_as_h2(w.x), v2) | __hge2_mask(u32_as_h2(w.y), v2) |
          __hge2_mask(u32_as_h2(w.z), v2) | __hge2_mask(u32_as_h2(w.w), v2)) != 0;
}

// This thread's 8 vectors (tid*8 .. tid*8+7): exact candidate mask of vector j, with the
// segment-boundary and take-all (no threshold yet) cases.
// Half e (element order) of a 16-byte vector, picked by selects, so neither a compile-time
// nor a run-time e indexes a register array.
__device__ __forceinline__ uint32_t vec_half(const uint4& w, int e) {
  const uint32_t word = e < 2 ? w.x : (e < 4 ? w.y : (e < 6 ? w.z : w.w));
  return (e & 1) ? (word >> 16) : (word & 0xFFFFu);
}

template <bool STRICT>
__device__ __forceinline__ uint32_t vec_mask(const StageInfo& si, const uint8_t* buf, int vi,
                                             h2t v2, bool take_all) {
  const uint4 w = lds128(buf + vi * 16);
  uint32_t m = take_all ? 0xFFu : pass_mask8<STRICT>(w, v2);
  if (vi == si.vlo || vi == si.vhi) m &= valid_mask8(si.cv0 + vi, si.a0, si.a1);
  return m;
}

// Flags (bit j: vector tid*8+j holds a candidate) and the exact candidate count of this
// thread.  Without DIRECT, a pre-test against the maximum of the thread's 64 values (three
// paired max instructions per vector) decides first, and exact masks follow only on a hit:
// cheapest when nothing passes.  With DIRECT (a count follows anyway), the masks are built in
// one pass: each 128-bit smem load is compared (four paired compares), and only the vectors
// that pass are counted exactly.
template <bool STRICT, bool DIRECT = false>
__device__ __forceinline__ uint32_t thread_flags(const StageInfo& si, const uint8_t* buf,
                                                 h2t v2, bool take_all, uint32_t* count) {
  const int tid = threadIdx.x;
  const int vbase = tid * kVecPerThread;
  const int sw = tid & 7;
  const bool edge = take_all || (si.vlo >= vbase && si.vlo < vbase + kVecPerThread) ||
                    (si.vhi >= vbase && si.vhi < vbase + kVecPerThread);
  uint32_t flags = 0, cnt = 0;
  if (!edge) {
    if (!DIRECT && vbase + kVecPerThread <= si.nvc) {
      // Common case: the maximum of the thread's 64 values (max ignores NaN, which never
      // passes) against the threshold; exact masks only when something passes.
      h2t acc = u32_as_h2(kNaN2);
#pragma unroll
      for (int jj = 0; jj < kVecPerThread; ++jj) {
        const uint4 w = lds128(buf + (vbase + (jj ^ sw)) * 16);  // rotated: conflict-free
        const h2t m01 = __hmax2(u32_as_h2(w.x), u32_as_h2(w.y));
        const h2t m23 = __hmax2(u32_as_h2(w.z), u32_as_h2(w.w));
        acc = __hmax2(acc, __hmax2(m01, m23));
      }
      const uint32_t hit = STRICT ? __hgt2_mask(acc, v2) : __hge2_mask(acc, v2);
      if (hit == 0) {
        *count = 0;
        return 0;
      }
    }
#pragma unroll
    for (int jj = 0; jj < kVecPerThread; ++jj) {
      const int j = jj ^ sw;
      const int vi = vbase + j;
      if (vi < si.nvc) {
        const uint4 w = lds128(buf + vi * 16);
        if (pass_any<STRICT>(w, v2)) {
          flags |= 1u << j;
          cnt += __popc(pass_mask8<STRICT>(w, v2));
        }
      }
    }
  } else {
    for (int j = 0; j < kVecPerThread; ++j) {
      const int vi = vbase + j;
      if (vi < si.nvc) {
        const uint32_t m = vec_mask<STRICT>(si, buf, vi, v2, take_all);
        if (m) {
          flags |= 1u << j;
          cnt += __popc(m);
        }
      }
    }
  }
  *count = cnt;
  return flags;
}

__device__ __forceinline__ unsigned long long make_composite(uint32_t word, long long chunk_elem0,
                                                             long long a0) {
  const uint32_t raw = word >> 16;
  const long long idx = chunk_elem0 + (word & 0xFFFFu) - a0;
  return (static_cast<unsigned long long>(desc_key(raw)) << 48) |
         (static_cast<unsigned long long>(idx) << 16) | raw;
}

// Block-wide k-th smallest key among the n composites of the segment buffer: two 8-bit digit
// histograms.  Each thread takes a contiguous run of entries (the buffer is in index order, so
// tie-heavy and sorted data give long runs of one bin) and adds run lengths with plain shared
// atomics.  kFewerThanK when n < k.  The histograms are zero on entry and left zero.
template <bool BIG>
__device__ uint32_t buffer_kth_key_block(Scratch<BIG>& sm, uint32_t n, uint32_t k) {
  if (n < k) return kFewerThanK;
  const int tid = threadIdx.x;
  const uint32_t R = (n + kThreads - 1) / kThreads;
  const uint32_t i0 = tid * R < n ? tid * R : n;
  const uint32_t i1 = i0 + R < n ? i0 + R : n;
  RunHist rh;
  for (uint32_t i = i0; i < i1; ++i) rh.add(sm.hist1, static_cast<uint32_t>(sm.cache[i] >> 56));
  rh.flush(sm.hist1);
  csync();
  if (tid < 32) warp_find_bin(sm.hist1, 0, k, &sm.bin1, &sm.before1);
  csync();
  const uint32_t b1 = static_cast<uint32_t>(sm.bin1);
  for (uint32_t i = i0; i < i1; ++i) {
    const uint32_t key = static_cast<uint32_t>(sm.cache[i] >> 48);
    if ((key >> 8) == b1) rh.add(sm.hist2, key & 0xFFu);
  }
  rh.flush(sm.hist2);
  csync();
  if (tid < 32) warp_find_bin(sm.hist2, sm.before1, k, &sm.bin2, &sm.before2);
  csync();
  const uint32_t kk = (b1 << 8) | static_cast<uint32_t>(sm.bin2);
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  csync();
  return kk;
}

// Exact top-k selection among the chunk's candidates under threshold K (strict or not, or
// take-all): the reference's two 8-bit digit passes plus ordered tie ranks.  Returns the
// cutoff key; *S gets this thread's selected elements (bit 8*j+e), *sbase their first output
// position and *stot the block total (== k).  Rare path.

// Writes this thread's selected elements (bit 8 j + e of S: element e of its vector j), in
// index order, as (key, index, bits) composites at out[0 ...]; e0 is the chunk's first aligned
// element, a0 the segment's.  A plain loop (no lambda capturing the running count, which
// would keep it in local memory).
__device__ __forceinline__ void write_selected(const uint8_t* buf, uint64_t S, long long e0,
                                               long long a0, unsigned long long* out) {
  const int tid = threadIdx.x;
  uint32_t r = 0;
#pragma unroll 1
  for (int j = 0; j < kVecPerThread; ++j) {
    uint32_t m8 = static_cast<uint32_t>(S >> (8 * j)) & 0xFFu;
    if (m8 == 0) continue;
    const uint4 w = lds128(buf + (tid * kVecPerThread + j) * 16);
    for (; m8; m8 &= m8 - 1) {
      const int e = __ffs(m8) - 1;
      const uint32_t lidx = static_cast<uint32_t>(tid * 64 + 8 * j + e);
      out[r++] = make_composite((vec_half(w, e) << 16) | lidx, e0, a0);
    }
  }
}

template <class SM>
__device__ uint32_t exact_local_select(const TopkParams& p, const StageInfo& si,
                                       const uint8_t* buf, SM& sm, uint32_t K, bool strict,
                                       uint64_t* S_out, uint32_t* sbase_out, uint32_t* stot_out) {
  const int tid = threadIdx.x;
  const bool take_all = K == kNoThreshold;
  const uint32_t vb = key_to_bits(K);
  const h2t v2 = u32_as_h2(vb | (vb << 16));
  uint64_t M = 0;
  for (int j = 0; j < kVecPerThread; ++j) {
    const int vi = tid * kVecPerThread + j;
    if (vi < si.nvc) {
      const uint32_t m = strict ? vec_mask<true>(si, buf, vi, v2, take_all)
                                : vec_mask<false>(si, buf, vi, v2, take_all);
      M |= static_cast<uint64_t>(m) << (8 * j);
    }
  }
  // The candidate passes walk all 64 element positions of the thread in the same order in
  // every lane, with predicated shared atomics: lane-dependent loops over set bits diverged,
  // and warp-aggregated adds (match_any, or a ballot for the first lane's bin) cost more than
  // the atomics they saved.
  const int sw = tid & 7;  // rotated vector order: a quarter-warp's 16-byte loads hit all banks
#pragma unroll 1
  for (int jj = 0; jj < kVecPerThread; ++jj) {
    const int j = jj ^ sw;
    const uint32_t m8 = static_cast<uint32_t>(M >> (8 * j)) & 0xFFu;
    const uint4 w = lds128(buf + (tid * kVecPerThread + j) * 16);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if ((m8 >> e) & 1u) atomicAdd(&sm.hist1[desc_key(vec_half(w, e)) >> 8], 1u);
    }
  }
  csync();
  if (tid < 32) warp_find_bin(sm.hist1, 0, p.k, &sm.bin1, &sm.before1);
  csync();
  const uint32_t b1 = static_cast<uint32_t>(sm.bin1);
#pragma unroll 1
  for (int jj = 0; jj < kVecPerThread; ++jj) {
    const int j = jj ^ sw;
    const uint32_t m8 = static_cast<uint32_t>(M >> (8 * j)) & 0xFFu;
    const uint4 w = lds128(buf + (tid * kVecPerThread + j) * 16);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t key = desc_key(vec_half(w, e));
      if (((m8 >> e) & 1u) && (key >> 8) == b1) atomicAdd(&sm.hist2[key & 0xFFu], 1u);
    }
  }
  csync();
  if (tid < 32) warp_find_bin(sm.hist2, sm.before1, p.k, &sm.bin2, &sm.before2);
  csync();
  const uint32_t kstar = (b1 << 8) | static_cast<uint32_t>(sm.bin2);
  const uint32_t need = static_cast<uint32_t>(p.k) - sm.before2;
  // keys below the cutoff, and this thread's ties at it, in index order
  uint64_t S = 0, T = 0;
#pragma unroll 1
  for (int jj = 0; jj < kVecPerThread; ++jj) {
    const int j = jj ^ sw;
    const uint32_t m8 = static_cast<uint32_t>(M >> (8 * j)) & 0xFFu;
    const uint4 w = lds128(buf + (tid * kVecPerThread + j) * 16);
    uint32_t lt = 0, eq = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t key = desc_key(vec_half(w, e));
      lt |= static_cast<uint32_t>(key < kstar) << e;
      eq |= static_cast<uint32_t>(key == kstar) << e;
    }
    S |= static_cast<uint64_t>(lt & m8) << (8 * j);
    T |= static_cast<uint64_t>(eq & m8) << (8 * j);
  }
  uint32_t ttot;
  const uint32_t tbase = block_excl_scan<kThreads, true>(static_cast<uint32_t>(__popcll(T)), &ttot,
                                                         sm.warp_tot);
  // the ties ranked below `need` by index join the selection
  for (uint32_t tr = tbase; T != 0 && tr < need; ++tr) {
    S |= T & (~T + 1);  // lowest remaining tie
    T &= T - 1;
  }
  *sbase_out =
      block_excl_scan<kThreads, true>(static_cast<uint32_t>(__popcll(S)), stot_out, sm.warp_tot);
  *S_out = S;
  if (tid == 0 && p.stats) atomicAdd(&p.status[1], 1u);
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  return kstar;
}

enum ChunkResult { kChunkDone = 0, kChunkOverflow = 1, kChunkFail = 2 };

// Keeps, in order, the segment buffer's composites with key < K and the first `need` with
// key == K, and returns the new count.  The buffer is in index order, so the ties dropped come
// after `need` earlier ties at K and all keys below K: with K the buffer's k-th key and need =
// k - (keys below K), they can no longer reach the top k, and exactly k composites remain.
// Each thread holds its kCacheCap / kThreads entries in registers across the scan's barriers,
// so the in-place writes never overtake a read.
template <bool BIG>
__device__ uint32_t compact_cache(Scratch<BIG>& sm, uint32_t n, uint32_t K, uint32_t need) {
  constexpr int kPer = Cfg<BIG>::kCacheCap / kThreads;
  const uint32_t i0 = threadIdx.x * kPer;
  unsigned long long v[kPer];
  uint32_t lt = 0, eq = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t i = i0 + j;
    v[j] = i < n ? sm.cache[i] : ~0ull;
    const uint32_t key = static_cast<uint32_t>(v[j] >> 48);
    lt += (i < n && key < K) ? 1u : 0u;
    eq += (i < n && key == K) ? 1u : 0u;
  }
  // both counts in one scan: each total is at most kCacheCap < 2^16
  uint32_t tot;
  const uint32_t pre = block_excl_scan<kThreads, true>(lt | (eq << 16), &tot, sm.warp_tot);
  uint32_t e = pre >> 16;  // ties before this thread's entries
  uint32_t w = (pre & 0xFFFFu) + (e < need ? e : need);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t i = i0 + j;
    const uint32_t key = static_cast<uint32_t>(v[j] >> 48);
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

#include "bt_small.cuh"
#include "bt_large.cuh"


// 96 registers: each SM sub-partition (16K registers) holds 5 warps, so two blocks of 9 or 10
// warps fit on an SM (with 112, a sub-partition would hold only 4 warps: one block per SM).
template <bool BIG>
__global__ void __maxnreg__(96)
topk_kernel(TopkParams p) {
  using L = SmemLayout<BIG>;
  constexpr int S = L::S;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  Scratch<BIG>& sm = *reinterpret_cast<Scratch<BIG>*>(smem + L::off_scratch);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::off_full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L::off_empty);
  StageInfo* info = reinterpret_cast<StageInfo*>(smem + L::off_info);
  const int tid = threadIdx.x;

  if (tid == 0) {
    if constexpr (!BIG) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&sm.batch_full[b], kWarps);
        mbar_init(&sm.batch_free[b], 1);
      }
      sm.kpub = ~0ull;  // tagged with segment -1: matches nothing
    }
    for (int st = 0; st < S; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kWarps);  // one arrival per consumer warp
      StageInfo z{};
      z.s = -1;
      z.part = kStopPart;
      z.vlo = z.vhi = -1;
      info[st] = z;  // a wait that times out then sees the stop item, never garbage
    }
    fence_mbar_init();
    sm.fail = 0u;
    if constexpr (BIG) sm.probe_req = 0u;
  }
  if (tid < 256) {
    sm.hist1[tid] = 0;
    sm.hist2[tid] = 0;
  }
  __syncthreads();
  grid_dep_wait();  // the set-up kernel's resets are complete and visible from here on
  // The next call's set-up kernel may launch now: it waits for this grid to complete (and
  // its memory to be visible) before it touches the workspace, so only its launch overlaps.
  grid_dep_launch();
  if (tid >= kThreads) {
    if (tid == kThreads) {
      if constexpr (BIG) {
        producer_loop<BIG>(p, stages, full, empty, info, &sm.fail, &sm.probe_req);
      } else {
        producer_loop<BIG>(p, stages, full, empty, info, &sm.fail);
      }
    } else if (!BIG && tid >= kThreads + 32) {
      if constexpr (!BIG) merger_loop(p, sm);
    }
    return;
  }
  if constexpr (BIG) {
    consumer_loop_large(p, stages, full, empty, info, sm);
  } else {
    consumer_loop_small(p, stages, full, empty, info, sm);
  }
}

}  // namespace BT_ELEM_NS
}  // namespace bt
