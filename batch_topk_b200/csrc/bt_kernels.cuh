// bt_kernels.cuh -- the batched fp16 top-k pipeline for sm_100a.
//
// One streaming pass over HBM replaces the reference's three full reads
// (src/radix_histogram.cuh K1/K2 and src/candidate_compact.cuh K9):
//
//  chunk_kernel (persistent, 2 CTAs/SM, 3-stage cp.async.bulk pipeline of 32 KiB chunks)
//    For each chunk of a segment (<= 16384 values):
//      1. certified threshold: the k-th best of the chunk's group maxima.  Each maximum
//         is a distinct element, so at least k elements of the chunk are >= it, and every
//         member of the segment's top-k is >= it.  The chunk publishes it with atomicMin on
//         the segment's descending key; later chunks try the published value first.
//      2. ordered compaction: values >= threshold are written, in index order, to the
//         chunk's candidate slot (fp16 bits << 16 | chunk-local index).  Ballot-free: an
//         8-bit half2 compare mask per 16-byte vector, popc, one block exclusive scan.
//      3. if more than `cap` candidates survive, an exact local select (two 8-bit digit
//         passes over smem, the reference's radix_boundary_select logic) keeps exactly the
//         chunk's k best, lowest index first among ties.
//  merge_kernel (one CTA per segment)
//    Concatenates the segment's chunk lists (index order), drops entries worse than the
//    segment's final threshold, finds the exact cutoff key with two 8-bit digit passes,
//    keeps keys below the cutoff plus the first ties by index, and bitonic-sorts those <= k
//    entries by (key, index).  This is the reference's boundary select + compaction + final
//    sort (src/radix_boundary_select.cuh, src/candidate_compact.cuh, src/final_topk50.cuh)
//    applied to a few hundred candidates instead of the whole segment.
#pragma once

#include <cstddef>
#include <cstdint>

#include "bt_device.cuh"

namespace bt {

struct TopkParams {
  const uint16_t* base;          // d_input rounded down to 16 bytes
  int shift;                     // d_input - base, in elements (0..7)
  int seg_num;
  long long seg_len;             // fixed-length rows (offsets == nullptr)
  const int* offsets;            // CSR offsets (seg_num + 1) or nullptr
  int p_max;                     // fixed-length: chunk slots per segment
  uint32_t* chunk_start;         // CSR: first slot of each segment (seg_num + 1)
  long long slot_capacity;       // chunk slots in the workspace
  int k;
  int groups;                    // group maxima per thread in the threshold select
  int cap;                       // candidate capacity per chunk slot
  int reuse;                     // try the published segment threshold first
  int stats;                     // count events into status[1..4]
  uint32_t* seg_thresh;          // [seg_num]
  uint32_t* chunk_count;         // [slot_capacity]
  uint32_t* cand;                // [slot_capacity * cap]
  uint32_t* status;              // [16]
  uint16_t* out_values;          // [seg_num * k]
  int* out_indices;              // [seg_num * k]
};

struct SegGeom {
  long long a0, a1;  // aligned element coordinates of the segment [start, end)
  long long v0;      // first aligned 16-byte vector
  long long nv;      // vectors spanned
  int nchunks;
  int chunk_vecs;    // vectors per chunk (the last one may hold fewer)
};

__device__ __forceinline__ SegGeom seg_geom(const TopkParams& p, int s) {
  long long g0, g1;
  if (p.offsets) {
    g0 = p.offsets[s];
    g1 = p.offsets[s + 1];
    if (g0 < 0 || g1 < g0) g1 = g0 = 0;
  } else {
    g0 = static_cast<long long>(s) * p.seg_len;
    g1 = g0 + p.seg_len;
  }
  SegGeom g;
  g.a0 = g0 + p.shift;
  g.a1 = g1 + p.shift;
  g.v0 = g.a0 >> 3;
  g.nv = (g.a1 > g.a0) ? ((g.a1 + 7) >> 3) - g.v0 : 0;
  g.nchunks = static_cast<int>((g.nv + kVecPerChunk - 1) / kVecPerChunk);
  g.chunk_vecs = g.nchunks ? static_cast<int>((g.nv + g.nchunks - 1) / g.nchunks) : 0;
  return g;
}

struct StageInfo {
  long long cv0;   // first aligned vector of the chunk
  long long a0, a1;
  long long slot;
  int s;
  int nvc;         // vectors in the chunk; 0 = nothing to do
  uint32_t g_prev; // the segment's published threshold when the load was issued
  int pad;
};

struct alignas(16) ChunkSmem {
  uint32_t hist1[256];  // 16-byte aligned: warp_find_bin reads it with 128-bit loads
  uint32_t hist2[256];
  uint32_t warp_tot[kWarps];
  int bin1, bin2;
  uint32_t before1, before2;
};

// Dynamic shared memory: [stages | ChunkSmem | mbarriers | StageInfo].
constexpr size_t kSmemOffScratch = static_cast<size_t>(kStages) * kStageBytes;
constexpr size_t kSmemOffBars = kSmemOffScratch + sizeof(ChunkSmem);
constexpr size_t kSmemOffInfo = kSmemOffBars + kStages * sizeof(uint64_t);
constexpr size_t kChunkSmemBytes = kSmemOffInfo + kStages * sizeof(StageInfo);
static_assert(kSmemOffScratch % 16 == 0 && sizeof(ChunkSmem) % 16 == 0, "hist alignment");
static_assert(kSmemOffBars % 8 == 0 && kSmemOffInfo % 8 == 0, "mbarrier/info alignment");

// Processing order of chunk work items.  Fixed-length rows go chunk-major (all segments'
// chunk 0, then chunk 1, ...) so later chunks find a published threshold.  CSR batches go
// in slot order.
__device__ __forceinline__ void decode_work(const TopkParams& p, long long q, int* s, int* c,
                                            long long* slot) {
  if (!p.offsets) {
    *c = static_cast<int>(q / p.seg_num);
    *s = static_cast<int>(q % p.seg_num);
    *slot = static_cast<long long>(*s) * p.p_max + *c;
  } else {
    int lo = 0, hi = p.seg_num;  // chunk_start[lo] <= q < chunk_start[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (static_cast<long long>(p.chunk_start[mid]) <= q) lo = mid; else hi = mid;
    }
    *s = lo;
    *c = static_cast<int>(q - p.chunk_start[lo]);
    *slot = q;
  }
}

// Issued by one thread: fills the stage's info and starts its bulk load.
__device__ __forceinline__ void issue_chunk(const TopkParams& p, long long q, StageInfo* info,
                                            uint8_t* buf, uint64_t* bar, uint64_t policy) {
  int s, c;
  long long slot;
  decode_work(p, q, &s, &c, &slot);
  const SegGeom g = seg_geom(p, s);
  StageInfo si;
  si.s = s;
  si.slot = slot;
  si.a0 = g.a0;
  si.a1 = g.a1;
  si.pad = 0;
  if (c >= g.nchunks) {
    si.nvc = 0;
    si.cv0 = 0;
  } else {
    si.cv0 = g.v0 + static_cast<long long>(c) * g.chunk_vecs;
    const long long rem = g.v0 + g.nv - si.cv0;
    si.nvc = static_cast<int>(rem < g.chunk_vecs ? rem : g.chunk_vecs);
  }
  si.g_prev = si.nvc > 0 ? __ldcg(&p.seg_thresh[s]) : kNoThreshold;
  *info = si;
  if (si.nvc > 0) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(si.nvc) * 16u);
    bulk_load(buf, p.base + si.cv0 * 8, static_cast<uint32_t>(si.nvc) * 16u, bar, policy);
  } else {
    mbar_arrive(bar);
  }
}

// k-th best group maximum of the chunk (descending key), or kNoThreshold when the chunk has
// fewer than k non-NaN maxima.  Publishes it on the segment.  Block-uniform result.
__device__ uint32_t chunk_select(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                                 ChunkSmem& sm) {
  const int tid = threadIdx.x;
  uint32_t acc0 = 0x7E007E00u, acc1 = 0x7E007E00u, acc2 = 0x7E007E00u, acc3 = 0x7E007E00u;
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int vi = j * kThreads + tid;  // strided groups: 8 values kThreads vectors apart
    if (vi < si.nvc) {
      uint4 w = lds128(buf + vi * 16);
      const long long gv = si.cv0 + vi;
      if (gv * 8 < si.a0 || gv * 8 + 8 > si.a1) w = nan_fill(w, valid_mask8(gv, si.a0, si.a1));
      acc0 = h2_as_u32(__hmax2(u32_as_h2(acc0), u32_as_h2(w.x)));
      acc1 = h2_as_u32(__hmax2(u32_as_h2(acc1), u32_as_h2(w.y)));
      acc2 = h2_as_u32(__hmax2(u32_as_h2(acc2), u32_as_h2(w.z)));
      acc3 = h2_as_u32(__hmax2(u32_as_h2(acc3), u32_as_h2(w.w)));
    }
  }
  uint32_t keys[8];
  int ng;
  if (p.groups >= 8) {
    keys[0] = desc_key(acc0); keys[1] = desc_key(acc0 >> 16);
    keys[2] = desc_key(acc1); keys[3] = desc_key(acc1 >> 16);
    keys[4] = desc_key(acc2); keys[5] = desc_key(acc2 >> 16);
    keys[6] = desc_key(acc3); keys[7] = desc_key(acc3 >> 16);
    ng = 8;
  } else {
    const uint32_t m0 = h2_as_u32(__hmax2(u32_as_h2(acc0), u32_as_h2(acc2)));
    const uint32_t m1 = h2_as_u32(__hmax2(u32_as_h2(acc1), u32_as_h2(acc3)));
    if (p.groups == 4) {
      keys[0] = desc_key(m0); keys[1] = desc_key(m0 >> 16);
      keys[2] = desc_key(m1); keys[3] = desc_key(m1 >> 16);
      ng = 4;
    } else {
      const uint32_t m = h2_as_u32(__hmax2(u32_as_h2(m0), u32_as_h2(m1)));
      if (p.groups == 2) {
        keys[0] = desc_key(m); keys[1] = desc_key(m >> 16);
        ng = 2;
      } else {
        const __half2 mh = u32_as_h2(m);
        const __half top = __hmax(__low2half(mh), __high2half(mh));
        keys[0] = desc_key(*reinterpret_cast<const uint16_t*>(&top));
        ng = 1;
      }
    }
  }
  // round 1: high byte
  for (int i = 0; i < ng; ++i) hist_add_match(sm.hist1, keys[i] >> 8, true);
  __syncthreads();
  if (tid < 32) warp_find_bin(sm.hist1, 0, p.k, &sm.bin1, &sm.before1);
  __syncthreads();
  const int b1 = sm.bin1;
  uint32_t kc = kNoThreshold;
  if (b1 < 255) {
    // round 2: low byte inside the boundary bin
    for (int i = 0; i < ng; ++i) {
      hist_add_match(sm.hist2, keys[i] & 0xFFu, (keys[i] >> 8) == static_cast<uint32_t>(b1));
    }
    __syncthreads();
    if (tid < 32) warp_find_bin(sm.hist2, sm.before1, p.k, &sm.bin2, &sm.before2);
    __syncthreads();
    kc = (static_cast<uint32_t>(b1) << 8) | static_cast<uint32_t>(sm.bin2);
  }
  if (tid == 0) {
    if (kc < si.g_prev) atomicMin(&p.seg_thresh[si.s], kc);
    if (p.stats) atomicAdd(&p.status[3], 1u);
  }
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  return kc;
}

// 64-bit mask of this thread's candidates: bit 8*j+e for element e of vector tid*8+j.
__device__ __forceinline__ uint64_t candidate_mask(const StageInfo& si, const uint8_t* buf,
                                                   uint32_t kuse) {
  const int tid = threadIdx.x;
  const uint32_t vb = key_to_bits(kuse);
  const __half2 v2 = u32_as_h2(vb | (vb << 16));
  const bool take_all = kuse == kNoThreshold;
  const int sw = tid & 7;
  uint64_t M = 0;
#pragma unroll
  for (int jj = 0; jj < kVecPerThread; ++jj) {
    const int j = jj ^ sw;  // rotate the read order: conflict-free 16-byte smem reads
    const int vi = tid * kVecPerThread + j;
    if (vi < si.nvc) {
      const uint4 w = lds128(buf + vi * 16);
      uint32_t m = take_all ? 0xFFu : ge_mask8(w, v2);
      const long long gv = si.cv0 + vi;
      if (gv * 8 < si.a0 || gv * 8 + 8 > si.a1) m &= valid_mask8(gv, si.a0, si.a1);
      M |= static_cast<uint64_t>(m) << (8 * j);
    }
  }
  return M;
}

__device__ __forceinline__ void write_candidates(const TopkParams& p, const StageInfo& si,
                                                 const uint8_t* buf, uint64_t M,
                                                 uint32_t base) {
  const int tid = threadIdx.x;
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(buf) + tid * 64;
  uint32_t* out = p.cand + si.slot * p.cap + base;
  uint32_t r = 0;
  while (M) {
    const int pos = __ffsll(static_cast<long long>(M)) - 1;
    M &= M - 1;
    out[r++] = (static_cast<uint32_t>(v16[pos]) << 16) | static_cast<uint32_t>(tid * 64 + pos);
  }
}

// Exact top-k of the chunk's candidates (more than cap of them survived the threshold).
__device__ void exact_local(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                            ChunkSmem& sm, uint64_t M) {
  const int tid = threadIdx.x;
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(buf) + tid * 64;
  RunHist rh;
  for (uint64_t m = M; m; m &= m - 1) rh.add(sm.hist1, desc_key(v16[__ffsll(static_cast<long long>(m)) - 1]) >> 8);
  rh.flush(sm.hist1);
  __syncthreads();
  if (tid < 32) warp_find_bin(sm.hist1, 0, p.k, &sm.bin1, &sm.before1);
  __syncthreads();
  const uint32_t b1 = static_cast<uint32_t>(sm.bin1);
  for (uint64_t m = M; m; m &= m - 1) {
    const uint32_t key = desc_key(v16[__ffsll(static_cast<long long>(m)) - 1]);
    if ((key >> 8) == b1) rh.add(sm.hist2, key & 0xFFu);
  }
  rh.flush(sm.hist2);
  __syncthreads();
  if (tid < 32) warp_find_bin(sm.hist2, sm.before1, p.k, &sm.bin2, &sm.before2);
  __syncthreads();
  const uint32_t kstar = (b1 << 8) | static_cast<uint32_t>(sm.bin2);
  const uint32_t need = static_cast<uint32_t>(p.k) - sm.before2;
  uint32_t tcnt = 0;
  for (uint64_t m = M; m; m &= m - 1) {
    tcnt += desc_key(v16[__ffsll(static_cast<long long>(m)) - 1]) == kstar ? 1u : 0u;
  }
  uint32_t ttot;
  const uint32_t tbase = block_excl_scan<kThreads>(tcnt, &ttot, sm.warp_tot);
  uint64_t S = 0;
  uint32_t tr = tbase;
  for (uint64_t m = M; m; m &= m - 1) {
    const int pos = __ffsll(static_cast<long long>(m)) - 1;
    const uint32_t key = desc_key(v16[pos]);
    if (key < kstar) {
      S |= 1ull << pos;
    } else if (key == kstar) {
      if (tr < need) S |= 1ull << pos;
      ++tr;
    }
  }
  uint32_t stot;
  const uint32_t sbase = block_excl_scan<kThreads>(static_cast<uint32_t>(__popcll(S)), &stot,
                                                   sm.warp_tot);
  write_candidates(p, si, buf, S, sbase);
  if (tid == 0) {
    p.chunk_count[si.slot] = stot;
    if (p.stats) atomicAdd(&p.status[1], 1u);
  }
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
}

__device__ void process_chunk(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                              ChunkSmem& sm) {
  uint32_t kuse = si.g_prev;
  bool selected = false;
  if (kuse == kNoThreshold || !p.reuse) {
    const uint32_t kc = chunk_select(p, si, buf, sm);
    kuse = kc < kuse ? kc : kuse;
    selected = true;
  }
  for (;;) {
    const uint64_t M = candidate_mask(si, buf, kuse);
    uint32_t total;
    const uint32_t base = block_excl_scan<kThreads>(static_cast<uint32_t>(__popcll(M)), &total,
                                                    sm.warp_tot);
    if (total <= static_cast<uint32_t>(p.cap)) {
      write_candidates(p, si, buf, M, base);
      if (threadIdx.x == 0) {
        p.chunk_count[si.slot] = total;
        if (p.stats && !selected) atomicAdd(&p.status[2], 1u);
      }
      return;
    }
    if (!selected) {
      const uint32_t kc = chunk_select(p, si, buf, sm);
      kuse = kc < kuse ? kc : kuse;
      selected = true;
      continue;
    }
    exact_local(p, si, buf, sm, M);
    return;
  }
}

__global__ void __launch_bounds__(kThreads, 2)
chunk_kernel(TopkParams p, long long total_work) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>(smem + kSmemOffScratch);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemOffBars);
  StageInfo* info = reinterpret_cast<StageInfo*>(smem + kSmemOffInfo);
  const int tid = threadIdx.x;

  long long total = total_work;
  if (p.offsets) {
    const long long t = static_cast<long long>(p.chunk_start[p.seg_num]);
    total = t < p.slot_capacity ? t : p.slot_capacity;
  }
  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) mbar_init(&bars[st], 1);
    fence_mbar_init();
  }
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  __syncthreads();
  const uint64_t policy = policy_evict_first();
  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) {
      const long long q = blockIdx.x + static_cast<long long>(st) * gridDim.x;
      if (q < total) issue_chunk(p, q, &info[st], stages + st * kStageBytes, &bars[st], policy);
    }
  }
  for (long long i = 0;; ++i) {
    const long long q = blockIdx.x + i * gridDim.x;
    if (q >= total) break;
    const int st = static_cast<int>(i % kStages);
    const uint32_t parity = static_cast<uint32_t>((i / kStages) & 1);
    const bool ok = mbar_wait(&bars[st], parity);
    if (__syncthreads_or(!ok)) {
      // A bulk copy never completed: flag it, give in-flight copies one more bounded wait so
      // no copy lands after this block's shared memory is released, and stop.
      if (tid == 0) {
        atomicOr(&p.status[0], kStatusWaitTimeout);
        for (long long r = i; r < i + kStages; ++r) {
          const long long qq = blockIdx.x + r * gridDim.x;
          if (qq >= total) break;
          mbar_wait(&bars[r % kStages], static_cast<uint32_t>((r / kStages) & 1));
        }
      }
      __syncthreads();
      return;
    }
    const StageInfo si = info[st];
    if (si.nvc > 0) process_chunk(p, si, stages + st * kStageBytes, sm);
    __syncthreads();
    if (tid == 0) {
      const long long q2 = q + static_cast<long long>(kStages) * gridDim.x;
      if (q2 < total) issue_chunk(p, q2, &info[st], stages + st * kStageBytes, &bars[st], policy);
    }
  }
}

// ---- merge -----------------------------------------------------------------------------

struct alignas(16) MergeSmem {
  uint32_t hist1[256];  // first: 16-byte aligned for warp_find_bin's 128-bit loads
  uint32_t hist2[256];
  unsigned long long sel[kMaxK];
  uint32_t coff[kMaxChunksPerSegment + 1];
  uint32_t warp_tot[kMergeThreads / 32];
  int bin1, bin2;
  uint32_t before1, before2;
};
static_assert(offsetof(MergeSmem, hist2) % 16 == 0, "hist alignment");

// Walks this thread's contiguous range of the segment's concatenated candidate lists.
struct ItemCursor {
  const TopkParams* p;
  const MergeSmem* sm;
  long long slot0;
  long long first_elem;  // aligned element index of chunk 0's first vector
  long long a0;
  int chunk_vecs;
  int nch;
  uint32_t i0, i1;

  template <typename F>
  __device__ __forceinline__ void for_each(F&& f) const {
    if (i0 >= i1) return;
    int lo = 0, hi = nch;  // largest c with coff[c] <= i0
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (sm->coff[mid] <= i0) lo = mid; else hi = mid;
    }
    int c = lo;
    for (uint32_t i = i0; i < i1; ++i) {
      while (sm->coff[c + 1] <= i) ++c;
      const uint32_t w = __ldcg(&p->cand[(slot0 + c) * p->cap + (i - sm->coff[c])]);
      const uint32_t raw = w >> 16;
      const long long elem = first_elem + static_cast<long long>(c) * chunk_vecs * 8 + (w & 0xFFFFu);
      f(desc_key(raw), raw, static_cast<uint32_t>(elem - a0));
    }
  }
};

__global__ void __launch_bounds__(kMergeThreads) merge_kernel(TopkParams p) {
  __shared__ __align__(16) MergeSmem sm;
  constexpr int T = kMergeThreads;
  const int tid = threadIdx.x;
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  __syncthreads();
  const uint32_t k = static_cast<uint32_t>(p.k);
  for (int s = blockIdx.x; s < p.seg_num; s += gridDim.x) {
    const SegGeom g = seg_geom(p, s);
    const long long slot0 = p.offsets ? static_cast<long long>(p.chunk_start[s])
                                      : static_cast<long long>(s) * p.p_max;
    const int nch = g.nchunks;
    const bool bad = nch > kMaxChunksPerSegment ||
                     (p.offsets && (slot0 + nch > p.slot_capacity ||
                                    static_cast<long long>(p.chunk_start[s + 1]) - slot0 != nch));
    uint16_t* ov = p.out_values + static_cast<long long>(s) * k;
    int* oi = p.out_indices + static_cast<long long>(s) * k;
    if (bad) {
      if (tid == 0) {
        atomicOr(&p.status[0], nch > kMaxChunksPerSegment ? kStatusSegmentTooLong : kStatusBadOffsets);
      }
      for (uint32_t r = tid; r < k; r += T) {
        ov[r] = 0xFC00u;
        oi[r] = -1;
      }
      continue;
    }
    // prefix of the per-chunk candidate counts
    const int per = (nch + T - 1) / T;
    const int c0 = tid * per < nch ? tid * per : nch;
    const int c1 = c0 + per < nch ? c0 + per : nch;
    uint32_t local = 0;
    for (int c = c0; c < c1; ++c) {
      const uint32_t n = __ldcg(&p.chunk_count[slot0 + c]);
      local += n < static_cast<uint32_t>(p.cap) ? n : static_cast<uint32_t>(p.cap);
    }
    uint32_t n_all;
    uint32_t run = block_excl_scan<T>(local, &n_all, sm.warp_tot);
    for (int c = c0; c < c1; ++c) {
      sm.coff[c] = run;
      const uint32_t n = __ldcg(&p.chunk_count[slot0 + c]);
      run += n < static_cast<uint32_t>(p.cap) ? n : static_cast<uint32_t>(p.cap);
    }
    if (tid == 0) sm.coff[nch] = n_all;
    __syncthreads();
    const uint32_t kf = __ldcg(&p.seg_thresh[s]);
    ItemCursor cur;
    cur.p = &p;
    cur.sm = &sm;
    cur.slot0 = slot0;
    cur.first_elem = g.v0 * 8;
    cur.a0 = g.a0;
    cur.chunk_vecs = g.chunk_vecs;
    cur.nch = nch;
    const uint32_t R = (n_all + T - 1) / T;
    cur.i0 = tid * R < n_all ? tid * R : n_all;
    cur.i1 = cur.i0 + R < n_all ? cur.i0 + R : n_all;

    // exact cutoff over candidates with key <= kf: two 8-bit digit passes
    RunHist rh;
    cur.for_each([&](uint32_t key, uint32_t, uint32_t) {
      if (key <= kf) rh.add(sm.hist1, key >> 8);
    });
    rh.flush(sm.hist1);
    __syncthreads();
    if (tid < 32) warp_find_bin(sm.hist1, 0, k, &sm.bin1, &sm.before1);
    __syncthreads();
    const int b1 = sm.bin1;
    uint32_t kstar, need;
    if (b1 >= 256) {  // fewer than k candidates (segment shorter than k): keep them all
      kstar = 0x10000u;
      need = 0;
    } else {
      cur.for_each([&](uint32_t key, uint32_t, uint32_t) {
        if (key <= kf && (key >> 8) == static_cast<uint32_t>(b1)) rh.add(sm.hist2, key & 0xFFu);
      });
      rh.flush(sm.hist2);
      __syncthreads();
      if (tid < 32) warp_find_bin(sm.hist2, sm.before1, k, &sm.bin2, &sm.before2);
      __syncthreads();
      kstar = (static_cast<uint32_t>(b1) << 8) | static_cast<uint32_t>(sm.bin2);
      need = k - sm.before2;
    }
    // ties at the cutoff: ordered ranks
    uint32_t tcnt = 0;
    cur.for_each([&](uint32_t key, uint32_t, uint32_t) { tcnt += (key <= kf && key == kstar); });
    uint32_t ttot;
    const uint32_t tbase = block_excl_scan<T>(tcnt, &ttot, sm.warp_tot);
    uint32_t scnt = 0;
    {
      uint32_t tr = tbase;
      cur.for_each([&](uint32_t key, uint32_t, uint32_t) {
        if (key > kf) return;
        if (key < kstar) {
          ++scnt;
        } else if (key == kstar) {
          scnt += tr < need;
          ++tr;
        }
      });
    }
    uint32_t nsel;
    const uint32_t sbase = block_excl_scan<T>(scnt, &nsel, sm.warp_tot);
    {
      uint32_t tr = tbase, w = sbase;
      cur.for_each([&](uint32_t key, uint32_t raw, uint32_t idx) {
        if (key > kf) return;
        bool take = key < kstar;
        if (key == kstar) {
          take = tr < need;
          ++tr;
        }
        if (take) {
          sm.sel[w++] = (static_cast<unsigned long long>(key) << 48) |
                        (static_cast<unsigned long long>(idx) << 16) | raw;
        }
      });
    }
    int n2 = 1;
    while (n2 < static_cast<int>(nsel)) n2 <<= 1;
    for (int i = static_cast<int>(nsel) + tid; i < n2; i += T) sm.sel[i] = ~0ull;
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < n2 / 2; i += T) {
          const int lo = 2 * i - (i & (stride - 1));
          const int hi = lo + stride;
          const bool up = (lo & size) == 0;
          const unsigned long long a = sm.sel[lo], b = sm.sel[hi];
          if ((a > b) == up) {
            sm.sel[lo] = b;
            sm.sel[hi] = a;
          }
        }
        __syncthreads();
      }
    }
    for (uint32_t r = tid; r < k; r += T) {
      if (r < nsel) {
        const unsigned long long c = sm.sel[r];
        ov[r] = static_cast<uint16_t>(c & 0xFFFFu);
        oi[r] = static_cast<int>((c >> 16) & 0xFFFFFFFFu);
      } else {
        ov[r] = 0xFC00u;
        oi[r] = -1;
      }
    }
    if (tid == 0) {
      if (nsel < k && g.a1 - g.a0 >= static_cast<long long>(k)) atomicOr(&p.status[0], kStatusCertifyFailed);
      if (p.stats) atomicAdd(&p.status[4], 1u);
    }
    sm.hist1[tid] = 0;
    sm.hist2[tid] = 0;
    __syncthreads();
  }
}

// ---- set-up kernels -------------------------------------------------------------------

// Fixed-length rows: reset the per-segment thresholds and the status words.
__global__ void init_kernel(TopkParams p) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i < 16) p.status[i] = 0;
  for (long long s = i; s < p.seg_num; s += static_cast<long long>(gridDim.x) * blockDim.x) {
    p.seg_thresh[s] = kNoThreshold;
  }
}

// CSR batches: thresholds, status, and the chunk-slot prefix over segments (one block).
__global__ void __launch_bounds__(1024) csr_prep_kernel(TopkParams p) {
  __shared__ uint32_t warp_tot[32];
  const int tid = threadIdx.x;
  if (tid < 16) p.status[tid] = 0;
  __syncthreads();
  uint32_t carry = 0;
  for (int base = 0; base < p.seg_num; base += 1024) {
    const int s = base + tid;
    uint32_t nch = 0;
    if (s < p.seg_num) {
      p.seg_thresh[s] = kNoThreshold;
      nch = static_cast<uint32_t>(seg_geom(p, s).nchunks);
      if (p.offsets[s] < 0 || p.offsets[s + 1] < p.offsets[s]) atomicOr(&p.status[0], kStatusBadOffsets);
    }
    uint32_t tot;
    const uint32_t pre = block_excl_scan<1024>(nch, &tot, warp_tot);
    if (s < p.seg_num) p.chunk_start[s] = carry + pre;
    carry += tot;
  }
  if (tid == 0) {
    p.chunk_start[p.seg_num] = carry;
    if (static_cast<long long>(carry) > p.slot_capacity) atomicOr(&p.status[0], kStatusBadOffsets);
  }
}

}  // namespace bt
