// bt_kernels.cuh -- the batched fp16 top-k pipeline for sm_100a.
//
// One streaming pass over HBM replaces the reference's three full reads (the high-byte and
// low-byte histograms, src/radix_histogram.cuh, and the compaction,
// src/candidate_compact.cuh).
//
// topk_kernel<BIG>: persistent, 2 blocks per SM (96 registers a thread), warp-specialised.
//   * Producer warp (one elected lane): claims work parts (a segment, or a run of its
//     chunks when there are fewer segments than blocks) from a global counter, in segment
//     order, and streams each chunk (<= 16384 fp16 values, 32 KiB) into a shared-memory
//     stage with one cp.async.bulk (no multicast), signalling a "full" mbarrier.
//   * 8 consumer warps, per chunk:
//       1. threshold: on the first chunk of a segment the k-th best of the chunk's group
//          maxima (a certified bound: every member of the segment's top-k is >= it), or the
//          previous segment's threshold when it still leaves between k and `cap` values.
//       2. candidate test: a 16-byte vector is skipped after four half2 compares against its
//          maximum; passing vectors give an 8-bit mask, and one block scan orders them.
//       3. strict mode: once k candidates with key <= K exist at lower indices, later
//          chunks only need keys strictly below K (ties at K can no longer win), which keeps
//          tie-heavy rows near k candidates.
//       4. more than `cap` survivors: an exact local select (two 8-bit digit passes, the
//          reference's radix_boundary_select logic) keeps exactly the chunk's k best.
//     then release the stage on an "empty" mbarrier.
//   * k <= 128 (bt_small.cuh): survivors go as (key, index, bits) composites to a merger
//     warp that keeps the segment's exact running top-k in registers (bitonic merges) and
//     publishes its k-th key back as the consumers' threshold.
//   * k > 128: chunk lists go to the workspace; at the segment's end the block that finishes
//     it (per-segment arrival counter) merges them: drops keys above the final threshold,
//     finds the exact cutoff with two 8-bit digit passes, keeps keys below it plus the first
//     ties by index, and places each survivor at its rank by (key, index).  This is the
//     reference's boundary select, compaction and final sort (src/radix_boundary_select.cuh,
//     src/candidate_compact.cuh, src/final_topk50.cuh, src/final_block_sort.cuh) on ~k
//     candidates, while the producer keeps prefetching the next chunks.
// Every wait (mbarrier, batch hand-off) has an iteration cap; on expiry the kernel sets
// BT_STATUS_WAIT_TIMEOUT in the workspace status word and finishes without further waits.
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
  uint32_t* part_start;          // CSR: first work part of each segment (seg_num + 1)
  long long slot_capacity;       // chunk slots in the workspace
  long long parts_total;         // fixed-length: number of work parts
  int part_chunks;               // at most this many chunks per work part
  int tail_seg0;                 // fixed-length: segments from here on are cut into
  int tail_parts;                //   tail_parts parts each (the last wave ends evenly)
  int steal;                     // whole segments, chunks claimed one by one, idle blocks help
  int help_window;               // how many of the last-claimed segments idle blocks may help
  uint32_t* chunk_next;          // [seg_num] next unclaimed chunk of each segment (steal)
  int k;
  int groups;                    // group maxima per thread in the threshold select
  int cap;                       // candidate capacity per chunk slot
  int stats;                     // count events into status[1..4]
  uint32_t* seg_thresh;          // [seg_num] thresholds shared by CTAs splitting a segment
  uint32_t* seg_done;            // [seg_num] chunks finished (arrival counter)
  uint32_t* chunk_count;         // [slot_capacity]
  uint32_t* chunk_off;           // [slot_capacity] merge scratch for very long segments
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

// Small k keeps three 32 KiB load stages; large k gives one up for a bigger merge buffer.
template <bool BIG>
struct Cfg {
  static constexpr int kStagesN = BIG ? 2 : 3;
  static constexpr int kSelCap = BIG ? kMaxK : 128;      // >= k
  static constexpr int kCacheCap = BIG ? 2048 : 1024;    // merge cache, 64-bit composites
  static constexpr int kCoffCap = 128;                   // chunks per segment in smem
  static constexpr int kGroupWords = BIG ? 4 : 1;        // packed group-max key words/thread
};

struct StageInfo {
  long long cv0;   // first aligned vector of the chunk
  long long a0, a1;
  long long slot;
  long long v0;    // first aligned vector of the segment
  int s, c;
  int nvc;         // vectors in the chunk; 0 = empty work item
  int nchunks;     // chunks of the segment
  int chunk_vecs;
  int vlo, vhi;    // chunk-relative vectors that straddle the segment ends (-1: none)
  int last;        // last chunk of this work part
  int part;        // work part id (kStopPart: no more work)
};
constexpr int kStopPart = -1;
constexpr uint32_t kWorkCounter = 8;  // status[8]: next work part to claim (reset per call)
constexpr uint32_t kHelpCounter = 9;  // status[9]: next segment an idle block helps
constexpr int kHelpMinChunks = 3;     // a helper joins a segment with at least this many left

template <bool BIG>
struct alignas(16) Scratch {
  uint32_t hist1[256];  // 16-byte aligned: warp_find_bin reads it with 128-bit loads
  uint32_t hist2[256];
  unsigned long long cache[Cfg<BIG>::kCacheCap];
  unsigned long long sel[Cfg<BIG>::kSelCap];
  alignas(16) uint32_t gkeys[Cfg<BIG>::kGroupWords * kThreads];  // 128-bit reads
  uint32_t coff[Cfg<BIG>::kCoffCap + 1];
  uint32_t coff2[Cfg<BIG>::kCoffCap + 1];  // per-chunk offsets of the survivors of the merge filter
  unsigned long long tmask[kThreads];      // balanced write: each thread's candidate bits
  uint32_t tbase[kThreads];                // balanced write: each thread's first output slot
  uint32_t warp_tot[kWarps];
  alignas(16) uint32_t wcnt[2][kWarps];  // per-warp candidate counts, double-buffered
  int bin1, bin2;
  uint32_t before1, before2;
  uint32_t bcast[4];
  uint32_t fail;
};

// k <= 128: per-segment state lives with the merger warp (bt_small.cuh).
constexpr int kBatchCap = 512;  // >= cap for k <= 128 (max(4k, 256))

struct BatchMeta {
  long long len;        // segment length (values)
  long long part_slot;  // slot of the first chunk of this block's part of the segment
  long long seg_slot;   // slot of the segment's chunk 0
  int s;
  uint32_t n;           // candidates in the batch
  int flags;            // kBatchEnd | kBatchStop
  int mycnt;            // chunks of the segment in this block's part, up to this batch
  int nchunks;
  uint32_t K;           // consumers' threshold for the segment
};
constexpr int kBatchEnd = 1;
constexpr int kBatchStop = 2;

template <>
struct alignas(16) Scratch<false> {
  uint32_t hist1[256];  // 16-byte aligned: warp_find_bin reads it with 128-bit loads
  uint32_t hist2[256];
  unsigned long long batch[2][kBatchCap];  // consumer -> merger candidate batches
  BatchMeta meta[2];
  uint64_t batch_full[2];                  // mbarriers: one arrival per consumer warp
  uint64_t batch_free[2];                  // mbarriers: one arrival by the merger
  unsigned long long kpub;                 // merger: (segment << 32) | k-th key
  alignas(16) uint32_t gkeys[Cfg<false>::kGroupWords * kThreads];  // 128-bit reads
  uint32_t warp_tot[kWarps];
  alignas(16) uint32_t wcnt[2][kWarps];  // per-warp candidate counts (128-bit reads)
  uint32_t kuse[2];
  int bin1, bin2;
  uint32_t before1, before2;
  uint32_t bcast[4];
  uint32_t fail;
};
using SmallScratch = Scratch<false>;

// Every array read with 128-bit shared loads (lds128) must start on a 16-byte boundary.
static_assert(offsetof(Scratch<false>, hist1) % 16 == 0 && offsetof(Scratch<false>, hist2) % 16 == 0 &&
              offsetof(Scratch<false>, gkeys) % 16 == 0 && offsetof(Scratch<false>, wcnt) % 16 == 0,
              "16-byte alignment of lds128 operands");
static_assert(offsetof(Scratch<true>, hist1) % 16 == 0 && offsetof(Scratch<true>, hist2) % 16 == 0 &&
              offsetof(Scratch<true>, gkeys) % 16 == 0, "16-byte alignment of lds128 operands");

// Dynamic shared memory: [stages | Scratch | full[] | empty[] | StageInfo[]].
template <bool BIG>
struct SmemLayout {
  static constexpr int S = Cfg<BIG>::kStagesN;
  static constexpr size_t off_scratch = static_cast<size_t>(S) * kStageBytes;
  static constexpr size_t off_full = off_scratch + sizeof(Scratch<BIG>);
  static constexpr size_t off_empty = off_full + S * sizeof(uint64_t);
  static constexpr size_t off_info = off_empty + S * sizeof(uint64_t);
  static constexpr size_t bytes = off_info + S * sizeof(StageInfo);
  static_assert(off_scratch % 16 == 0 && sizeof(Scratch<BIG>) % 16 == 0, "scratch alignment");
  static_assert(off_full % 8 == 0 && off_info % 8 == 0, "mbarrier/info alignment");
};

// k > 128: 8 consumer warps + 1 producer warp.  k <= 128: plus 1 merger warp.
template <bool BIG>
constexpr int block_threads() { return BIG ? kThreads + 32 : kThreads + 64; }

__device__ __forceinline__ void csync() { group_sync<kThreads>(); }

// ---- producer ------------------------------------------------------------------------

// Work parts: each segment's chunks are cut into ceil(nchunks / part_chunks) parts of
// near-equal size; blocks claim parts dynamically, in segment order.
__device__ __forceinline__ long long total_parts(const TopkParams& p) {
  return p.offsets ? static_cast<long long>(p.part_start[p.seg_num]) : p.parts_total;
}

// Part id -> segment and chunk range [*c0, *c1).
__device__ __forceinline__ void decode_part(const TopkParams& p, long long part, int* s, int* c0,
                                            int* c1, SegGeom* g, long long* slot0) {
  int seg, j, pps;
  if (!p.offsets) {
    const int per = (p.p_max + p.part_chunks - 1) / p.part_chunks;
    const long long head = static_cast<long long>(p.tail_seg0) * per;
    if (part < head) {
      seg = static_cast<int>(part / per);
      j = static_cast<int>(part - static_cast<long long>(seg) * per);
      pps = per;
    } else {
      const long long q = part - head;
      seg = p.tail_seg0 + static_cast<int>(q / p.tail_parts);
      j = static_cast<int>(q - static_cast<long long>(seg - p.tail_seg0) * p.tail_parts);
      pps = p.tail_parts;
    }
    *slot0 = static_cast<long long>(seg) * p.p_max;
  } else {
    int lo = 0, hi = p.seg_num;  // part_start[lo] <= part < part_start[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (static_cast<long long>(p.part_start[mid]) <= part) lo = mid; else hi = mid;
    }
    seg = lo;
    j = static_cast<int>(part - p.part_start[lo]);
    pps = static_cast<int>(p.part_start[lo + 1] - p.part_start[lo]);
    *slot0 = static_cast<long long>(p.chunk_start[seg]);
  }
  *g = seg_geom(p, seg);
  const int n = g->nchunks;
  *s = seg;
  *c0 = static_cast<int>(static_cast<long long>(j) * n / pps);
  *c1 = static_cast<int>(static_cast<long long>(j + 1) * n / pps);
}

template <bool BIG>
__device__ void producer_loop(const TopkParams& p, uint8_t* stages, uint64_t* full,
                              uint64_t* empty, StageInfo* info) {
  constexpr int S = Cfg<BIG>::kStagesN;
  const uint64_t policy = policy_evict_first();
  const long long nparts = total_parts(p);
  long long issued = 0;
  int st = 0;     // stage of the next load
  int round = 0;  // how many times every stage has been filled
  bool ok = true;
  // one stage: wait for it to be free, fill its info, start the copy (or just signal)
  auto put = [&](const StageInfo& si) -> bool {
    if (round > 0 && !mbar_wait(&empty[st], static_cast<uint32_t>((round - 1) & 1))) {
      atomicOr(&p.status[0], kStatusWaitTimeout);
      return false;
    }
    info[st] = si;
    if (si.nvc > 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(si.nvc) * 16u);
      bulk_load(stages + static_cast<size_t>(st) * kStageBytes, p.base + si.cv0 * 8,
                static_cast<uint32_t>(si.nvc) * 16u, &full[st], policy);
    } else {
      mbar_arrive(&full[st]);
    }
    ++issued;
    if (++st == S) {
      st = 0;
      ++round;
    }
    return true;
  };
  // chunk c of segment s (geometry g, chunk slots from slot0) as work part `part`
  auto chunk_info = [&](int s, const SegGeom& g, long long slot0, int c, int part, bool last_c) {
    StageInfo si;
    si.s = s;
    si.c = c;
    si.part = part;
    si.slot = slot0 + c;
    si.a0 = g.a0;
    si.a1 = g.a1;
    si.v0 = g.v0;
    si.nchunks = g.nchunks;
    si.chunk_vecs = g.chunk_vecs;
    si.last = last_c ? 1 : 0;
    si.cv0 = g.v0 + static_cast<long long>(c) * g.chunk_vecs;
    const long long rem = g.v0 + g.nv - si.cv0;
    si.nvc = static_cast<int>(rem < g.chunk_vecs ? rem : g.chunk_vecs);
    const long long first = g.v0 - si.cv0;
    const long long last = ((g.a1 - 1) >> 3) - si.cv0;
    si.vlo = ((g.a0 & 7) && first >= 0 && first < si.nvc) ? static_cast<int>(first) : -1;
    si.vhi = ((g.a1 & 7) && last >= 0 && last < si.nvc) ? static_cast<int>(last) : -1;
    return si;
  };
  if (p.steal) {
    // Whole segments, claimed in order.  A segment's chunks are claimed one at a time (one
    // ahead, so the claim's latency hides behind the stage wait).  Once every segment is
    // claimed, a block that has run dry helps one of the segments claimed last: it takes
    // the chunks the owner has not claimed yet, and the split-segment merge joins the two
    // lists.  Each visit of a block to a segment is one work part (numbered per block).
    int visit = 0;
    long long s = atomicAdd(&p.status[kWorkCounter], 1u);
    bool own = true;
    while (ok) {
      if (s >= p.seg_num) {
        own = false;
        const long long h = atomicAdd(&p.status[kHelpCounter], 1u);
        if (h >= p.help_window) break;
        s = p.seg_num - 1 - h;
      }
      const SegGeom g = seg_geom(p, static_cast<int>(s));
      const long long slot0 = s * p.p_max;
      if (!own && static_cast<int>(__ldcg(&p.chunk_next[s])) + kHelpMinChunks > g.nchunks) {
        s = p.seg_num;  // too little left to repay a helper's first chunk: try the next one
        continue;
      }
      int c = static_cast<int>(atomicAdd(&p.chunk_next[s], 1u));
      while (ok && c < g.nchunks) {
        const int cn = static_cast<int>(atomicAdd(&p.chunk_next[s], 1u));
        ok = put(chunk_info(static_cast<int>(s), g, slot0, c, visit, cn >= g.nchunks));
        c = cn;
      }
      ++visit;
      s = own ? static_cast<long long>(atomicAdd(&p.status[kWorkCounter], 1u)) : p.seg_num;
    }
  } else {
    long long part = atomicAdd(&p.status[kWorkCounter], 1u);
    while (ok && part < nparts) {
      const long long next = atomicAdd(&p.status[kWorkCounter], 1u);  // claim ahead
      int s, c0, c1;
      SegGeom g;
      long long slot0;
      decode_part(p, part, &s, &c0, &c1, &g, &slot0);
      for (int c = c0; c < c1 && ok; ++c) {
        ok = put(chunk_info(s, g, slot0, c, static_cast<int>(part), c == c1 - 1));
      }
      part = next;
    }
  }
  if (ok) {  // the stop sentinel
    StageInfo z{};
    z.s = -1;
    z.part = kStopPart;
    z.vlo = z.vhi = -1;
    ok = put(z);
  }
  // Do not retire while a bulk copy may still land in this block's shared memory.
  for (long long r = issued - S; r < issued; ++r) {
    if (r < 0) continue;
    mbar_wait(&full[r % S], static_cast<uint32_t>((r / S) & 1));
  }
}

// ---- consumer: per-chunk work ---------------------------------------------------------

// A consumer warp is done with a stage: one arrival per warp, after all its lanes.
__device__ __forceinline__ void release_stage(uint64_t* empty) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(empty);
}

struct SegState {
  int s = -1;
  int part = -2;              // work part (kStopPart never matches: -2)
  uint32_t K = kNoThreshold;  // current threshold key (desc)
  bool strict = false;        // later chunks need key < K
  bool spilled = false;       // the shared-memory candidate buffer overflowed
  int mycnt = 0;              // chunks of this segment processed here
  int nchunks = 0;
  int chunk_vecs = 0;
  uint32_t nbuf = 0;          // candidates of this segment in sm.cache
  uint32_t added = 0;         // candidates added since the threshold was last tightened
  bool quiet = false;         // the previous chunk of the part sent nothing
  bool rising = false;        // the previous chunk overflowed its threshold (large k)
  long long slot0 = 0, v0 = 0, a0 = 0, a1 = 0;
};


// k-th smallest of the packed 16-bit keys a warp holds at src (words [lane * per, +per) per
// lane; 0xFFFF keys are NaN maxima or padding), or 0xFFFF when fewer than k keys are
// numeric.  The search runs over [min, max] of the numeric keys in 4-ary steps: three
// independent warp counts per step instead of one dependent count per bit.
__device__ __forceinline__ uint32_t kth_packed_keys(const uint32_t* src, int per, uint32_t k) {
  uint32_t lo = 0xFFFFu, hi = 0u;
  for (int i = 0; i < per; i += 4) {
    const uint4 w = lds128(src + i);
    const uint32_t v[8] = {w.x & 0xFFFFu, w.x >> 16, w.y & 0xFFFFu, w.y >> 16,
                           w.z & 0xFFFFu, w.z >> 16, w.w & 0xFFFFu, w.w >> 16};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      lo = v[j] < lo ? v[j] : lo;
      hi = (v[j] < 0xFFFFu && v[j] > hi) ? v[j] : hi;
    }
  }
  lo = __reduce_min_sync(0xFFFFFFFFu, lo);
  hi = __reduce_max_sync(0xFFFFFFFFu, hi);
  auto count_le = [&](uint32_t m1, uint32_t m2, uint32_t m3, uint32_t* c1, uint32_t* c2,
                      uint32_t* c3) {
    uint32_t a = 0, b = 0, c = 0;
    for (int i = 0; i < per; i += 4) {
      const uint4 w = lds128(src + i);
      const uint32_t v[8] = {w.x & 0xFFFFu, w.x >> 16, w.y & 0xFFFFu, w.y >> 16,
                             w.z & 0xFFFFu, w.z >> 16, w.w & 0xFFFFu, w.w >> 16};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        a += v[j] <= m1 ? 1u : 0u;
        b += v[j] <= m2 ? 1u : 0u;
        c += v[j] <= m3 ? 1u : 0u;
      }
    }
    *c1 = __reduce_add_sync(0xFFFFFFFFu, a);
    *c2 = __reduce_add_sync(0xFFFFFFFFu, b);
    *c3 = __reduce_add_sync(0xFFFFFFFFu, c);
  };
  if (lo >= 0xFFFFu) return 0xFFFFu;
  uint32_t c1, c2, c3;
  count_le(hi, hi, hi, &c1, &c2, &c3);
  if (c1 < k) return 0xFFFFu;  // fewer than k numeric keys
  // invariant: the answer lies in [lo, hi] and at least k keys are <= hi
  while (lo < hi) {
    const uint32_t m2 = (lo + hi) >> 1;
    const uint32_t m1 = (lo + m2) >> 1;
    const uint32_t m3 = (m2 + 1u + hi) >> 1;
    count_le(m1, m2, m3, &c1, &c2, &c3);
    if (c1 >= k) {
      hi = m1;
    } else if (c2 >= k) {
      lo = m1 + 1u;
      hi = m2;
    } else if (c3 >= k) {
      lo = m2 + 1u;
      hi = m3;
    } else {
      lo = m3 + 1u;
    }
  }
  return lo;
}

// kth_packed_keys for 16 keys a lane (8 words at src), held in registers across the search
// steps instead of re-read from shared memory at each step.
__device__ __forceinline__ uint32_t kth_keys16(const uint32_t* src, uint32_t k) {
  const uint4 wa = lds128(src), wb = lds128(src + 4);
  const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
  uint32_t lo = 0xFFFFu, hi = 0u;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t v = (w[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu;
    lo = v < lo ? v : lo;
    hi = (v < 0xFFFFu && v > hi) ? v : hi;
  }
  lo = __reduce_min_sync(0xFFFFFFFFu, lo);
  hi = __reduce_max_sync(0xFFFFFFFFu, hi);
  if (lo >= 0xFFFFu) return 0xFFFFu;
  auto count3 = [&](uint32_t m1, uint32_t m2, uint32_t m3, uint32_t* c1, uint32_t* c2,
                    uint32_t* c3) {
    uint32_t a = 0, b = 0, c = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t v = (w[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu;
      a += v <= m1 ? 1u : 0u;
      b += v <= m2 ? 1u : 0u;
      c += v <= m3 ? 1u : 0u;
    }
    *c1 = __reduce_add_sync(0xFFFFFFFFu, a);
    *c2 = __reduce_add_sync(0xFFFFFFFFu, b);
    *c3 = __reduce_add_sync(0xFFFFFFFFu, c);
  };
  uint32_t c1, c2, c3;
  count3(hi, hi, hi, &c1, &c2, &c3);
  if (c1 < k) return 0xFFFFu;  // fewer than k numeric keys
  // invariant: the answer lies in [lo, hi] and at least k keys are <= hi
  while (lo < hi) {
    const uint32_t m2 = (lo + hi) >> 1;
    const uint32_t m1 = (lo + m2) >> 1;
    const uint32_t m3 = (m2 + 1u + hi) >> 1;
    count3(m1, m2, m3, &c1, &c2, &c3);
    if (c1 >= k) {
      hi = m1;
    } else if (c2 >= k) {
      lo = m1 + 1u;
      hi = m2;
    } else if (c3 >= k) {
      lo = m2 + 1u;
      hi = m3;
    } else {
      lo = m3 + 1u;
    }
  }
  return lo;
}

// k-th best group maximum of the chunk (descending key), or kNoThreshold when the chunk has
// fewer than k non-NaN maxima.  Each maximum is a distinct element, so at least k elements
// of the chunk are >= it and every member of the segment's top-k is >= it.  Two barriers:
// the group keys go to shared memory, warp 0 selects, and the result is broadcast.
template <bool BIG>
__device__ uint32_t chunk_select(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                                 Scratch<BIG>& sm) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  uint32_t acc0 = 0x7E007E00u, acc1 = 0x7E007E00u, acc2 = 0x7E007E00u, acc3 = 0x7E007E00u;
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
        const __half2 mh = u32_as_h2(m);
        const __half top = __hmax(__low2half(mh), __high2half(mh));
        kw[0] = desc_key(*reinterpret_cast<const uint16_t*>(&top)) | 0xFFFF0000u;
      }
      nw = 1;
    }
  }
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

// Threshold test of one 16-byte vector: 8-bit element mask (bit e = element e) of values
// passing `key < K` (STRICT) or `key <= K`, i.e. value > V or value >= V (never NaN).
template <bool STRICT>
__device__ __forceinline__ uint32_t pass_mask8(const uint4& w, __half2 v2) {
  return STRICT ? gt_mask8(w, v2) : ge_mask8(w, v2);
}

// Is any half of the vector passing?  (OR of the four compares, no compression.)
template <bool STRICT>
__device__ __forceinline__ bool pass_any(const uint4& w, __half2 v2) {
  if (STRICT) {
    return (__hgt2_mask(u32_as_h2(w.x), v2) | __hgt2_mask(u32_as_h2(w.y), v2) |
            __hgt2_mask(u32_as_h2(w.z), v2) | __hgt2_mask(u32_as_h2(w.w), v2)) != 0;
  }
  return (__hge2_mask(u32_as_h2(w.x), v2) | __hge2_mask(u32_as_h2(w.y), v2) |
          __hge2_mask(u32_as_h2(w.z), v2) | __hge2_mask(u32_as_h2(w.w), v2)) != 0;
}

// This thread's 8 vectors (tid*8 .. tid*8+7): exact candidate mask of vector j, with the
// segment-boundary and take-all (no threshold yet) cases.
template <bool STRICT>
__device__ __forceinline__ uint32_t vec_mask(const StageInfo& si, const uint8_t* buf, int vi,
                                             __half2 v2, bool take_all) {
  const uint4 w = lds128(buf + vi * 16);
  uint32_t m = take_all ? 0xFFu : pass_mask8<STRICT>(w, v2);
  if (vi == si.vlo || vi == si.vhi) m &= valid_mask8(si.cv0 + vi, si.a0, si.a1);
  return m;
}

// Flags (bit j: vector tid*8+j holds a candidate) and the exact candidate count of this
// thread.  The common case costs one 128-bit smem load, four half2 compares and an OR per
// vector; exact counting only runs on the rare vectors that pass.
template <bool STRICT>
__device__ __forceinline__ uint32_t thread_flags(const StageInfo& si, const uint8_t* buf,
                                                 __half2 v2, bool take_all, uint32_t* count) {
  const int tid = threadIdx.x;
  const int vbase = tid * kVecPerThread;
  const int sw = tid & 7;
  const bool edge = take_all || (si.vlo >= vbase && si.vlo < vbase + kVecPerThread) ||
                    (si.vhi >= vbase && si.vhi < vbase + kVecPerThread);
  uint32_t flags = 0, cnt = 0;
  if (!edge) {
    if (vbase + kVecPerThread <= si.nvc) {
      // Common case: the maximum of the thread's 64 values (max ignores NaN, which never
      // passes) against the threshold; exact masks only when something passes.
      __half2 acc = u32_as_h2(0x7E007E00u);
#pragma unroll
      for (int jj = 0; jj < kVecPerThread; ++jj) {
        const uint4 w = lds128(buf + (vbase + (jj ^ sw)) * 16);  // rotated: conflict-free
        const __half2 m01 = __hmax2(u32_as_h2(w.x), u32_as_h2(w.y));
        const __half2 m23 = __hmax2(u32_as_h2(w.z), u32_as_h2(w.w));
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

// Writes this thread's candidates (flagged vectors, index order) at [base, ...) of the
// chunk's slot, and as (key, index, bits) composites at nbuf + base of the segment's
// shared-memory buffer when to_smem.
template <bool STRICT, bool BIG>
__device__ __forceinline__ void write_flagged(const TopkParams& p, const StageInfo& si,
                                              const uint8_t* buf, uint32_t flags, __half2 v2,
                                              bool take_all, uint32_t base, Scratch<BIG>& sm,
                                              uint32_t nbuf, bool to_smem) {
  const int tid = threadIdx.x;
  uint32_t* out = p.cand + si.slot * p.cap + base;
  const long long e0 = si.cv0 * 8;
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(buf);
  uint32_t r = 0;
  while (flags) {
    const int j = __ffs(flags) - 1;
    flags &= flags - 1;
    const int vi = tid * kVecPerThread + j;
    uint32_t m = vec_mask<STRICT>(si, buf, vi, v2, take_all);
    while (m) {
      const int e = __ffs(m) - 1;
      m &= m - 1;
      const uint32_t lidx = static_cast<uint32_t>(vi * 8 + e);
      const uint32_t w = (static_cast<uint32_t>(v16[lidx]) << 16) | lidx;
      out[r] = w;
      if (to_smem) sm.cache[nbuf + base + r] = make_composite(w, e0, si.a0);
      ++r;
    }
  }
}

// k-th smallest key among the n composites of the segment buffer, searched in [0, hi]
// (kFewerThanK when fewer than k of them have key <= hi: then every candidate qualifies).  Each warp computes it independently (no barrier).
template <bool BIG>
__device__ __forceinline__ uint32_t buffer_kth_key(const Scratch<BIG>& sm, uint32_t n, uint32_t k,
                                                   uint32_t hi) {
  if (n < k) return kFewerThanK;
  const int lane = threadIdx.x & 31;
  {
    uint32_t cnt = 0;
    for (uint32_t i = lane; i < n; i += 32) cnt += static_cast<uint32_t>(sm.cache[i] >> 48) <= hi;
    if (__reduce_add_sync(0xFFFFFFFFu, cnt) < k) return kFewerThanK;
  }
  uint32_t lo = 0;
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    uint32_t cnt = 0;
    for (uint32_t i = lane; i < n; i += 32) {
      cnt += static_cast<uint32_t>(sm.cache[i] >> 48) <= mid ? 1u : 0u;
    }
    if (__reduce_add_sync(0xFFFFFFFFu, cnt) >= k) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// Block-wide k-th smallest key among the n composites of the segment buffer: two 8-bit digit
// histograms (aggregated shared atomics) instead of a per-warp search over the whole buffer.
// kFewerThanK when n < k.  The histograms are zero on entry and left zero.
template <bool BIG>
__device__ uint32_t buffer_kth_key_block(Scratch<BIG>& sm, uint32_t n, uint32_t k) {
  if (n < k) return kFewerThanK;
  const int tid = threadIdx.x;
  for (uint32_t i0 = 0; i0 < n; i0 += kThreads) {
    const uint32_t i = i0 + tid;
    const uint32_t key = i < n ? static_cast<uint32_t>(sm.cache[i] >> 48) : 0u;
    hist_add_match(sm.hist1, key >> 8, i < n);
  }
  csync();
  if (tid < 32) warp_find_bin(sm.hist1, 0, k, &sm.bin1, &sm.before1);
  csync();
  const uint32_t b1 = static_cast<uint32_t>(sm.bin1);
  for (uint32_t i0 = 0; i0 < n; i0 += kThreads) {
    const uint32_t i = i0 + tid;
    const uint32_t key = i < n ? static_cast<uint32_t>(sm.cache[i] >> 48) : 0u;
    hist_add_match(sm.hist2, key & 0xFFu, i < n && (key >> 8) == b1);
  }
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
template <class SM>
__device__ uint32_t exact_local_select(const TopkParams& p, const StageInfo& si,
                                       const uint8_t* buf, SM& sm, uint32_t K, bool strict,
                                       uint64_t* S_out, uint32_t* sbase_out, uint32_t* stot_out) {
  const int tid = threadIdx.x;
  const bool take_all = K == kNoThreshold;
  const uint32_t vb = key_to_bits(K);
  const __half2 v2 = u32_as_h2(vb | (vb << 16));
  uint64_t M = 0;
  for (int j = 0; j < kVecPerThread; ++j) {
    const int vi = tid * kVecPerThread + j;
    if (vi < si.nvc) {
      const uint32_t m = strict ? vec_mask<true>(si, buf, vi, v2, take_all)
                                : vec_mask<false>(si, buf, vi, v2, take_all);
      M |= static_cast<uint64_t>(m) << (8 * j);
    }
  }
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(buf) + tid * 64;
  RunHist rh;
  for (uint64_t m = M; m; m &= m - 1) {
    rh.add(sm.hist1, desc_key(v16[__ffsll(static_cast<long long>(m)) - 1]) >> 8);
  }
  rh.flush(sm.hist1);
  csync();
  if (tid < 32) warp_find_bin(sm.hist1, 0, p.k, &sm.bin1, &sm.before1);
  csync();
  const uint32_t b1 = static_cast<uint32_t>(sm.bin1);
  for (uint64_t m = M; m; m &= m - 1) {
    const uint32_t key = desc_key(v16[__ffsll(static_cast<long long>(m)) - 1]);
    if ((key >> 8) == b1) rh.add(sm.hist2, key & 0xFFu);
  }
  rh.flush(sm.hist2);
  csync();
  if (tid < 32) warp_find_bin(sm.hist2, sm.before1, p.k, &sm.bin2, &sm.before2);
  csync();
  const uint32_t kstar = (b1 << 8) | static_cast<uint32_t>(sm.bin2);
  const uint32_t need = static_cast<uint32_t>(p.k) - sm.before2;
  uint32_t tcnt = 0;
  for (uint64_t m = M; m; m &= m - 1) {
    tcnt += desc_key(v16[__ffsll(static_cast<long long>(m)) - 1]) == kstar ? 1u : 0u;
  }
  uint32_t ttot;
  const uint32_t tbase = block_excl_scan<kThreads, true>(tcnt, &ttot, sm.warp_tot);
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
  *sbase_out =
      block_excl_scan<kThreads, true>(static_cast<uint32_t>(__popcll(S)), stot_out, sm.warp_tot);
  *S_out = S;
  if (tid == 0 && p.stats) atomicAdd(&p.status[1], 1u);
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  return kstar;
}

// Large-k path: exact local select, written to the chunk's global slot and the segment's
// shared-memory buffer.
template <bool BIG>
__device__ uint32_t exact_local(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                                Scratch<BIG>& sm, SegState& ss) {
  const int tid = threadIdx.x;
  uint64_t S;
  uint32_t sbase, stot;
  const uint32_t kstar = exact_local_select(p, si, buf, sm, ss.K, ss.strict, &S, &sbase, &stot);
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(buf) + tid * 64;
  const bool to_smem = !ss.spilled && ss.nbuf + stot <= static_cast<uint32_t>(Cfg<BIG>::kCacheCap);
  uint32_t* out = p.cand + si.slot * p.cap + sbase;
  const long long e0 = si.cv0 * 8;
  uint32_t r = 0;
  for (uint64_t m = S; m; m &= m - 1) {
    const int pos = __ffsll(static_cast<long long>(m)) - 1;
    const uint32_t lidx = static_cast<uint32_t>(tid * 64 + pos);
    const uint32_t w = (static_cast<uint32_t>(v16[pos]) << 16) | lidx;
    out[r] = w;
    if (to_smem) sm.cache[ss.nbuf + sbase + r] = make_composite(w, e0, si.a0);
    ++r;
  }
  if (to_smem) ss.nbuf += stot; else ss.spilled = true;
  if (tid == 0) p.chunk_count[si.slot] = stot;
  return kstar;
}

enum ChunkResult { kChunkDone = 0, kChunkOverflow = 1, kChunkFail = 2 };

// Drops the segment buffer's composites with key > K, keeping their order; returns the new
// count.  Each thread holds its kCacheCap / kThreads entries in registers across the scan's
// barriers, so the in-place writes never overtake a read.
template <bool BIG>
__device__ uint32_t compact_cache(Scratch<BIG>& sm, uint32_t n, uint32_t K) {
  constexpr int kPer = Cfg<BIG>::kCacheCap / kThreads;
  const uint32_t i0 = threadIdx.x * kPer;
  unsigned long long v[kPer];
  uint32_t keep = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t i = i0 + j;
    v[j] = i < n ? sm.cache[i] : ~0ull;
    keep += (i < n && static_cast<uint32_t>(v[j] >> 48) <= K) ? 1u : 0u;
  }
  uint32_t tot;
  uint32_t w = block_excl_scan<kThreads, true>(keep, &tot, sm.warp_tot);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t i = i0 + j;
    if (i < n && static_cast<uint32_t>(v[j] >> 48) <= K) sm.cache[w++] = v[j];
  }
  csync();
  return tot;
}

// Position of the r-th set bit (r from 0) of a 64-bit mask.
__device__ __forceinline__ int select_bit64(unsigned long long m, uint32_t r) {
  const uint32_t lo = static_cast<uint32_t>(m);
  const uint32_t pl = static_cast<uint32_t>(__popc(lo));
  uint32_t w = r < pl ? lo : static_cast<uint32_t>(m >> 32);
  uint32_t rr = r < pl ? r : r - pl;
  int pos = r < pl ? 0 : 32;
#pragma unroll
  for (int width = 16; width >= 1; width >>= 1) {
    const uint32_t c = static_cast<uint32_t>(__popc(w & ((1u << width) - 1u)));
    if (rr >= c) {
      rr -= c;
      w >>= width;
      pos += width;
    }
  }
  return pos;
}

// Writes the chunk's `total` candidates in index order like write_flagged, but spread over the
// block: every thread takes output slots tid, tid + kThreads, ... and finds each one's owner
// thread (binary search over the prefixes) and element (the rank-th set bit of the owner's
// mask).  For clustered candidates (a sorted row's top values sit in a few threads) this keeps
// the block from waiting on a few serial writers.
template <bool STRICT, bool BIG>
__device__ void write_balanced(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                               uint32_t flags, __half2 v2, bool take_all, uint32_t base,
                               uint32_t total, Scratch<BIG>& sm, uint32_t nbuf, bool to_smem) {
  const int tid = threadIdx.x;
  unsigned long long M = 0;
  for (uint32_t f = flags; f; f &= f - 1) {
    const int j = __ffs(f) - 1;
    M |= static_cast<unsigned long long>(vec_mask<STRICT>(si, buf, tid * kVecPerThread + j, v2,
                                                          take_all)) << (8 * j);
  }
  sm.tmask[tid] = M;
  sm.tbase[tid] = base;
  csync();
  uint32_t* out = p.cand + si.slot * p.cap;
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(buf);
  const long long e0 = si.cv0 * 8;
  for (uint32_t i = tid; i < total; i += kThreads) {
    int lo = 0, hi = kThreads - 1;  // owner: the last thread whose first slot is <= i
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sm.tbase[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int pos = select_bit64(sm.tmask[lo], i - sm.tbase[lo]);
    const uint32_t lidx = static_cast<uint32_t>(lo * 64 + pos);
    const uint32_t w = (static_cast<uint32_t>(v16[lidx]) << 16) | lidx;
    out[i] = w;
    if (to_smem) sm.cache[nbuf + i] = make_composite(w, e0, si.a0);
  }
  csync();  // tmask / tbase are free again
}

// Counts the chunk's candidates under (ss.K, STRICT) with one barrier, then writes them in
// index order.  `par` selects the double-buffered warp-count slots.
template <bool STRICT, bool BIG>
__device__ int stream_chunk(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                            Scratch<BIG>& sm, SegState& ss, int par) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const bool take_all = ss.K == kNoThreshold;
  const uint32_t vb = key_to_bits(ss.K);
  const __half2 v2 = u32_as_h2(vb | (vb << 16));
  uint32_t cnt;
  const uint32_t flags = thread_flags<STRICT>(si, buf, v2, take_all, &cnt);
  uint32_t incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) sm.wcnt[par][warp] = incl;
  csync();
  if (sm.fail) return kChunkFail;
  uint32_t total = 0, wpre = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t t = sm.wcnt[par][w];
    wpre += w < warp ? t : 0u;
    total += t;
  }
  if (total == 0) {
    if (tid == 0) {
      p.chunk_count[si.slot] = 0;
      if (p.stats) atomicAdd(&p.status[2], 1u);
    }
    return kChunkDone;
  }
  if (total > static_cast<uint32_t>(p.cap)) return kChunkOverflow;
  const uint32_t base = wpre + incl - cnt;
  bool to_smem = !ss.spilled && ss.nbuf + total <= static_cast<uint32_t>(Cfg<BIG>::kCacheCap);
  if (BIG && !to_smem && !ss.spilled && ss.nbuf >= static_cast<uint32_t>(p.k)) {
    // make room: the buffer's k-th key is a tighter threshold (k composites at lower
    // indices beat it), and the buffered composites beyond it can go
    const uint32_t kk = buffer_kth_key_block(sm, ss.nbuf, static_cast<uint32_t>(p.k));
    if (kk < ss.K) {
      ss.K = kk;
      ss.strict = true;
    }
    ss.nbuf = compact_cache<BIG>(sm, ss.nbuf, ss.K);
    ss.added = 0;
    to_smem = ss.nbuf + total <= static_cast<uint32_t>(Cfg<BIG>::kCacheCap);
  }
  if (BIG && total >= 512) {
    write_balanced<STRICT, BIG>(p, si, buf, flags, v2, take_all, base, total, sm, ss.nbuf, to_smem);
  } else if (flags) {
    write_flagged<STRICT, BIG>(p, si, buf, flags, v2, take_all, base, sm, ss.nbuf, to_smem);
  }
  if (tid == 0) p.chunk_count[si.slot] = total;
  if (to_smem) {
    ss.nbuf += total;
    ss.added += total;
  } else {
    ss.spilled = true;
  }
  if (!take_all) {
    // >= k values with key <= K are now written (certified by this segment's own select or
    // exact pass, earlier in index order): later chunks only need key < K.  Once k more
    // candidates have arrived, tighten K to the exact k-th best of the buffer.
    ss.strict = true;
    // once k more candidates have arrived, tighten K to the buffer's k-th key (k composites at
    // lower indices beat it, so it is a strict threshold)
    if (ss.added >= static_cast<uint32_t>(p.k) && !ss.spilled) {
      csync();
      const uint32_t kk = buffer_kth_key_block(sm, ss.nbuf, static_cast<uint32_t>(p.k));
      if (kk < ss.K) ss.K = kk;
      ss.added = 0;
    }
  }
  return kChunkDone;
}

// First chunk of a segment (or one after an uncertified chunk): select a threshold, stream,
// and fall back to the exact local select when too many values pass.
template <bool BIG>
__device__ int first_chunk(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                           Scratch<BIG>& sm, SegState& ss, int par, bool* adopted = nullptr) {
  const uint32_t kc = chunk_select(p, si, buf, sm);
  if (adopted) *adopted = kc < ss.K;
  if (kc < ss.K) {
    ss.K = kc;
    ss.strict = false;
  }
  int r = ss.strict ? stream_chunk<true, BIG>(p, si, buf, sm, ss, par)
                    : stream_chunk<false, BIG>(p, si, buf, sm, ss, par);
  if (r == kChunkOverflow) {
    ss.K = exact_local(p, si, buf, sm, ss);
    ss.strict = true;
    ss.added = 0;
    r = kChunkDone;
  }
  return r;
}

// ---- consumer: segment merge -----------------------------------------------------------

// Candidate source for the merge: the shared-memory cache or the chunk lists in global
// memory (very long segments, many candidates, or a segment split across blocks).
struct CacheSrc {
  const unsigned long long* cache;
  __device__ __forceinline__ unsigned long long get(uint32_t i) const { return cache[i]; }
};

struct GlobalSrc {
  const TopkParams* p;
  const uint32_t* coff;  // P + 1 prefix entries (shared or global memory)
  int P;
  long long slot0, v0, a0;
  int chunk_vecs;
  __device__ __forceinline__ unsigned long long get(uint32_t i) const {
    int lo = 0, hi = P;  // largest c with coff[c] <= i
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (coff[mid] <= i) lo = mid; else hi = mid;
    }
    const uint32_t w = __ldcg(&p->cand[(slot0 + lo) * p->cap + (i - coff[lo])]);
    return make_composite(w, (v0 + static_cast<long long>(lo) * chunk_vecs) * 8, a0);
  }
};

// Each of the n candidates with key <= kf takes the output slot given by its rank in
// (key, index) order among them; composites are distinct, so ranks are exact.  Every
// candidate ranking below another one with key <= kf also has key <= kf.
__device__ __forceinline__ void rank_emit(const TopkParams& p, const unsigned long long* items,
                                          uint32_t n, uint32_t kf, int s, long long len) {
  const int tid = threadIdx.x;
  const uint32_t k = static_cast<uint32_t>(p.k);
  uint16_t* ov = p.out_values + static_cast<long long>(s) * k;
  int* oi = p.out_indices + static_cast<long long>(s) * k;
  for (uint32_t e = tid; e < n; e += kThreads) {
    const unsigned long long c = items[e];
    if (static_cast<uint32_t>(c >> 48) > kf) continue;
    uint32_t rank = 0;
    for (uint32_t j = 0; j < n; ++j) rank += items[j] < c ? 1u : 0u;
    if (rank < k) {
      ov[rank] = static_cast<uint16_t>(c & 0xFFFFu);
      oi[rank] = static_cast<int>((c >> 16) & 0xFFFFFFFFu);
    }
  }
  // A segment shorter than k never certifies a threshold, so all n candidates are its
  // values; the rest of the row is padding.
  if (len < static_cast<long long>(k)) {
    for (uint32_t r = n + tid; r < k; r += kThreads) {
      ov[r] = 0xFC00u;
      oi[r] = -1;
    }
  }
  if (tid == 0 && p.stats) atomicAdd(&p.status[4], 1u);
}

// Exact top-k of the n candidates of `src` (index order) with key <= kf; writes row s.
template <bool BIG, class Src>
__device__ void select_and_emit(const TopkParams& p, const Src& src, uint32_t n, uint32_t kf,
                                int s, long long seg_len, Scratch<BIG>& sm) {
  const int tid = threadIdx.x;
  const uint32_t k = static_cast<uint32_t>(p.k);
  const uint32_t R = (n + kThreads - 1) / kThreads;
  const uint32_t i0 = tid * R < n ? tid * R : n;
  const uint32_t i1 = i0 + R < n ? i0 + R : n;
  for (uint32_t j = 0; j < R; ++j) {
    const uint32_t i = i0 + j;
    uint32_t key = 0xFFFFFFFFu;
    if (i < i1) key = static_cast<uint32_t>(src.get(i) >> 48);
    hist_add_match(sm.hist1, key >> 8, key <= kf);
  }
  csync();
  if (tid < 32) warp_find_bin(sm.hist1, 0, k, &sm.bin1, &sm.before1);
  csync();
  const int b1 = sm.bin1;
  uint32_t kstar, need;
  if (b1 >= 256) {  // fewer than k candidates (a segment shorter than k): keep them all
    kstar = 0x10000u;
    need = 0;
  } else {
    for (uint32_t j = 0; j < R; ++j) {
      const uint32_t i = i0 + j;
      uint32_t key = 0xFFFFFFFFu;
      if (i < i1) key = static_cast<uint32_t>(src.get(i) >> 48);
      hist_add_match(sm.hist2, key & 0xFFu, key <= kf && (key >> 8) == static_cast<uint32_t>(b1));
    }
    csync();
    if (tid < 32) warp_find_bin(sm.hist2, sm.before1, k, &sm.bin2, &sm.before2);
    csync();
    kstar = (static_cast<uint32_t>(b1) << 8) | static_cast<uint32_t>(sm.bin2);
    need = k - sm.before2;
  }
  // ordered ranks of the ties at the cutoff
  uint32_t tcnt = 0;
  for (uint32_t i = i0; i < i1; ++i) {
    const uint32_t key = static_cast<uint32_t>(src.get(i) >> 48);
    tcnt += (key <= kf && key == kstar) ? 1u : 0u;
  }
  uint32_t ttot;
  const uint32_t tbase = block_excl_scan<kThreads, true>(tcnt, &ttot, sm.warp_tot);
  uint32_t scnt = 0;
  {
    uint32_t tr = tbase;
    for (uint32_t i = i0; i < i1; ++i) {
      const uint32_t key = static_cast<uint32_t>(src.get(i) >> 48);
      if (key > kf) continue;
      if (key < kstar) {
        ++scnt;
      } else if (key == kstar) {
        scnt += tr < need ? 1u : 0u;
        ++tr;
      }
    }
  }
  uint32_t nsel;
  const uint32_t sbase = block_excl_scan<kThreads, true>(scnt, &nsel, sm.warp_tot);
  {
    uint32_t tr = tbase, w = sbase;
    for (uint32_t i = i0; i < i1; ++i) {
      const unsigned long long c = src.get(i);
      const uint32_t key = static_cast<uint32_t>(c >> 48);
      if (key > kf) continue;
      bool take = key < kstar;
      if (key == kstar) {
        take = tr < need;
        ++tr;
      }
      if (take) sm.sel[w++] = c;
    }
  }
  csync();
  uint16_t* ov = p.out_values + static_cast<long long>(s) * k;
  int* oi = p.out_indices + static_cast<long long>(s) * k;
  if (nsel <= static_cast<uint32_t>(kThreads)) {
    rank_emit(p, sm.sel, nsel, 0xFFFFu, s, 0);
  } else {
    int n2 = 1;
    while (n2 < static_cast<int>(nsel)) n2 <<= 1;
    for (int i = static_cast<int>(nsel) + tid; i < n2; i += kThreads) sm.sel[i] = ~0ull;
    csync();
    for (int size = 2; size <= n2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < n2 / 2; i += kThreads) {
          const int lo = 2 * i - (i & (stride - 1));
          const int hi = lo + stride;
          const bool up = (lo & size) == 0;
          const unsigned long long a = sm.sel[lo], b = sm.sel[hi];
          if ((a > b) == up) {
            sm.sel[lo] = b;
            sm.sel[hi] = a;
          }
        }
        csync();
      }
    }
    for (uint32_t r = tid; r < nsel; r += kThreads) {
      const unsigned long long c = sm.sel[r];
      ov[r] = static_cast<uint16_t>(c & 0xFFFFu);
      oi[r] = static_cast<int>((c >> 16) & 0xFFFFFFFFu);
    }
    if (tid == 0 && p.stats) atomicAdd(&p.status[4], 1u);
  }
  for (uint32_t r = nsel + tid; r < k; r += kThreads) {
    ov[r] = 0xFC00u;
    oi[r] = -1;
  }
  if (tid == 0 && nsel < k && seg_len >= static_cast<long long>(k)) {
    atomicOr(&p.status[0], kStatusCertifyFailed);
  }
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  csync();
}

// Emits row s from the n candidates in sm.cache (key <= kf qualifies).
template <bool BIG>
__device__ __forceinline__ void emit_from_cache(const TopkParams& p, Scratch<BIG>& sm, uint32_t n,
                                                uint32_t kf, int s, long long len) {
  const uint32_t k = static_cast<uint32_t>(p.k);
  if (!BIG) {
    const uint32_t kk = buffer_kth_key(sm, n, k, kf);  // exact cutoff key of the row
    if (kk == kFewerThanK && len >= static_cast<long long>(k) && threadIdx.x == 0) {
      atomicOr(&p.status[0], kStatusCertifyFailed);  // fewer than k candidates survived
    }
    rank_emit(p, sm.cache, n, kk, s, len);
  } else {
    CacheSrc cs{sm.cache};
    select_and_emit<BIG>(p, cs, n, kf, s, len, sm);
  }
}

// Merges segment ss.s from the chunk lists in global memory (split or overflowing segments).
template <bool BIG>
__device__ void merge_from_global(const TopkParams& p, const SegState& ss, uint32_t kf,
                                  Scratch<BIG>& sm) {
  using C = Cfg<BIG>;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int P = ss.nchunks;
  const bool small_p = P <= C::kCoffCap;
  uint32_t* coff = small_p ? sm.coff : p.chunk_off + ss.slot0;
  if (tid < 32) {  // prefix of the per-chunk candidate counts
    uint32_t carry = 0;
    for (int base = 0; base < P; base += 32) {
      const int c = base + lane;
      uint32_t n = 0;
      if (c < P) {
        n = __ldcg(&p.chunk_count[ss.slot0 + c]);
        n = n < static_cast<uint32_t>(p.cap) ? n : static_cast<uint32_t>(p.cap);
      }
      uint32_t incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      if (c < P) coff[c] = carry + incl - n;
      carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) {
      coff[P] = carry;
      sm.bcast[2] = carry;
    }
  }
  if (!small_p) __threadfence_block();
  csync();
  const uint32_t n = sm.bcast[2];
  const long long len = ss.a1 - ss.a0;
  if (small_p && n > static_cast<uint32_t>(C::kCacheCap)) {
    // Too many candidates for the cache: keep only those with key <= kf (the segment's final
    // threshold), in index order.  Pass 1 counts them per chunk, pass 2 compacts them, one
    // warp per chunk with ballot ranks.  Usually they fit, and the cache merge runs.
    const int warp = tid >> 5;
    for (int c = warp; c < P; c += kWarps) {
      const uint32_t cnt = sm.coff[c + 1] - sm.coff[c];
      const uint32_t* src = p.cand + (ss.slot0 + c) * p.cap;
      uint32_t keep = 0;
      for (uint32_t i = lane; i < cnt; i += 32) keep += desc_key(__ldcg(src + i) >> 16) <= kf ? 1u : 0u;
      keep = __reduce_add_sync(0xFFFFFFFFu, keep);
      if (lane == 0) sm.coff2[c] = keep;
    }
    csync();
    if (tid < 32) {
      uint32_t carry = 0;
      for (int base = 0; base < P; base += 32) {
        const int c = base + lane;
        const uint32_t v = c < P ? sm.coff2[c] : 0u;
        uint32_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        if (c < P) sm.coff2[c] = carry + incl - v;
        carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
      }
      if (lane == 0) sm.bcast[2] = carry;
    }
    csync();
    const uint32_t nkeep = sm.bcast[2];
    if (nkeep <= static_cast<uint32_t>(C::kCacheCap)) {
      for (int c = warp; c < P; c += kWarps) {
        const uint32_t cnt = sm.coff[c + 1] - sm.coff[c];
        const uint32_t* src = p.cand + (ss.slot0 + c) * p.cap;
        const long long e0 = (ss.v0 + static_cast<long long>(c) * ss.chunk_vecs) * 8;
        uint32_t dst = sm.coff2[c];
        for (uint32_t i0 = 0; i0 < cnt; i0 += 32) {
          const uint32_t i = i0 + lane;
          uint32_t w = 0;
          bool keep = false;
          if (i < cnt) {
            w = __ldcg(src + i);
            keep = desc_key(w >> 16) <= kf;
          }
          const unsigned b = __ballot_sync(0xFFFFFFFFu, keep);
          if (keep) sm.cache[dst + __popc(b & ((1u << lane) - 1u))] = make_composite(w, e0, ss.a0);
          dst += __popc(b);
        }
      }
      csync();
      emit_from_cache<BIG>(p, sm, nkeep, kf, ss.s, len);
      return;
    }
    // still too many: the merge reads the chunk lists in place (below)
  }
  if (small_p && n <= static_cast<uint32_t>(C::kCacheCap)) {
    const int warp = tid >> 5;
    for (int c = warp; c < P; c += kWarps) {
      const uint32_t o = sm.coff[c];
      const uint32_t cnt = sm.coff[c + 1] - o;
      const uint32_t* src = p.cand + (ss.slot0 + c) * p.cap;
      const long long e0 = (ss.v0 + static_cast<long long>(c) * ss.chunk_vecs) * 8;
      for (uint32_t i = lane; i < cnt; i += 32) {
        sm.cache[o + i] = make_composite(__ldcg(src + i), e0, ss.a0);
      }
    }
    csync();
    emit_from_cache<BIG>(p, sm, n, kf, ss.s, len);
  } else {
    GlobalSrc gs{&p, coff, P, ss.slot0, ss.v0, ss.a0, ss.chunk_vecs};
    select_and_emit<BIG>(p, gs, n, kf, ss.s, len, sm);
  }
}

// The CTA has finished its chunks of segment ss.s: merge it here if no other CTA still
// holds some of them.
template <bool BIG>
__device__ void close_segment(const TopkParams& p, const SegState& ss, Scratch<BIG>& sm) {
  if (ss.mycnt == 0) return;
  uint32_t kf = ss.K;
  const bool split = ss.mycnt != ss.nchunks;
  if (split) {
    __threadfence();  // this thread's candidate writes, before the arrival below
    csync();
    if (threadIdx.x == 0) {
      if (ss.K < kNoThreshold) atomicMin(&p.seg_thresh[ss.s], ss.K);
      __threadfence();
      const uint32_t old = atomicAdd(&p.seg_done[ss.s], static_cast<uint32_t>(ss.mycnt));
      const bool last = old + static_cast<uint32_t>(ss.mycnt) == static_cast<uint32_t>(ss.nchunks);
      uint32_t k2 = ss.K;
      if (last) {
        __threadfence();
        const uint32_t g = __ldcg(&p.seg_thresh[ss.s]);
        k2 = g < k2 ? g : k2;
      }
      sm.bcast[0] = last ? 1u : 0u;
      sm.bcast[1] = k2;
    }
    csync();
    if (!sm.bcast[0]) return;
    kf = sm.bcast[1];
    __threadfence();
  }
  csync();  // every consumer's candidate writes for this segment are done
  if (!split && !ss.spilled) {
    emit_from_cache<BIG>(p, sm, ss.nbuf, kf, ss.s, ss.a1 - ss.a0);
    return;
  }
  merge_from_global<BIG>(p, ss, kf, sm);
}

template <bool BIG>
__device__ void consumer_loop(const TopkParams& p, uint8_t* stages, uint64_t* full,
                              uint64_t* empty, const StageInfo* info, Scratch<BIG>& sm) {
  constexpr int S = Cfg<BIG>::kStagesN;
  SegState ss;
  int st = 0, par = 0;
  uint32_t ph = 0;
  for (;;) {
    const bool ok = mbar_wait(&full[st], ph);
    if (!ok) sm.fail = 1u;
    const StageInfo& si = info[st];  // read in place: valid until this stage is released
    const uint8_t* buf = stages + static_cast<size_t>(st) * kStageBytes;
    int r = kChunkDone;
    if (si.part == ss.part && ss.strict && si.nvc > 0) {  // uniform: stage info is shared
      // steady state: one barrier per chunk, usually nothing to write.  After an overflow
      // (values rising along the row) the next chunk starts from its own threshold instead
      // of counting everything under the stale one first.
      if (ss.rising) {
        bool adopted;
        r = first_chunk<BIG>(p, si, buf, sm, ss, par, &adopted);
        ss.rising = adopted;  // still rising while the chunk's own threshold beats the old one
      } else {
        r = stream_chunk<true, BIG>(p, si, buf, sm, ss, par);
        if (r == kChunkOverflow) {
          r = first_chunk<BIG>(p, si, buf, sm, ss, par);  // values ramped up
          ss.rising = true;
        }
      }
    } else {
      if (group_or<kThreads>(!ok)) r = kChunkFail;
      if (r != kChunkFail) {
        if (si.part != ss.part) {
          close_segment<BIG>(p, ss, sm);
          if (si.part == kStopPart) break;
          ss = SegState{};
          ss.s = si.s;
          ss.part = si.part;
          ss.nchunks = si.nchunks;
          ss.chunk_vecs = si.chunk_vecs;
          ss.slot0 = si.slot - si.c;  // the segment's chunk 0 (the global merge walks all)
          ss.v0 = si.v0;
          ss.a0 = si.a0;
          ss.a1 = si.a1;
        }
        if (si.nvc > 0) r = first_chunk<BIG>(p, si, buf, sm, ss, par);
      }
    }
    if (r == kChunkFail) {  // a bulk copy never arrived: stop (the stage contents are not valid)
      if (threadIdx.x == 0) atomicOr(&p.status[0], kStatusWaitTimeout);
      return;
    }
    if (si.nvc > 0) {
      ++ss.mycnt;
      par ^= 1;
    }
    release_stage(&empty[st]);
    if (++st == S) {
      st = 0;
      ph ^= 1u;
    }
  }
}

}  // namespace bt

#include "bt_small.cuh"

namespace bt {

// 96 registers: each SM sub-partition (16K registers) holds 5 warps, so two 9-warp blocks fit.
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
      producer_loop<BIG>(p, stages, full, empty, info);
    } else if (!BIG && tid >= kThreads + 32) {
      if constexpr (!BIG) merger_loop(p, sm);
    }
    return;
  }
  if constexpr (BIG) {
    consumer_loop<true>(p, stages, full, empty, info, sm);
  } else {
    consumer_loop_small(p, stages, full, empty, info, sm);
  }
}

// ---- set-up kernels -------------------------------------------------------------------

// Fixed-length rows: reset the per-segment thresholds, arrival counters and status words.
__global__ void init_kernel(TopkParams p) {
  grid_dep_launch();  // the streaming kernel may set up meanwhile; it waits before any use
  grid_dep_wait();    // launched early behind the previous kernel: wait for its completion
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  if (i < 16) p.status[i] = 0;
  for (long long s = i; s < p.seg_num; s += stride) {
    p.seg_thresh[s] = kNoThreshold;
    p.seg_done[s] = 0;
    if (p.steal) p.chunk_next[s] = 0;
  }
  // a split segment's partial lists are found by their non-zero slot count
  for (long long c = i; c < p.slot_capacity; c += stride) p.chunk_count[c] = 0;
}

// CSR batches: the same resets, the chunk-slot prefix over segments, and the padding rows of
// empty segments (which no chunk work item covers).  One block.
__global__ void __launch_bounds__(1024) csr_prep_kernel(TopkParams p) {
  __shared__ uint32_t warp_tot[32];
  grid_dep_launch();  // the streaming kernel may set up meanwhile; it waits before any use
  grid_dep_wait();    // launched early behind the previous kernel: wait for its completion
  const int tid = threadIdx.x;
  if (tid < 16) p.status[tid] = 0;
  for (long long c = tid; c < p.slot_capacity; c += 1024) p.chunk_count[c] = 0;
  __syncthreads();
  uint32_t carry = 0, pcarry = 0;
  for (int base = 0; base < p.seg_num; base += 1024) {
    const int s = base + tid;
    uint32_t nch = 0;
    if (s < p.seg_num) {
      p.seg_thresh[s] = kNoThreshold;
      p.seg_done[s] = 0;
      nch = static_cast<uint32_t>(seg_geom(p, s).nchunks);
      if (p.offsets[s] < 0 || p.offsets[s + 1] < p.offsets[s]) {
        atomicOr(&p.status[0], kStatusBadOffsets);
      }
      if (nch == 0) {
        for (int r = 0; r < p.k; ++r) {
          p.out_values[static_cast<long long>(s) * p.k + r] = 0xFC00u;
          p.out_indices[static_cast<long long>(s) * p.k + r] = -1;
        }
      }
    }
    uint32_t tot;
    const uint32_t pre = block_excl_scan<1024>(nch, &tot, warp_tot);
    if (s < p.seg_num) p.chunk_start[s] = carry + pre;
    carry += tot;
    const uint32_t npart = (nch + p.part_chunks - 1) / p.part_chunks;
    uint32_t ptot;
    const uint32_t ppre = block_excl_scan<1024>(npart, &ptot, warp_tot);
    if (s < p.seg_num) p.part_start[s] = pcarry + ppre;
    pcarry += ptot;
  }
  if (tid == 0) {
    p.chunk_start[p.seg_num] = carry;
    // chunks beyond the workspace capacity: process no part at all and flag the call
    const bool over = static_cast<long long>(carry) > p.slot_capacity;
    p.part_start[p.seg_num] = over ? 0u : pcarry;
    if (over) atomicOr(&p.status[0], kStatusBadOffsets);
  }
}

}  // namespace bt
