// bt_kernels.cuh -- the batched top-k pipeline for 16-bit floats (fp16, bf16) on sm_100a.
//
// One streaming pass over HBM replaces the reference's three full reads (the high-byte and
// low-byte histograms, src/radix_histogram.cuh, and the compaction,
// src/candidate_compact.cuh).
//
// topk_kernel<BIG>: persistent, 2 blocks per SM (96 registers a thread), warp-specialised.
//   * Producer warp (one elected lane): claims work parts (a segment, or a run of its
//     chunks when there are fewer segments than blocks) from a global counter, in segment
//     order, and streams each chunk (<= 16384 values, 32 KiB) into a shared-memory
//     stage with one cp.async.bulk (no multicast), signalling a "full" mbarrier.
//   * 8 consumer warps, per chunk:
//       1. threshold: on the first chunk of a segment the k-th best of the chunk's group
//          maxima (a certified bound: every member of the segment's top-k is >= it), or the
//          previous segment's threshold when it still leaves between k and `cap` values.
//       2. candidate test: a 16-byte vector is skipped after four paired compares against its
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
//
// This header holds what does not touch input values (types, the producer, key-only
// selection, the set-up kernels); bt_body.cuh holds the rest and is compiled once per
// element type, into bt::f16 (topk_kernel for fp16) and bt::bf16 (for bf16).
#pragma once

#include <cstddef>
#include <cstdint>

#include "bt_common.cuh"
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
  int steal;                     // whole segments, chunks claimed one by one, idle blocks help
  int help_window;               // how many of the last-claimed segments idle blocks may help
  int help_min;                  // a helper joins a segment with at least this many chunks left
  uint32_t* chunk_next;          // [seg_num] next unclaimed chunk of each segment (steal)
  int k;
  int groups;                    // group maxima per thread in the threshold select
  int cap;                       // candidate capacity per chunk slot
  int stats;                     // count events into status[1..4]
  uint32_t* seg_thresh;          // [seg_num] the running strict threshold of the segment's
                                 // first part and the last chunk it covers, (key << 16) | chunk
                                 // (kNoOwnerKey: none yet), for the segment's other parts
  uint32_t* seg_done;            // [seg_num] chunks finished (arrival counter)
  uint32_t* chunk_count;         // [slot_capacity]
  uint32_t* chunk_off;           // [slot_capacity] merge scratch for very long segments
  uint32_t* cand;                // [slot_capacity * cap]
  uint32_t* status;              // [16]
  uint16_t* out_values;          // [seg_num * k]
  int* out_indices;              // [seg_num * k]
  uint32_t pad_bits;             // -inf of the element type: the value of a missing entry
  int epv_shift;                 // log2 of the elements in a 16-byte vector: 3 (16-bit), 2 (fp32)
  uint32_t* out_values32;        // [seg_num * k] value bits of 32-bit elements (fp32 entry points)
  uint32_t handoff_tries;        // tries of each consumer <-> merger hand-off wait (kWaitCap;
                                 // fewer only through the failure-path test hook)
  long long max_total_len;       // CSR: the caller's bound on offsets[seg_num] - offsets[0]
};

struct SegGeom {
  long long a0, a1;  // aligned element coordinates of the segment [start, end) (elements of the
                     // input's own type, counted from the 16-byte boundary below the input)
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
  const int sh = p.epv_shift;
  g.v0 = g.a0 >> sh;
  g.nv = (g.a1 > g.a0) ? ((g.a1 + (1 << sh) - 1) >> sh) - g.v0 : 0;
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
  static constexpr int kGroupWords = 1;                  // packed group-max key words/thread
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
  int probe;       // k > 128: a look at the segment's last chunk ahead of order (not its turn)
  uint32_t ext_k;  // a strict threshold for this chunk certified by the segment's first part
                   // (k values with key <= it at lower indices), or kNoThreshold
};
constexpr int kStopPart = -1;
constexpr uint32_t kNoOwnerKey = 0xFFFFFFFFu;  // seg_thresh: the first part has no k-th key yet

// The strict threshold a chunk c of another part may take from the first part's published
// (key << 16) | last_chunk word: the k values behind the key lie in chunks <= last_chunk, so
// they precede every value of chunk c when last_chunk < c (ties at the key lose by index).
__device__ __forceinline__ uint32_t owner_threshold(uint32_t word, int c) {
  const uint32_t key = word >> 16;
  return (key < kNoThreshold && (word & 0xFFFFu) < static_cast<uint32_t>(c)) ? key : kNoThreshold;
}
constexpr uint32_t kWorkCounter = 8;  // status[8]: next work part to claim (reset per call)
constexpr uint32_t kHelpCounter = 9;  // status[9]: next segment an idle block helps
constexpr int kHelpMinChunks = 3;     // k <= 128: a helper joins a segment with >= 3 chunks left
constexpr int kHelpMinChunksBig = 12;  // k > 128 (a costlier first chunk of a visit)

template <bool BIG>
struct alignas(16) Scratch {
  uint32_t hist1[256];  // 16-byte aligned: warp_find_bin reads it with 128-bit loads
  uint32_t hist2[256];
  unsigned long long cache[Cfg<BIG>::kCacheCap];
  uint32_t tbase[kThreads];                // split-segment merge: list lengths of 256 slots
  uint32_t warp_tot[kWarps];
  alignas(16) uint32_t wcnt[2][kWarps];  // per-warp candidate counts, double-buffered
  alignas(16) uint32_t rw[2][kWarps][8];  // strided counts: per-warp round totals (16-bit packed)
  int bin1, bin2;
  uint32_t before1, before2;
  uint32_t bcast[4];
  uint32_t fail;
  uint32_t probe_req;  // k > 128: part id + 1 whose segment's last chunk should be probed next
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
  int c;                // the chunk this batch comes from
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
              offsetof(Scratch<true>, wcnt) % 16 == 0 && offsetof(Scratch<true>, rw) % 16 == 0,
              "16-byte alignment of lds128 operands");

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
    seg = static_cast<int>(part / per);
    j = static_cast<int>(part - static_cast<long long>(seg) * per);
    pps = per;
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

// `abort` is the block's failure flag: once the consumers have failed and stopped releasing
// stages, a wait for a free stage gives up at once instead of running out its tries.
template <bool BIG>
__device__ void producer_loop(const TopkParams& p, uint8_t* stages, uint64_t* full,
                              uint64_t* empty, StageInfo* info, const uint32_t* abort,
                              const volatile uint32_t* probe_req = nullptr) {
  constexpr int S = Cfg<BIG>::kStagesN;
  const uint64_t policy = policy_evict_first();
  const long long nparts = total_parts(p);
  long long issued = 0;
  int st = 0;     // stage of the next load
  int round = 0;  // how many times every stage has been filled
  bool ok = true;
  // one stage: wait for it to be free, fill its info, start the copy (or just signal).  `ow`
  // is the segment's published first-part word for another part's chunk (kNoOwnerKey: none);
  // its load was issued before the call, so the round trip overlaps the wait for the stage.
  auto put = [&](StageInfo si, uint32_t ow) -> bool {
    if (round > 0 && !mbar_wait_abort(&empty[st], static_cast<uint32_t>((round - 1) & 1),
                                      abort)) {
      atomicOr(&p.status[0], kStatusWaitTimeout);
      return false;
    }
    si.ext_k = owner_threshold(ow, si.c);
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
    si.probe = 0;
    si.ext_k = kNoThreshold;
    si.cv0 = g.v0 + static_cast<long long>(c) * g.chunk_vecs;
    const long long rem = g.v0 + g.nv - si.cv0;
    si.nvc = static_cast<int>(rem < g.chunk_vecs ? rem : g.chunk_vecs);
    const long long first = g.v0 - si.cv0;
    const long long emask = (1ll << p.epv_shift) - 1;  // element position within a vector
    const long long last = ((g.a1 - 1) >> p.epv_shift) - si.cv0;
    si.vlo = ((g.a0 & emask) && first >= 0 && first < si.nvc) ? static_cast<int>(first) : -1;
    si.vhi = ((g.a1 & emask) && last >= 0 && last < si.nvc) ? static_cast<int>(last) : -1;
    return si;
  };
  if (p.steal) {
    // Whole segments, claimed in order.  A segment's chunks are claimed one at a time (one
    // ahead, so the claim's latency hides behind the stage wait).  Once every segment is
    // claimed, a block that has run dry helps one of the segments claimed last: it takes
    // the chunks the owner has not claimed yet, one at a time as well, so the two share out
    // what is left at the pace each works at, and the split-segment merge joins the two
    // lists (their chunks interleave).  Each visit of a block to a segment is one work part
    // (numbered per block).
    int visit = 0;
    // the first segment of block b is segment b (no claim round trip before the first load;
    // the grid never exceeds the segments here); later ones come from the work counter
    const long long b0 = static_cast<long long>(blockIdx.x);
    long long s = b0 < p.seg_num ? b0 : static_cast<long long>(p.seg_num);
    bool own = true;
    // CSR: the set-up kernel clears the part count when the offsets are invalid (or every
    // segment is empty): then no segment is touched, and only the stop item goes out
    const bool work = !(p.offsets && p.part_start[p.seg_num] == 0u);
    while (ok && work) {
      if (s >= p.seg_num) {
        own = false;
        // k > 128: help only once this block's consumers are through every stage filled so
        // far (a part's close there takes long): a chunk claimed earlier would wait in a stage
        // while the owner could have taken it.
        if (BIG && issued > 0) {
          const int last = st == 0 ? S - 1 : st - 1;
          const int rl = st == 0 ? round - 1 : round;  // the round that filled it
          if (!mbar_wait_abort(&empty[last], static_cast<uint32_t>(rl & 1), abort)) {
            atomicOr(&p.status[0], kStatusWaitTimeout);
            ok = false;
            break;
          }
        }
        // k > 128 (rows of very uneven cost) walks the window twice: a second helper may join
        const long long h = atomicAdd(&p.status[kHelpCounter], 1u);
        if (h >= (BIG ? 2 : 1) * static_cast<long long>(p.help_window)) break;
        s = p.seg_num - 1 - h % p.help_window;
      }
      const SegGeom g = seg_geom(p, static_cast<int>(s));
      const long long slot0 = p.offsets ? static_cast<long long>(p.chunk_start[s]) : s * p.p_max;
      if (!own && static_cast<int>(__ldcg(&p.chunk_next[s])) + p.help_min > g.nchunks) {
        s = p.seg_num;  // too little left to repay a helper's first chunk: try the next one
        continue;
      }
      // the first claim takes two chunks: the first load waits for one round trip, not two
      int c = static_cast<int>(atomicAdd(&p.chunk_next[s], 2u));
      int pre = c + 1;  // claimed with c (past the end when c is the last chunk)
      bool probed = false;
      while (ok && c < g.nchunks) {
        // k > 128: the owner's consumers found the values rising; the segment's last chunk
        // goes in next, out of turn (once, unclaimed: it is read again in its turn)
        if (probe_req != nullptr && !probed && c + 2 < g.nchunks &&
            *probe_req == static_cast<uint32_t>(visit) + 1u) {
          StageInfo si = chunk_info(static_cast<int>(s), g, slot0, g.nchunks - 1, visit, false);
          si.probe = 1;
          ok = put(si, kNoOwnerKey);
          probed = true;
          continue;
        }
        // a helper reads the owner's latest threshold with each claim (both round trips overlap)
        const uint32_t ow = own ? kNoOwnerKey : ld_relaxed_gpu(&p.seg_thresh[s]);
        int cn = pre;
        if (pre < 0) cn = static_cast<int>(atomicAdd(&p.chunk_next[s], 1u));
        pre = -1;
        ok = put(chunk_info(static_cast<int>(s), g, slot0, c, visit, cn >= g.nchunks), ow);
        c = cn;
      }
      ++visit;
      s = own ? static_cast<long long>(gridDim.x) +
                    static_cast<long long>(atomicAdd(&p.status[kWorkCounter], 1u))
              : p.seg_num;
    }
  } else {
    long long part = atomicAdd(&p.status[kWorkCounter], 1u);
    while (ok && part < nparts) {
      const long long next = atomicAdd(&p.status[kWorkCounter], 1u);  // claim ahead
      int s, c0, c1;
      SegGeom g;
      long long slot0;
      decode_part(p, part, &s, &c0, &c1, &g, &slot0);
      // k > 128: when the consumers find this part's values rising chunk after chunk, the
      // segment's last chunk goes in next, out of turn (once), so its certified threshold can
      // stop the climb; it is read again in its own turn.  One copy of the stage fill serves
      // both, which keeps this loop as short as without the probe.
      bool probed = false;
      int c = c0;
      while (ok && c < c1) {
        const bool probe_now = probe_req != nullptr && !probed && c + 2 < c1 &&
                               *probe_req == static_cast<uint32_t>(part) + 1u;
        StageInfo si = chunk_info(s, g, slot0, probe_now ? g.nchunks - 1 : c,
                                  static_cast<int>(part), !probe_now && c == c1 - 1);
        si.probe = probe_now ? 1 : 0;
        // a later part's chunks after its first may take the first part's threshold
        const bool ext = c0 > 0 && c > c0;
        ok = put(si, ext ? ld_relaxed_gpu(&p.seg_thresh[s]) : kNoOwnerKey);
        probed = probed || probe_now;
        if (!probe_now) ++c;
      }
      part = next;
    }
  }
  if (ok) {  // the stop sentinel
    StageInfo z{};
    z.s = -1;
    z.part = kStopPart;
    z.vlo = z.vhi = -1;
    ok = put(z, kNoOwnerKey);
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

// ---- set-up kernels -------------------------------------------------------------------

// Fixed-length rows: reset the per-segment thresholds, arrival counters and status words.
__global__ void init_kernel(TopkParams p) {
  grid_dep_launch();  // the streaming kernel may set up meanwhile; it waits before any use
  grid_dep_wait();    // launched early behind the previous kernel: wait for its completion
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  if (i < 16) p.status[i] = 0;
  for (long long s = i; s < p.seg_num; s += stride) {
    p.seg_thresh[s] = kNoOwnerKey;
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
  // Each thread takes kPrepPer consecutive segments a round (C4's 4096 segments: one round of
  // two block scans, not four): the offsets' loads are in flight together.
  constexpr int kPrepPer = 4;
  uint32_t carry = 0, pcarry = 0;
  for (int base = 0; base < p.seg_num; base += 1024 * kPrepPer) {
    uint32_t nch[kPrepPer];
    uint32_t csum = 0, psum = 0;
#pragma unroll
    for (int r = 0; r < kPrepPer; ++r) {
      const int s = base + tid * kPrepPer + r;
      nch[r] = 0;
      if (s < p.seg_num) {
        p.seg_thresh[s] = kNoOwnerKey;
        p.seg_done[s] = 0;
        if (p.steal) p.chunk_next[s] = 0;
        nch[r] = static_cast<uint32_t>(seg_geom(p, s).nchunks);
        if (p.offsets[s] < 0 || p.offsets[s + 1] < p.offsets[s]) {
          atomicOr(&p.status[0], kStatusBadOffsets);
        }
        if (nch[r] == 0) {
          for (int q = 0; q < p.k; ++q) {
            const long long o = static_cast<long long>(s) * p.k + q;
            if (p.out_values32) p.out_values32[o] = p.pad_bits;
            else p.out_values[o] = static_cast<uint16_t>(p.pad_bits);
            p.out_indices[o] = -1;
          }
        }
      }
      csum += nch[r];
      psum += (nch[r] + p.part_chunks - 1) / p.part_chunks;
    }
    uint32_t tot, ptot;
    uint32_t run = carry + block_excl_scan<1024>(csum, &tot, warp_tot);
    uint32_t prun = pcarry + block_excl_scan<1024>(psum, &ptot, warp_tot);
#pragma unroll
    for (int r = 0; r < kPrepPer; ++r) {
      const int s = base + tid * kPrepPer + r;
      if (s < p.seg_num) {
        p.chunk_start[s] = run;
        p.part_start[s] = prun;
      }
      run += nch[r];
      prun += (nch[r] + p.part_chunks - 1) / p.part_chunks;
    }
    carry += tot;
    pcarry += ptot;
  }
  if (tid == 0) {
    p.chunk_start[p.seg_num] = carry;
    // offsets spanning more than max_total_len values, or chunks beyond the workspace
    // capacity: process no part at all and flag the call
    const long long span = static_cast<long long>(p.offsets[p.seg_num]) - p.offsets[0];
    const bool over = static_cast<long long>(carry) > p.slot_capacity || span > p.max_total_len;
    p.part_start[p.seg_num] = over ? 0u : pcarry;
    if (over) atomicOr(&p.status[0], kStatusBadOffsets);
  }
}

}  // namespace bt

// The value-facing kernels, compiled once per element type (bt_body.cuh): bt::f16 for
// IEEE binary16 and bt::bf16 for bfloat16 inputs.
#define BT_ELEM_NS f16
#include "bt_body.cuh"
#undef BT_ELEM_NS
#define BT_ELEM_NS bf16
#define BT_ELEM_BF16 1
#include "bt_body.cuh"
#undef BT_ELEM_BF16
#undef BT_ELEM_NS

// 32-bit floats: a separate consumer on the same producer, set-up kernels and workspace layout.
#include "bt_f32.cuh"
