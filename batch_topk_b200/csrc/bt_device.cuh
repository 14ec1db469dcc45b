// bt_device.cuh -- shared device primitives for the batched top-k kernels (sm_100a).
//
//   * the inverse of the descending key codec (the codec itself: bt_elem.cuh);
//   * mbarrier and bulk-copy (cp.async.bulk, no multicast) wrappers with bounded waits;
//   * block scans, bin search over 256-bin histograms, and aggregated smem histogram adds.
#pragma once

#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace bt {

// ---- geometry and limits -----------------------------------------------------------
constexpr int kThreads = 256;                         // chunk kernel block size
constexpr int kWarps = kThreads / 32;
constexpr int kVecPerThread = 8;                      // 16-byte vectors per thread
constexpr int kVecPerChunk = kThreads * kVecPerThread;  // 2048 vectors
constexpr int kChunkElems = kVecPerChunk * 8;         // 16384 16-bit values
constexpr int kStageBytes = kVecPerChunk * 16;        // 32 KiB per pipeline stage
constexpr int kStages = 3;
constexpr int kMaxK = 1024;
constexpr int kMergeThreads = 256;
constexpr int kMaxChunksPerSegment = 4097;            // 2^26 values, misaligned start
constexpr uint32_t kNoThreshold = 0xFFFFu;  // key bound that admits every value, NaN too
constexpr uint32_t kFewerThanK = 0x10000u;  // "fewer than k candidates": all of them qualify
constexpr uint32_t kWaitCap = 1u << 16;               // bounded mbarrier waits
constexpr uint32_t kWaitHintNs = 20000;               // per-try suspend limit

// status word bits (mirrors BT_STATUS_* in include/batch_topk_b200.h)
constexpr uint32_t kStatusWaitTimeout = 1;
constexpr uint32_t kStatusBadOffsets = 2;
constexpr uint32_t kStatusSegmentTooLong = 4;
constexpr uint32_t kStatusCertifyFailed = 8;

// ---- codec (element-independent part) ---------------------------------------------
// The descending key codec itself (NaN test, +-0) depends on the element type: bt_elem.cuh.
// Bit pattern of the (non-NaN) value whose key is `key` (+0 for key 0x7FFF): the inverse map
// is the same for fp16 and bf16.
__host__ __device__ __forceinline__ uint32_t key_to_bits(uint32_t key) {
  return key < 0x8000u ? (key ^ 0x7FFFu) : key;
}

// 8-bit mask of the elements of aligned vector gv that lie inside [a0, a1).
__device__ __forceinline__ uint32_t valid_mask8(long long gv, long long a0, long long a1) {
  const long long e0 = gv * 8;
  long long lo = a0 - e0;
  long long hi = a1 - e0;
  lo = lo < 0 ? 0 : (lo > 8 ? 8 : lo);
  hi = hi < 0 ? 0 : (hi > 8 ? 8 : hi);
  if (hi <= lo) return 0u;
  return ((0xFFu << lo) & (0xFFu >> (8 - hi))) & 0xFFu;
}

// ---- PTX wrappers: mbarrier + bulk copy ---------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  // The suspend-time hint lets the thread sleep until the phase completes (or the hint
  // expires) instead of polling and taking issue slots from the working warps.
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kWaitHintNs)
      : "memory");
  return ok != 0;
}

// Non-blocking query of the same phase (acquire semantics as for try_wait): issued early, its
// latency overlaps other work, and a phase found complete needs no wait later.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false if the phase did not complete within kWaitCap tries (each
// try suspends for at most kWaitHintNs, so the bound is about a second).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t it = 0; it < kWaitCap; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// Bounded wait with a caller-given number of tries (0: fail at once without looking).
__device__ __forceinline__ bool mbar_wait_n(uint64_t* bar, uint32_t parity, uint32_t tries) {
  for (uint32_t it = 0; it < tries; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// Bounded wait that also gives up as soon as *abort becomes non-zero (set by the warps that
// would complete the phase once they have failed and stopped).
__device__ __forceinline__ bool mbar_wait_abort(uint64_t* bar, uint32_t parity,
                                                const volatile uint32_t* abort) {
  for (uint32_t it = 0; it < kWaitCap; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
  }
  return false;
}

// One bulk global->shared copy (16-byte aligned addresses, size a multiple of 16), completing
// transaction bytes on `bar`.  No multicast.  Evict-first L2 hint: the input is read once.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Relaxed GPU-scope load and store of a word that other blocks write or read (not cached in
// L1; no ordering with other accesses is implied).
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_relaxed_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialisation may
// start while the previous kernel in the stream still runs; grid_dep_wait() returns once that
// kernel has completed and its memory is visible (a no-op without such a launch).
// grid_dep_launch() lets the next kernel start early.
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// ---- block and warp collectives ----------------------------------------------------
// Named barrier 1 over the first THREADS threads of the block (the consumer warps of a
// warp-specialised kernel; the producer warp never joins it).
template <int THREADS>
__device__ __forceinline__ void group_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(THREADS) : "memory");
}

// OR-reduction of a predicate over the same group, returned to every member.
template <int THREADS>
__device__ __forceinline__ bool group_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "n"(THREADS)
      : "memory");
  return r != 0;
}

// Exclusive scan over the THREADS threads that call it; synchronises with group_sync when
// GROUP is true (warp-specialised kernels) and __syncthreads otherwise.
template <int THREADS, bool GROUP = false>
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* total,
                                                    uint32_t* warp_tot) {
  constexpr int NW = THREADS / 32;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  if (GROUP) group_sync<THREADS>(); else __syncthreads();
  uint32_t pre = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const uint32_t t = warp_tot[w];
    pre += (w < warp) ? t : 0u;
    tot += t;
  }
  *total = tot;
  if (GROUP) group_sync<THREADS>(); else __syncthreads();
  return pre + x - v;
}

// Warp-collective (call from one full warp): first bin b of hist[256] where
// base + sum(hist[0..b]) >= target.  Lane 0 writes *out_bin (256 when never reached) and
// *out_before (count before that bin, or the grand total when never reached).
__device__ __forceinline__ void warp_find_bin(const uint32_t* hist, uint32_t base,
                                              uint32_t target, int* out_bin,
                                              uint32_t* out_before) {
  const int lane = threadIdx.x & 31;
  const uint4 a = lds128(hist + lane * 8);
  const uint4 b = lds128(hist + lane * 8 + 4);
  const uint32_t c[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += c[i];
  uint32_t incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - tot;
  const uint32_t grand = __shfl_sync(0xFFFFFFFFu, incl, 31);
  const unsigned hit = __ballot_sync(0xFFFFFFFFu, base + incl >= target);
  if (hit == 0) {
    if (lane == 0) {
      *out_bin = 256;
      *out_before = base + grand;
    }
    return;
  }
  const int L = __ffs(hit) - 1;
  if (lane == L) {
    uint32_t run = base + excl;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (run + c[i] >= target) {
        *out_bin = lane * 8 + i;
        *out_before = run;
        break;
      }
      run += c[i];
    }
  }
}

// Per-thread run-length aggregation of histogram adds (for sequential scans where equal
// bins cluster, e.g. tie-heavy or sorted data).
struct RunHist {
  uint32_t bin = 0xFFFFFFFFu;
  uint32_t count = 0;
  __device__ __forceinline__ void add(uint32_t* hist, uint32_t b) {
    if (b == bin) {
      ++count;
      return;
    }
    if (count) atomicAdd(&hist[bin], count);
    bin = b;
    count = 1;
  }
  __device__ __forceinline__ void flush(uint32_t* hist) {
    if (count) atomicAdd(&hist[bin], count);
    count = 0;
    bin = 0xFFFFFFFFu;
  }
};

}  // namespace bt
