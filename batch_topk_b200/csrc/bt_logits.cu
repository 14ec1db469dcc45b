// bt_logits.cu -- the logits producer with the top-k fused into its epilogue.
//
// logits[M, V] = H[M, D] . W[V, D]^T for a decode-sized batch (M <= 128 rows of hidden state,
// V vocabulary rows of the output projection), fp16 in, fp32 accumulation on the tcgen05
// tensor cores, rounded to fp16 in the epilogue exactly as a plain GEMM that stores fp16
// would.  Two entry points share the kernel:
//   * bt_logits_f16 stores the logits (the unfused producer);
//   * bt_logits_topk_f16 never stores them: each CTA keeps, per row, the exact top k of the
//     vocabulary columns it produced, and only those lists reach HBM; the streaming top-k
//     kernel (bt_topk_half) then selects each row's top k from the CTAs' lists.
//
// The kernel is warp-specialised, one CTA per SM, persistent over a contiguous range of
// 128-column vocabulary tiles:
//   warp 0     TMA producer: 128x64 tiles of H and W into a 4-stage shared-memory ring
//              (128-byte swizzle, no multicast), completion counted on mbarriers;
//   warp 1     allocates 256 TMEM columns (two 128x128 fp32 accumulators) and issues
//              tcgen05.mma (kind::f16, M=128, N=128, K=16) from one thread, committing each
//              stage back to the producer and each finished accumulator to the epilogue;
//   warps 2-5  epilogue: tcgen05.ld of their 32 TMEM lanes (one accumulator row, i.e. one
//              token row, per thread), fp32 -> fp16, and either the store or the row's
//              running top-k filter; the accumulator is handed back as soon as it is read,
//              so the next tile's MMAs overlap this epilogue.
// Every mbarrier wait is bounded; a wait that gives up sets a status flag and stops the CTA.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include "../../include/batch_topk_b200.h"
#include "bt_device.cuh"

namespace btl {

namespace f16 {
#include "bt_elem.cuh"
}  // namespace f16

constexpr int kBM = 128;                 // accumulator rows (token rows; rows >= M are zero)
constexpr int kBN = 128;                 // vocabulary columns per tile
constexpr int kBK = 64;                  // 64 fp16 = one 128-byte swizzle row
constexpr int kStages = 4;
constexpr int kThreads = 192;            // 6 warps: TMA, MMA, 4 x epilogue
constexpr uint32_t kTileABytes = kBM * kBK * 2;
constexpr uint32_t kTileBBytes = kBN * kBK * 2;
constexpr uint32_t kStageBytes = kTileABytes + kTileBBytes;  // 32 KiB
constexpr uint32_t kTmemCols = 2 * kBN;  // two accumulators
constexpr int kMaxCap = 256;             // per-row candidate buffer of the fused epilogue (max)
constexpr int kMaxTilesPerCta = 511;     // column offsets inside a CTA's range fit 16 bits

constexpr size_t kBarOff = static_cast<size_t>(kStages) * kStageBytes;
constexpr size_t kCandOff = kBarOff + 128;
constexpr size_t kSmemPlain = kCandOff + 1024;  // + slack for aligning the base to 1 KiB
constexpr size_t kRowOff = kCandOff;    // fused: the rows' final counts, then the row buffers
constexpr size_t kBufOff = kRowOff + static_cast<size_t>(kBM) * 4;
constexpr size_t kSmemFused = 232448;    // the per-block opt-in maximum: buffers take the rest
constexpr size_t kBufBytes = kSmemFused - 1024 - kBufOff;

struct LogitsParams {
  int M, V, D, k;
  int tiles;          // ceil(V / kBN)
  int tiles_per_cta;  // CTA c owns tiles [c * tiles_per_cta, min(tiles, (c + 1) * tiles_per_cta))
  int ktiles;         // ceil(D / kBK)
  int L;              // fused: candidates per row (the CTAs' lists back to back)
  int vec_store;      // plain: 16-byte row stores allowed (V % 8 == 0, 16-byte aligned logits)
  int cap;            // fused: candidate buffer entries per row (>= k + 32, <= kMaxCap)
  uint16_t* logits;   // plain: [M, V]
  uint16_t* cand_vals;  // fused: [M, L] value bits
  int* cand_idx;        // fused: [M, L] vocabulary indices
  uint32_t* status;     // bit 0: a bounded wait gave up
};

// ---- tcgen05 / TMA wrappers --------------------------------------------------------------

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 2-D tiled TMA load (coordinates: x = column in elements, y = row), no multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(bt::smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bt::smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the 128-byte swizzle:
// rows of 128 bytes, 8-row swizzle atoms 1024 bytes apart (stride byte offset), leading byte
// offset unused (1), descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: fp16 A and B (both K-major), fp32 accumulator,
// N = kBN, M = kBM.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) |
                            (static_cast<uint32_t>(kBN >> 3) << 17) |
                            (static_cast<uint32_t>(kBM >> 4) << 24);

// D (+)= A . B^T for one K=16 slice; acc = 0 overwrites D.  No output lane is disabled.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t acc) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(da), "l"(db), "r"(kIdesc), "r"(acc), "r"(z)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bt::smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"  // in the same statement: no use of v before the wait
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

// ---- fused epilogue: per-row candidate buffers ------------------------------------------
//
// Each token row keeps a buffer of candidates in shared memory: 32-bit entries
// (key << 16 | column offset in the CTA's range) and the value bits beside them, in column
// order.  Comparing entries compares (key, column): exactly the tie rule (equal values, lower
// index first), so "the k best" of a row are its k smallest entries, and a column can only
// enter while its entry is below the row's threshold T (the k-th smallest kept so far).
// Each epilogue thread filters its own row (one compare a value, an append when it passes); a
// row that runs out of room is cut by its whole warp together (a bitwise select by warp
// reductions over the row's contiguous buffer), so no lane ever runs a cut alone.

// Cuts the row's n (<= kMaxCap) entries, keeping their order, and returns the row's new
// threshold.  The key bits are resolved from the top by a bitwise select, one warp reduction a
// bit, starting below the bits every entry shares; [xk, U) is the key range still holding the
// k-th smallest key.  EXACT: down to that key, keeping every entry with a smaller key and the
// first k - (those) entries with it in buffer order (which is column order); returns the k-th
// smallest entry.  *kept receives the entries kept.  Otherwise the select stops as soon as the entries with key < U number at
// most `target`: those are kept (at least k of them, so U is certified) and U << 16 is
// returned -- unless ties at the k-th key leave more, when the exact cut is made.
template <bool EXACT>
__device__ __forceinline__ uint32_t warp_cut_row(uint32_t* ent, uint16_t* vb, int n, int k,
                                                 int target, int* kept) {
  constexpr int NJ = kMaxCap / 32;
  const int lane = threadIdx.x & 31;
  const int nj = (n + 31) >> 5;
  uint32_t key[NJ];
  bool val[NJ];
  uint32_t kor = 0, kand = 0xFFFFu;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    val[j] = j < nj && lane + 32 * j < n;
    key[j] = val[j] ? ent[lane + 32 * j] >> 16 : 0xFFFFu;
    if (val[j]) {
      kor |= key[j];
      kand &= key[j];
    }
  }
  kor = __reduce_or_sync(0xFFFFFFFFu, kor);
  kand = __reduce_and_sync(0xFFFFFFFFu, kand);
  const uint32_t diff = kor ^ kand;  // key bits that vary
  const int top = diff ? 31 - __clz(diff) : -1;
  // bits above `top` are common to every key
  uint32_t xk = top >= 0 ? (kand & ~((2u << top) - 1u)) : kand;
  uint32_t U = top >= 0 ? xk + (2u << top) : xk + 1u;
  uint32_t cU = static_cast<uint32_t>(n);  // entries with key < U
  int bit = top;
#pragma unroll 1
  for (; bit >= 0; --bit) {
    if (!EXACT && cU <= static_cast<uint32_t>(target)) break;
    const uint32_t y = xk | (1u << bit);
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < NJ; ++j) c += (val[j] && key[j] < y) ? 1u : 0u;
    c = __reduce_add_sync(0xFFFFFFFFu, c);
    if (c < static_cast<uint32_t>(k)) {
      xk = y;
    } else {
      U = y;
      cU = c;
    }
  }
  const bool coarse = !EXACT && cU <= static_cast<uint32_t>(target);
  int need = 0;
  if (!coarse) {  // xk is the k-th smallest key
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < NJ; ++j) c += (val[j] && key[j] < xk) ? 1u : 0u;
    need = k - static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, c));  // ties kept, >= 1
  }
  uint32_t e[NJ];
  uint16_t b[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    e[j] = val[j] ? ent[lane + 32 * j] : 0u;
    b[j] = val[j] ? vb[lane + 32 * j] : 0;
  }
  __syncwarp();  // every lane has read the buffer before it is rewritten
  const uint32_t lt = (1u << lane) - 1u;
  int base = 0, eq_seen = 0;
  uint32_t kth = 0;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    if (j < nj) {
      bool keep;
      bool eq = false;
      int eq_rank = 0;
      if (coarse) {
        keep = val[j] && key[j] < U;
      } else {
        eq = val[j] && key[j] == xk;
        const uint32_t meq = __ballot_sync(0xFFFFFFFFu, eq);
        eq_rank = eq_seen + __popc(meq & lt);
        keep = val[j] && (key[j] < xk || (eq && eq_rank < need));
        eq_seen += __popc(meq);
      }
      const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
      if (keep) {
        const int at = base + __popc(m & lt);
        ent[at] = e[j];
        vb[at] = b[j];
        if (eq && eq_rank == need - 1) kth = e[j];
      }
      base += __popc(m);
    }
  }
  __syncwarp();
  *kept = base;
  if (coarse) return U >= 0x10000u ? 0xFFFFFFFFu : (U << 16);
  return __reduce_max_sync(0xFFFFFFFFu, kth);  // one lane holds the k-th entry
}


__device__ __forceinline__ void set_fail(volatile uint32_t* fail, uint32_t* status) {
  *fail = 1u;
  atomicOr(status, 1u);
}

// ---- the kernel ---------------------------------------------------------------------------

template <bool FUSED>
__global__ void __launch_bounds__(kThreads, 1)
    logits_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const LogitsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;  // [2] accumulator b holds a finished tile
  uint64_t* tempty = tfull + 2;       // [2] the epilogue has read accumulator b
  uint64_t* drain = tempty + 2;       // every MMA issued has completed (teardown)
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(drain + 1);
  volatile uint32_t* fail = tmem_slot + 1;
  int* rowN = reinterpret_cast<int*>(smem + kRowOff);             // [kBM] final row counts
  const int mpad = (p.M + 31) & ~31;                             // rows with a buffer
  uint32_t* ent = reinterpret_cast<uint32_t*>(smem + kBufOff);   // [mpad][cap]
  uint16_t* vbits = reinterpret_cast<uint16_t*>(ent + static_cast<size_t>(mpad) * p.cap);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * p.tiles_per_cta;
  const int t1 = min(p.tiles, t0 + p.tiles_per_cta);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      bt::mbar_init(&full[s], 1);
      bt::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      bt::mbar_init(&tfull[b], 1);
      bt::mbar_init(&tempty[b], 4);  // one arrival per epilogue warp
    }
    bt::mbar_init(drain, 1);
    *fail = 0u;
    bt::fence_mbar_init();
  }
  if (warp == 1) {  // the whole warp allocates; the address lands in tmem_slot
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     bt::smem_addr(const_cast<uint32_t*>(tmem_slot))),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      const uint64_t pol_w = bt::policy_evict_first();  // W streams through once
      const uint64_t pol_h = policy_evict_last();       // H is re-read for every tile
      int s = 0;
      uint32_t ph = 0;
      long long issued = 0;
      for (int t = t0; t < t1 && !*fail; ++t) {
        for (int kt = 0; kt < p.ktiles; ++kt) {
          if (!bt::mbar_wait_abort(&empty[s], ph ^ 1u, fail)) {
            set_fail(fail, p.status);
            break;
          }
          uint8_t* st = smem + static_cast<size_t>(s) * kStageBytes;
          bt::mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_2d(st, &tmA, kt * kBK, 0, &full[s], pol_h);
          tma_load_2d(st + kTileABytes, &tmB, kt * kBK, t * kBN, &full[s], pol_w);
          ++issued;
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Do not retire while a tensor copy may still land in shared memory (after a failure the
      // consumer may not have waited for the last stages); a copy always completes.
      for (long long r = issued - kStages; r < issued; ++r) {
        if (r >= 0) bt::mbar_wait(&full[r % kStages], static_cast<uint32_t>((r / kStages) & 1));
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int t = t0, i = 0; t < t1 && !*fail; ++t, ++i) {
        const int b = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        if (!bt::mbar_wait_abort(&tempty[b], (use & 1u) ^ 1u, fail)) {
          set_fail(fail, p.status);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * kBN);
        bool ok = true;
        for (int kt = 0; kt < p.ktiles; ++kt) {
          if (!bt::mbar_wait_abort(&full[s], ph, fail)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = bt::smem_addr(smem + static_cast<size_t>(s) * kStageBytes);
          const uint32_t b0 = a0 + kTileABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {  // K=16 slices: 32 bytes along each row
            mma_f16(d, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                    (kt | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) {
          set_fail(fail, p.status);
          break;
        }
        mma_commit(&tfull[b]);
      }
      // nothing may still write TMEM when it is freed
      mma_commit(drain);
      if (!bt::mbar_wait(drain, 0u)) atomicOr(p.status, 1u);
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31 ----
    const int q = warp & 3;
    const int r = q * 32 + lane;  // this thread's accumulator row
    const int ew = warp - 2;      // fused: rows ew, ew + 4, ... are this warp's to filter
    const int colbase = t0 * kBN;
    int cnt = 0;               // fused: entries in this thread's row buffer
    uint32_t T = 0xFFFFFFFFu;  // fused: the row's threshold (column offsets stay below 0xFFFF)
    for (int t = t0, i = 0; t < t1; ++t, ++i) {
      const int b = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      const bool got = bt::mbar_wait_abort(&tfull[b], use & 1u, fail);
      // uniform over the warps that go on together (tcgen05.ld needs whole warps, and the
      // fused epilogue's warps meet at named barriers)
      const bool lost = FUSED ? bt::group_or<128>(!got) : !__all_sync(0xFFFFFFFFu, got);
      if (lost) {
        if (lane == 0) set_fail(fail, p.status);
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < kBN; c0 += 32) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * kBN + c0),
                  v);
        const int col0 = t * kBN + c0;
        if constexpr (FUSED) {
          // Each thread filters its own row's 32 values against the row's threshold (one
          // compare a value; appends are rare once the row has a threshold) ...
          if (r < p.M) {
            // entries of all 32 values first (independent of one another), then the appends
            const uint32_t ob = static_cast<uint32_t>(col0 - colbase);
            uint32_t e[32], hw2[16];
            uint32_t pm = 0;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const __half2 h2 = __floats2half2_rn(__uint_as_float(v[j]), __uint_as_float(v[j + 1]));
              const uint32_t hw = *reinterpret_cast<const uint32_t*>(&h2);
              hw2[j >> 1] = hw;
              e[j] = (f16::desc_key(hw & 0xFFFFu) << 16) | (ob + static_cast<uint32_t>(j));
              e[j + 1] = (f16::desc_key(hw >> 16) << 16) | (ob + static_cast<uint32_t>(j + 1));
              pm |= (e[j] < T ? 1u : 0u) << j;
              pm |= (e[j + 1] < T ? 1u : 0u) << (j + 1);
            }
            if (col0 + 32 > p.V) pm &= p.V > col0 ? (1u << (p.V - col0)) - 1u : 0u;
            if (pm) {
              uint32_t* re = ent + r * p.cap;
              uint16_t* rb = vbits + r * p.cap;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if ((pm >> j) & 1u) {
                  re[cnt] = e[j];
                  rb[cnt] = static_cast<uint16_t>(hw2[j >> 1] >> (16 * (j & 1)));
                  ++cnt;
                }
              }
            }
          }
          // ... and a row that could not take another 32 values is cut by the whole warp
          uint32_t full_rows = __ballot_sync(0xFFFFFFFFu, cnt > p.cap - 32);
          while (full_rows) {
            const int rr = __ffs(full_rows) - 1;
            full_rows &= full_rows - 1u;
            const int row = q * 32 + rr;
            const int n = __shfl_sync(0xFFFFFFFFu, cnt, rr);
            int kept;
            const uint32_t tn = warp_cut_row<false>(ent + row * p.cap, vbits + row * p.cap, n, p.k,
                                                    p.k + (p.cap - 32 - p.k) / 4, &kept);
            if (lane == rr) {
              cnt = kept;
              T = tn;
            }
          }
        } else {
          if (r < p.M) {
            uint32_t w[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint32_t lo = __half_as_ushort(__float2half_rn(__uint_as_float(v[2 * j])));
              const uint32_t hi = __half_as_ushort(__float2half_rn(__uint_as_float(v[2 * j + 1])));
              w[j] = lo | (hi << 16);
            }
            uint16_t* dst = p.logits + static_cast<size_t>(r) * p.V + col0;
            if (p.vec_store && col0 + 32 <= p.V) {
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col0 + j < p.V) dst[j] = static_cast<uint16_t>((w[j >> 1] >> (16 * (j & 1))) & 0xFFFFu);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bt::mbar_arrive(&tempty[b]);  // the MMA warp may overwrite accumulator b
    }
    if constexpr (FUSED) {
      rowN[r] = cnt;
      if (!bt::group_or<128>(*fail != 0u)) {  // also orders the counts for the other warps
        // each row's exact top k of this CTA's columns (min(k, columns) entries), in column
        // order, to this CTA's slot of the row's candidate list; rows spread over the 4 warps
        for (int row = ew; row < p.M; row += 4) {
          uint32_t* re = ent + row * p.cap;
          uint16_t* rb = vbits + row * p.cap;
          int n = rowN[row];
          if (n > p.k) {
            int kept;
            warp_cut_row<true>(re, rb, n, p.k, 0, &kept);
            n = kept;  // == k
          }
          __syncwarp();
          const size_t base = static_cast<size_t>(row) * p.L + static_cast<size_t>(blockIdx.x) * p.k;
          for (int i2 = lane; i2 < n; i2 += 32) {
            p.cand_vals[base + i2] = rb[i2];
            p.cand_idx[base + i2] = colbase + static_cast<int>(re[i2] & 0xFFFFu);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// Candidate indices back to vocabulary indices after the second-stage select:
// out_idx[r, j] = cand_idx[r, local[r, j]].
__global__ void gather_indices(const int* __restrict__ cand_idx, const int* __restrict__ local,
                               int* __restrict__ out_idx, int M, int L, int k) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * k) return;
  const int r = i / k;
  const int l = local[i];
  out_idx[i] = l >= 0 ? cand_idx[static_cast<size_t>(r) * L + l] : -1;
}



// ---- host side ----------------------------------------------------------------------------

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_mu;
__device__ uint32_t g_plain_status;  // status word of bt_logits_f16 (it takes no workspace)
EncodeTiledFn g_encode = nullptr;
bool g_encode_tried = false;
int g_sms[64] = {0};
bool g_attr[64] = {false};

// The driver's tensor-map encoder, looked up once through the runtime (no libcuda link).
EncodeTiledFn encoder() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_encode_tried) {
    g_encode_tried = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  return g_encode;
}

// SM count of the current device, and the kernels' shared-memory opt-in (once per device).
cudaError_t device_setup(int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_attr[dev]) {
    e = cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(logits_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemPlain));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(logits_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemFused));
    if (e != cudaSuccess) return e;
    g_attr[dev] = true;
  }
  *sms = g_sms[dev];
  return cudaSuccess;
}

// [rows, cols] row-major fp16, 128x64 boxes (64 columns = 128 bytes) with the 128-byte swizzle;
// out-of-range rows and columns read as zero.
bool make_map(CUtensorMap* m, const void* base, int rows, int cols) {
  EncodeTiledFn fn = encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), 128u};
  const cuuint32_t estr[2] = {1u, 1u};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Plan {
  int tiles, tpc, grid, ktiles, L;
};

// Shape checks shared by both entry points; k = 0 for the plain producer.
bool plan(int M, int V, int D, int k, int sms, Plan* pl) {
  if (M < 1 || M > kBM || V < 1 || D < 8 || (D & 7) != 0) return false;
  if (k < 0 || k > BT_LOGITS_MAX_K || k > V) return false;
  pl->tiles = (V + kBN - 1) / kBN;
  pl->tpc = (pl->tiles + sms - 1) / sms;
  if (pl->tpc > kMaxTilesPerCta) return false;
  pl->grid = (pl->tiles + pl->tpc - 1) / pl->tpc;
  pl->ktiles = (D + kBK - 1) / kBK;
  const int last_cols = V - (pl->grid - 1) * pl->tpc * kBN;
  pl->L = (pl->grid - 1) * k + (last_cols < k ? last_cols : k);
  return true;
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct FusedLayout {
  size_t status, vals, idx, local, topk_ws, total;
};

FusedLayout fused_layout(int M, const Plan& pl, int k) {
  FusedLayout f;
  f.status = 0;
  f.vals = 256;
  f.idx = f.vals + align256(static_cast<size_t>(M) * pl.L * 2);
  f.local = f.idx + align256(static_cast<size_t>(M) * pl.L * 4);
  f.topk_ws = f.local + align256(static_cast<size_t>(M) * k * 4);
  f.total = f.topk_ws + align256(bt_topk_half_workspace_size(M, pl.L, k));
  return f;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace btl

extern "C" {

int bt_logits_f16(const void* d_hidden, const void* d_weight, int M, int V, int D,
                  void* d_logits, void* stream) {
  using namespace btl;
  if (!d_hidden || !d_weight || !d_logits || !aligned16(d_hidden) || !aligned16(d_weight) ||
      (reinterpret_cast<uintptr_t>(d_logits) & 1u)) {
    return cudaErrorInvalidValue;
  }
  int sms = 0;
  cudaError_t e = device_setup(&sms);
  if (e != cudaSuccess) return e;
  Plan pl;
  if (!plan(M, V, D, 0, sms, &pl)) return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  if (!make_map(&ta, d_hidden, M, D) || !make_map(&tb, d_weight, V, D)) return cudaErrorInvalidValue;
  LogitsParams p{};
  p.M = M;
  p.V = V;
  p.D = D;
  p.k = 0;
  p.tiles = pl.tiles;
  p.tiles_per_cta = pl.tpc;
  p.ktiles = pl.ktiles;
  p.L = 0;
  p.logits = static_cast<uint16_t*>(d_logits);
  p.vec_store = (V % 8 == 0) && aligned16(d_logits);
  // no caller workspace here: a wait that gives up is reported to the library's own word
  void* sw = nullptr;
  e = cudaGetSymbolAddress(&sw, g_plain_status);
  if (e != cudaSuccess) return e;
  p.status = static_cast<uint32_t*>(sw);
  logits_kernel<false><<<pl.grid, kThreads, kSmemPlain, static_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  return cudaGetLastError();
}

size_t bt_logits_topk_f16_workspace_size(int M, int V, int D, int k) {
  using namespace btl;
  int sms = 0;
  if (device_setup(&sms) != cudaSuccess) return 0;
  Plan pl;
  if (k < 1 || !plan(M, V, D, k, sms, &pl)) return 0;
  return fused_layout(M, pl, k).total;
}

int bt_logits_topk_f16(const void* d_hidden, const void* d_weight, int M, int V, int D, int k,
                       void* d_out_values, int* d_out_indices, void* d_workspace,
                       size_t workspace_bytes, void* stream) {
  using namespace btl;
  if (!d_hidden || !d_weight || !d_out_values || !d_out_indices || !d_workspace ||
      !aligned16(d_hidden) || !aligned16(d_weight) || (reinterpret_cast<uintptr_t>(d_workspace) & 255u) ||
      (reinterpret_cast<uintptr_t>(d_out_values) & 1u) || (reinterpret_cast<uintptr_t>(d_out_indices) & 3u)) {
    return cudaErrorInvalidValue;
  }
  int sms = 0;
  cudaError_t e = device_setup(&sms);
  if (e != cudaSuccess) return e;
  Plan pl;
  if (k < 1 || !plan(M, V, D, k, sms, &pl)) return cudaErrorInvalidValue;
  const FusedLayout f = fused_layout(M, pl, k);
  if (workspace_bytes < f.total) return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  if (!make_map(&ta, d_hidden, M, D) || !make_map(&tb, d_weight, V, D)) return cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(d_workspace);
  e = cudaMemsetAsync(ws + f.status, 0, 4, st);
  if (e != cudaSuccess) return e;
  LogitsParams p{};
  p.M = M;
  p.V = V;
  p.D = D;
  p.k = k;
  p.tiles = pl.tiles;
  p.tiles_per_cta = pl.tpc;
  p.ktiles = pl.ktiles;
  p.L = pl.L;
  const int mpad = (M + 31) & ~31;
  p.cap = static_cast<int>(kBufBytes / (static_cast<size_t>(mpad) * 6));
  if (p.cap > kMaxCap) p.cap = kMaxCap;
  p.cap = (p.cap - 1) | 1;  // odd: the rows' appends at equal counts fall in distinct banks
  if (p.cap < k + 32) return cudaErrorInvalidValue;  // cannot happen for M <= 128, k <= 64
  p.cand_vals = reinterpret_cast<uint16_t*>(ws + f.vals);
  p.cand_idx = reinterpret_cast<int*>(ws + f.idx);
  p.status = reinterpret_cast<uint32_t*>(ws + f.status);
  logits_kernel<true><<<pl.grid, kThreads, kSmemFused, st>>>(ta, tb, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // second stage: each row's top k among its L candidates (kept in column order, so ties
  // still go to the lower vocabulary index), then candidate slots -> vocabulary indices
  int* local = reinterpret_cast<int*>(ws + f.local);
  const int rc = bt_topk_half(p.cand_vals, M, pl.L, k, d_out_values, local, ws + f.topk_ws,
                              bt_topk_half_workspace_size(M, pl.L, k), stream);
  if (rc != 0) return rc;
  const int n = M * k;
  gather_indices<<<(n + 255) / 256, 256, 0, st>>>(p.cand_idx, local, d_out_indices, M, pl.L, k);
  return cudaGetLastError();
}

int bt_logits_topk_status(const void* d_workspace, int M, int V, int D, int k, void* stream) {
  using namespace btl;
  int sms = 0;
  cudaError_t e = device_setup(&sms);
  if (e != cudaSuccess) return -static_cast<int>(e);
  Plan pl;
  if (!d_workspace || k < 1 || !plan(M, V, D, k, sms, &pl)) {
    return -static_cast<int>(cudaErrorInvalidValue);
  }
  const FusedLayout f = fused_layout(M, pl, k);
  uint32_t s = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  e = cudaMemcpyAsync(&s, static_cast<const uint8_t*>(d_workspace) + f.status, 4,
                      cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return -static_cast<int>(e);
  // the producer's flag (a bounded wait gave up) is reported as BT_STATUS_WAIT_TIMEOUT, OR-ed
  // with the second stage's own status word
  const int s2 = bt_workspace_status(static_cast<const uint8_t*>(d_workspace) + f.topk_ws, M,
                                     stream, nullptr);
  if (s2 < 0) return s2;
  return static_cast<int>((s ? BT_STATUS_WAIT_TIMEOUT : 0u) | static_cast<uint32_t>(s2));
}

}  // extern "C"
