// bt_small.cuh -- the k <= 128 pipeline: streaming consumers + a merger warp.
//
// Consumers (8 warps) test each chunk against the segment's threshold and hand the
// survivors, as (key, index, bits) composites, to the merger through a double-buffered
// shared-memory batch.  The merger warp keeps the exact running top-k of the segment (a
// sorted list of <= k composites) and publishes its k-th key; consumers adopt it as a
// strict threshold at their next chunk barrier (k candidates with that key or better, all
// at lower indices, already exist).  At the segment's last chunk the list is the answer.
// A segment shared by two blocks goes through global partial lists and an arrival counter;
// the last block to arrive merges them.
// No include guard: part of bt_body.cuh, compiled once per element namespace.



// ---- consumer ----------------------------------------------------------------------------

struct Counted {
  uint32_t flags, cnt, base, total, knext;
  bool fail;
};

// Counts this chunk's candidates under (K, STRICT) with one barrier and picks up the merger's
// latest threshold for segment `seg` (uniform: staged through kuse[par] by one thread).
// Flips `par`: consecutive counts alternate between the two slot sets.
template <bool STRICT>
__device__ __forceinline__ Counted count_chunk(const StageInfo& si, const uint8_t* buf,
                                               SmallScratch& sm, uint32_t K, int& par, int seg) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const bool take_all = K == kNoThreshold;
  const uint32_t vb = key_to_bits(K);
  const h2t v2 = u32_as_h2(vb | (vb << 16));
  Counted c;
  // A count is needed anyway: masks in one pass, without the maximum pre-test that pays off
  // only when nothing passes.
  c.flags = thread_flags<STRICT, true>(si, buf, v2, take_all, &c.cnt);
  uint32_t incl = 0;
  if (__ballot_sync(0xFFFFFFFFu, c.cnt != 0)) {  // warp scan only when something passed
    incl = c.cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
  }
  if (lane == 31) sm.wcnt[par][warp] = incl;
  if (tid == kThreads - 1) {  // the last warp has the fewest vectors: it stages the threshold
    const unsigned long long kp = *reinterpret_cast<volatile unsigned long long*>(&sm.kpub);
    sm.kuse[par] = (static_cast<int>(kp >> 32) == seg) ? static_cast<uint32_t>(kp & 0xFFFFu)
                                                       : kNoThreshold;
  }
  csync();
  c.fail = sm.fail != 0;
  const uint4 wa = lds128(&sm.wcnt[par][0]);
  const uint4 wb = lds128(&sm.wcnt[par][4]);
  const uint32_t t[kWarps] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
  uint32_t total = 0, wpre = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    wpre += w < warp ? t[w] : 0u;
    total += t[w];
  }
  c.total = total;
  c.base = wpre + incl - c.cnt;
  c.knext = sm.kuse[par];
  par ^= 1;  // the next count uses the other slots: no barrier separates it from these reads
  return c;
}

// Writes this thread's flagged candidates as composites at batch[base ...].
template <bool STRICT>
__device__ __forceinline__ void write_batch(const StageInfo& si, const uint8_t* buf, uint32_t flags,
                                            uint32_t K, uint32_t base, unsigned long long* batch) {
  const int tid = threadIdx.x;
  const bool take_all = K == kNoThreshold;
  const uint32_t vb = key_to_bits(K);
  const h2t v2 = u32_as_h2(vb | (vb << 16));
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(buf);
  const long long e0 = si.cv0 * 8;
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
      batch[base + r++] =
          make_composite((static_cast<uint32_t>(v16[lidx]) << 16) | lidx, e0, si.a0);
    }
  }
}

// Waits until batch buffer b may be overwritten (the merger released its previous use).
__device__ __forceinline__ bool wait_batch_free(const TopkParams& p, SmallScratch& sm,
                                                long long nb) {
  if (nb < 2) return true;
  return mbar_wait_n(&sm.batch_free[nb & 1], static_cast<uint32_t>(((nb >> 1) - 1) & 1),
                     p.handoff_tries);
}

__device__ __forceinline__ void send_batch(SmallScratch& sm, int b, const BatchMeta& meta) {
  if (threadIdx.x == 0) sm.meta[b] = meta;
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.batch_full[b]);
}

// One non-empty chunk: threshold, count, write the batch, hand it to the merger.
__device__ int small_chunk(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                           SmallScratch& sm, SegState& ss, int& par, long long* nbp,
                           uint32_t* guess, uint32_t* tight, bool* tight_hot) {
  const long long nb = *nbp;
  const uint32_t k = static_cast<uint32_t>(p.k);
  const uint32_t cap = static_cast<uint32_t>(p.cap);
  uint32_t K = ss.K;
  bool strict = ss.strict;
  Counted c;
  if (strict) {
    c = count_chunk<true>(si, buf, sm, K, par, ss.s);
  } else {
    bool have = false;
    if (ss.mycnt == 0 && *tight_hot && *tight != kNoThreshold && *tight != *guess) {
      // the previous segment's final threshold: on tie-heavy rows it holds in this chunk
      // already (>= k values at or beyond it), and then every later chunk is strict at it
      c = count_chunk<false>(si, buf, sm, *tight, par, ss.s);
      if (c.fail) return kChunkFail;
      if (c.total >= k && c.total <= cap) {
        K = *tight;
        have = true;
      } else {
        *tight_hot = false;  // retried after one segment without it
      }
    } else if (ss.mycnt == 0) {
      *tight_hot = true;
    }
    if (!have && ss.mycnt == 0 && *guess != kNoThreshold) {
      // the previous segment's first-chunk threshold, verified on this chunk: accepted when
      // it leaves between k and cap candidates here (then it is certified by this chunk)
      c = count_chunk<false>(si, buf, sm, *guess, par, ss.s);
      if (c.fail) return kChunkFail;
      if (c.total >= k && c.total <= cap) {
        K = *guess;
        have = true;
        if (threadIdx.x == 0 && p.stats) atomicAdd(&p.status[5], 1u);
      }
    }
    if (!have) {
      K = chunk_select(p, si, buf, sm);
      if (ss.mycnt == 0) *guess = K;
      c = count_chunk<false>(si, buf, sm, K, par, ss.s);
    }
    strict = false;
  }
  if (c.fail) return kChunkFail;
  const int b = static_cast<int>(nb & 1);
  uint32_t n = c.total;
  bool written = false;
  if (n > cap) {
    // too many survivors (rising values): a tighter chunk threshold, else the exact select
    if (strict) {
      const uint32_t kc = chunk_select(p, si, buf, sm);
      if (kc < K) {
        const Counted c2 = count_chunk<false>(si, buf, sm, kc, par, ss.s);
        if (c2.fail) return kChunkFail;
        if (c2.total <= cap) {
          K = kc;
          strict = false;
          c = c2;
          n = c2.total;
        }
      }
    }
    if (n > cap) {
      uint64_t S;
      uint32_t sbase, stot;
      const uint32_t kstar = exact_local_select(p, si, buf, sm, K, strict, &S, &sbase, &stot);
      if (!wait_batch_free(p, sm, nb)) sm.fail = 1u;  // caught at the next barrier
      write_selected(buf, S, si.cv0 * 8, si.a0, sm.batch[b] + sbase);
      K = kstar;
      strict = true;
      n = stot;
      written = true;
    }
  }
  const bool send = n > 0 || si.last;  // empty middle chunks need no hand-off
  if (!written && send) {
    if (!wait_batch_free(p, sm, nb)) sm.fail = 1u;  // caught at the next barrier
    if (c.flags) {
      if (strict) write_batch<true>(si, buf, c.flags, K, c.base, sm.batch[b]);
      else write_batch<false>(si, buf, c.flags, K, c.base, sm.batch[b]);
    }
  }
  // >= k values with key <= K are in the batches now (this chunk certified K, or an earlier
  // one did): later chunks of the segment only need key < K.
  if (K != kNoThreshold) {
    ss.K = K;
    ss.strict = true;
  }
  if (c.knext < ss.K) {  // the merger's k-th key: k candidates at lower indices beat ties
    ss.K = c.knext;
    ss.strict = true;
  }
  if (threadIdx.x == 0 && p.stats && n == 0) atomicAdd(&p.status[2], 1u);
  if (!send) return kChunkDone;
  BatchMeta meta;
  meta.len = si.a1 - si.a0;
  meta.part_slot = ss.slot0;
  meta.seg_slot = si.slot - si.c;
  meta.s = si.s;
  meta.n = n;
  meta.flags = si.last ? kBatchEnd : 0;
  meta.mycnt = ss.mycnt + 1;
  meta.nchunks = si.nchunks;
  meta.c = si.c;
  meta.K = ss.K;
  send_batch(sm, b, meta);
  *nbp = nb + 1;
  return kChunkDone;
}

__device__ void consumer_loop_small(const TopkParams& p, uint8_t* stages, uint64_t* full,
                                    uint64_t* empty, const StageInfo* info, SmallScratch& sm) {
  constexpr int S = Cfg<false>::kStagesN;
  SegState ss;
  uint32_t guess = kNoThreshold;  // the previous part's first-chunk threshold
  uint32_t tight = kNoThreshold;  // the previous part's final threshold
  bool tight_hot = true;
  bool second_hot = true;  // the test on a part's second chunk found it quiet last time it ran
  long long nb = 0;  // batches sent
  int st = 0, par = 0;
  uint32_t ph = 0;   // full-barrier phase parity of stage st
  bool failed = false;
  bool ready = false;  // stage st's full phase was already seen complete
  for (;;) {
    // A failed wait is noticed by everyone at the next barrier (sm.fail), so every consumer
    // thread keeps taking the same branches; stage info is never garbage (initialised).
    if (!ready && !mbar_wait(&full[st], ph)) sm.fail = 1u;
    ready = false;
    const StageInfo& si = info[st];  // read in place: valid until this stage is released
    if (si.part == kStopPart) break;
    if (si.nvc > 0) {
      if (si.part != ss.part) {
        tight = ss.K;
        ss = SegState{};
        ss.s = si.s;
        ss.part = si.part;
        ss.slot0 = si.slot;  // first slot of this part
      }
      const uint8_t* buf = stages + static_cast<size_t>(st) * kStageBytes;
      // The segment's first part certified a strict threshold for this chunk (another part):
      // take it when it is at least as tight as this part's own.
      bool adopted = false;
      if (si.ext_k < ss.K || (si.ext_k == ss.K && !ss.strict && si.ext_k < kNoThreshold)) {
        ss.K = si.ext_k;
        ss.strict = true;
        adopted = ss.mycnt == 0;
      }
      // Fast path for a middle chunk after a quiet one under a strict threshold: the max test
      // and one OR-barrier; only when some value passes (or a wait failed) does the chunk go
      // through the full count/compaction below.
      // The chunk right after the part's first one is tried too: once the first chunk has
      // certified a strict threshold, tie-heavy rows have nothing left to pass.
      bool done = false;
      // After a miss on a second chunk the next part skips that test once (rows whose first
      // threshold is loose rarely have a quiet second chunk; tie-heavy rows always do).
      const bool second = ss.mycnt == 1 && !ss.quiet;
      bool try_second = second && second_hot;
      if (second && !second_hot) second_hot = true;  // skipped once: the next part tries again
      if (ss.strict && ss.K < kNoThreshold && (ss.quiet || try_second || adopted)) {
        const bool last = si.last != 0;  // read before the barrier
        const uint32_t vb = key_to_bits(ss.K);
        uint32_t cnt;
        const uint32_t f = thread_flags<true>(si, buf, u32_as_h2(vb | (vb << 16)), false, &cnt);
        // Query the next stage now: the query's latency overlaps the OR-barrier, and a stage
        // that has landed needs no wait at the top of the loop (its phase cannot advance
        // before this thread releases it).
        ready = mbar_test_wait(&full[st + 1 == S ? 0 : st + 1], st + 1 == S ? ph ^ 1u : ph);
        done = !group_or<kThreads>(f != 0 || sm.fail != 0);
        if (done) ss.quiet = true;
        if (done && last) {  // nothing passed in the part's last chunk: the end marker
          if (!wait_batch_free(p, sm, nb)) sm.fail = 1u;  // seen by all at the next barrier
          BatchMeta meta;
          meta.len = si.a1 - si.a0;
          meta.part_slot = ss.slot0;
          meta.seg_slot = si.slot - si.c;
          meta.s = si.s;
          meta.n = 0;
          meta.flags = kBatchEnd;
          meta.mycnt = ss.mycnt + 1;
          meta.nchunks = si.nchunks;
          meta.c = si.c;
          meta.K = ss.K;
          send_batch(sm, static_cast<int>(nb & 1), meta);
          ++nb;
        }
      }
      if (try_second && !done && ss.strict && ss.K < kNoThreshold) second_hot = false;
      if (!done) {
        const long long nb0 = nb;
        const int r = small_chunk(p, si, buf, sm, ss, par, &nb, &guess, &tight, &tight_hot);
        if (r == kChunkFail) {
          failed = true;
          break;
        }
        ss.quiet = nb == nb0;
      }
      ++ss.mycnt;
    }
    release_stage(&empty[st]);
    if (++st == S) {
      st = 0;
      ph ^= 1u;
    }
  }
  // tell the merger to stop (bounded wait for the buffer)
  wait_batch_free(p, sm, nb);
  csync();
  if ((failed || sm.fail) && threadIdx.x == 0) atomicOr(&p.status[0], kStatusWaitTimeout);
  BatchMeta stop{};
  stop.flags = kBatchStop;
  send_batch(sm, static_cast<int>(nb & 1), stop);
}

// ---- merger ----------------------------------------------------------------------------------
//
// The running top-k is held in registers: a sorted (ascending) sequence of N = 32*R 64-bit
// composites, element r*32+lane in x[r] of lane `lane`.  A batch is loaded in the same layout,
// sorted with a bitonic network, and merged in: C[i] = min(L[i], B[N-1-i]) holds the N
// smallest of L and B as a bitonic sequence, and one bitonic merge pass sorts it.

constexpr unsigned long long kEmpty = ~0ull;  // never a composite (indices are < 2^32 - 1)

// L <- the N smallest of L and B, both ascending.
template <int R>
__device__ __forceinline__ void merge_sorted(unsigned long long (&L)[R], const unsigned long long (&B)[R]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const unsigned long long b = shfl64(B[R - 1 - r], 31 - lane);  // B[N-1-i]
    L[r] = L[r] < b ? L[r] : b;
  }
#pragma unroll
  for (int stride = 16 * R; stride > 0; stride >>= 1) bitonic_step<R>(L, 0, stride);
}

// Element i of the striped array (all lanes get it).
template <int R>
__device__ __forceinline__ unsigned long long element(const unsigned long long (&x)[R], int i) {
  unsigned long long v = x[0];
#pragma unroll
  for (int r = 1; r < R; ++r) v = (i >> 5) == r ? x[r] : v;
  return shfl64(v, i & 31);
}

// L <- the N smallest of L (ascending, N = 32R) and the 32*RB-entry ascending batch B
// (RB <= R): C[i] = min(L[i], B[N-1-i]) only touches L's top RB registers, and one bitonic
// merge pass over L sorts the result.
template <int R, int RB>
__device__ __forceinline__ void merge_sorted_top(unsigned long long (&L)[R], const unsigned long long (&B)[RB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = R - RB; r < R; ++r) {
    const unsigned long long b = shfl64(B[R - 1 - r], 31 - lane);  // B[N-1-i]
    L[r] = L[r] < b ? L[r] : b;
  }
#pragma unroll
  for (int stride = 16 * R; stride > 0; stride >>= 1) bitonic_step<R>(L, 0, stride);
}

// Merges m composites from `src` (shared or global memory; `sorted` when already ascending).
// An unsorted remainder of at most 32(R-1) entries goes in 32 at a time, each sorted in a
// single register: for R = 4 that is 15 + 28 exchange steps per 32 entries against 112 + 28
// for a full 128-entry sort.
template <int R>
__device__ __forceinline__ void absorb(unsigned long long (&L)[R], const unsigned long long* src,
                                       int m, bool sorted) {
  const int lane = threadIdx.x & 31;
  int base = 0;
  for (; base < m && (sorted || m - base > 32 * (R - 1)); base += 32 * R) {
    unsigned long long B[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = base + (r << 5) + lane;
      B[r] = i < m ? src[i] : kEmpty;
    }
    if (!sorted) warp_sort_regs<R>(B);
    merge_sorted<R>(L, B);
  }
  for (; base < m; base += 32) {
    unsigned long long B1[1];
    const int i = base + lane;
    B1[0] = i < m ? src[i] : kEmpty;
    warp_sort_regs<1>(B1);
    merge_sorted_top<R, 1>(L, B1);
  }
}

template <int R>
__device__ __forceinline__ void emit_row(const TopkParams& p, int s, const unsigned long long (&L)[R],
                                         int nl, long long len) {
  const int lane = threadIdx.x & 31;
  const int k = p.k;
  uint16_t* ov = p.out_values + static_cast<long long>(s) * k;
  int* oi = p.out_indices + static_cast<long long>(s) * k;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int pos = (r << 5) + lane;
    if (pos < k) {
      if (pos < nl) {
        ov[pos] = static_cast<uint16_t>(L[r] & 0xFFFFu);
        oi[pos] = static_cast<int>((L[r] >> 16) & 0xFFFFFFFFu);
      } else {
        ov[pos] = kNegInfBits;
        oi[pos] = -1;
      }
    }
  }
  if (lane == 0) {
    if (nl < k && len >= k) atomicOr(&p.status[0], kStatusCertifyFailed);
    if (p.stats) atomicAdd(&p.status[4], 1u);
  }
}

// End of this block's part of a segment: emit the row, or publish the partial list and, if
// this block arrives last, merge all parts.
template <int R>
__device__ void finalize_part(const TopkParams& p, const BatchMeta& m, unsigned long long (&L)[R],
                              int nl) {
  const int lane = threadIdx.x & 31;
  const int k = p.k;
  if (m.mycnt == m.nchunks) {
    emit_row<R>(p, m.s, L, nl, m.len);
    return;
  }
  // partial list (its first min(nl, k) entries) -> the cand region of this part's first slot
  const int np = nl < k ? nl : k;
  unsigned long long* dst = reinterpret_cast<unsigned long long*>(p.cand + m.part_slot * p.cap);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int pos = (r << 5) + lane;
    if (pos < np) dst[pos] = L[r];
  }
  // only the part's first slot carries a count (every slot count starts at zero per call:
  // a part's chunks need not be contiguous when idle blocks help)
  if (lane == 0) p.chunk_count[m.part_slot] = static_cast<uint32_t>(np);
  __threadfence();
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    const uint32_t old = atomicAdd(&p.seg_done[m.s], static_cast<uint32_t>(m.mycnt));
    last = old + static_cast<uint32_t>(m.mycnt) == static_cast<uint32_t>(m.nchunks);
  }
  last = __shfl_sync(0xFFFFFFFFu, last, 0);
  if (!last) return;
  __threadfence();
  int n = nl;
  // the slot counts of the whole segment in one round trip (lanes in parallel); only each
  // part's first slot holds a list
  for (int c0 = 0; c0 < m.nchunks; c0 += 32) {
    const long long slot = m.seg_slot + c0 + lane;
    int cnt = 0;
    if (c0 + lane < m.nchunks && slot != m.part_slot) {  // own part: already in L
      cnt = static_cast<int>(__ldcg(&p.chunk_count[slot]));
    }
    for (unsigned todo = __ballot_sync(0xFFFFFFFFu, cnt > 0); todo; todo &= todo - 1) {
      const int q = __ffs(todo) - 1;
      int cq = __shfl_sync(0xFFFFFFFFu, cnt, q);
      cq = cq < k ? cq : k;  // a partial list holds at most k entries, ascending
      const long long sq = m.seg_slot + c0 + q;
      absorb<R>(L, reinterpret_cast<const unsigned long long*>(p.cand + sq * p.cap), cq, true);
      n += cq;
    }
  }
  emit_row<R>(p, m.s, L, n < 32 * R ? n : 32 * R, m.len);
}

template <int R>
__device__ void merger_loop_r(const TopkParams& p, SmallScratch& sm) {
  const int lane = threadIdx.x & 31;
  const int k = p.k;
  unsigned long long L[R];
#pragma unroll
  for (int r = 0; r < R; ++r) L[r] = kEmpty;
  long long nbm = 0;
  int cur = -1;
  int nl = 0;
  for (;;) {
    const int b = static_cast<int>(nbm & 1);
    if (!mbar_wait_n(&sm.batch_full[b], static_cast<uint32_t>((nbm >> 1) & 1), p.handoff_tries)) {
      if (lane == 0) atomicOr(&p.status[0], kStatusWaitTimeout);
      return;
    }
    const BatchMeta m = sm.meta[b];
    if (m.flags & kBatchStop) return;
    if (m.s != cur) {
      cur = m.s;
      nl = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) L[r] = kEmpty;
    }
    const int nb = static_cast<int>(m.n);
    if (nb > 0) {
      absorb<R>(L, sm.batch[b], nb, false);
      nl = nl + nb < 32 * R ? nl + nb : 32 * R;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.batch_free[b]);
    if (nb > 0 && nl >= k) {
      const unsigned long long kth = element<R>(L, k - 1);
      if (lane == 0) {
        *reinterpret_cast<volatile unsigned long long*>(&sm.kpub) =
            (static_cast<unsigned long long>(static_cast<uint32_t>(m.s)) << 32) |
            static_cast<uint32_t>(kth >> 48);
        // the segment's first part also publishes it for the other parts (helpers), with the
        // last chunk it covers: their later chunks may take it as a strict threshold
        if (m.part_slot == m.seg_slot && m.mycnt < m.nchunks) {
          st_relaxed_gpu(&p.seg_thresh[m.s],
                         (static_cast<uint32_t>(kth >> 48) << 16) | static_cast<uint32_t>(m.c));
        }
      }
    }
    if (m.flags & kBatchEnd) {
      finalize_part<R>(p, m, L, nl);
      cur = -1;
      nl = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) L[r] = kEmpty;
    }
    ++nbm;
  }
}

__device__ void merger_loop(const TopkParams& p, SmallScratch& sm) {
  if (p.k <= 32) {
    merger_loop_r<1>(p, sm);
  } else if (p.k <= 64) {
    merger_loop_r<2>(p, sm);
  } else {
    merger_loop_r<4>(p, sm);
  }
}

