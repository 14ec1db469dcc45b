// bt_large.cuh -- the k > 128 pipeline: streaming consumers with a per-segment shared-memory
// candidate cache.
//
// Each block keeps the candidates of the segment part it is working on in a 2048-entry cache
// of (key, index, bits) composites, in index order.  A chunk's survivors under the segment's
// certified threshold are appended; when the cache has no room, the entries that can no longer
// reach the top k are dropped (filtered against a threshold the current chunk certifies, or cut
// to the exact k best), so at least k entries of room always exist and nothing spills to global
// memory.  At the end of a part the cache holds a superset of the part's top k; a whole segment
// is selected and written from it directly, a split segment's parts publish their exact top-k
// lists and the block that finishes the segment last merges them.  This replaces the
// reference's boundary select, compaction and final sort (src/radix_boundary_select.cuh,
// src/candidate_compact.cuh, src/final_block_sort.cuh) for k above its 128 limit.
// No include guard: part of bt_body.cuh, compiled once per element namespace.

using LargeScratch = Scratch<true>;

struct LargeState {
  int s = -1;
  int part = -2;              // work part (kStopPart never matches: -2)
  uint32_t K = kNoThreshold;  // certified threshold key (desc)
  bool strict = false;        // later chunks need key < K (always, once K is set)
  bool quiet = false;         // the previous chunk of the part added nothing
  bool rising = false;        // the previous chunk beat the stale threshold (values ramp up)
  uint32_t nbuf = 0;          // candidates in sm.cache
  uint32_t added = 0;         // candidates appended since K was last tightened from the cache
  int mycnt = 0;              // chunks of this part processed
  int nchunks = 0;            // chunks of the segment
  long long part_slot = 0;    // slot of the part's first chunk: its partial list lives there
  long long seg_slot = 0;     // slot of the segment's chunk 0
  long long a0 = 0, a1 = 0;   // aligned element coordinates of the segment
  uint32_t pub = kNoThreshold;  // thread 0 of a first part: the threshold it last published
};

// ---- strided count and append --------------------------------------------------------
//
// For the count and the append, thread t owns vectors t + kThreads * j of the chunk, j = 0..7
// ("round j").  Round-major order (round, thread, element) is index order, and survivors
// clustered in one stretch of the chunk (sorted rows) spread over every thread.  Positions come
// from per-round warp scans of 16-bit packed counts and one barrier.
struct SCount {
  uint64_t M;         // survivors: bit 8 j + e = element e of the thread's round-j vector
  uint64_t E;         // tie mode: the survivors whose key equals the threshold (subset of M)
  uint32_t base[4];   // per round (16-bit fields): index-order rank of the thread's first
                      // survivor among the round-major survivors (tie mode: among key < T)
  uint32_t ebase[4];  // tie mode, per round: survivors with key == T ahead of the thread's first
  uint32_t total;     // survivors (tie mode: those with key < T)
  uint32_t total_eq;  // tie mode: survivors with key == T
  bool fail;
};

// Counts the chunk's survivors under threshold T: key < T (STRICT), key <= T, or every value
// (take_all, T == kNoThreshold).  TIES (non-strict, not take-all): survivors with key == T are
// counted apart, so the caller can keep only the first ones by index.  One barrier.
template <bool STRICT, bool TIES>
__device__ __forceinline__ SCount strided_count(const StageInfo& si, const uint8_t* buf,
                                                LargeScratch& sm, uint32_t T, int& par) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const bool take_all = T == kNoThreshold;
  const uint32_t vb = key_to_bits(T);
  const h2t v2 = u32_as_h2(vb | (vb << 16));
  SCount c;
  c.M = 0;
  c.E = 0;
  uint32_t own[4] = {0, 0, 0, 0}, owne[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int vi = j * kThreads + tid;
    if (vi < si.nvc) {
      const uint4 w = lds128(buf + vi * 16);
      uint32_t m, e = 0;
      if (TIES) {
        const uint32_t lt = gt_mask8(w, v2);  // value > V: key < T
        m = ge_mask8(w, v2);                  // value >= V: key <= T
        e = m & ~lt;
      } else {
        m = take_all ? 0xFFu : pass_mask8<STRICT>(w, v2);
      }
      if (vi == si.vlo || vi == si.vhi) {
        const uint32_t vm = valid_mask8(si.cv0 + vi, si.a0, si.a1);
        m &= vm;
        e &= vm;
      }
      c.M |= static_cast<uint64_t>(m) << (8 * j);
      c.E |= static_cast<uint64_t>(e) << (8 * j);
      const uint32_t cl = static_cast<uint32_t>(__popc(m & ~e));
      own[j >> 1] |= cl << ((j & 1) * 16);
      if (TIES) owne[j >> 1] |= static_cast<uint32_t>(__popc(e)) << ((j & 1) * 16);
    }
  }
  uint32_t incl[4] = {own[0], own[1], own[2], own[3]};
  uint32_t incle[4] = {owne[0], owne[1], owne[2], owne[3]};
  if (__ballot_sync(0xFFFFFFFFu, c.M != 0)) {
    warp_scan4(incl);
    if (TIES) warp_scan4(incle);
  }
  if (lane == 31) {
    *reinterpret_cast<uint4*>(&sm.rw[par][warp][0]) = make_uint4(incl[0], incl[1], incl[2], incl[3]);
    if (TIES) {
      *reinterpret_cast<uint4*>(&sm.rw[par][warp][4]) =
          make_uint4(incle[0], incle[1], incle[2], incle[3]);
    }
  }
  csync();
  c.fail = sm.fail != 0;
  c.total = round_bases(sm.rw[par], 0, incl, own, c.base);
  c.total_eq = 0;
  if (TIES) c.total_eq = round_bases(sm.rw[par], 1, incle, owne, c.ebase);
  par ^= 1;
  return c;
}

// Appends the counted survivors at sm.cache[nbuf ...] in index order.  Tie mode keeps every
// survivor with key < T and the first `need` with key == T.  Each thread visits only its set
// bits, and in tie mode skips the rounds that hold nothing it still keeps.
template <bool TIES>
__device__ __forceinline__ void strided_append(const StageInfo& si, const uint8_t* buf,
                                               const SCount& c, uint32_t need, LargeScratch& sm,
                                               uint32_t nbuf) {
  const int tid = threadIdx.x;
  const long long e0 = si.cv0 * 8;
  unsigned long long* out = sm.cache + nbuf;
#pragma unroll 1
  for (int j = 0; j < kVecPerThread; ++j) {
    uint32_t m = static_cast<uint32_t>(c.M >> (8 * j)) & 0xFFu;
    const uint32_t em = static_cast<uint32_t>(c.E >> (8 * j)) & 0xFFu;
    uint32_t lpos = field16(c.base, j);
    uint32_t epos = TIES ? field16(c.ebase, j) : 0u;
    if (TIES && epos >= need) m &= ~em;  // every tie of this round is past the first `need`
    if (m == 0) continue;
    const int vi = j * kThreads + tid;
    const uint4 w = lds128(buf + vi * 16);
    // key < T survivors and the ties in front of them, in element order
    for (uint32_t f = m; f; f &= f - 1) {
      const int e = __ffs(f) - 1;
      const uint32_t lidx = static_cast<uint32_t>(vi * 8 + e);
      const unsigned long long comp = make_composite((vec_half(w, e) << 16) | lidx, e0, si.a0);
      if (TIES && ((em >> e) & 1u)) {
        // ties ahead of this one: epos plus those of this vector below element e
        const uint32_t r = epos + static_cast<uint32_t>(__popc(em & ((1u << e) - 1u)));
        if (r < need) out[lpos + static_cast<uint32_t>(__popc(m & ~em & ((1u << e) - 1u))) + r] = comp;
      } else {
        const uint32_t lt_before = static_cast<uint32_t>(__popc(m & ~em & ((1u << e) - 1u)));
        uint32_t r = 0;
        if (TIES) {
          r = epos + static_cast<uint32_t>(__popc(em & ((1u << e) - 1u)));
          r = r < need ? r : need;
        }
        out[lpos + lt_before + r] = comp;
      }
    }
  }
  csync();  // the appended entries are visible to the whole block
}

// Exact cutoff of the survivors counted in c: the k-th smallest key among them and the number
// of survivors with a smaller key (two 8-bit digit histograms over the survivors only).
// Requires c.total + c.total_eq >= k.  The histograms are zero on entry and left zero.
__device__ __forceinline__ uint32_t survivor_cutoff(const uint8_t* buf, const SCount& c,
                                                    uint32_t k, LargeScratch& sm,
                                                    uint32_t* before) {
  // Every lane walks all 64 of its element positions in the same order, with predicated
  // shared atomics (lane-dependent loops over set bits diverge).
  const int tid = threadIdx.x;
#pragma unroll 1
  for (int j = 0; j < kVecPerThread; ++j) {
    const uint32_t m = static_cast<uint32_t>(c.M >> (8 * j)) & 0xFFu;
    const uint4 w = lds128(buf + (j * kThreads + tid) * 16);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if ((m >> e) & 1u) atomicAdd(&sm.hist1[desc_key(vec_half(w, e)) >> 8], 1u);
    }
  }
  csync();
  if (tid < 32) warp_find_bin(sm.hist1, 0, k, &sm.bin1, &sm.before1);
  csync();
  const uint32_t b1 = static_cast<uint32_t>(sm.bin1);
#pragma unroll 1
  for (int j = 0; j < kVecPerThread; ++j) {
    const uint32_t m = static_cast<uint32_t>(c.M >> (8 * j)) & 0xFFu;
    const uint4 w = lds128(buf + (j * kThreads + tid) * 16);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t key = desc_key(vec_half(w, e));
      if (((m >> e) & 1u) && (key >> 8) == b1) atomicAdd(&sm.hist2[key & 0xFFu], 1u);
    }
  }
  csync();
  if (tid < 32) warp_find_bin(sm.hist2, sm.before1, k, &sm.bin2, &sm.before2);
  csync();
  const uint32_t kk = (b1 << 8) | static_cast<uint32_t>(sm.bin2);
  *before = sm.before2;
  sm.hist1[tid] = 0;
  sm.hist2[tid] = 0;
  csync();
  return kk;
}

// Cuts the cache to its exact k best (keys below the k-th key, then the first ties at it by
// index; the cache is in index order) and makes that k-th key the strict threshold.
__device__ __forceinline__ void cut_to_k(LargeScratch& sm, LargeState& ls, uint32_t k) {
  const uint32_t kk = buffer_kth_key_block(sm, ls.nbuf, k);
  const uint32_t need = k - sm.before2;  // ties at kk within the k best
  ls.nbuf = compact_cache<true>(sm, ls.nbuf, kk, need);
  if (kk < ls.K || !ls.strict) {
    ls.K = kk < ls.K ? kk : ls.K;
    ls.strict = true;
  }
  ls.added = 0;
}

// Drops the cache entries with key > kc: after this chunk certified at least k of its values
// with key <= kc (at higher indices than every cache entry), such entries can no longer reach
// the top k.  Index order is kept.
__device__ __forceinline__ void drop_above(LargeScratch& sm, LargeState& ls, uint32_t kc) {
  ls.nbuf = compact_cache<true>(sm, ls.nbuf, kc + 1u, 0u);
}

// Exact top-k of this chunk's candidates under (T, strict), appended to the cache; returns
// the cutoff key (the chunk's k-th best under T).  Rare: only when even a chunk-certified
// threshold leaves more candidates than the cache has room for (heavy ties at it).
__device__ uint32_t large_exact(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                                LargeScratch& sm, LargeState& ls, uint32_t T, bool strict) {
  uint64_t S;
  uint32_t sbase, stot;
  const uint32_t kstar = exact_local_select(p, si, buf, sm, T, strict, &S, &sbase, &stot);
  const long long e0 = si.cv0 * 8;
  write_selected(buf, S, e0, si.a0, sm.cache + ls.nbuf + sbase);
  ls.nbuf += stot;
  csync();
  return kstar;
}

// ---- contiguous count and append ------------------------------------------------------
//
// The steady-state form: thread t owns vectors 8t .. 8t+7, one warp scan and one barrier give
// every thread its first output position, and each thread writes its own survivors.  That is
// cheapest while survivors are few and spread; when one thread holds many (survivors clustered
// in a stretch of the chunk), the strided form above spreads the writes instead.
struct CCount {
  uint32_t flags, cnt, base, total, maxcnt;
  bool fail;
};

template <bool STRICT>
__device__ __forceinline__ CCount contig_count(const StageInfo& si, const uint8_t* buf,
                                               LargeScratch& sm, uint32_t K, int& par) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint32_t vb = key_to_bits(K);
  const h2t v2 = u32_as_h2(vb | (vb << 16));
  CCount c;
  c.flags = thread_flags<STRICT, true>(si, buf, v2, false, &c.cnt);
  uint32_t incl = 0, wmax = 0;
  if (__ballot_sync(0xFFFFFFFFu, c.cnt != 0)) {
    incl = c.cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    wmax = __reduce_max_sync(0xFFFFFFFFu, c.cnt);
  }
  if (lane == 31) sm.wcnt[par][warp] = incl | (wmax << 16);  // total <= 16384, max <= 64
  csync();
  c.fail = sm.fail != 0;
  const uint4 wa = lds128(&sm.wcnt[par][0]);
  const uint4 wb = lds128(&sm.wcnt[par][4]);
  const uint32_t t[kWarps] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
  uint32_t total = 0, wpre = 0, mx = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t tw = t[w] & 0xFFFFu;
    wpre += w < warp ? tw : 0u;
    total += tw;
    mx = (t[w] >> 16) > mx ? (t[w] >> 16) : mx;
  }
  c.total = total;
  c.maxcnt = mx;
  c.base = wpre + incl - c.cnt;
  par ^= 1;
  return c;
}

// Writes this thread's survivors under K (key < K with STRICT, else key <= K; flagged
// vectors, index order) at sm.cache[nbuf + base ...].
template <bool STRICT>
__device__ __forceinline__ void contig_append(const StageInfo& si, const uint8_t* buf,
                                              const CCount& c, uint32_t K, LargeScratch& sm,
                                              uint32_t nbuf) {
  const int tid = threadIdx.x;
  const uint32_t vb = key_to_bits(K);
  const h2t v2 = u32_as_h2(vb | (vb << 16));
  const long long e0 = si.cv0 * 8;
  unsigned long long* out = sm.cache + nbuf + c.base;
  uint32_t r = 0;
  for (uint32_t flags = c.flags; flags; flags &= flags - 1) {
    const int j = __ffs(flags) - 1;
    const int vi = tid * kVecPerThread + j;
    const uint4 w = lds128(buf + vi * 16);
    uint32_t m = pass_mask8<STRICT>(w, v2);
    if (vi == si.vlo || vi == si.vhi) m &= valid_mask8(si.cv0 + vi, si.a0, si.a1);
    for (; m; m &= m - 1) {
      const int e = __ffs(m) - 1;
      const uint32_t lidx = static_cast<uint32_t>(vi * 8 + e);
      out[r++] = make_composite((vec_half(w, e) << 16) | lidx, e0, si.a0);
    }
  }
  csync();
}

// A thread holding more survivors than this writes too long alone: the strided form is used.
constexpr uint32_t kClusterMax = 16;

// Appends this chunk's exact top k among the survivors counted in t (survivors under a
// threshold certified for this chunk, at least k of them): the k-th smallest survivor key T2
// (t's own threshold when fewer than k survivors beat it, else a digit select over the
// survivors), every survivor with key < T2 and the first ties at T2 by index.  The cache first
// drops what these k entries beat and, if still short of room, is cut to its own k best.
// Afterwards T2 is the segment's strict threshold.  Returns false when a wait failed.
__device__ bool append_chunk_topk(const StageInfo& si, const uint8_t* buf, SCount& t, uint32_t T,
                                  bool tie_counted, LargeScratch& sm, LargeState& ls,
                                  uint32_t k, int& par) {
  constexpr uint32_t C = Cfg<true>::kCacheCap;
  uint32_t T2 = T;
  if (!tie_counted || t.total >= k) {
    uint32_t before;
    T2 = survivor_cutoff(buf, t, k, sm, &before);
    if (T2 == kNoThreshold) return false;  // the k-th survivor is a NaN: the caller's fallback
    t = strided_count<false, true>(si, buf, sm, T2, par);
    if (t.fail) return false;
  }
  const uint32_t need = k - t.total;  // ties at T2 within the chunk's top k
  if (k > C - ls.nbuf && ls.nbuf > 0) drop_above(sm, ls, T2);
  if (k > C - ls.nbuf) cut_to_k(sm, ls, k);
  strided_append<true>(si, buf, t, need, sm, ls.nbuf);
  ls.nbuf += k;
  ls.added = 0;
  ls.quiet = false;
  if (ls.K == kNoThreshold || T2 < ls.K) ls.K = T2;
  ls.strict = true;
  return true;
}

// One non-empty chunk of the current part.  Returns false when a wait failed (sm.fail).
__device__ bool large_chunk(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                            LargeScratch& sm, LargeState& ls, int& par) {
  constexpr uint32_t C = Cfg<true>::kCacheCap;
  const uint32_t k = static_cast<uint32_t>(p.k);
  const bool probe = si.probe != 0;
  // A chunk after a quiet one under a strict threshold: the maximum test and one OR-barrier.
  if (!probe && ls.quiet && ls.K < kNoThreshold) {
    const uint32_t vb = key_to_bits(ls.K);
    uint32_t cnt;
    const uint32_t f = thread_flags<true>(si, buf, u32_as_h2(vb | (vb << 16)), false, &cnt);
    if (!group_or<kThreads>(f != 0 || sm.fail != 0)) return true;
  }
  // Steady state: survivors under the segment's strict threshold, if the cache has room.
  SCount c;
  bool counted = false;
  if (!probe && ls.K != kNoThreshold && !ls.rising) {
    CCount cc = contig_count<true>(si, buf, sm, ls.K, par);
    if (cc.fail) return false;
    if (cc.total > C - ls.nbuf && ls.nbuf > k) {
      // The cache's own k-th key is usually far tighter than anything this chunk certifies
      // alone (the k-th of every value seen so far): cut to it and count again.
      const uint32_t K1 = ls.K;
      cut_to_k(sm, ls, k);
      if (ls.K != K1) {
        cc = contig_count<true>(si, buf, sm, ls.K, par);
        if (cc.fail) return false;
      }
    }
    if (cc.total <= C - ls.nbuf) {
      if (cc.maxcnt <= kClusterMax) {
        contig_append<true>(si, buf, cc, ls.K, sm, ls.nbuf);
      } else {
        c = strided_count<true, false>(si, buf, sm, ls.K, par);
        if (c.fail) return false;
        strided_append<false>(si, buf, c, 0u, sm, ls.nbuf);
      }
      ls.nbuf += cc.total;
      ls.added += cc.total;
      ls.quiet = cc.total == 0;
      if (ls.added >= k && ls.nbuf >= k) {  // k more since the last tightening: the cache's
        const uint32_t kk = buffer_kth_key_block(sm, ls.nbuf, k);  // k-th key is tighter
        if (kk < ls.K) ls.K = kk;
        ls.added = 0;
      }
      return true;
    }
    counted = true;  // the stale threshold overflowed the cache
  }
  // The threshold this chunk certifies by itself: its k-th best group maximum kc (at least k
  // of its values have key <= kc).
  const uint32_t kc = chunk_select<true>(p, si, buf, sm);
  if (sm.fail) return false;
  if (probe) {
    // The segment's last chunk, out of turn: at least k of its values have key <= kc, and
    // every value of this part precedes them, so this part's values with key <= kc (ties
    // included) must stay candidates: the strict threshold kc + 1 (keys are integers).  The
    // chunk is counted again in its own turn.
    if (kc + 1u < kNoThreshold && kc + 1u < ls.K) {
      ls.K = kc + 1u;
      ls.strict = true;
      ls.rising = false;
      ls.quiet = false;
      ls.added = 0;
    }
    return true;
  }
  const bool own = kc != kNoThreshold && (ls.K == kNoThreshold || kc < ls.K);
  const bool was_rising = ls.rising;
  ls.rising = (counted || ls.rising) && own;  // values ramp up: skip the stale count next time
  if (ls.rising && !was_rising && threadIdx.x == 0 && ls.part_slot == ls.seg_slot) {
    // ask the producer for a look at the segment's last chunk: on rising rows its certified
    // threshold makes the chunks in between quiet
    *reinterpret_cast<volatile uint32_t*>(&sm.probe_req) = static_cast<uint32_t>(ls.part) + 1u;
  }
  // Every value with key <= kc, when the cache has room for them (the usual first chunk).
  // With less room than about k (rising rows after their first chunk) that seldom fits, and
  // the exact top k below is taken directly.
  if (own && C - ls.nbuf >= k + k / 8) {
    const CCount cc = contig_count<false>(si, buf, sm, kc, par);
    if (cc.fail) return false;
    if (cc.total <= C - ls.nbuf) {
      if (cc.maxcnt <= kClusterMax) {
        contig_append<false>(si, buf, cc, kc, sm, ls.nbuf);
      } else {
        c = strided_count<false, false>(si, buf, sm, kc, par);
        if (c.fail) return false;
        strided_append<false>(si, buf, c, 0u, sm, ls.nbuf);
      }
      ls.nbuf += cc.total;
      ls.added = 0;
      ls.quiet = false;
      ls.K = kc;  // certified: >= k values with key <= kc are in the cache now
      ls.strict = true;
      return true;
    }
  }
  if (own) {
    // too many (heavy ties, or a loose kc): the chunk's exact top k
    c = strided_count<false, true>(si, buf, sm, kc, par);
    if (c.fail) return false;
    if (append_chunk_topk(si, buf, c, kc, true, sm, ls, k, par)) return true;
    if (sm.fail) return false;
  } else {
    // kc is no better than the segment's threshold (or there is neither): survivors under
    // that threshold, or every value
    c = ls.K == kNoThreshold ? strided_count<false, false>(si, buf, sm, kNoThreshold, par)
                             : strided_count<true, false>(si, buf, sm, ls.K, par);
    if (c.fail) return false;
    if (c.total > C - ls.nbuf && ls.nbuf > k) {
      const uint32_t K1 = ls.K;
      cut_to_k(sm, ls, k);
      if (ls.K != K1) {
        c = strided_count<true, false>(si, buf, sm, ls.K, par);
        if (c.fail) return false;
      }
    }
    if (c.total <= C - ls.nbuf) {
      strided_append<false>(si, buf, c, 0u, sm, ls.nbuf);
      ls.nbuf += c.total;
      ls.quiet = c.total == 0;
      return true;
    }
    if (append_chunk_topk(si, buf, c, ls.K, false, sm, ls, k, par)) return true;
    if (sm.fail) return false;
  }
  // The chunk's k-th best is a NaN (fewer than k numbers in it): the ordered exact select,
  // which places NaNs by index.
  if (ls.nbuf > C - k) cut_to_k(sm, ls, k);
  const uint32_t T = own ? kc : ls.K;
  const bool st = !own && ls.K != kNoThreshold;
  const uint32_t kstar = large_exact(p, si, buf, sm, ls, T, st);
  if (ls.K == kNoThreshold || kstar < ls.K) ls.K = kstar;
  ls.strict = true;
  ls.quiet = false;
  return true;
}

// ---- row output ----------------------------------------------------------------------

// Writes row s from the n <= 1024 composites at sm.cache[0 .. n): the first k in ascending
// composite order (key, then index: the reference's order, include/batch_topk_types.cuh:50-92)
// as value bits and indices; when n < k, slots n .. k-1 get the padding (-inf, index -1).  Warp w sorts entries
// [128 w, 128 w + 128) in registers (bitonic, 4 a lane); then every entry's rank is its place
// in its own run plus, per other run, a binary search for the entries below it, and it is
// written straight to that slot of the row.
__device__ void sort_emit(const TopkParams& p, LargeScratch& sm, uint32_t n, int s,
                          long long len) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const uint32_t warp = static_cast<uint32_t>(tid >> 5);
  const uint32_t k = static_cast<uint32_t>(p.k);
  const uint32_t runs = (n + 127) / 128;  // <= 8 runs of 128 (n <= 1024)
  unsigned long long x[4];
  if (warp < runs) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t i = warp * 128 + r * 32 + lane;
      x[r] = i < n ? sm.cache[i] : ~0ull;
    }
    warp_sort_regs<4>(x);  // element r * 32 + lane of the run in x[r]
  }
  csync();
  if (warp < runs) {
#pragma unroll
    for (int r = 0; r < 4; ++r) sm.cache[warp * 128 + r * 32 + lane] = x[r];
  }
  csync();
  uint16_t* ov = p.out_values + static_cast<long long>(s) * k;
  int* oi = p.out_indices + static_cast<long long>(s) * k;
  if (warp < runs) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const unsigned long long v = x[r];
      if (v == ~0ull) continue;  // padding past n
      uint32_t rank = static_cast<uint32_t>(r * 32 + lane);
      for (uint32_t q = 0; q < runs; ++q) {
        if (q == warp) continue;
        const unsigned long long* run = sm.cache + q * 128;
        uint32_t lo = 0;  // entries of run q below v (composites are distinct)
#pragma unroll
        for (uint32_t step = 128; step > 0; step >>= 1) {
          if (lo + step <= 128 && run[lo + step - 1] < v) lo += step;
        }
        rank += lo;
      }
      if (rank < k) {
        ov[rank] = static_cast<uint16_t>(v & 0xFFFFu);
        oi[rank] = static_cast<int>((v >> 16) & 0xFFFFFFFFu);
      }
    }
  }
  for (uint32_t r = n + tid; r < k; r += kThreads) {
    ov[r] = kNegInfBits;
    oi[r] = -1;
  }
  if (tid == 0) {
    // fewer than k candidates can only come from a segment shorter than k
    if (n < k && len >= static_cast<long long>(k)) atomicOr(&p.status[0], kStatusCertifyFailed);
    if (p.stats) atomicAdd(&p.status[4], 1u);
  }
  csync();  // the cache is free again
}

// Loads n composites from a partial list in global memory into sm.cache[at ...].
__device__ __forceinline__ void load_list(const unsigned long long* src, uint32_t n,
                                          LargeScratch& sm, uint32_t at) {
  for (uint32_t i = threadIdx.x; i < n; i += kThreads) sm.cache[at + i] = __ldcg(src + i);
}

// Merges the adjacent runs sm.cache[0, n) and sm.cache[n, n + m), each in index order, into
// one run in index order: each entry moves to its own position plus the number of entries of
// the other run with a smaller index (a binary search; indices are distinct).  Each thread
// holds its kCacheCap / kThreads entries in registers across the barrier, so the in-place
// writes never overtake a read.
__device__ void merge_index_runs(LargeScratch& sm, uint32_t n, uint32_t m) {
  constexpr int kPer = Cfg<true>::kCacheCap / kThreads;
  const uint32_t tot = n + m;
  unsigned long long v[kPer];
  uint32_t pos[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t i = threadIdx.x * kPer + j;
    v[j] = i < tot ? sm.cache[i] : 0ull;
    pos[j] = i;
    if (i < tot) {
      const bool first = i < n;
      const uint32_t base = first ? n : 0u;
      const uint32_t idx = static_cast<uint32_t>(v[j] >> 16);
      uint32_t lo = 0, hi = first ? m : n;  // entries of the other run with a smaller index
      while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (static_cast<uint32_t>(sm.cache[base + mid] >> 16) < idx) lo = mid + 1u; else hi = mid;
      }
      pos[j] = (first ? i : i - n) + lo;
    }
  }
  csync();
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (threadIdx.x * kPer + j < tot) sm.cache[pos[j]] = v[j];
  }
  csync();
}

// End of this block's part of segment ls.s: write the row, or publish the part's top k and,
// if this block finishes the segment, merge all parts in index order.
__device__ void large_close(const TopkParams& p, LargeState& ls, LargeScratch& sm) {
  if (ls.mycnt == 0) return;
  constexpr uint32_t C = Cfg<true>::kCacheCap;
  const uint32_t k = static_cast<uint32_t>(p.k);
  const long long len = ls.a1 - ls.a0;
  if (ls.mycnt == ls.nchunks) {
    // the sort ranks up to 1024 entries and writes the first k: no cut below that
    if (ls.nbuf > 1024) cut_to_k(sm, ls, k);
    sort_emit(p, sm, ls.nbuf, ls.s, len);
    return;
  }
  // split segment: this part's exact top k, in index order, to its first slot
  if (ls.nbuf > k) cut_to_k(sm, ls, k);
  const int tid = threadIdx.x;
  unsigned long long* dst = reinterpret_cast<unsigned long long*>(p.cand + ls.part_slot * p.cap);
  for (uint32_t i = tid; i < ls.nbuf; i += kThreads) dst[i] = sm.cache[i];
  __threadfence();
  csync();
  if (tid == 0) {
    p.chunk_count[ls.part_slot] = ls.nbuf;  // zeroed per call: only parts' first slots hold one
    __threadfence();
    const uint32_t old = atomicAdd(&p.seg_done[ls.s], static_cast<uint32_t>(ls.mycnt));
    sm.bcast[0] = old + static_cast<uint32_t>(ls.mycnt) == static_cast<uint32_t>(ls.nchunks);
  }
  csync();
  if (!sm.bcast[0]) return;
  __threadfence();
  // last to arrive: every part's list, joined in index order
  uint32_t n = 0;
  for (int c0 = 0; c0 < ls.nchunks; c0 += kThreads) {
    const int c = c0 + tid;
    const uint32_t cnt = c < ls.nchunks ? __ldcg(&p.chunk_count[ls.seg_slot + c]) : 0u;
    sm.tbase[tid] = cnt;
    csync();
    const int m = ls.nchunks - c0 < kThreads ? ls.nchunks - c0 : kThreads;
    for (int j = 0; j < m; ++j) {
      const uint32_t cj = sm.tbase[j];  // uniform
      if (cj == 0) continue;
      if (n + cj > C) {
        ls.nbuf = n;
        cut_to_k(sm, ls, k);
        n = ls.nbuf;
      }
      load_list(reinterpret_cast<const unsigned long long*>(p.cand + (ls.seg_slot + c0 + j) * p.cap),
                cj, sm, n);
      csync();
      // parts that took turns at a segment's chunks (helping) hold interleaved index ranges:
      // the lists meet by index, as the cuts and the tie rule need
      if (p.steal && n > 0) merge_index_runs(sm, n, cj);
      n += cj;
    }
    csync();  // tbase is rewritten by the next round
  }
  ls.nbuf = n;
  if (ls.nbuf > 1024) cut_to_k(sm, ls, k);
  sort_emit(p, sm, ls.nbuf, ls.s, len);
}

__device__ void consumer_loop_large(const TopkParams& p, uint8_t* stages, uint64_t* full,
                                    uint64_t* empty, const StageInfo* info, LargeScratch& sm) {
  constexpr int S = Cfg<true>::kStagesN;
  LargeState ls;
  int st = 0, par = 0;
  uint32_t ph = 0;
  bool failed = false;
  for (;;) {
    // A failed wait is noticed by every consumer at the next barrier (sm.fail), so all keep
    // taking the same branches; stage info is never garbage (initialised).
    if (!mbar_wait(&full[st], ph)) sm.fail = 1u;
    const StageInfo& si = info[st];  // read in place: valid until this stage is released
    if (si.part != ls.part) {
      if (group_or<kThreads>(sm.fail != 0)) {
        failed = true;
        break;
      }
      large_close(p, ls, sm);
      if (si.part == kStopPart) break;
      ls = LargeState{};
      ls.s = si.s;
      ls.part = si.part;
      ls.nchunks = si.nchunks;
      ls.part_slot = si.slot;
      ls.seg_slot = si.slot - si.c;
      ls.a0 = si.a0;
      ls.a1 = si.a1;
    }
    if (si.nvc > 0) {
      const uint8_t* buf = stages + static_cast<size_t>(st) * kStageBytes;
      // another part's chunk: the segment's first part may have certified a tighter strict
      // threshold from chunks that all precede this one
      if (si.ext_k < ls.K) {
        ls.K = si.ext_k;
        ls.strict = true;
      }
      if (!large_chunk(p, si, buf, sm, ls, par)) {
        failed = true;
        break;
      }
      if (!si.probe) ++ls.mycnt;
      // the segment's first part publishes its threshold for helpers, with the last chunk
      // it covers (strict K: k values with key <= K lie in chunks <= si.c, or, from a probe
      // of the last chunk, anywhere with key < K, which bounds every chunk)
      if (threadIdx.x == 0 && !si.probe && ls.part_slot == ls.seg_slot &&
          ls.mycnt < ls.nchunks && ls.K < kNoThreshold && ls.K != ls.pub) {
        st_relaxed_gpu(&p.seg_thresh[ls.s], (ls.K << 16) | static_cast<uint32_t>(si.c));
        ls.pub = ls.K;
      }
    }
    release_stage(&empty[st]);
    if (++st == S) {
      st = 0;
      ph ^= 1u;
    }
  }
  if (failed && threadIdx.x == 0) atomicOr(&p.status[0], kStatusWaitTimeout);
  if (failed) sm.fail = 1u;  // the producer stops waiting for stages nobody will release
}
