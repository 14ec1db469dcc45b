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
  uint32_t added = 0;         // candidates added since K was last tightened from the cache
  int mycnt = 0;              // chunks of this part processed
  int nchunks = 0;            // chunks of the segment
  long long part_slot = 0;    // slot of the part's first chunk: its partial list lives there
  long long seg_slot = 0;     // slot of the segment's chunk 0
  long long a0 = 0, a1 = 0;   // aligned element coordinates of the segment
};

struct LCount {
  uint32_t flags, cnt, base, total;
  bool fail;
};

// Counts the chunk's candidates under (K, STRICT) with one barrier: per-thread vector flags and
// counts, the thread's first output position and the block total.  `par` alternates the
// per-warp count slots so consecutive counts need no barrier between them.
template <bool STRICT>
__device__ __forceinline__ LCount large_count(const StageInfo& si, const uint8_t* buf,
                                              LargeScratch& sm, uint32_t K, int& par) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const bool take_all = K == kNoThreshold;
  const uint32_t vb = key_to_bits(K);
  const h2t v2 = u32_as_h2(vb | (vb << 16));
  LCount c;
  c.flags = thread_flags<STRICT, true>(si, buf, v2, take_all, &c.cnt);
  uint32_t incl = 0;
  if (__ballot_sync(0xFFFFFFFFu, c.cnt != 0)) {
    incl = c.cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
  }
  if (lane == 31) sm.wcnt[par][warp] = incl;
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
  par ^= 1;
  return c;
}

__device__ __forceinline__ LCount count_under(const StageInfo& si, const uint8_t* buf,
                                              LargeScratch& sm, uint32_t K, bool strict,
                                              int& par) {
  return strict ? large_count<true>(si, buf, sm, K, par) : large_count<false>(si, buf, sm, K, par);
}

// Appends the counted candidates (in index order) at sm.cache[nbuf ...].
__device__ __forceinline__ void large_append(const StageInfo& si, const uint8_t* buf,
                                             const LCount& c, uint32_t K, bool strict,
                                             LargeScratch& sm, uint32_t nbuf) {
  const bool take_all = K == kNoThreshold;
  const uint32_t vb = key_to_bits(K);
  const h2t v2 = u32_as_h2(vb | (vb << 16));
  if (c.total >= 512) {  // clustered survivors: spread the writes over the block
    if (strict) write_balanced<true>(si, buf, c.flags, v2, take_all, c.base, c.total, sm, nbuf);
    else write_balanced<false>(si, buf, c.flags, v2, take_all, c.base, c.total, sm, nbuf);
  } else if (c.flags) {
    if (strict) write_flagged<true>(si, buf, c.flags, v2, take_all, c.base, sm, nbuf);
    else write_flagged<false>(si, buf, c.flags, v2, take_all, c.base, sm, nbuf);
  }
  csync();  // the appended entries are visible to the whole block
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
  const int tid = threadIdx.x;
  uint64_t S;
  uint32_t sbase, stot;
  const uint32_t kstar = exact_local_select(p, si, buf, sm, T, strict, &S, &sbase, &stot);
  const long long e0 = si.cv0 * 8;
  uint32_t r = 0;
  const uint32_t at = ls.nbuf + sbase;
  for_each_candidate<true>(buf, S, [&](uint32_t bits, int pos) {
    const uint32_t w = (bits << 16) | static_cast<uint32_t>(tid * 64 + pos);
    sm.cache[at + r] = make_composite(w, e0, si.a0);
    ++r;
  });
  ls.nbuf += stot;
  csync();
  return kstar;
}

// One non-empty chunk of the current part.  Returns false when a wait failed (sm.fail).
__device__ bool large_chunk(const TopkParams& p, const StageInfo& si, const uint8_t* buf,
                            LargeScratch& sm, LargeState& ls, int& par) {
  constexpr uint32_t C = Cfg<true>::kCacheCap;
  const uint32_t k = static_cast<uint32_t>(p.k);
  // A chunk after a quiet one under a strict threshold: the maximum test and one OR-barrier.
  if (ls.quiet && ls.strict && ls.K < kNoThreshold) {
    const uint32_t vb = key_to_bits(ls.K);
    uint32_t cnt;
    const uint32_t f = thread_flags<true>(si, buf, u32_as_h2(vb | (vb << 16)), false, &cnt);
    if (!group_or<kThreads>(f != 0 || sm.fail != 0)) return true;
  }
  LCount c;
  bool counted = false;
  if (ls.K != kNoThreshold && !ls.rising) {
    c = count_under(si, buf, sm, ls.K, ls.strict, par);
    if (c.fail) return false;
    counted = true;
    if (c.total <= C - ls.nbuf) {
      large_append(si, buf, c, ls.K, ls.strict, sm, ls.nbuf);
      ls.nbuf += c.total;
      ls.added += c.total;
      ls.quiet = c.total == 0;
      if (ls.added >= k && ls.nbuf >= k) {  // k more candidates: a tighter threshold
        const uint32_t kk = buffer_kth_key_block(sm, ls.nbuf, k);
        if (kk < ls.K) ls.K = kk;
        ls.strict = true;
        ls.added = 0;
      }
      return true;
    }
  }
  // The threshold this chunk certifies by itself: its k-th best group maximum.
  const uint32_t kc = chunk_select<true>(p, si, buf, sm);
  if (sm.fail) return false;
  const bool own = kc < ls.K || ls.K == kNoThreshold;  // kc (key <= kc) is the tighter bound
  ls.rising = counted ? own : (ls.rising && own);
  uint32_t T = own ? kc : ls.K;
  bool st = own ? false : ls.strict;
  if (own && kc != kNoThreshold && ls.nbuf > 0) {
    // every cache entry with key > kc is beaten by >= k values of this chunk: drop them when
    // the room is short (rising rows lose their whole cache here)
    if (ls.nbuf > C - k) drop_above(sm, ls, kc);
  }
  if (own || !counted) {  // otherwise T is the threshold just counted
    c = count_under(si, buf, sm, T, st, par);
    if (c.fail) return false;
  }
  if (c.total > C - ls.nbuf && ls.nbuf > k) {
    cut_to_k(sm, ls, k);  // room for at least k more
    if (ls.K < T || (ls.K == T && !st)) {
      T = ls.K;
      st = true;
      c = count_under(si, buf, sm, T, st, par);
      if (c.fail) return false;
    }
  }
  if (c.total <= C - ls.nbuf) {
    large_append(si, buf, c, T, st, sm, ls.nbuf);
    ls.nbuf += c.total;
    ls.added += c.total;
    ls.quiet = c.total == 0;
    if (T != kNoThreshold && (c.total > 0 || st)) {
      // T is certified: by this chunk (kc: >= k values with key <= kc, all written now), or it
      // is the segment's own strict threshold
      if (T < ls.K || ls.K == kNoThreshold) ls.K = T;
      ls.strict = true;
    }
  } else {
    // more ties at the chunk's threshold than the cache has room for: exact top k of the chunk
    const uint32_t kstar = large_exact(p, si, buf, sm, ls, T, st);
    if (kstar < ls.K || ls.K == kNoThreshold) ls.K = kstar;
    ls.strict = true;
    ls.added = 0;
    ls.quiet = false;
  }
  return true;
}

// Loads n composites from a partial list in global memory into sm.cache[at ...].
__device__ __forceinline__ void load_list(const unsigned long long* src, uint32_t n,
                                          LargeScratch& sm, uint32_t at) {
  for (uint32_t i = threadIdx.x; i < n; i += kThreads) sm.cache[at + i] = __ldcg(src + i);
}

// End of this block's part of segment ls.s: write the row, or publish the part's top k and,
// if this block finishes the segment, merge all parts in index order.
__device__ void large_close(const TopkParams& p, LargeState& ls, LargeScratch& sm) {
  if (ls.mycnt == 0) return;
  constexpr uint32_t C = Cfg<true>::kCacheCap;
  const uint32_t k = static_cast<uint32_t>(p.k);
  const long long len = ls.a1 - ls.a0;
  if (ls.mycnt == ls.nchunks) {
    CacheSrc cs{sm.cache};
    select_and_emit<true>(p, cs, ls.nbuf, 0xFFFFu, ls.s, len, sm);
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
  // last to arrive: every part's list, in slot (= index) order
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
      n += cj;
      csync();
    }
    csync();  // tbase is rewritten by the next round
  }
  CacheSrc cs{sm.cache};
  select_and_emit<true>(p, cs, n, 0xFFFFu, ls.s, len, sm);
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
      if (!large_chunk(p, si, buf, sm, ls, par)) {
        failed = true;
        break;
      }
      ++ls.mycnt;
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
