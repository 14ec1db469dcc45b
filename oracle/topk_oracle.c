/*
 * topk_oracle.c -- CPU restatement of the reference's batched fp16 top-k.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.  The
 * product library never links or calls it.
 *
 * What it restates (paths are inside the fire-emblem/batch_topk project):
 *   - include/type_codec.cuh:13-23   normalize_half_bits (any NaN -> 0xFFFF, +-0 -> 0x0000)
 *   - include/type_codec.cuh:25-38   encode_half_asc / encode_half_desc (desc = ~asc)
 *   - include/batch_topk_types.cuh:50-92  cpu_reference_topk: stable sort of the index
 *     permutation by (NaN last, larger float first, lower index first), then the first
 *     min(k, len) entries.
 *   - src/radix_select_state.cuh:9-51     simulate_radix_boundary (high-byte select state)
 *   - src/radix_histogram.cuh:158-186     histogram_pass_kernel (digit histogram with prefix mask)
 *   - src/radix_boundary_select.cuh:9-78  boundary select + cutoff finalisation state
 *
 * Two top-k methods give identical output:
 *   method 0 ("sort")  : merge sort of the index permutation with the reference comparator,
 *                        written on float values exactly as the reference does.
 *   method 1 ("count") : two 8-bit counting passes over the descending key, then the
 *                        ordered collection of keys below the cutoff plus the first ties
 *                        by index, then a sort of those <= k entries.  Key order equals the
 *                        comparator's order (the codec is a bijection on values with -0==+0
 *                        and all NaNs equal), so this is the same total order, in O(n).
 *
 * Short segments (len < k) produce len entries; the batch drivers pad the rest of the row
 * with value 0xFC00 (-inf) and index -1.
 *
 * bfloat16 rows (the *_bf16 drivers): the reference has no bf16 path (other input types are
 * a listed non-goal), so this restates the same comparator on bfloat16 values converted
 * exactly to float, and the same descending key with bfloat16's NaN test (exponent field
 * 0x7F80); padding is bfloat16 -inf, 0xFF80.
 *
 * float32 rows (the *_f32 drivers, 32-bit bit patterns): likewise no reference path; the same
 * comparator on the float values themselves, and for the count method a 32-bit descending key
 * (any NaN -> 0xFFFFFFFF, +-0 -> 0x7FFFFFFF, else bits ^ (sign ? 0 : 0x7FFFFFFF)) selected with
 * four 8-bit counting passes; padding is float32 -inf, 0xFF800000.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- codec: include/type_codec.cuh:13-38 ---------------------------------------- */

uint16_t oracle_normalize_half_bits(uint16_t bits) {
  if ((bits & 0x7c00u) == 0x7c00u && (bits & 0x03ffu) != 0) return 0xffffu; /* any NaN */
  if ((bits & 0x7fffu) == 0) return 0x0000u;                                 /* +-0 */
  return bits;
}

uint16_t oracle_encode_asc(uint16_t raw) {
  const uint16_t bits = oracle_normalize_half_bits(raw);
  return (bits & 0x8000u) ? (uint16_t)~bits : (uint16_t)(bits ^ 0x8000u);
}

uint16_t oracle_encode_desc(uint16_t raw) { return (uint16_t)~oracle_encode_asc(raw); }

/* bfloat16: the same sign-magnitude codec with an 8-bit exponent field. */
uint16_t oracle_encode_desc_bf16(uint16_t raw) {
  uint16_t bits = raw;
  if ((bits & 0x7fffu) > 0x7f80u) bits = 0xffffu; /* any NaN */
  else if ((bits & 0x7fffu) == 0) bits = 0x0000u; /* +-0 */
  const uint16_t asc = (bits & 0x8000u) ? (uint16_t)~bits : (uint16_t)(bits ^ 0x8000u);
  return (uint16_t)~asc;
}

/* Exact bfloat16 -> fp32 conversion (bfloat16 is the top half of an fp32). */
float oracle_bf16_to_float(uint16_t b) {
  const uint32_t f = (uint32_t)b << 16;
  float out;
  memcpy(&out, &f, sizeof(out));
  return out;
}

/* Exact fp16 -> fp32 conversion (every fp16 value is representable in fp32). */
float oracle_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t f;
  if (exp == 0) {
    if (man == 0) {
      f = sign;
    } else {
      int shift = 0;
      while (!(man & 0x400u)) {
        man <<= 1;
        ++shift;
      }
      man &= 0x3ffu;
      f = sign | ((uint32_t)(113 - shift) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    f = sign | 0x7f800000u | (man << 13);
  } else {
    f = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float out;
  memcpy(&out, &f, sizeof(out));
  return out;
}

/* ---- comparator: include/batch_topk_types.cuh:70-81 ------------------------------ */

/* Returns nonzero when element lhs ranks strictly before rhs. */
static int ref_before(const float* v, int lhs, int rhs) {
  const float a = v[lhs], b = v[rhs];
  const int an = isnan(a), bn = isnan(b);
  if (an != bn) return bn;
  if (!an && a != b) return a > b;
  return lhs < rhs;
}

static void merge_sort_idx(const float* v, int* idx, int* tmp, int n) {
  /* bottom-up merge sort; stable, but the comparator is a total order anyway */
  for (int width = 1; width < n; width *= 2) {
    for (int lo = 0; lo < n; lo += 2 * width) {
      int mid = lo + width < n ? lo + width : n;
      int hi = lo + 2 * width < n ? lo + 2 * width : n;
      int i = lo, j = mid, o = lo;
      while (i < mid && j < hi) tmp[o++] = ref_before(v, idx[j], idx[i]) ? idx[j++] : idx[i++];
      while (i < mid) tmp[o++] = idx[i++];
      while (j < hi) tmp[o++] = idx[j++];
    }
    memcpy(idx, tmp, sizeof(int) * (size_t)n);
  }
}

/* method 0: the reference's algorithm (sort whole permutation, take min(k,len)). */
static int topk_sort_segment(const uint16_t* in, int len, int k, uint16_t* out_v, int32_t* out_i,
                             int bf16) {
  if (len <= 0 || k <= 0) return 0;
  float* v = (float*)malloc(sizeof(float) * (size_t)len);
  int* idx = (int*)malloc(sizeof(int) * (size_t)len);
  int* tmp = (int*)malloc(sizeof(int) * (size_t)len);
  for (int i = 0; i < len; ++i) {
    v[i] = bf16 ? oracle_bf16_to_float(in[i]) : oracle_half_to_float(in[i]);
    idx[i] = i;
  }
  merge_sort_idx(v, idx, tmp, len);
  const int kk = k < len ? k : len;
  for (int r = 0; r < kk; ++r) {
    out_i[r] = idx[r];
    out_v[r] = in[idx[r]];
  }
  free(v);
  free(idx);
  free(tmp);
  return kk;
}

/* method 1: counting select on the descending key (same total order, O(n)). */
static int cmp_key_idx(const void* a, const void* b) {
  const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return x < y ? -1 : (x > y ? 1 : 0);
}

static int topk_count_segment(const uint16_t* in, int len, int k, uint16_t* out_v, int32_t* out_i,
                              int bf16) {
  if (len <= 0 || k <= 0) return 0;
  uint16_t (*encode)(uint16_t) = bf16 ? oracle_encode_desc_bf16 : oracle_encode_desc;
  const int kk = k < len ? k : len;
  uint32_t h1[256], h2[256];
  memset(h1, 0, sizeof(h1));
  memset(h2, 0, sizeof(h2));
  for (int i = 0; i < len; ++i) ++h1[encode(in[i]) >> 8];
  uint32_t cum = 0;
  int b1 = 0;
  for (; b1 < 256; ++b1) {
    if (cum + h1[b1] >= (uint32_t)kk) break;
    cum += h1[b1];
  }
  for (int i = 0; i < len; ++i) {
    const uint16_t key = encode(in[i]);
    if ((key >> 8) == b1) ++h2[key & 0xffu];
  }
  int b2 = 0;
  for (; b2 < 256; ++b2) {
    if (cum + h2[b2] >= (uint32_t)kk) break;
    cum += h2[b2];
  }
  const uint16_t cutoff = (uint16_t)((b1 << 8) | b2);
  int need = kk - (int)cum; /* ties at the cutoff that make it, lowest index first */
  uint64_t* sel = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)kk);
  int n = 0;
  for (int i = 0; i < len; ++i) {
    const uint16_t key = encode(in[i]);
    if (key < cutoff || (key == cutoff && need > 0)) {
      if (key == cutoff) --need;
      sel[n++] = ((uint64_t)key << 32) | (uint32_t)i;
    }
  }
  qsort(sel, (size_t)n, sizeof(uint64_t), cmp_key_idx);
  for (int r = 0; r < n; ++r) {
    const int i = (int)(uint32_t)sel[r];
    out_i[r] = i;
    out_v[r] = in[i];
  }
  free(sel);
  return n;
}

static int topk_segment(const uint16_t* in, int len, int k, uint16_t* out_v, int32_t* out_i,
                        int method, int bf16) {
  return method == 0 ? topk_sort_segment(in, len, k, out_v, out_i, bf16)
                     : topk_count_segment(in, len, k, out_v, out_i, bf16);
}

int oracle_topk_segment(const uint16_t* in, int len, int k, uint16_t* out_v, int32_t* out_i,
                        int method) {
  return topk_segment(in, len, k, out_v, out_i, method, 0);
}

/* ---- batch drivers (fixed-length rows and CSR offsets), threaded ------------------ */

typedef struct {
  const uint16_t* in;
  const int64_t* offsets; /* CSR: seg_num+1 element offsets; NULL for fixed length */
  int64_t seg_len;
  int k;
  int method;
  int bf16;
  uint16_t* out_v;
  int32_t* out_i;
  int64_t seg_begin, seg_end;
} job_t;

static void* run_job(void* arg) {
  job_t* j = (job_t*)arg;
  for (int64_t s = j->seg_begin; s < j->seg_end; ++s) {
    int64_t start, len;
    if (j->offsets) {
      start = j->offsets[s];
      len = j->offsets[s + 1] - j->offsets[s];
    } else {
      start = s * j->seg_len;
      len = j->seg_len;
    }
    uint16_t* ov = j->out_v + s * (int64_t)j->k;
    int32_t* oi = j->out_i + s * (int64_t)j->k;
    int n = topk_segment(j->in + start, (int)len, j->k, ov, oi, j->method, j->bf16);
    for (int r = n; r < j->k; ++r) {
      ov[r] = j->bf16 ? 0xff80u : 0xfc00u;
      oi[r] = -1;
    }
  }
  return NULL;
}

static int run_batch(const uint16_t* in, const int64_t* offsets, int64_t seg_num, int64_t seg_len,
                     int k, uint16_t* out_v, int32_t* out_i, int method, int threads, int bf16) {
  if (seg_num <= 0 || k <= 0) return -1;
  if (threads < 1) threads = 1;
  if (threads > seg_num) threads = (int)seg_num;
  pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  job_t* jobs = (job_t*)malloc(sizeof(job_t) * (size_t)threads);
  for (int t = 0; t < threads; ++t) {
    jobs[t].in = in;
    jobs[t].offsets = offsets;
    jobs[t].seg_len = seg_len;
    jobs[t].k = k;
    jobs[t].method = method;
    jobs[t].bf16 = bf16;
    jobs[t].out_v = out_v;
    jobs[t].out_i = out_i;
    jobs[t].seg_begin = seg_num * t / threads;
    jobs[t].seg_end = seg_num * (t + 1) / threads;
    pthread_create(&tid[t], NULL, run_job, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
  free(tid);
  free(jobs);
  return 0;
}

int oracle_topk_batch(const uint16_t* in, int64_t seg_num, int64_t seg_len, int k, uint16_t* out_v,
                      int32_t* out_i, int method, int threads) {
  if (seg_len <= 0) return -1;
  return run_batch(in, NULL, seg_num, seg_len, k, out_v, out_i, method, threads, 0);
}

int oracle_topk_csr(const uint16_t* in, const int64_t* offsets, int64_t seg_num, int k,
                    uint16_t* out_v, int32_t* out_i, int method, int threads) {
  return run_batch(in, offsets, seg_num, 0, k, out_v, out_i, method, threads, 0);
}

int oracle_topk_batch_bf16(const uint16_t* in, int64_t seg_num, int64_t seg_len, int k,
                           uint16_t* out_v, int32_t* out_i, int method, int threads) {
  if (seg_len <= 0) return -1;
  return run_batch(in, NULL, seg_num, seg_len, k, out_v, out_i, method, threads, 1);
}

int oracle_topk_csr_bf16(const uint16_t* in, const int64_t* offsets, int64_t seg_num, int k,
                         uint16_t* out_v, int32_t* out_i, int method, int threads) {
  return run_batch(in, offsets, seg_num, 0, k, out_v, out_i, method, threads, 1);
}

/* ---- float32 rows ------------------------------------------------------------------ */

uint32_t oracle_encode_desc_f32(uint32_t bits) {
  if ((bits & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu; /* any NaN */
  if ((bits & 0x7fffffffu) == 0) return 0x7fffffffu;          /* +-0 */
  return (bits & 0x80000000u) ? bits : (bits ^ 0x7fffffffu);
}

static int topk_sort_segment_f32(const uint32_t* in, int len, int k, uint32_t* out_v,
                                 int32_t* out_i) {
  if (len <= 0 || k <= 0) return 0;
  float* v = (float*)malloc(sizeof(float) * (size_t)len);
  int* idx = (int*)malloc(sizeof(int) * (size_t)len);
  int* tmp = (int*)malloc(sizeof(int) * (size_t)len);
  memcpy(v, in, sizeof(float) * (size_t)len);
  for (int i = 0; i < len; ++i) idx[i] = i;
  merge_sort_idx(v, idx, tmp, len);
  const int kk = k < len ? k : len;
  for (int r = 0; r < kk; ++r) {
    out_i[r] = idx[r];
    out_v[r] = in[idx[r]];
  }
  free(v);
  free(idx);
  free(tmp);
  return kk;
}

static int topk_count_segment_f32(const uint32_t* in, int len, int k, uint32_t* out_v,
                                  int32_t* out_i) {
  if (len <= 0 || k <= 0) return 0;
  const int kk = k < len ? k : len;
  uint32_t h[256];
  uint32_t prefix = 0, cum = 0;
  for (int d = 3; d >= 0; --d) { /* most significant digit first */
    memset(h, 0, sizeof(h));
    const int sh = 8 * d;
    for (int i = 0; i < len; ++i) {
      const uint32_t key = oracle_encode_desc_f32(in[i]);
      if (d == 3 || (key >> (sh + 8)) == (prefix >> (sh + 8))) ++h[(key >> sh) & 0xffu];
    }
    int b = 0;
    for (; b < 256; ++b) {
      if (cum + h[b] >= (uint32_t)kk) break;
      cum += h[b];
    }
    prefix |= (uint32_t)b << sh;
  }
  const uint32_t cutoff = prefix;
  int need = kk - (int)cum; /* ties at the cutoff that make it, lowest index first */
  uint64_t* sel = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)kk);
  int n = 0;
  for (int i = 0; i < len; ++i) {
    const uint32_t key = oracle_encode_desc_f32(in[i]);
    if (key < cutoff || (key == cutoff && need > 0)) {
      if (key == cutoff) --need;
      sel[n++] = ((uint64_t)key << 32) | (uint32_t)i;
    }
  }
  qsort(sel, (size_t)n, sizeof(uint64_t), cmp_key_idx);
  for (int r = 0; r < n; ++r) {
    const int i = (int)(uint32_t)sel[r];
    out_i[r] = i;
    out_v[r] = in[i];
  }
  free(sel);
  return n;
}

typedef struct {
  const uint32_t* in;
  const int64_t* offsets;
  int64_t seg_len;
  int k;
  int method;
  uint32_t* out_v;
  int32_t* out_i;
  int64_t seg_begin, seg_end;
} job32_t;

static void* run_job_f32(void* arg) {
  job32_t* j = (job32_t*)arg;
  for (int64_t s = j->seg_begin; s < j->seg_end; ++s) {
    int64_t start, len;
    if (j->offsets) {
      start = j->offsets[s];
      len = j->offsets[s + 1] - j->offsets[s];
    } else {
      start = s * j->seg_len;
      len = j->seg_len;
    }
    uint32_t* ov = j->out_v + s * (int64_t)j->k;
    int32_t* oi = j->out_i + s * (int64_t)j->k;
    const int n = j->method == 0 ? topk_sort_segment_f32(j->in + start, (int)len, j->k, ov, oi)
                                 : topk_count_segment_f32(j->in + start, (int)len, j->k, ov, oi);
    for (int r = n; r < j->k; ++r) {
      ov[r] = 0xff800000u;
      oi[r] = -1;
    }
  }
  return NULL;
}

static int run_batch_f32(const uint32_t* in, const int64_t* offsets, int64_t seg_num,
                         int64_t seg_len, int k, uint32_t* out_v, int32_t* out_i, int method,
                         int threads) {
  if (seg_num <= 0 || k <= 0) return -1;
  if (threads < 1) threads = 1;
  if (threads > seg_num) threads = (int)seg_num;
  pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  job32_t* jobs = (job32_t*)malloc(sizeof(job32_t) * (size_t)threads);
  for (int t = 0; t < threads; ++t) {
    jobs[t].in = in;
    jobs[t].offsets = offsets;
    jobs[t].seg_len = seg_len;
    jobs[t].k = k;
    jobs[t].method = method;
    jobs[t].out_v = out_v;
    jobs[t].out_i = out_i;
    jobs[t].seg_begin = seg_num * t / threads;
    jobs[t].seg_end = seg_num * (t + 1) / threads;
    pthread_create(&tid[t], NULL, run_job_f32, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
  free(tid);
  free(jobs);
  return 0;
}

int oracle_topk_batch_f32(const uint32_t* in, int64_t seg_num, int64_t seg_len, int k,
                          uint32_t* out_v, int32_t* out_i, int method, int threads) {
  if (seg_len <= 0) return -1;
  return run_batch_f32(in, NULL, seg_num, seg_len, k, out_v, out_i, method, threads);
}

int oracle_topk_csr_f32(const uint32_t* in, const int64_t* offsets, int64_t seg_num, int k,
                        uint32_t* out_v, int32_t* out_i, int method, int threads) {
  return run_batch_f32(in, offsets, seg_num, 0, k, out_v, out_i, method, threads);
}

/* ---- select-state restatements, for the reference's known-answer tests ----------- */

/* src/radix_histogram.cuh:158-186: 256-bin count of (key >> shift) & 0xff over keys with
 * (key & prefix_mask) == prefix. */
void oracle_histogram_pass(const uint16_t* in, int len, int shift, uint16_t prefix,
                           uint16_t prefix_mask, uint32_t* hist256) {
  memset(hist256, 0, sizeof(uint32_t) * 256);
  for (int i = 0; i < len; ++i) {
    const uint16_t key = oracle_encode_desc(in[i]);
    if ((key & prefix_mask) == prefix) ++hist256[(key >> shift) & 0xffu];
  }
}

/* src/radix_boundary_select.cuh:9-78 (and src/radix_select_state.cuh:9-51 for the first
 * six fields): fills out[8] = {prefix, prefix_mask, cutoff_key, selected_count,
 * live_count, boundary_digit, strictly_better_count, remaining_slots}. */
void oracle_select_state(const uint16_t* in, int len, int k, int32_t* out) {
  uint32_t hi[256], lo[256];
  oracle_histogram_pass(in, len, 8, 0, 0, hi);
  int prefix = 0, prefix_mask = 0, cutoff = 0xffff, selected = 0, live = 0, digit = 0;
  int strictly_better = 0, remaining = 0;
  int found = 0;
  for (int b = 0; b < 256; ++b) {
    if (selected + (int)hi[b] < k) {
      selected += (int)hi[b];
      continue;
    }
    digit = b;
    prefix = b << 8;
    prefix_mask = 0xff00;
    live = (int)hi[b];
    found = 1;
    break;
  }
  if (!found) {
    prefix = 0xffff;
    prefix_mask = 0xffff;
    cutoff = 0xffff;
    live = 0;
    digit = 255;
    strictly_better = selected;
    remaining = k > selected ? k - selected : 0;
  }
  /* finalisation runs on the low-byte histogram of the boundary digit in both cases */
  oracle_histogram_pass(in, len, 0, (uint16_t)(digit << 8), 0xff00u, lo);
  int sel = selected;
  int done = 0;
  for (int b = 0; b < 256; ++b) {
    if (sel + (int)lo[b] < k) {
      sel += (int)lo[b];
      continue;
    }
    cutoff = (digit << 8) | b;
    strictly_better = sel;
    remaining = k - sel;
    done = 1;
    break;
  }
  if (!done) {
    cutoff = 0xffff;
    strictly_better = sel;
    remaining = k > sel ? k - sel : 0;
  }
  out[0] = prefix;
  out[1] = prefix_mask;
  out[2] = cutoff;
  out[3] = selected;
  out[4] = live;
  out[5] = digit;
  out[6] = strictly_better;
  out[7] = remaining;
}
