/*
 * batch_topk_b200.h -- C ABI of the B200 batched fp16 top-k engine.
 *
 * Semantics follow fire-emblem/batch_topk (the reference):
 *   - For each segment, return the top-k values and their segment-local int32 indices.
 *   - Order: values descending; equal values go to the LOWER index; every NaN ranks below
 *     every number, -inf included, and NaNs tie among themselves by index; -0 == +0.
 *     (include/batch_topk_types.cuh:50-92 cpu_reference_topk, :100-113 candidate_better,
 *      include/type_codec.cuh:13-38.)
 *   - Output values are the input's own fp16 bit patterns at the returned indices.
 *   - Outputs are row-major [seg_num, k].  All calls are asynchronous on `stream`; the
 *     caller owns every buffer.  The workspace needs no initialisation.
 *
 * Return values are cudaError_t codes (0 = cudaSuccess, 1 = cudaErrorInvalidValue).
 * fp16 data is passed as `const void*` (IEEE binary16 bit patterns); `stream` is a
 * cudaStream_t (NULL = legacy default stream).
 *
 * Differences from the reference's limits (deliberate):
 *   - seg_len up to BT_MAX_SEG_LEN (the reference stops at 10000);
 *   - k up to BT_MAX_K (the reference stops at 128);
 *   - a CSR (segment-offsets) entry point, which the reference does not have; on it a
 *     segment shorter than k is valid: its first len slots hold the result and the rest
 *     hold value 0xFC00 (-inf) and index -1.
 */
#ifndef BATCH_TOPK_B200_H_
#define BATCH_TOPK_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BT_MAX_K 1024
#define BT_MAX_SEG_LEN (1 << 26)

/* Replaces radix_topk::batch_topk_half (include/batch_topk.cuh:10-19).  Same arguments and
 * error contract: cudaErrorInvalidValue for seg_num <= 0, seg_len <= 0, k <= 0, k > seg_len,
 * k > BT_MAX_K, seg_len > BT_MAX_SEG_LEN, a NULL pointer, or workspace_bytes below
 * bt_topk_half_workspace_size(seg_num, seg_len, k).  Launch errors are returned as is. */
int bt_topk_half(const void* d_input, int seg_num, int seg_len, int k, void* d_output_values,
                 int* d_output_indices, void* d_workspace, size_t workspace_bytes, void* stream);

/* Replaces radix_topk::batch_topk_half_workspace_size (include/batch_topk.cuh:21).
 * Returns 0 for an unsupported shape, as the reference does (src/batch_topk.cu:35-40). */
size_t bt_topk_half_workspace_size(int seg_num, int seg_len, int k);

/* Variable-length (CSR) batch; no reference counterpart (the reference is fixed-length only,
 * include/batch_topk.cuh:10-19).  Segment s is d_input[d_offsets[s] .. d_offsets[s+1]);
 * d_offsets holds seg_num+1 non-decreasing int32 element offsets on the device.
 * max_total_len bounds d_offsets[seg_num] - d_offsets[0] and sizes the workspace.
 * Segments shorter than k are valid (padding as described above). */
int bt_topk_half_segmented(const void* d_input, const int* d_offsets, int seg_num,
                           long long max_total_len, int k, void* d_output_values,
                           int* d_output_indices, void* d_workspace, size_t workspace_bytes,
                           void* stream);

size_t bt_topk_half_segmented_workspace_size(int seg_num, long long max_total_len, int k);

/* bfloat16 inputs; no reference counterpart (the reference is fp16 only and lists other types
 * as a non-goal).  The same arguments, layouts, limits, error contract and order as the fp16
 * entry points above, with values ordered as bfloat16: descending, equal values by lower
 * index, -0 equal to +0, NaN last.  Output values are the input's own bit patterns; a missing
 * entry of a short CSR segment is -inf (0xFF80) with index -1.  The workspace sizes are those
 * of the fp16 entry points. */
int bt_topk_bf16(const void* d_input, int seg_num, int seg_len, int k, void* d_output_values,
                 int* d_output_indices, void* d_workspace, size_t workspace_bytes, void* stream);

size_t bt_topk_bf16_workspace_size(int seg_num, int seg_len, int k);

int bt_topk_bf16_segmented(const void* d_input, const int* d_offsets, int seg_num,
                           long long max_total_len, int k, void* d_output_values,
                           int* d_output_indices, void* d_workspace, size_t workspace_bytes,
                           void* stream);

size_t bt_topk_bf16_segmented_workspace_size(int seg_num, long long max_total_len, int k);

/* float32 inputs; no reference counterpart (the reference is fp16 only and lists other types as
 * a non-goal).  The same arguments, layouts, limits, error contract and order as the fp16 entry
 * points, with float32 values and values out: d_input and d_output_values hold 32-bit bit
 * patterns and must be 4-byte aligned.  Order: descending, equal values (-0 == +0) by lower
 * index, every NaN last.  Output values are the input's own bit patterns; a missing entry of a
 * short CSR segment is -inf (0xFF800000) with index -1.  The workspace sizes are these
 * functions' own (a 16-byte vector holds 4 values here, not 8). */
int bt_topk_f32(const void* d_input, int seg_num, int seg_len, int k, void* d_output_values,
                int* d_output_indices, void* d_workspace, size_t workspace_bytes, void* stream);

size_t bt_topk_f32_workspace_size(int seg_num, int seg_len, int k);

int bt_topk_f32_segmented(const void* d_input, const int* d_offsets, int seg_num,
                          long long max_total_len, int k, void* d_output_values,
                          int* d_output_indices, void* d_workspace, size_t workspace_bytes,
                          void* stream);

size_t bt_topk_f32_segmented_workspace_size(int seg_num, long long max_total_len, int k);

/* bt_topk_half without a caller workspace; NO COUNTERPART IN THE REFERENCE, which always takes
 * a caller-allocated workspace (include/batch_topk.cuh:10-19).
 *
 * Meant for callers that may not allocate device memory at the moment they need a top-k:
 * code running inside a custom allocator or an out-of-memory handler (allocating there
 * re-enters the allocator or fails outright), and hosts whose device-memory budget is fixed
 * up front and accounted by someone else, such as an inference server that hands each plugin
 * a pre-sized pool.  The call allocates nothing: its scratch is a fixed array of
 * BT_NOALLOC_SCRATCH_BYTES in this library's device image, and the kernels reset the parts of
 * it that must start at zero on every call.
 *
 * Limit: calls whose bt_topk_half_workspace_size(seg_num, seg_len, k) exceeds
 * BT_NOALLOC_SCRATCH_BYTES (or is 0, an unsupported shape) return cudaErrorInvalidValue and
 * launch nothing; use bt_topk_half with a workspace for those.  Other arguments and results
 * are those of bt_topk_half.
 *
 * Set-up: the first call on each device (the current one) looks up the array's device
 * address and the kernels' launch attributes; make that first call before beginning any
 * stream capture on that device.  Later calls only launch.
 *
 * Concurrency: every call on a device shares the one array, so calls that can overlap on the
 * GPU (different streams without ordering between them, or several host threads) race on it
 * and give wrong results.  Serialise them, e.g. on a single stream. */
#define BT_NOALLOC_SCRATCH_BYTES (32u << 20)
int bt_topk_half_noalloc(const void* d_input, int seg_num, int seg_len, int k,
                         void* d_output_values, int* d_output_indices, void* stream);

/* Reads back (synchronously, on `stream`) the device status word of the last call that used
 * this workspace: 0 when every device-side check passed, otherwise a bitwise OR of
 * BT_STATUS_* flags.  stats (may be NULL) receives BT_STATS_WORDS counters, filled only when
 * the process runs with BT_STATS=1: chunks that needed the exact local select, chunks with no
 * candidate, group-max threshold selects, rows emitted, first chunks whose threshold was the
 * previous segment's (verified), and one reserved word. */
#define BT_STATS_WORDS 6
#define BT_STATUS_OK 0
#define BT_STATUS_WAIT_TIMEOUT 1    /* a bounded wait (bulk copy, hand-off) hit its cap */
#define BT_STATUS_BAD_OFFSETS 2     /* CSR offsets decreasing or beyond max_total_len */
#define BT_STATUS_SEGMENT_TOO_LONG 4
#define BT_STATUS_CERTIFY_FAILED 8  /* fewer candidates than the threshold certified */
int bt_workspace_status(const void* d_workspace, int seg_num, void* stream, unsigned* stats);

/* bt_workspace_status for the no-allocation entry point: reads back (synchronously, on
 * `stream`) the status word and counters of the last bt_topk_half_noalloc call on the current
 * device, from the library's fixed scratch array.  No reference counterpart (the reference
 * reports device-side problems only through cudaGetLastError, src/batch_topk.cu:85-193).
 * Allocates nothing.  Returns the BT_STATUS_* flags, or a negated cudaError_t code. */
int bt_noalloc_status(void* stream, unsigned* stats);

/* Logits producer with the top-k fused into its epilogue; no reference counterpart (the
 * reference selects from logits already in memory, include/batch_topk.cuh:10-19).
 *
 * logits[M, V] = hidden[M, D] . weight[V, D]^T: fp16 inputs (row-major, 16-byte aligned),
 * fp32 accumulation on the tensor cores, rounded to fp16 (round to nearest even) -- the values
 * a GEMM that stores fp16 logits produces.  1 <= M <= 128, V >= 1, D >= 8 with D % 8 == 0.
 *
 * bt_logits_f16 stores the logits, row-major [M, V] (2-byte aligned).
 *
 * bt_logits_topk_f16 returns, per row, the top k of those logits with the order and output
 * layout of bt_topk_half (values descending, equal values by lower vocabulary index, NaN last;
 * values are the fp16 logits' bit patterns, indices are vocabulary rows), without writing the
 * logits to memory.  1 <= k <= min(BT_LOGITS_MAX_K, V).  The workspace (256-byte aligned) holds
 * each CTA's per-row candidate lists and the second stage's scratch; its size comes from
 * bt_logits_topk_f16_workspace_size (0: unsupported shape).  The results equal bt_topk_half
 * applied to bt_logits_f16's output, bit for bit.
 *
 * bt_logits_topk_status reads back (synchronously) the status of the last call on a workspace:
 * BT_STATUS_* flags, or a negated cudaError_t code. */
#define BT_LOGITS_MAX_K 64
int bt_logits_f16(const void* d_hidden, const void* d_weight, int M, int V, int D,
                  void* d_logits, void* stream);

size_t bt_logits_topk_f16_workspace_size(int M, int V, int D, int k);

int bt_logits_topk_f16(const void* d_hidden, const void* d_weight, int M, int V, int D, int k,
                       void* d_out_values, int* d_out_indices, void* d_workspace,
                       size_t workspace_bytes, void* stream);

int bt_logits_topk_status(const void* d_workspace, int M, int V, int D, int k, void* stream);

/* Failure-path test hook (no reference counterpart): the number of tries each consumer <->
 * merger hand-off wait of the k <= 128 kernel makes before it gives up, for calls launched
 * after this one, process-wide.  0 makes those waits fail at once, so a call ends early with
 * BT_STATUS_WAIT_TIMEOUT set and its outputs undefined; a negative value restores the default
 * (about a second of waiting).  The waits for bulk copies already in flight are never
 * shortened.  Not for concurrent callers. */
void bt_set_handoff_wait_tries(int tries);

/* Optional timing hook: when both are non-NULL cudaEvent_t handles, every later call records
 * ev_start just before its main (streaming) kernel and ev_stop just after it, on the call's
 * stream.  Pass NULLs to switch it off.  Process-wide; not for concurrent callers. */
void bt_set_profile_events(void* ev_start, void* ev_stop);

/* Launch facts for the current device (initialises the per-device set-up on first use):
 * info[0..5] = {SM count, resident blocks per SM for k <= 128, for k > 128, dynamic shared
 * memory bytes per block for k <= 128, for k > 128, threads per block}.  Writes min(n, 6)
 * entries; returns a cudaError_t code. */
int bt_device_info(int* info, int n);

/* Human-readable text for a return code or status flag set. */
const char* bt_error_string(int code);

/* Library version, major * 10000 + minor * 100 + patch. */
int bt_version(void);

#ifdef __cplusplus
}
#endif

#endif /* BATCH_TOPK_B200_H_ */
