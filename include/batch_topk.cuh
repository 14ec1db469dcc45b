// batch_topk.cuh -- C++ drop-in for fire-emblem/batch_topk's operator header.
//
// Keeps the reference's names and signatures (include/batch_topk.cuh:10-21 of the reference:
// radix_topk::batch_topk_half and radix_topk::batch_topk_half_workspace_size) so its host
// callers recompile unchanged and link against libbatch_topk_b200.so instead.  Each function
// forwards to the C ABI in batch_topk_b200.h; nothing here computes.
//
// Deliberate differences from the reference (documented in batch_topk_b200.h): seg_len up to
// BT_MAX_SEG_LEN instead of 10000, k up to BT_MAX_K instead of 128.
#pragma once

#include <cstddef>

#include <cuda_fp16.h>
#include <cuda_runtime_api.h>

#include "batch_topk_b200.h"

namespace radix_topk {

inline cudaError_t batch_topk_half(const half* d_input, int seg_num, int seg_len, int k,
                                   half* d_output_values, int* d_output_indices,
                                   void* d_workspace, size_t workspace_bytes,
                                   cudaStream_t stream) {
  return static_cast<cudaError_t>(bt_topk_half(d_input, seg_num, seg_len, k, d_output_values,
                                               d_output_indices, d_workspace, workspace_bytes,
                                               static_cast<void*>(stream)));
}

inline size_t batch_topk_half_workspace_size(int seg_num, int seg_len, int k) {
  return bt_topk_half_workspace_size(seg_num, seg_len, k);
}

// Variable-length batch (no reference counterpart): segment s is
// d_input[d_offsets[s] .. d_offsets[s+1]) with d_offsets on the device.
inline cudaError_t batch_topk_half_segmented(const half* d_input, const int* d_offsets,
                                             int seg_num, long long max_total_len, int k,
                                             half* d_output_values, int* d_output_indices,
                                             void* d_workspace, size_t workspace_bytes,
                                             cudaStream_t stream) {
  return static_cast<cudaError_t>(bt_topk_half_segmented(
      d_input, d_offsets, seg_num, max_total_len, k, d_output_values, d_output_indices,
      d_workspace, workspace_bytes, static_cast<void*>(stream)));
}

inline size_t batch_topk_half_segmented_workspace_size(int seg_num, long long max_total_len,
                                                       int k) {
  return bt_topk_half_segmented_workspace_size(seg_num, max_total_len, k);
}

}  // namespace radix_topk
