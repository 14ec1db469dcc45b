// ref_gpu.cu -- a C ABI over the reference's OWN GPU path, for a same-box timing comparison.
//
// TEST INFRASTRUCTURE ONLY, never part of the product.  oracle/Makefile compiles this file
// together with the reference's unmodified src/batch_topk.cu (fire-emblem/batch_topk), where
// the reference tree lies, into oracle/_ref/libref_gpu.so for sm_100a.  The two functions
// forward to radix_topk::batch_topk_half and radix_topk::batch_topk_half_workspace_size
// (reference include/batch_topk.cuh:10-21, src/batch_topk.cu:35-193) so a ctypes caller can
// time the reference's kernels on its own supported shapes (seg_len <= 10000, k <= 128; the
// tuned path at seg_len 10000, k 50) next to this library's entry point.
#include <cstddef>

#include "batch_topk.cuh"

extern "C" {

int ref_gpu_topk_half(const void* d_input, int seg_num, int seg_len, int k,
                      void* d_output_values, int* d_output_indices, void* d_workspace,
                      size_t workspace_bytes, void* stream) {
  return static_cast<int>(radix_topk::batch_topk_half(
      static_cast<const half*>(d_input), seg_num, seg_len, k, static_cast<half*>(d_output_values),
      d_output_indices, d_workspace, workspace_bytes, static_cast<cudaStream_t>(stream)));
}

size_t ref_gpu_workspace_size(int seg_num, int seg_len, int k) {
  return radix_topk::batch_topk_half_workspace_size(seg_num, seg_len, k);
}

}  // extern "C"
