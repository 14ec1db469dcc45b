// batch_topk.cu -- C ABI, argument validation, workspace layout and launch sequence.
//
// The public contract is the reference's radix_topk::batch_topk_half /
// batch_topk_half_workspace_size (include/batch_topk.cuh:10-21, src/batch_topk.cu:13-60 of
// fire-emblem/batch_topk): caller-owned buffers, cudaErrorInvalidValue on bad arguments,
// asynchronous on the caller's stream, no host synchronisation, no allocation.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "../../include/batch_topk_b200.h"
#include "bt_kernels.cuh"

namespace bt {
namespace {

constexpr int kVersion = 100;  // 0.1.0

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int groups_for_k(int k) { return k <= 64 ? 1 : (k <= 128 ? 2 : (k <= 256 ? 4 : 8)); }
int cap_for_k(int k) { return k * 4 < 256 ? 256 : k * 4; }

// Chunk slots one fixed-length segment may need: its 16-byte vectors (epv elements each) span
// at most ceil(len / epv) + 1 when the row start is not 16-byte aligned.
long long slots_per_segment(long long seg_len, int epv = 8) {
  const long long nv = (seg_len + epv - 1) / epv + 1;
  return (nv + kVecPerChunk - 1) / kVecPerChunk;
}

// Upper bound on chunk slots for a CSR batch of seg_num segments totalling total_len values.
long long csr_slot_bound(long long seg_num, long long total_len, int epv = 8) {
  return (total_len / epv + 2 * seg_num) / kVecPerChunk + seg_num + 1;
}

struct Layout {
  size_t status, thresh, done, next, chunk_start, part_start, counts, offs, cand, total;
};

// status | seg_thresh | seg_done | chunk_next | chunk_start, part_start (CSR) |
// chunk_count | chunk_off | candidates, each region 256-byte aligned.
Layout make_layout(long long seg_num, long long slots, int cap, bool csr) {
  Layout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  L.status = take(16 * sizeof(uint32_t));
  L.thresh = take(static_cast<size_t>(seg_num) * sizeof(uint32_t));
  L.done = take(static_cast<size_t>(seg_num) * sizeof(uint32_t));
  L.next = take(static_cast<size_t>(seg_num) * sizeof(uint32_t));
  L.chunk_start = csr ? take(static_cast<size_t>(seg_num + 1) * sizeof(uint32_t)) : 0;
  L.part_start = csr ? take(static_cast<size_t>(seg_num + 1) * sizeof(uint32_t)) : 0;
  L.counts = take(static_cast<size_t>(slots) * sizeof(uint32_t));
  L.offs = take(static_cast<size_t>(slots + 1) * sizeof(uint32_t));
  L.cand = take(static_cast<size_t>(slots) * cap * sizeof(uint32_t));
  L.total = off;
  return L;
}

bool fixed_shape_ok(int seg_num, int seg_len, int k) {
  return seg_num > 0 && seg_len > 0 && k > 0 && k <= kMaxK && k <= seg_len &&
         static_cast<long long>(seg_len) <= BT_MAX_SEG_LEN;
}

bool csr_shape_ok(int seg_num, long long max_total_len, int k) {
  return seg_num > 0 && k > 0 && k <= kMaxK && max_total_len >= 0 &&
         max_total_len < (1ll << 31);
}

using TopkKernel = void (*)(TopkParams);

// Element types of the entry points: IEEE binary16, bfloat16, binary32.
enum Elem { kF16 = 0, kBF16 = 1, kF32 = 2 };

// The streaming kernel for k <= 128 (small) or larger k, per 16-bit element type.
TopkKernel topk_kernel_for(bool big, bool bf16) {
  if (bf16) return big ? bf16::topk_kernel<true> : bf16::topk_kernel<false>;
  return big ? f16::topk_kernel<true> : f16::topk_kernel<false>;
}

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int blocks_per_sm[3] = {0, 0, 0};  // topk_kernel<false>, topk_kernel<true>, f32::topk_kernel
};

std::mutex g_mu;
DeviceInfo g_dev[64];
cudaEvent_t g_prof_start = nullptr, g_prof_stop = nullptr;
int g_stats = -1;
int g_steal_env = -1;        // BT_STEAL: 0 turns helping off
uint32_t g_handoff_tries = kWaitCap;  // bt_set_handoff_wait_tries (failure-path tests)

// Chunks per work part.  With at least as many segments as resident blocks every block is
// busy with whole segments, and a segment is never split: each extra part costs its own
// first-chunk threshold and a cross-block merge of partial lists.  With fewer segments,
// about one part per block.
int choose_part_chunks(long long total_chunks, long long seg_num, long long resident) {
  if (seg_num >= resident) return kMaxChunksPerSegment;
  long long u = (total_chunks + resident - 1) / resident;
  if (u < 1) u = 1;
  if (u > kMaxChunksPerSegment) u = kMaxChunksPerSegment;
  return static_cast<int>(u);
}

cudaError_t device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    // Both element types' kernels: the shared-memory opt-in, and the smaller occupancy of the
    // two (the same code shape, so in practice the same number).
    for (int big = 0; big < 2; ++big) {
      const size_t smem = big ? SmemLayout<true>::bytes : SmemLayout<false>::bytes;
      const int threads = big ? block_threads<true>() : block_threads<false>();
      int best = 1 << 30;
      for (int bf = 0; bf < 2; ++bf) {
        const TopkKernel kern = topk_kernel_for(big != 0, bf != 0);
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        int n = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem);
        if (e != cudaSuccess) return e;
        best = n < best ? n : best;
      }
      d.blocks_per_sm[big] = best;
    }
    e = cudaFuncSetAttribute(f32::topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(f32::FLayout::bytes));
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.blocks_per_sm[2], f32::topk_kernel,
                                                      f32::kBlockThreads, f32::FLayout::bytes);
    if (e != cudaSuccess) return e;
    if (d.blocks_per_sm[0] < 1 || d.blocks_per_sm[1] < 1 || d.blocks_per_sm[2] < 1) {
      return cudaErrorInvalidConfiguration;
    }
    if (g_stats < 0) {
      const char* s = std::getenv("BT_STATS");
      g_stats = (s && s[0] == '1') ? 1 : 0;
    }
    if (g_steal_env < 0) {
      const char* s = std::getenv("BT_STEAL");
      g_steal_env = s ? std::atoi(s) : 1;
    }
    d.ready = true;
  }
  *out = d;
  return cudaSuccess;
}

// The streaming kernel with programmatic stream serialisation: its prologue overlaps the
// set-up kernel, which it waits for (grid_dep_wait) before touching the workspace.
// The set-up kernels are launched with programmatic stream serialisation as well: behind the
// previous call's streaming kernel (which lets dependents launch early) their blocks are placed
// while it drains, and each waits (griddepcontrol.wait) for the preceding grid to complete
// before touching the workspace.  Behind any other kernel this is plain stream order.
cudaError_t launch_setup(void (*kernel)(TopkParams), const TopkParams& p, int grid, int threads,
                         cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

cudaError_t launch_topk(TopkKernel kernel, int threads, size_t smem, const TopkParams& p,
                        int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

cudaError_t launch_pipeline(TopkParams p, bool csr, long long work_items, Elem elem,
                            cudaStream_t stream) {
  DeviceInfo di;
  cudaError_t e = device_info(&di);
  if (e != cudaSuccess) return e;
  p.stats = g_stats > 0 ? 1 : 0;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    p.handoff_tries = g_handoff_tries;
  }
  // fp32 rows always take the cache kernel; 16-bit rows the merger kernel up to k = 128
  const bool f32 = elem == kF32;
  const bool big = f32 || p.k > Cfg<false>::kSelCap;
  const int kind = f32 ? 2 : (big ? 1 : 0);
  const long long resident = static_cast<long long>(di.sms) * di.blocks_per_sm[kind];
  p.part_chunks = choose_part_chunks(work_items, p.seg_num, resident);
  long long parts = work_items;  // CSR: an upper bound (every part holds a chunk)
  // CSR parts are whole segments when there are at least as many segments as resident blocks
  bool whole = p.part_chunks == kMaxChunksPerSegment;
  if (!csr) {
    const long long per = (p.p_max + p.part_chunks - 1) / p.part_chunks;
    p.parts_total = static_cast<long long>(p.seg_num) * per;
    parts = p.parts_total;
    whole = per == 1;
  }
  // Whole segments: claim chunk by chunk and let blocks that run dry help (BT_STEAL=0: off).
  // 16-bit inputs: for k > 128 a helper's first chunk (a select, often an exact select)
  // costs more, so it joins only segments with more chunks left.  With whole segments the
  // grid never exceeds the segments.
  p.steal = (!f32 && whole && g_steal_env != 0) ? 1 : 0;
  p.help_min = big ? kHelpMinChunksBig : kHelpMinChunks;
  if (csr) {
    e = launch_setup(csr_prep_kernel, p, 1, 1024, stream);
  } else {
    e = launch_setup(init_kernel, p, static_cast<int>((p.seg_num + 255) / 256), 256, stream);
  }
  if (e != cudaSuccess) return e;
  long long grid_ll = parts < resident ? (parts > 0 ? parts : 1) : resident;
  const int grid = static_cast<int>(grid_ll);
  p.help_window = p.steal ? (grid < p.seg_num ? grid : p.seg_num) : 0;
  if (g_prof_start) cudaEventRecord(g_prof_start, stream);
  if (f32) {
    e = launch_topk(f32::topk_kernel, f32::kBlockThreads, f32::FLayout::bytes, p, grid, stream);
  } else if (big) {
    e = launch_topk(topk_kernel_for(true, elem == kBF16), block_threads<true>(),
                    SmemLayout<true>::bytes, p, grid, stream);
  } else {
    e = launch_topk(topk_kernel_for(false, elem == kBF16), block_threads<false>(),
                    SmemLayout<false>::bytes, p, grid, stream);
  }
  if (e != cudaSuccess) return e;
  if (g_prof_stop) cudaEventRecord(g_prof_stop, stream);
  return cudaSuccess;
}

// Elements per 16-byte vector.
int epv_of(Elem elem) { return elem == kF32 ? 4 : 8; }

TopkParams base_params(const void* d_input, int seg_num, int k, void* d_out_values,
                       int* d_out_indices, void* d_workspace, const Layout& L, long long slots,
                       Elem elem) {
  TopkParams p{};
  p.pad_bits = elem == kF32 ? 0xFF800000u : (elem == kBF16 ? 0xFF80u : 0xFC00u);  // -inf
  p.epv_shift = elem == kF32 ? 2 : 3;
  const uintptr_t in = reinterpret_cast<uintptr_t>(d_input);
  p.base = reinterpret_cast<const uint16_t*>(in & ~static_cast<uintptr_t>(15));
  p.shift = static_cast<int>((in & 15) / (elem == kF32 ? 4 : 2));
  p.seg_num = seg_num;
  p.k = k;
  p.groups = groups_for_k(k);
  p.cap = cap_for_k(k);
  p.slot_capacity = slots;
  uint8_t* ws = static_cast<uint8_t*>(d_workspace);
  p.status = reinterpret_cast<uint32_t*>(ws + L.status);
  p.seg_thresh = reinterpret_cast<uint32_t*>(ws + L.thresh);
  p.seg_done = reinterpret_cast<uint32_t*>(ws + L.done);
  p.chunk_next = reinterpret_cast<uint32_t*>(ws + L.next);
  p.chunk_start = reinterpret_cast<uint32_t*>(ws + L.chunk_start);
  p.part_start = reinterpret_cast<uint32_t*>(ws + L.part_start);
  p.chunk_count = reinterpret_cast<uint32_t*>(ws + L.counts);
  p.chunk_off = reinterpret_cast<uint32_t*>(ws + L.offs);
  p.cand = reinterpret_cast<uint32_t*>(ws + L.cand);
  p.out_values = elem == kF32 ? nullptr : static_cast<uint16_t*>(d_out_values);
  p.out_values32 = elem == kF32 ? static_cast<uint32_t*>(d_out_values) : nullptr;
  p.out_indices = d_out_indices;
  return p;
}

bool pointers_ok(const void* in, const void* ov, const int* oi, const void* ws, Elem elem) {
  if (!in || !ov || !oi || !ws) return false;
  const uintptr_t a = reinterpret_cast<uintptr_t>(in), b = reinterpret_cast<uintptr_t>(ov),
                  c = reinterpret_cast<uintptr_t>(oi), d = reinterpret_cast<uintptr_t>(ws);
  const uintptr_t es = elem == kF32 ? 4 : 2;  // element size: values must be element-aligned
  return (a % es == 0) && (b % es == 0) && (c % 4 == 0) && (d % 16 == 0);
}

size_t fixed_workspace(int seg_num, int seg_len, int k, Elem elem) {
  if (!fixed_shape_ok(seg_num, seg_len, k)) return 0;
  const long long slots =
      static_cast<long long>(seg_num) * slots_per_segment(seg_len, epv_of(elem));
  return make_layout(seg_num, slots, cap_for_k(k), false).total;
}

size_t csr_workspace(int seg_num, long long max_total_len, int k, Elem elem) {
  if (!csr_shape_ok(seg_num, max_total_len, k)) return 0;
  const long long slots = csr_slot_bound(seg_num, max_total_len, epv_of(elem));
  return make_layout(seg_num, slots, cap_for_k(k), true).total;
}

// Fixed-length rows of one element type.
int topk_fixed(const void* d_input, int seg_num, int seg_len, int k, void* d_output_values,
               int* d_output_indices, void* d_workspace, size_t workspace_bytes, void* stream,
               Elem elem) {
  if (!fixed_shape_ok(seg_num, seg_len, k)) return cudaErrorInvalidValue;
  if (!pointers_ok(d_input, d_output_values, d_output_indices, d_workspace, elem)) {
    return cudaErrorInvalidValue;
  }
  const long long p_max = slots_per_segment(seg_len, epv_of(elem));
  const long long slots = static_cast<long long>(seg_num) * p_max;
  const Layout L = make_layout(seg_num, slots, cap_for_k(k), false);
  if (workspace_bytes < L.total) return cudaErrorInvalidValue;
  TopkParams p = base_params(d_input, seg_num, k, d_output_values, d_output_indices,
                             d_workspace, L, slots, elem);
  p.seg_len = seg_len;
  p.offsets = nullptr;
  p.p_max = static_cast<int>(p_max);
  return launch_pipeline(p, false, slots, elem, static_cast<cudaStream_t>(stream));
}

// CSR batches of one element type.
int topk_csr(const void* d_input, const int* d_offsets, int seg_num, long long max_total_len,
             int k, void* d_output_values, int* d_output_indices, void* d_workspace,
             size_t workspace_bytes, void* stream, Elem elem) {
  if (!csr_shape_ok(seg_num, max_total_len, k)) return cudaErrorInvalidValue;
  if (!d_offsets || reinterpret_cast<uintptr_t>(d_offsets) % 4 != 0) return cudaErrorInvalidValue;
  if (!pointers_ok(d_input, d_output_values, d_output_indices, d_workspace, elem)) {
    return cudaErrorInvalidValue;
  }
  const long long slots = csr_slot_bound(seg_num, max_total_len, epv_of(elem));
  const Layout L = make_layout(seg_num, slots, cap_for_k(k), true);
  if (workspace_bytes < L.total) return cudaErrorInvalidValue;
  TopkParams p = base_params(d_input, seg_num, k, d_output_values, d_output_indices,
                             d_workspace, L, slots, elem);
  p.seg_len = 0;
  p.offsets = d_offsets;
  p.p_max = 0;
  p.max_total_len = max_total_len;
  return launch_pipeline(p, true, slots, elem, static_cast<cudaStream_t>(stream));
}

}  // namespace
}  // namespace bt

// Scratch for bt_topk_half_noalloc: a fixed device array that lives as long as the module,
// so that entry point never asks the runtime for memory.  BT_NOALLOC_SCRATCH_BYTES (32 MiB)
// covers, for example, 1024 rows of 151936 values at k <= 128 (about 10.5 MB).
static __device__ __align__(256) unsigned char g_noalloc_scratch[BT_NOALLOC_SCRATCH_BYTES];

namespace bt {
namespace {

void* g_noalloc_ptr[64] = {};

// Device address of g_noalloc_scratch on the current device, looked up once per device.
// The lookup may load this library's device code onto the device, so it runs on the first
// call there and not on later ones.
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    if (!ptr || reinterpret_cast<uintptr_t>(ptr) % 256 != 0) return cudaErrorInvalidDevicePointer;
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace bt

extern "C" {

size_t bt_topk_half_workspace_size(int seg_num, int seg_len, int k) {
  return bt::fixed_workspace(seg_num, seg_len, k, bt::kF16);
}

int bt_topk_half(const void* d_input, int seg_num, int seg_len, int k, void* d_output_values,
                 int* d_output_indices, void* d_workspace, size_t workspace_bytes, void* stream) {
  return bt::topk_fixed(d_input, seg_num, seg_len, k, d_output_values, d_output_indices,
                        d_workspace, workspace_bytes, stream, bt::kF16);
}

int bt_topk_half_noalloc(const void* d_input, int seg_num, int seg_len, int k,
                         void* d_output_values, int* d_output_indices, void* stream) {
  const size_t need = bt_topk_half_workspace_size(seg_num, seg_len, k);
  if (need == 0 || need > BT_NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  // Device info (shared-memory opt-in, occupancy) is set up before the scratch lookup so that
  // both happen on the first call on a device, outside any stream capture the caller begins
  // later.
  bt::DeviceInfo di;
  cudaError_t e = bt::device_info(&di);
  if (e != cudaSuccess) return e;
  void* scratch = nullptr;
  e = bt::noalloc_scratch(&scratch);
  if (e != cudaSuccess) return e;
  return bt_topk_half(d_input, seg_num, seg_len, k, d_output_values, d_output_indices, scratch,
                      need, stream);
}

size_t bt_topk_half_segmented_workspace_size(int seg_num, long long max_total_len, int k) {
  return bt::csr_workspace(seg_num, max_total_len, k, bt::kF16);
}

int bt_topk_half_segmented(const void* d_input, const int* d_offsets, int seg_num,
                           long long max_total_len, int k, void* d_output_values,
                           int* d_output_indices, void* d_workspace, size_t workspace_bytes,
                           void* stream) {
  return bt::topk_csr(d_input, d_offsets, seg_num, max_total_len, k, d_output_values,
                      d_output_indices, d_workspace, workspace_bytes, stream, bt::kF16);
}

size_t bt_topk_bf16_workspace_size(int seg_num, int seg_len, int k) {
  return bt_topk_half_workspace_size(seg_num, seg_len, k);
}

int bt_topk_bf16(const void* d_input, int seg_num, int seg_len, int k, void* d_output_values,
                 int* d_output_indices, void* d_workspace, size_t workspace_bytes, void* stream) {
  return bt::topk_fixed(d_input, seg_num, seg_len, k, d_output_values, d_output_indices,
                        d_workspace, workspace_bytes, stream, bt::kBF16);
}

size_t bt_topk_bf16_segmented_workspace_size(int seg_num, long long max_total_len, int k) {
  return bt_topk_half_segmented_workspace_size(seg_num, max_total_len, k);
}

int bt_topk_bf16_segmented(const void* d_input, const int* d_offsets, int seg_num,
                           long long max_total_len, int k, void* d_output_values,
                           int* d_output_indices, void* d_workspace, size_t workspace_bytes,
                           void* stream) {
  return bt::topk_csr(d_input, d_offsets, seg_num, max_total_len, k, d_output_values,
                      d_output_indices, d_workspace, workspace_bytes, stream, bt::kBF16);
}

size_t bt_topk_f32_workspace_size(int seg_num, int seg_len, int k) {
  return bt::fixed_workspace(seg_num, seg_len, k, bt::kF32);
}

int bt_topk_f32(const void* d_input, int seg_num, int seg_len, int k, void* d_output_values,
                int* d_output_indices, void* d_workspace, size_t workspace_bytes, void* stream) {
  return bt::topk_fixed(d_input, seg_num, seg_len, k, d_output_values, d_output_indices,
                        d_workspace, workspace_bytes, stream, bt::kF32);
}

size_t bt_topk_f32_segmented_workspace_size(int seg_num, long long max_total_len, int k) {
  return bt::csr_workspace(seg_num, max_total_len, k, bt::kF32);
}

int bt_topk_f32_segmented(const void* d_input, const int* d_offsets, int seg_num,
                          long long max_total_len, int k, void* d_output_values,
                          int* d_output_indices, void* d_workspace, size_t workspace_bytes,
                          void* stream) {
  return bt::topk_csr(d_input, d_offsets, seg_num, max_total_len, k, d_output_values,
                      d_output_indices, d_workspace, workspace_bytes, stream, bt::kF32);
}

int bt_workspace_status(const void* d_workspace, int seg_num, void* stream, unsigned* stats) {
  (void)seg_num;
  if (!d_workspace) return cudaErrorInvalidValue;
  uint32_t words[16];
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(words, d_workspace, sizeof(words), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return -static_cast<int>(e);
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return -static_cast<int>(e);
  if (stats) {
    for (int i = 0; i < BT_STATS_WORDS; ++i) stats[i] = words[1 + i];
  }
  return static_cast<int>(words[0]);
}

int bt_noalloc_status(void* stream, unsigned* stats) {
  void* scratch = nullptr;
  const cudaError_t e = bt::noalloc_scratch(&scratch);
  if (e != cudaSuccess) return -static_cast<int>(e);
  // the status words open the scratch, as they open every workspace (make_layout)
  return bt_workspace_status(scratch, 0, stream, stats);
}

void bt_set_handoff_wait_tries(int tries) {
  std::lock_guard<std::mutex> lock(bt::g_mu);
  bt::g_handoff_tries = tries < 0 ? bt::kWaitCap : static_cast<uint32_t>(tries);
}

void bt_set_profile_events(void* ev_start, void* ev_stop) {
  std::lock_guard<std::mutex> lock(bt::g_mu);
  if (ev_start && ev_stop) {
    bt::g_prof_start = static_cast<cudaEvent_t>(ev_start);
    bt::g_prof_stop = static_cast<cudaEvent_t>(ev_stop);
  } else {
    bt::g_prof_start = nullptr;
    bt::g_prof_stop = nullptr;
  }
}

const char* bt_error_string(int code) {
  if (code < 0) return cudaGetErrorString(static_cast<cudaError_t>(-code));
  switch (code) {
    case 0: return "success";
    case cudaErrorInvalidValue: return "invalid argument (shape, pointer, or workspace size)";
    default: return cudaGetErrorString(static_cast<cudaError_t>(code));
  }
}

int bt_device_info(int* info, int n) {
  bt::DeviceInfo di;
  const cudaError_t e = bt::device_info(&di);
  if (e != cudaSuccess) return static_cast<int>(e);
  const int v[6] = {di.sms, di.blocks_per_sm[0], di.blocks_per_sm[1],
                    static_cast<int>(bt::SmemLayout<false>::bytes),
                    static_cast<int>(bt::SmemLayout<true>::bytes), bt::block_threads<false>()};
  for (int i = 0; i < n && i < 6; ++i) info[i] = v[i];
  return 0;
}

int bt_version(void) { return bt::kVersion; }

}  // extern "C"
