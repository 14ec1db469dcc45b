// Host-only caller of the C++ drop-in headers (include/batch_topk.cuh, batch_topk_types.cuh,
// batch_topk_benchmark.cuh), built with g++ and linked against libbatch_topk_b200.so.  It runs
// without a GPU: the operator calls below are all rejected on the host.  Prints one line per
// check, "ok <name>" or "FAIL <name>", and exits non-zero on any failure.
#include <cmath>
#include <cstdio>
#include <vector>

#include "batch_topk.cuh"
#include "batch_topk_benchmark.cuh"
#include "batch_topk_types.cuh"

static int failures = 0;
static void check(bool ok, const char* name) {
  std::printf("%s %s\n", ok ? "ok" : "FAIL", name);
  if (!ok) ++failures;
}

int main() {
  using namespace radix_topk;
  {
    const ReferenceTopKResult r = cpu_reference_topk({5.0f, 7.0f, 7.0f, 1.0f}, 4, 2);
    check(r.indices == std::vector<int>{1, 2} && r.values == std::vector<float>{7.0f, 7.0f},
          "ordering");
  }
  {
    const ReferenceTopKResult r = cpu_reference_topk({NAN, 3.0f, -1.0f, NAN}, 4, 3);
    check(r.indices == std::vector<int>{1, 2, 0} && std::isnan(r.values[2]), "nan_ordering");
  }
  {
    const ReferenceTopKResult r = cpu_reference_topk({2.0f, 1.0f}, 4, 4);
    check(r.indices == std::vector<int>{0, 1}, "bounded_seg_len");
    check(cpu_reference_topk({1.0f}, 0, 1).indices.empty(), "empty_for_zero_len");
  }
  check(encode_half_desc(__float2half(3.0f)) < encode_half_desc(__float2half(-1.0f)) &&
            encode_half_desc(__float2half(NAN)) > encode_half_desc(__float2half(-1.0f)),
        "codec_order");
  check(encode_half_desc(__float2half(1.0f)) == 0x43FF &&
            encode_half_desc(__float2half(INFINITY)) == 0x03FF &&
            encode_half_desc(__float2half(-INFINITY)) == 0xFC00 &&
            encode_half_desc(__float2half(0.0f)) == encode_half_desc(__float2half(-0.0f)),
        "codec_keys");
  {
    Candidate a{}, b{};
    a.value = __float2half(5.0f);
    a.index = 2;
    b.value = __float2half(5.0f);
    b.index = 1;
    check(!candidate_better(a, b) && candidate_better(b, a), "tie_break");
    a.value = __float2half(NAN);
    a.index = 0;
    check(!candidate_better(a, b) && candidate_better(b, a), "nan_loses");
  }
  {
    SegmentSelectState s{};
    check(s.cutoff_key == 0xFFFFu && s.prefix == 0 && s.remaining_slots == 0, "state_defaults");
  }
  check(kPrimaryBenchmarkCases.size() == 5 && kPrimaryBenchmarkCases[0].seg_len == 10000,
        "benchmark_table");
  check(batch_topk_half_workspace_size(0, 10000, 50) == 0 &&
            batch_topk_half_workspace_size(1, 10, 11) == 0 &&
            batch_topk_half_workspace_size(1, 10000, 50) > 0,
        "workspace_size");
  const size_t need = batch_topk_half_workspace_size(2, 100, 5);
  half* fake_h = reinterpret_cast<half*>(1 << 20);
  int* fake_i = reinterpret_cast<int*>(1 << 20);
  void* fake_w = reinterpret_cast<void*>(1 << 20);
  check(batch_topk_half(nullptr, 2, 100, 5, fake_h, fake_i, fake_w, need, 0) ==
            cudaErrorInvalidValue,
        "null_input");
  check(batch_topk_half(fake_h, 2, 100, 101, fake_h, fake_i, fake_w, need, 0) ==
            cudaErrorInvalidValue,
        "k_above_seg_len");
  check(batch_topk_half(fake_h, 2, 100, 5, fake_h, fake_i, fake_w, need - 1, 0) ==
            cudaErrorInvalidValue,
        "short_workspace");
  check(batch_topk_half_segmented(fake_h, nullptr, 2, 100, 5, fake_h, fake_i, fake_w, 1 << 20,
                                  0) == cudaErrorInvalidValue,
        "segmented_null_offsets");
  return failures == 0 ? 0 : 1;
}
