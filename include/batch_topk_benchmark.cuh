// batch_topk_benchmark.cuh -- the reference's primary benchmark table, same names and values
// (include/batch_topk_benchmark.cuh of fire-emblem/batch_topk), so its benchmark driver builds
// against this library unchanged.  ref_us is the reference's own latency target per case, in
// microseconds, on its hardware; this library does not use the table.
#pragma once

#include <array>

namespace radix_topk {

struct BenchmarkCase {
  int seg_num;
  int seg_len;
  int k;
  float ref_us;
};

inline constexpr std::array<BenchmarkCase, 5> kPrimaryBenchmarkCases = {{
    {128, 10000, 50, 11.0f},
    {1500, 10000, 50, 82.0f},
    {3000, 10000, 50, 161.0f},
    {4500, 10000, 50, 241.0f},
    {6000, 10000, 50, 319.0f},
}};

}  // namespace radix_topk
