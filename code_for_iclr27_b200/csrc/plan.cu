// Recall merge plan on the device (recall/planning.py:34-52).
//
// The reference builds, per touched layer and head, the merged order of the
// head's resident rows and its recalled rows by a stable argsort of their
// positions on the host, after copying the layer's positions to the host
// (cache.py:216-217).  A head's resident positions are ascending (appends add
// increasing positions, compactions keep order, merges write position
// order), and duplicates are refused, so the merged order is two merges of
// sorted lists, one element at a time:
//
// * resident row j of head h goes to new row start'(h) + j + (the number of
//   h's recalled positions below its position);
// * the k-th recalled position of head h (sorted) goes to new row
//   start'(h) + k + (the number of h's resident positions below it);
//
// with start'(h) = start(h) + (recalled rows of the heads before h).  One
// thread per resident or recalled row, each a binary search.  A position that
// is recalled twice, recalled while resident, or a head whose resident
// positions are not ascending sets *flag (1: duplicate, 2: not ascending; 4:
// inconsistent head bounds): the caller reads it before it adopts the merged
// tensors, as the reference raises before it changes the cache.
#include <algorithm>

#include "common.cuh"

namespace lrk {
namespace {

constexpr int kPlanThreads = 256;
constexpr int kPlanLayers = 64;

struct PlanTable {
  lrk_plan_layer layer[kPlanLayers];
};

// Number of entries of values[0 .. n) (ascending) below x.
__device__ __forceinline__ int64_t below(const float *values, int64_t n, float x) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (values[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// The index h with starts[h] <= i < starts[h + 1] (starts ascending, heads + 1 entries).
__device__ __forceinline__ int head_of(const int32_t *starts, int heads, int64_t i) {
  int lo = 0, hi = heads;  // answer in [0, heads)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (starts[mid] <= i) lo = mid; else hi = mid;
  }
  return lo;
}

// starts[h] clamped into [0, limit]: bounds that are not ascending or do
// not end at the row count (the host validates neither) cannot move a read
// or a write out of the layer's arrays; *flag bit 4 reports them.
__device__ __forceinline__ int64_t bound_at(const int32_t *starts, int h, int64_t limit) {
  return min(max(static_cast<int64_t>(starts[h]), int64_t{0}), limit);
}

__global__ void __launch_bounds__(kPlanThreads) merge_plan_kernel(PlanTable table, int heads,
                                                                  unsigned int *__restrict__ flag) {
  const lrk_plan_layer &l = table.layer[blockIdx.y];
  const int64_t total = l.rows + l.recalled;
  if (blockIdx.x == 0 && threadIdx.x < 2) {
    const int32_t *starts = threadIdx.x == 0 ? l.head_starts : l.recalled_starts;
    bool ok = starts[0] == 0 && starts[heads] == (threadIdx.x == 0 ? l.rows : l.recalled);
    for (int h = 0; h < heads; ++h) ok = ok && starts[h] <= starts[h + 1];
    if (!ok) atomicOr(flag, 4u);
  }
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kPlanThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kPlanThreads) {
    const bool resident = i < l.rows;
    const int64_t e = resident ? i : i - l.rows;
    const int h = head_of(resident ? l.head_starts : l.recalled_starts, heads, e);
    const int64_t start = bound_at(l.head_starts, h, l.rows), end = bound_at(l.head_starts, h + 1, l.rows);
    const int64_t first = bound_at(l.recalled_starts, h, l.recalled);
    const int64_t last = bound_at(l.recalled_starts, h + 1, l.recalled);
    int64_t to = -1, from = 0;
    if (resident && i >= start && i < end) {
      const float p = l.positions[i];
      if (i > start && !(l.positions[i - 1] < p)) atomicOr(flag, 2u);
      const int64_t k = below(l.recalled_positions + first, last - first, p);
      if (first + k < last && l.recalled_positions[first + k] == p) atomicOr(flag, 1u);
      to = start + first + (i - start) + k;
      from = i;
    } else if (!resident && e >= first && e < last) {
      const float r = l.recalled_positions[e];
      if (e > first && !(l.recalled_positions[e - 1] < r)) atomicOr(flag, 1u);
      to = start + e + below(l.positions + start, end - start, r);
      from = -(l.recalled_index ? l.recalled_index[e] : e) - 1;
    }
    if (to >= 0 && to < total) l.mapping[to] = from;
    else atomicOr(flag, 4u);
  }
}

}  // namespace
}  // namespace lrk

using namespace lrk;

extern "C" int lrk_merge_plan(const lrk_plan_layer *layers, int64_t count, int64_t heads, unsigned int *flag,
                              lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(count >= 0 && heads >= 1 && heads <= INT32_MAX, "invalid plan sizes");
  if (count == 0) return LRK_OK;
  LRK_REQUIRE(layers && flag, "null pointer");
  for (int64_t i = 0; i < count; ++i) {
    const lrk_plan_layer &l = layers[i];
    LRK_REQUIRE(l.rows >= 0 && l.recalled >= 0, "invalid plan layer sizes");
    LRK_REQUIRE(l.head_starts && l.recalled_starts && l.mapping, "null plan layer pointer");
    LRK_REQUIRE(l.rows == 0 || l.positions, "null positions");
    LRK_REQUIRE(l.recalled == 0 || l.recalled_positions, "null recalled positions");
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int64_t l0 = 0; l0 < count; l0 += kPlanLayers) {
    const int n = static_cast<int>(std::min<int64_t>(kPlanLayers, count - l0));
    PlanTable table{};
    int64_t longest = 0;
    for (int i = 0; i < n; ++i) {
      table.layer[i] = layers[l0 + i];
      longest = std::max(longest, layers[l0 + i].rows + layers[l0 + i].recalled);
    }
    if (longest == 0) continue;
    const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(ceil_div(longest, kPlanThreads), 4096));
    merge_plan_kernel<<<dim3(blocks, n), kPlanThreads, 0, s>>>(table, static_cast<int>(heads), flag);
    const int status = launch_status("lrk_merge_plan");
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
}
