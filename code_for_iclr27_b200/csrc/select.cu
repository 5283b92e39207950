// Selection kernels of liblrk: torch.topk(largest=False, sorted=True)
// semantics and the allocation-preserving refinement of selection.py:52-88.
//
// Order semantics reproduced (PyTorch CUDA topk, ties included):
// * Float scores are ranked by the order-preserving 32-bit map
//   bits ^ (sign ? 0xffffffff : 0x80000000), NaN -> 0xffffffff, the same map
//   PyTorch's radix select uses; the k chosen elements are the k smallest by
//   (key, index).
// * Output order is (key, index) -- PyTorch's stable sorts -- except for
//   2 <= k <= 32, where PyTorch sorts the gathered elements (keys below the
//   k-th in index order, then the k-th key's ties in index order) with an
//   unstable 32-wide bitonic network; that network is replayed here exactly.
//   This holds at every slice length (checked against torch 2.11 on B200).
//
// Machinery: a stable LSD radix sort of (64-bit key, 32-bit payload) pairs in
// 8-bit digits.  Each pass is a per-tile digit histogram, one exclusive scan
// over the digit-major count table, and a scatter that ranks each tile's
// elements stably with warp match masks.  The global raw-score sort keys on
// the 32-bit score; the per-segment sort keys on (segment << 32 | score), so
// one pass sequence sorts every segment at once.
#include <algorithm>

#include "common.cuh"

namespace lrk {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortRounds = 16;
constexpr int kSortTile = kSortThreads * kSortRounds;  // elements per scatter tile
constexpr int kBitonicMax = 32;
constexpr int kMaxSharedSegments = 4096;

__device__ __forceinline__ uint32_t radix_key(float v) {
  const uint32_t x = __float_as_uint(v);
  const uint32_t mask = (x & 0x80000000u) ? 0xffffffffu : 0x80000000u;
  return (v == v) ? (x ^ mask) : 0xffffffffu;
}

__global__ void __launch_bounds__(kSortThreads) histogram_kernel(const uint64_t *__restrict__ keys, int64_t n,
                                                                 int shift, uint32_t *__restrict__ counts,
                                                                 int64_t tiles) {
  __shared__ uint32_t hist[256];
  hist[threadIdx.x] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kSortTile;
  for (int i = threadIdx.x; i < kSortTile; i += kSortThreads) {
    const int64_t e = base + i;
    if (e < n) atomicAdd(&hist[(keys[e] >> shift) & 255u], 1u);
  }
  __syncthreads();
  counts[static_cast<int64_t>(threadIdx.x) * tiles + blockIdx.x] = hist[threadIdx.x];
}

// Exclusive scan of uint32 values in place with 1024-thread CTAs: CTA b scans
// [b span, min(total, (b + 1) span)) starting from carry_in[b] (0 without
// carry_in).  One CTA with span = total scans everything; for long tables
// the span is kScanSpan and carry_in holds the scanned block sums
// (block_sums_kernel, then this kernel on the sums).
constexpr int kScanItems = 8;
constexpr int64_t kScanSpan = 1024 * kScanItems;

__global__ void __launch_bounds__(1024) scan_kernel(uint32_t *__restrict__ data, int64_t total, int64_t span,
                                                    const uint32_t *__restrict__ carry_in) {
  constexpr int kItems = kScanItems;
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t carry_shared;
  if (threadIdx.x == 0) carry_shared = carry_in != nullptr ? carry_in[blockIdx.x] : 0u;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * span;
  const int64_t stop = lmin(total, first + span);
  for (int64_t base = first; base < stop; base += 1024 * kItems) {
    uint32_t v[kItems];
    uint32_t sum = 0;
    const int64_t start = base + static_cast<int64_t>(threadIdx.x) * kItems;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      v[j] = start + j < stop ? data[start + j] : 0u;
      sum += v[j];
    }
    uint32_t inclusive = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t other = __shfl_up_sync(0xffffffffu, inclusive, o);
      if (lane >= o) inclusive += other;
    }
    if (lane == 31) warp_sums[warp] = inclusive;
    __syncthreads();
    if (warp == 0) {
      uint32_t w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t other = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += other;
      }
      warp_sums[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const uint32_t carry = carry_shared;
    uint32_t running = carry + (warp > 0 ? warp_sums[warp - 1] : 0u) + inclusive - sum;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      if (start + j < stop) data[start + j] = running;
      running += v[j];
    }
    __syncthreads();
    if (threadIdx.x == 1023) carry_shared = carry + warp_sums[31];
    __syncthreads();
  }
}

// Sum of each kScanSpan block of `total` values (one CTA per block).
__global__ void __launch_bounds__(1024) block_sums_kernel(const uint32_t *__restrict__ data, int64_t total,
                                                          uint32_t *__restrict__ sums) {
  __shared__ uint32_t warp_sums[32];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kScanSpan;
  uint32_t sum = 0;
  for (int64_t i = first + threadIdx.x; i < lmin(total, first + kScanSpan); i += 1024) sum += data[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x < 32) {
    sum = warp_sums[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (threadIdx.x == 0) sums[blockIdx.x] = sum;
  }
}

// Extra uint32 entries a count table of `total` entries needs after it for
// the block sums of the multi-CTA scan.
inline int64_t scan_extra(int64_t total) { return total > 4 * kScanSpan ? ceil_div(total, kScanSpan) : 0; }

// Exclusive scan of counts[0, total) in place; the block sums (when used)
// live at counts + total.
void exclusive_scan(uint32_t *counts, int64_t total, cudaStream_t stream) {
  const int64_t blocks = scan_extra(total);
  if (blocks == 0) {
    scan_kernel<<<1, 1024, 0, stream>>>(counts, total, total, nullptr);
    return;
  }
  uint32_t *sums = counts + total;
  block_sums_kernel<<<static_cast<unsigned>(blocks), 1024, 0, stream>>>(counts, total, sums);
  scan_kernel<<<1, 1024, 0, stream>>>(sums, blocks, blocks, nullptr);
  scan_kernel<<<static_cast<unsigned>(blocks), 1024, 0, stream>>>(counts, total, kScanSpan, sums);
}

__global__ void __launch_bounds__(kSortThreads) scatter_kernel(
    const uint64_t *__restrict__ keys_in, const uint32_t *__restrict__ values_in, uint64_t *__restrict__ keys_out,
    uint32_t *__restrict__ values_out, int64_t n, int shift, const uint32_t *__restrict__ offsets,
    int64_t tiles) {
  __shared__ uint32_t running[256];
  __shared__ uint32_t warp_counts[kSortThreads / 32][256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  running[threadIdx.x] = offsets[static_cast<int64_t>(threadIdx.x) * tiles + blockIdx.x];
#pragma unroll
  for (int w = 0; w < kSortThreads / 32; ++w) warp_counts[w][threadIdx.x] = 0;
  __syncthreads();
  const uint32_t lower_lanes = (1u << lane) - 1u;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kSortTile;
  for (int round = 0; round < kSortRounds; ++round) {
    const int64_t e = base + round * kSortThreads + threadIdx.x;
    const bool valid = e < n;
    uint64_t key = 0;
    uint32_t value = 0;
    uint32_t digit = 256u + lane;  // invalid lanes match nobody
    if (valid) {
      key = keys_in[e];
      value = values_in[e];
      digit = static_cast<uint32_t>((key >> shift) & 255u);
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, digit);
    const uint32_t rank = __popc(peers & lower_lanes);
    if (valid && rank == 0) warp_counts[warp][digit] = __popc(peers);
    __syncthreads();
    if (valid) {
      uint32_t position = running[digit] + rank;
      for (int w = 0; w < warp; ++w) position += warp_counts[w][digit];
      keys_out[position] = key;
      values_out[position] = value;
    }
    __syncthreads();
    uint32_t total = 0;
#pragma unroll
    for (int w = 0; w < kSortThreads / 32; ++w) {
      total += warp_counts[w][threadIdx.x];
      warp_counts[w][threadIdx.x] = 0;
    }
    running[threadIdx.x] += total;
    __syncthreads();
  }
}

struct SortBuffers {
  uint64_t *keys[2];
  uint32_t *values[2];
  uint32_t *counts;
};

// Sort n pairs in buffers[0] by key bits [0, bits); returns the index (0/1)
// of the buffer holding the result.
int radix_sort(SortBuffers &b, int64_t n, int bits, cudaStream_t stream, int &status) {
  status = LRK_OK;
  int current = 0;
  if (n <= 1) return current;
  const int64_t tiles = ceil_div(n, kSortTile);
  for (int shift = 0; shift < bits; shift += 8) {
    histogram_kernel<<<static_cast<unsigned>(tiles), kSortThreads, 0, stream>>>(b.keys[current], n, shift, b.counts,
                                                                              tiles);
    exclusive_scan(b.counts, 256 * tiles, stream);
    scatter_kernel<<<static_cast<unsigned>(tiles), kSortThreads, 0, stream>>>(
        b.keys[current], b.values[current], b.keys[current ^ 1], b.values[current ^ 1], n, shift, b.counts, tiles);
    current ^= 1;
  }
  status = launch_status("radix sort");
  return current;
}

// Number of ends <= i, i.e. the segment holding element i.  Clamped to the
// last segment so that a table whose last end falls short of n can never
// index past the per-segment arrays.
__device__ __forceinline__ int64_t segment_of(const int64_t *ends, int64_t segments, int64_t i) {
  int64_t lo = 0, hi = segments;
  while (lo < hi) {
    const int64_t mid = (lo + hi) / 2;
    if (ends[mid] <= i) lo = mid + 1; else hi = mid;
  }
  return lo < segments ? lo : segments - 1;
}

// keys_raw[i] = radix(raw[i]); keys_seg[i] = segment << 32 | radix(pooled[i]).
__global__ void build_keys_kernel(const float *__restrict__ raw, const float *__restrict__ pooled, int64_t n,
                                  const int64_t *__restrict__ ends, int64_t segments, uint64_t *__restrict__ keys_raw,
                                  uint32_t *__restrict__ values_raw, uint64_t *__restrict__ keys_seg,
                                  uint32_t *__restrict__ values_seg) {
  __shared__ int64_t shared_ends[kMaxSharedSegments];
  const bool use_shared = segments <= kMaxSharedSegments;
  if (use_shared)
    for (int64_t s = threadIdx.x; s < segments; s += blockDim.x) shared_ends[s] = ends[s];
  __syncthreads();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    keys_raw[i] = radix_key(raw[i]);
    values_raw[i] = static_cast<uint32_t>(i);
    if (keys_seg != nullptr) {
      const int64_t s = segment_of(use_shared ? shared_ends : ends, segments, i);
      keys_seg[i] = (static_cast<uint64_t>(s) << 32) | radix_key(pooled[i]);
      values_seg[i] = static_cast<uint32_t>(i);
    }
  }
}

__device__ __forceinline__ bool lt_nan_last(float lhs, float rhs) {
  return (isnan(rhs) && !isnan(lhs)) || (lhs < rhs);
}

// Replays PyTorch's small-slice topk ordering on the k (<= 32) smallest
// entries of one sorted run: rebuild the gather order (keys below the k-th in
// index order, then the k-th key's ties in index order) and run the 16-thread,
// 32-slot bitonic network with a NaN-last less-than.  Runs in one thread; the
// network is data-parallel per stage, so iterating its 16 "threads" in order
// is equivalent.  `scores` maps a payload to its float value; `index_base` is
// subtracted from payloads to get slice-local indices for ordering.
__device__ void bitonic_replay(uint32_t *values, int k, const float *scores) {
  float key[kBitonicMax];
  uint32_t val[kBitonicMax];
  bool valid[kBitonicMax];
  // values[0..k) are in (radix key, index) order; the k-th key is the last.
  const uint32_t kth = radix_key(scores[values[k - 1]]);
  int w = 0;
  for (int pass = 0; pass < 2; ++pass) {
    // pass 0: strictly below the k-th key; pass 1: equal to it.  Each group
    // is emitted in ascending payload (= index) order.
    uint32_t last = 0;
    bool have_last = false;
    while (true) {
      int best = -1;
      for (int j = 0; j < k; ++j) {
        const uint32_t rk = radix_key(scores[values[j]]);
        const bool member = pass == 0 ? rk < kth : rk == kth;
        if (!member || (have_last && values[j] <= last)) continue;
        if (best < 0 || values[j] < values[best]) best = j;
      }
      if (best < 0) break;
      key[w] = scores[values[best]];
      val[w] = values[best];
      valid[w] = true;
      ++w;
      last = values[best];
      have_last = true;
    }
  }
  for (int j = w; j < kBitonicMax; ++j) {
    key[j] = 0.0f;
    val[j] = 0;
    valid[j] = false;
  }
  auto swap_step = [&](unsigned pos, unsigned stride, bool dir) {
    const unsigned a = pos, b = pos + stride;
    const bool swap = (lt_nan_last(key[a], key[b]) && valid[a]) || !valid[b];
    if (swap == dir) {
      const float tk = key[a]; key[a] = key[b]; key[b] = tk;
      const uint32_t tv = val[a]; val[a] = val[b]; val[b] = tv;
      const bool tb = valid[a]; valid[a] = valid[b]; valid[b] = tb;
    }
  };
  for (unsigned size = 2; size < kBitonicMax; size *= 2) {
    for (unsigned stride = size / 2; stride > 0; stride /= 2) {
      for (unsigned t = 0; t < kBitonicMax / 2; ++t) {
        const bool flag = (t & (size / 2)) != 0;
        swap_step(2 * t - (t & (stride - 1)), stride, flag);
      }
    }
  }
  for (unsigned stride = kBitonicMax / 2; stride > 0; stride /= 2)
    for (unsigned t = 0; t < kBitonicMax / 2; ++t) swap_step(2 * t - (t & (stride - 1)), stride, false);
  for (int j = 0; j < k; ++j) values[j] = val[j];
}

// Global pick fix-up (one thread): applies the small-slice network.
__global__ void global_bitonic_kernel(uint32_t *values, int k, const float *scores) {
  if (threadIdx.x == 0 && blockIdx.x == 0) bitonic_replay(values, k, scores);
}

// Per-segment fix-up: segments whose quota is in [2, 32].  One thread per
// segment.
__global__ void segment_bitonic_kernel(uint32_t *sorted_values, const int64_t *__restrict__ ends, int64_t segments,
                                       const uint32_t *__restrict__ quota, const float *scores) {
  const int64_t s = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (s >= segments) return;
  const int64_t start = s == 0 ? 0 : ends[s - 1];
  const int64_t length = ends[s] - start;
  const uint32_t q = quota[s];
  if (q >= 2 && q <= kBitonicMax && q <= length)
    bitonic_replay(sorted_values + start, q, scores);
}

// Global picks: values, segment ids, per-segment quotas, membership marks.
__global__ void picks_kernel(const uint32_t *__restrict__ picked, int64_t count, const float *__restrict__ raw,
                             const int64_t *__restrict__ ends, int64_t segments, float *__restrict__ values,
                             int64_t *__restrict__ segment_ids, uint32_t *__restrict__ quota,
                             uint8_t *__restrict__ mark, uint64_t *__restrict__ pick_keys,
                             uint32_t *__restrict__ pick_values) {
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < count;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t index = picked[j];
    const int64_t s = segment_of(ends, segments, index);
    values[j] = raw[index];
    segment_ids[j] = s;
    atomicAdd(&quota[s], 1u);
    mark[index] = 1;
    pick_keys[j] = static_cast<uint64_t>(s);
    pick_values[j] = static_cast<uint32_t>(j);
  }
}

// quota_start = exclusive scan of quota (segments small: one CTA).
__global__ void quota_scan_kernel(const uint32_t *__restrict__ quota, int64_t segments,
                                  uint32_t *__restrict__ quota_start) {
  if (threadIdx.x != 0) return;
  uint32_t running = 0;
  for (int64_t s = 0; s < segments; ++s) {
    quota_start[s] = running;
    running += quota[s];
  }
}

// Slot j (global raw order) of segment s is the r-th occurrence of s, r
// from the stable sort of picks by segment; it receives the segment's r-th
// refined pick.
__global__ void transplant_kernel(const uint32_t *__restrict__ by_segment, int64_t count,
                                  const int64_t *__restrict__ segment_ids, const uint32_t *__restrict__ quota_start,
                                  const uint32_t *__restrict__ refined, const int64_t *__restrict__ ends,
                                  const int64_t *__restrict__ position_starts, const uint8_t *__restrict__ mark,
                                  int64_t n, int64_t *__restrict__ positions, uint8_t *__restrict__ changed_segment,
                                  unsigned long long *__restrict__ changed) {
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < count;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t j = by_segment[p];
    const int64_t s = segment_ids[j];
    const int64_t r = p - quota_start[s];
    const int64_t start = s == 0 ? 0 : ends[s - 1];
    if (r < 0 || start + r >= n) continue;  // only for tables whose ends do not cover n
    const uint32_t index = refined[start + r];
    positions[j] = static_cast<int64_t>(index) - start + position_starts[s];
    if (!mark[index]) {
      atomicAdd(changed, 1ull);
      changed_segment[s] = 1;
    }
  }
}

__global__ void stats_kernel(const uint8_t *__restrict__ changed_segment, int64_t segments,
                             const unsigned long long *__restrict__ changed, int64_t *__restrict__ stats) {
  __shared__ int64_t total;
  if (threadIdx.x == 0) total = 0;
  __syncthreads();
  int64_t local = 0;
  for (int64_t s = threadIdx.x; s < segments; s += blockDim.x) local += changed_segment[s];
  atomicAdd(reinterpret_cast<unsigned long long *>(&total), static_cast<unsigned long long>(local));
  __syncthreads();
  if (threadIdx.x == 0) {
    stats[0] = static_cast<int64_t>(*changed);
    stats[1] = total;
  }
}

__global__ void gather_topk_kernel(const uint32_t *__restrict__ picked, int64_t k, const float *__restrict__ x,
                                   float *__restrict__ values, int64_t *__restrict__ indices) {
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < k;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t index = picked[j];
    values[j] = x[index];
    indices[j] = index;
  }
}

// ---------------------------------------------------------- workspace

struct Carver {
  char *base;
  size_t used = 0;
  template <typename T> T *take(int64_t count) {
    used = (used + 255) & ~static_cast<size_t>(255);
    T *p = reinterpret_cast<T *>(base == nullptr ? nullptr : base + used);
    used += static_cast<size_t>(count) * sizeof(T);
    return p;
  }
};

struct RefineLayout {
  SortBuffers raw_sort, seg_sort, pick_sort;
  uint8_t *mark, *changed_segment;
  uint32_t *quota, *quota_start;
  unsigned long long *changed;
  size_t bytes;
};

RefineLayout carve_refine(void *workspace, int64_t n, int64_t segments) {
  Carver c{static_cast<char *>(workspace)};
  RefineLayout l;
  const int64_t tiles = std::max<int64_t>(1, ceil_div(n, kSortTile));
  // The raw sort and the segment sort share storage: the raw result is copied
  // out (picks) before the segment sort starts.
  l.raw_sort.keys[0] = c.take<uint64_t>(n);
  l.raw_sort.keys[1] = c.take<uint64_t>(n);
  l.raw_sort.values[0] = c.take<uint32_t>(n);
  l.raw_sort.values[1] = c.take<uint32_t>(n);
  l.raw_sort.counts = c.take<uint32_t>(256 * tiles + scan_extra(256 * tiles));
  l.seg_sort.keys[0] = c.take<uint64_t>(n);
  l.seg_sort.keys[1] = c.take<uint64_t>(n);
  l.seg_sort.values[0] = c.take<uint32_t>(n);
  l.seg_sort.values[1] = c.take<uint32_t>(n);
  l.seg_sort.counts = l.raw_sort.counts;
  l.pick_sort.keys[0] = c.take<uint64_t>(n);
  l.pick_sort.keys[1] = c.take<uint64_t>(n);
  l.pick_sort.values[0] = c.take<uint32_t>(n);
  l.pick_sort.values[1] = c.take<uint32_t>(n);
  l.pick_sort.counts = l.raw_sort.counts;
  l.mark = c.take<uint8_t>(n);
  l.changed_segment = c.take<uint8_t>(segments);
  l.quota = c.take<uint32_t>(segments);
  l.quota_start = c.take<uint32_t>(segments);
  l.changed = c.take<unsigned long long>(1);
  l.bytes = c.used + 256;
  return l;
}

int bits_for(int64_t max_value) {
  int bits = 0;
  while (bits < 64 && (static_cast<uint64_t>(max_value) >> bits) != 0) ++bits;
  return ((bits + 7) / 8) * 8;
}

int grid_for(int64_t n, int threads = 256) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, threads), sm_count() * 8LL)));
}

}  // namespace
}  // namespace lrk

using namespace lrk;

extern "C" size_t lrk_refine_workspace_bytes(int64_t n, int64_t segments) {
  if (n < 0 || segments < 0) return 0;
  return carve_refine(nullptr, n, segments).bytes;
}

extern "C" int lrk_refine(const float *raw, const float *pooled, int64_t n, const int64_t *segment_ends,
                          const int64_t *position_starts, int64_t segments, int64_t count, void *workspace,
                          size_t workspace_bytes, float *values, int64_t *segment_ids, int64_t *positions,
                          int64_t *stats, lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(n >= 0 && segments >= 1 && count >= 0 && count <= n, "invalid refine sizes");
  LRK_REQUIRE(n < (int64_t{1} << 32) && segments < (int64_t{1} << 31), "refine too large");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LRK_REQUIRE(stats != nullptr, "null stats");
  if (count == 0) {
    cudaError_t e = cudaMemsetAsync(stats, 0, 2 * sizeof(int64_t), s);
    return e == cudaSuccess ? LRK_OK : fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  }
  LRK_REQUIRE(raw && pooled && segment_ends && position_starts && values && segment_ids && positions, "null pointer");
  RefineLayout l = carve_refine(workspace, n, segments);
  if (workspace == nullptr || workspace_bytes < l.bytes) return fail(LRK_ERR_WORKSPACE, "refine workspace too small");
  l = carve_refine(reinterpret_cast<void *>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t{255}), n,
                   segments);
  int status = LRK_OK;
  // Zero what accumulates: marks, quotas, changed flags and counter.
  cudaMemsetAsync(l.mark, 0, static_cast<size_t>(n), s);
  cudaMemsetAsync(l.changed_segment, 0, static_cast<size_t>(segments), s);
  cudaMemsetAsync(l.quota, 0, static_cast<size_t>(segments) * sizeof(uint32_t), s);
  cudaMemsetAsync(l.changed, 0, sizeof(unsigned long long), s);
  build_keys_kernel<<<grid_for(n), 256, 0, s>>>(raw, pooled, n, segment_ends, segments, l.raw_sort.keys[0],
                                                l.raw_sort.values[0], l.seg_sort.keys[0], l.seg_sort.values[0]);
  if ((status = launch_status("refine keys")) != LRK_OK) return status;
  // 1. Global bottom-count of raw scores.
  const int raw_at = radix_sort(l.raw_sort, n, 32, s, status);
  if (status != LRK_OK) return status;
  uint32_t *picked = l.raw_sort.values[raw_at];
  if (count >= 2 && count <= kBitonicMax) global_bitonic_kernel<<<1, 1, 0, s>>>(picked, static_cast<int>(count), raw);
  picks_kernel<<<grid_for(count), 256, 0, s>>>(picked, count, raw, segment_ends, segments, values, segment_ids,
                                               l.quota, l.mark, l.pick_sort.keys[0], l.pick_sort.values[0]);
  if ((status = launch_status("refine picks")) != LRK_OK) return status;
  // 2. Occurrence rank of each pick inside its segment.
  const int pick_at = radix_sort(l.pick_sort, count, bits_for(segments - 1), s, status);
  if (status != LRK_OK) return status;
  quota_scan_kernel<<<1, 32, 0, s>>>(l.quota, segments, l.quota_start);
  // 3. Every segment's pooled scores, sorted within the segment.
  const int seg_at = radix_sort(l.seg_sort, n, 32 + bits_for(segments - 1), s, status);
  if (status != LRK_OK) return status;
  uint32_t *refined = l.seg_sort.values[seg_at];
  segment_bitonic_kernel<<<static_cast<unsigned>(ceil_div(segments, 128)), 128, 0, s>>>(refined, segment_ends,
                                                                                      segments, l.quota, pooled);
  // 4. Transplant and change statistics.
  transplant_kernel<<<grid_for(count), 256, 0, s>>>(l.pick_sort.values[pick_at], count, segment_ids, l.quota_start,
                                                    refined, segment_ends, position_starts, l.mark, n, positions,
                                                    l.changed_segment, l.changed);
  stats_kernel<<<1, 256, 0, s>>>(l.changed_segment, segments, l.changed, stats);
  return launch_status("refine transplant");
}

extern "C" size_t lrk_topk_workspace_bytes(int64_t n) {
  if (n < 0) return 0;
  Carver c{nullptr};
  const int64_t tiles = std::max<int64_t>(1, ceil_div(n, kSortTile));
  c.take<uint64_t>(n);
  c.take<uint64_t>(n);
  c.take<uint32_t>(n);
  c.take<uint32_t>(n);
  c.take<uint32_t>(256 * tiles + scan_extra(256 * tiles));
  return c.used + 256;
}

extern "C" int lrk_topk_smallest(const float *x, int64_t n, int64_t k, void *workspace, size_t workspace_bytes,
                                 float *values, int64_t *indices, lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(n >= 0 && k >= 0 && k <= n, "selected index k out of range");
  LRK_REQUIRE(n < (int64_t{1} << 32), "topk too large");
  if (k == 0) return LRK_OK;
  LRK_REQUIRE(x && values && indices, "null pointer");
  if (workspace == nullptr || workspace_bytes < lrk_topk_workspace_bytes(n))
    return fail(LRK_ERR_WORKSPACE, "topk workspace too small");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  Carver c{reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t{255})};
  const int64_t tiles = std::max<int64_t>(1, ceil_div(n, kSortTile));
  SortBuffers b;
  b.keys[0] = c.take<uint64_t>(n);
  b.keys[1] = c.take<uint64_t>(n);
  b.values[0] = c.take<uint32_t>(n);
  b.values[1] = c.take<uint32_t>(n);
  b.counts = c.take<uint32_t>(256 * tiles + scan_extra(256 * tiles));
  build_keys_kernel<<<grid_for(n), 256, 0, s>>>(x, nullptr, n, nullptr, 0, b.keys[0], b.values[0], nullptr,
                                                nullptr);
  int status = launch_status("topk keys");
  if (status != LRK_OK) return status;
  const int at = radix_sort(b, n, 32, s, status);
  if (status != LRK_OK) return status;
  if (k >= 2 && k <= kBitonicMax) global_bitonic_kernel<<<1, 1, 0, s>>>(b.values[at], static_cast<int>(k), x);
  gather_topk_kernel<<<grid_for(k), 256, 0, s>>>(b.values[at], k, x, values, indices);
  return launch_status("topk gather");
}
