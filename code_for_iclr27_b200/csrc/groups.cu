// Layer-group selection kernels of liblrk: the request-wide "k smallest raw
// scores" question when one request's layers are split over several GPUs.
//
// refine_arrays (src/lazy_recall/selection.py:52-88) starts from the global
// bottom-`count` of a request's raw scores, ties taken in score-table order,
// which is layer-major (src/lazy_recall/scoring.py:218-287).  With layers
// split into contiguous groups, rank r holds a contiguous range of that order,
// so the request-wide choice is fixed by the k-th smallest key and how many of
// its ties each lower rank holds; a rank's share is then its local bottom-(share)
// by (key, index).  Both follow from radix histograms alone:
//
// * Scores map to order-preserving 32-bit keys (NaN last), the map of
//   PyTorch's radix select.
// * Three rounds of 12, 12 and 8 bits.  In each, every rank histograms the
//   current digit of its keys that still match the prefix fixed so far
//   (select_histogram_kernel); the histograms are all-gathered (NCCL over
//   NVLink, by the caller); and select_pick_kernel sums them over ranks, finds
//   the bin that holds the k-th key, and advances the per-(request, question)
//   state on the device.  Nothing comes back to the host between rounds.
// * After the last round the gathered histograms' bin of the k-th key holds
//   each rank's tie count, so a rank's share of the ties (ranks in index
//   order) needs no further exchange: share = its keys below the k-th key +
//   clamp(ties still needed - ties of lower ranks, 0, its ties).
//
// Several questions per request run side by side (the audit asks for the
// selected count and for the immediate-eviction prefix, a smaller k over the
// same keys: the bottom-immediate by (key, index) is a prefix of the
// bottom-count).
#include <algorithm>

#include "common.cuh"

namespace lrk {
namespace {

constexpr int kBins = LRK_SELECT_BINS;
constexpr int kHistThreads = 512;
constexpr int kHistItems = 16;  // elements per thread per tile
constexpr int kPickThreads = 256;

__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t x = __float_as_uint(v);
  const uint32_t mask = (x & 0x80000000u) ? 0xffffffffu : 0x80000000u;
  return (v == v) ? (x ^ mask) : 0xffffffffu;
}

struct RequestTable {
  const float *scores[LRK_SELECT_MAX_REQUESTS];
  int64_t n[LRK_SELECT_MAX_REQUESTS];
};

__device__ __forceinline__ int round_shift(int round) {
  int done = 0;
  for (int r = 0; r <= round; ++r) done += (r == 0 ? 12 : (r == 1 ? 12 : 8));
  return 32 - done;
}

// Histogram of one round's digit, per (request, question), of the keys that
// match the question's prefix.  Grid: (tiles, requests).  Round 0 has no
// prefix, so every question shares one histogram (counted once, added to
// each question's slot).  hist [requests][questions][kBins] u32, zeroed by
// the caller's launcher.
__global__ void __launch_bounds__(kHistThreads) select_histogram_kernel(RequestTable table, int base_request,
                                                                        int questions, int round,
                                                                        const int64_t *__restrict__ states,
                                                                        uint32_t *__restrict__ hist) {
  extern __shared__ uint32_t local[];  // [questions][kBins]
  const int request = base_request + blockIdx.y;
  const float *scores = table.scores[blockIdx.y];
  const int64_t n = table.n[blockIdx.y];
  const int counted = round == 0 ? 1 : questions;
  for (int i = threadIdx.x; i < counted * kBins; i += kHistThreads) local[i] = 0;
  const int shift = round_shift(round);
  const uint32_t digit_mask = (1u << (round == 2 ? 8 : 12)) - 1u;
  uint32_t prefix[LRK_SELECT_MAX_QUESTIONS];
  bool live[LRK_SELECT_MAX_QUESTIONS];
#pragma unroll
  for (int q = 0; q < LRK_SELECT_MAX_QUESTIONS; ++q) {
    const int64_t *state = states + (static_cast<int64_t>(request) * questions + (q < questions ? q : 0)) *
                                        LRK_SELECT_STATE_FIELDS;
    prefix[q] = static_cast<uint32_t>(state[LRK_SELECT_PREFIX]);
    live[q] = q < counted && state[LRK_SELECT_NEED] > 0;
  }
  __syncthreads();
  const int64_t tile = static_cast<int64_t>(kHistThreads) * kHistItems;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * tile; base < n;
       base += static_cast<int64_t>(gridDim.x) * tile) {
    // Coalesced: element base + j * threads + thread.
    float v[kHistItems];
#pragma unroll
    for (int j = 0; j < kHistItems; ++j) {
      const int64_t e = base + static_cast<int64_t>(j) * kHistThreads + threadIdx.x;
      v[j] = e < n ? __ldcs(scores + e) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kHistItems; ++j) {
      const int64_t e = base + static_cast<int64_t>(j) * kHistThreads + threadIdx.x;
      if (e >= n) continue;
      const uint32_t key = order_key(v[j]);
      const uint32_t digit = (key >> shift) & digit_mask;
      if (round == 0) {
        atomicAdd(&local[digit], 1u);
      } else {
        const uint32_t high = key >> (shift + (round == 2 ? 8 : 12));
#pragma unroll
        for (int q = 0; q < LRK_SELECT_MAX_QUESTIONS; ++q)
          if (live[q] && high == prefix[q]) atomicAdd(&local[q * kBins + digit], 1u);
      }
    }
  }
  __syncthreads();
  uint32_t *out = hist + static_cast<int64_t>(request) * questions * kBins;
  for (int i = threadIdx.x; i < counted * kBins; i += kHistThreads) {
    const uint32_t c = local[i];
    if (c == 0) continue;
    if (round == 0) {
      for (int q = 0; q < questions; ++q) atomicAdd(&out[q * kBins + i], c);
    } else {
      atomicAdd(&out[i], c);
    }
  }
}

// One CTA per (request, question): sum the gathered histograms over ranks,
// find the bin of the k-th key and advance the state; after the last round,
// this rank's share.  gathered [world][requests][questions][kBins] u32.
__global__ void __launch_bounds__(kPickThreads) select_pick_kernel(const uint32_t *__restrict__ gathered, int world,
                                                                   int rank, int requests, int questions, int round,
                                                                   int64_t *__restrict__ states) {
  constexpr int kPer = kBins / kPickThreads;  // 16 bins per thread
  __shared__ unsigned long long warp_sums[kPickThreads / 32];
  __shared__ int chosen;
  __shared__ unsigned long long chosen_before;
  const int pair = blockIdx.x;  // request * questions + question
  int64_t *state = states + static_cast<int64_t>(pair) * LRK_SELECT_STATE_FIELDS;
  const int64_t stride = static_cast<int64_t>(requests) * questions * kBins;
  const int bins = round == 2 ? 256 : kBins;
  // Per-thread bins [t * kPer, (t + 1) * kPer): request-wide totals and this rank's counts.
  unsigned long long total[kPer], mine[kPer];
  unsigned long long sum = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int bin = threadIdx.x * kPer + i;
    unsigned long long t = 0, m = 0;
    if (bin < bins) {
      for (int w = 0; w < world; ++w) {
        const uint32_t c = gathered[w * stride + static_cast<int64_t>(pair) * kBins + bin];
        t += c;
        if (w == rank) m = c;
      }
    }
    total[i] = t;
    mine[i] = m;
    sum += t;
  }
  // Exclusive scan of the per-thread sums (bins are thread-major, so this is
  // the scan in bin order).
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long inclusive = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long other = __shfl_up_sync(0xffffffffu, inclusive, o);
    if (lane >= o) inclusive += other;
  }
  if (lane == 31) warp_sums[warp] = inclusive;
  if (threadIdx.x == 0) chosen = -1;
  __syncthreads();
  unsigned long long before_warp = 0, grand = 0;
  for (int w = 0; w < kPickThreads / 32; ++w) {
    if (w < warp) before_warp += warp_sums[w];
    grand += warp_sums[w];
  }
  const unsigned long long exclusive = before_warp + inclusive - sum;
  if (round == 0) {
    // The request-wide key count; k beyond it asks for every key.
    if (threadIdx.x == 0) {
      state[LRK_SELECT_TOTAL] = static_cast<int64_t>(grand);
      const int64_t k = state[LRK_SELECT_K];
      state[LRK_SELECT_NEED] = k < 0 ? 0 : lmin(k, static_cast<int64_t>(grand));
    }
    __syncthreads();
  }
  const int64_t need = state[LRK_SELECT_NEED];
  if (need <= 0) {
    // k = 0 (or an empty request): the share is 0.  need < 0 marks a failed
    // search, whose share stays -1.
    if (threadIdx.x == 0 && round == LRK_SELECT_ROUNDS - 1 && need == 0) state[LRK_SELECT_SHARE] = 0;
    return;
  }
  // The thread whose bins contain cumulative rank `need` finds the bin.
  const unsigned long long target = static_cast<unsigned long long>(need);
  if (exclusive < target && target <= exclusive + sum) {
    unsigned long long running = exclusive;
    for (int i = 0; i < kPer; ++i) {
      if (running + total[i] >= target) {
        chosen = threadIdx.x * kPer + i;
        chosen_before = running;
        break;
      }
      running += total[i];
    }
  }
  __syncthreads();
  const int bin = chosen;
  if (bin < 0) {
    // Histograms that do not hold `need` keys (inconsistent inputs across
    // ranks): no bin is chosen; the share reads -1 and the state stops.
    if (threadIdx.x == 0) {
      state[LRK_SELECT_NEED] = -1;
      state[LRK_SELECT_SHARE] = -1;
    }
    return;
  }
  // This rank's keys in bins below the chosen one.
  unsigned long long mine_below = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (threadIdx.x * kPer + i < bin) mine_below += mine[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine_below += __shfl_xor_sync(0xffffffffu, mine_below, o);
  __syncthreads();
  if (lane == 0) warp_sums[warp] = mine_below;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long local_below = 0;
    for (int w = 0; w < kPickThreads / 32; ++w) local_below += warp_sums[w];
    const int width = round == 2 ? 8 : 12;
    state[LRK_SELECT_PREFIX] = static_cast<int64_t>((static_cast<uint64_t>(state[LRK_SELECT_PREFIX]) << width) |
                                                    static_cast<uint64_t>(bin));
    state[LRK_SELECT_BELOW] += static_cast<int64_t>(chosen_before);
    state[LRK_SELECT_LOCAL_BELOW] += static_cast<int64_t>(local_below);
    const int64_t remaining = need - static_cast<int64_t>(chosen_before);
    state[LRK_SELECT_NEED] = remaining;
    if (round == LRK_SELECT_ROUNDS - 1) {
      // Ties at the k-th key: lower ranks' ties come first (index order).
      int64_t ties_before = 0, my_ties = 0;
      for (int w = 0; w < world; ++w) {
        const int64_t c = gathered[w * stride + static_cast<int64_t>(pair) * kBins + bin];
        if (w < rank) ties_before += c;
        if (w == rank) my_ties = c;
      }
      const int64_t take = lmax(0, lmin(remaining - ties_before, my_ties));
      state[LRK_SELECT_SHARE] = state[LRK_SELECT_LOCAL_BELOW] + take;
    }
  }
}

}  // namespace
}  // namespace lrk

using namespace lrk;

extern "C" int lrk_select_histogram(const float *const *scores, const int64_t *counts, int64_t requests,
                                    int64_t questions, int round, const int64_t *states, uint32_t *histograms,
                                    lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(requests >= 0 && questions >= 1 && questions <= LRK_SELECT_MAX_QUESTIONS,
              "questions must be in [1, LRK_SELECT_MAX_QUESTIONS]");
  LRK_REQUIRE(round >= 0 && round < LRK_SELECT_ROUNDS, "round out of range");
  if (requests == 0) return LRK_OK;
  LRK_REQUIRE(scores && counts && states && histograms, "null pointer");
  for (int64_t r = 0; r < requests; ++r) {
    LRK_REQUIRE(counts[r] >= 0, "negative score count");
    LRK_REQUIRE(counts[r] == 0 || scores[r] != nullptr, "null score table");
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t hist_bytes = static_cast<size_t>(requests) * questions * kBins * sizeof(uint32_t);
  cudaError_t e = cudaMemsetAsync(histograms, 0, hist_bytes, s);
  if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  const int counted = round == 0 ? 1 : static_cast<int>(questions);
  const int shared = counted * kBins * static_cast<int>(sizeof(uint32_t));
  if (shared > 48 * 1024) {
    e = cudaFuncSetAttribute(select_histogram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, shared);
    if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  }
  const int64_t tile = static_cast<int64_t>(kHistThreads) * kHistItems;
  for (int64_t r0 = 0; r0 < requests; r0 += LRK_SELECT_MAX_REQUESTS) {
    const int batch = static_cast<int>(std::min<int64_t>(LRK_SELECT_MAX_REQUESTS, requests - r0));
    RequestTable table{};
    int64_t longest = 0;
    for (int i = 0; i < batch; ++i) {
      table.scores[i] = scores[r0 + i];
      table.n[i] = counts[r0 + i];
      longest = std::max(longest, counts[r0 + i]);
    }
    if (longest == 0) continue;
    // About two resident CTAs per SM over the batch.
    const int64_t want = std::max<int64_t>(1, 2 * sm_count() / batch);
    const unsigned tiles = static_cast<unsigned>(std::min<int64_t>(ceil_div(longest, tile), want));
    select_histogram_kernel<<<dim3(tiles, batch), kHistThreads, shared, s>>>(
        table, static_cast<int>(r0), static_cast<int>(questions), round, states, histograms);
    const int status = launch_status("lrk_select_histogram");
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
}

extern "C" int lrk_select_pick(const uint32_t *gathered, int64_t world, int64_t rank, int64_t requests,
                               int64_t questions, int round, int64_t *states, lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(world >= 1 && rank >= 0 && rank < world, "rank out of range");
  LRK_REQUIRE(requests >= 0 && questions >= 1 && questions <= LRK_SELECT_MAX_QUESTIONS,
              "questions must be in [1, LRK_SELECT_MAX_QUESTIONS]");
  LRK_REQUIRE(round >= 0 && round < LRK_SELECT_ROUNDS, "round out of range");
  if (requests == 0) return LRK_OK;
  LRK_REQUIRE(gathered && states, "null pointer");
  LRK_REQUIRE(requests * questions <= INT32_MAX, "too many questions");
  select_pick_kernel<<<static_cast<unsigned>(requests * questions), kPickThreads, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(gathered, static_cast<int>(world),
                                                                 static_cast<int>(rank), static_cast<int>(requests),
                                                                 static_cast<int>(questions), round, states);
  return launch_status("lrk_select_pick");
}
