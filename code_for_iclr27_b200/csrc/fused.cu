// Fused temporal scoring of liblrk: candidate risk straight from logits.
//
// The reference scores one head per call in two operators
// (csrc/scoring.cu:32-128): temporal_probabilities writes every fp32
// probability of a [window, groups, length] chunk, temporal_risk reads the
// candidate columns back.  Here the probabilities never reach HBM:
//
//   visibility     one CTA per segment: when the segment's key positions
//   kernel         are non-decreasing, each query's visible keys are a
//                  prefix; its length replaces the per-key position compare
//                  in the stats kernel (-1: compare positions).
//   stats kernel   one CTA per (segment, query, group) row: the exact row
//                  statistics of rows.cuh (max, denominator, value projection,
//                  in the reference's operation order), written to a small
//                  workspace.
//   risk kernel    one CTA per (segment, tile of 256 candidates): each thread
//                  owns one candidate column, walks every query and group,
//                  recomputes the reference's probability w / denominator for
//                  its column only, folds the margin drop
//                  sum_g p/max(1-p,eps) * (pv - op) into a running min / max /
//                  non-finite flag, and ends with the float64 risk.
//
// Every step repeats the reference operators' arithmetic in the same order
// (this file is compiled with --fmad=false), so the scores are bit-identical
// to temporal_probabilities + temporal_risk + the running maximum over query
// chunks (scoring.py:179-195): per-chunk risks are max(R(min), R(max)) of a
// convex R, so the maximum over chunks is the risk over all queries.
// Many (layer, head) segments go in one launch: their descriptors travel as a
// kernel parameter (up to kMaxScoreSegments per launch).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "common.cuh"
#include "rows.cuh"

namespace lrk {
namespace {

constexpr int kMaxScoreSegments = 48;
constexpr int kRiskThreads = 256;
constexpr int kQueryLanes = kRiskThreads / 32;
constexpr int kMaxGroups = 8;

struct ScoreTableParam {
  lrk_score_segment segment[kMaxScoreSegments];
  // Probability stash (risk from stored candidate probabilities): segment
  // i's rows start at stash + stash_offset[i], each row
  // stash_stride(candidates) floats.
  int64_t stash_offset[kMaxScoreSegments];
  int count;
};

// Floats per stashed row: the candidate count rounded up to 32 (128-byte
// rows: every row starts 16-byte aligned for 4-candidate vector copies, and
// the last tile of up to 32 candidates ends inside its row).
__host__ __device__ __forceinline__ int64_t stash_stride(int64_t candidates) { return (candidates + 31) & ~int64_t{31}; }

constexpr int kVisibilityThreads = 1024;

// One CTA per segment.  If key_positions[0 .. length) is non-decreasing (and
// free of NaN), visible[(segment * window) + q] = the number of keys with
// position <= the query's position (they are a prefix); otherwise -1.
// Every kVisibilitySample-th key position sits in shared memory, so a query's
// search takes a few shared-memory steps and one short search of global
// memory (the sortedness check's loads left the positions in L2).
constexpr int kVisibilitySample = 64;
constexpr int kVisibilitySamples = 2048;  // rows up to 131,072 keys use the samples

__global__ void __launch_bounds__(kVisibilityThreads) visibility_kernel(ScoreTableParam table,
                                                                        const int64_t *__restrict__ qpos, int window,
                                                                        int32_t *__restrict__ visible,
                                                                        int64_t segment_base) {
  __shared__ float samples[kVisibilitySamples];
  const lrk_score_segment &seg = table.segment[blockIdx.x];
  const float *kpos = seg.key_positions;
  const int64_t n = seg.length;
  // Non-decreasing and free of NaN; eight elements per thread per round, all
  // loads of a round issued before the comparisons.
  int ordered = 1;
  constexpr int kUnroll = 8;
  for (int64_t base = threadIdx.x; base < n; base += static_cast<int64_t>(kVisibilityThreads) * kUnroll) {
    float here[kUnroll], next[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t p = base + static_cast<int64_t>(u) * kVisibilityThreads;
      here[u] = p < n ? __ldg(kpos + p) : 0.0f;
      next[u] = p + 1 < n ? __ldg(kpos + p + 1) : INFINITY;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t p = base + static_cast<int64_t>(u) * kVisibilityThreads;
      if (p < n && (!(here[u] == here[u]) || !(here[u] <= next[u]))) ordered = 0;
    }
  }
  const int64_t sampled = (n + kVisibilitySample - 1) / kVisibilitySample;
  const bool use_samples = sampled <= kVisibilitySamples;
  if (use_samples)
    for (int64_t j = threadIdx.x; j < sampled; j += kVisibilityThreads) samples[j] = __ldg(kpos + j * kVisibilitySample);
  ordered = __syncthreads_and(ordered);
  int32_t *out = visible + (segment_base + blockIdx.x) * window;
  for (int q = threadIdx.x; q < window; q += kVisibilityThreads) {
    int64_t count = -1;
    if (ordered) {
      const float position = static_cast<float>(qpos[q]);
      int64_t lo = 0, hi = n;  // first key with position > the query's
      if (use_samples && sampled > 0) {
        // The last sample at or below the position bounds the search window.
        int slo = 0, shi = static_cast<int>(sampled);  // first sample > position
        while (slo < shi) {
          const int mid = (slo + shi) / 2;
          if (samples[mid] <= position) slo = mid + 1; else shi = mid;
        }
        if (slo == 0) {
          hi = 0;
        } else {
          lo = static_cast<int64_t>(slo - 1) * kVisibilitySample + 1;
          hi = lmin(n, static_cast<int64_t>(slo) * kVisibilitySample);
        }
      }
      while (lo < hi) {
        const int64_t mid = (lo + hi) / 2;
        if (__ldg(kpos + mid) <= position) lo = mid + 1; else hi = mid;
      }
      count = lo;
    }
    out[q] = static_cast<int32_t>(count);
  }
}

// One CTA per (segment, query, group) row: its exact statistics (rows.cuh).
// stats[(segment * window + query) * groups + group] = (max, denominator, projection).
// visible may be null (every row compares key positions).  With `stash`, the
// row's candidate-column probabilities are stored there (risk_stash_kernel
// reads them).
//
// CTAs start in grid order (x, then y), so the CTA of flattened row g asks L2
// for the row `ahead` places later (a whole row, one bulk prefetch, when the
// rows are 16-byte aligned): its pass A then reads from L2.
template <typename T, int MODE>
__global__ void __launch_bounds__(rows::kLanes, 3) stats_kernel(ScoreTableParam table, const int64_t *__restrict__ qpos,
                                                             int groups, float scale, float3 *__restrict__ stats,
                                                             const int32_t *__restrict__ visible,
                                                             int64_t segment_base, int64_t rows_per_segment,
                                                             int64_t ahead, float *__restrict__ stash) {
  extern __shared__ __align__(16) unsigned char stage[];
  __shared__ float scratch[rows::kLanes];
  const int64_t row = blockIdx.x;
  const int si = blockIdx.y;
  if (MODE == rows::kPacked && threadIdx.x == 0 && ahead > 0) {
    const int64_t later = si * rows_per_segment + row + ahead;
    if (later < rows_per_segment * gridDim.y) {
      const lrk_score_segment &next = table.segment[later / rows_per_segment];
      const T *start = static_cast<const T *>(next.logits) + (later % rows_per_segment) * next.logits_stride;
      const uint32_t bytes = static_cast<uint32_t>(lmin(next.length * static_cast<int64_t>(sizeof(T)), INT32_MAX)) & ~15u;
      if (bytes > 0) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(start), "r"(bytes) : "memory");
    }
  }
  const lrk_score_segment &seg = table.segment[si];
  const int group = static_cast<int>(row % groups);
  const int64_t query = row / groups;
  const int64_t window = rows_per_segment / groups;
  const rows::Visibility sees{seg.key_positions, static_cast<float>(qpos[query]),
                              visible != nullptr ? visible[(segment_base + si) * window + query] : -1};
  rows::CandidateOut candidates{nullptr, seg.first, seg.last};
  if (stash != nullptr) candidates.out = stash + table.stash_offset[si] + row * stash_stride(seg.last - seg.first);
  const rows::RowResult r = rows::row_statistics<T, MODE>(
      static_cast<const T *>(seg.logits) + row * seg.logits_stride, seg.length, sees,
      seg.projected_values + group * seg.projected_stride, scale, nullptr, stage, scratch, candidates);
  if (threadIdx.x == 0)
    stats[(segment_base + si) * rows_per_segment + row] = make_float3(r.maximum, r.denominator, r.projection);
}

template <typename K>
int allow_shared(K kernel, int64_t bytes) {
  if (bytes <= 48 * 1024) return LRK_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  return e == cudaSuccess ? LRK_OK : fail(LRK_ERR_CUDA, cudaGetErrorString(e));
}

// Every row of every segment starts on a 16-byte boundary.
template <typename T>
bool rows_aligned(const ScoreTableParam &table, int n) {
  for (int i = 0; i < n; ++i)
    if (!aligned(table.segment[i].logits, 16) ||
        (table.segment[i].logits_stride * static_cast<int64_t>(sizeof(T))) % 16 != 0)
      return false;
  return true;
}

template <typename T>
int launch_stats(const ScoreTableParam &table, int n, const int64_t *qpos, int window, int groups, float scale,
                 float3 *stats, int32_t *visible, int64_t s0, int64_t max_length, float *stash,
                 cudaStream_t stream) {
  if (visible != nullptr) {
    visibility_kernel<<<n, kVisibilityThreads, 0, stream>>>(table, qpos, window, visible, s0);
    const int status = launch_status("lrk_temporal_scores visibility");
    if (status != LRK_OK) return status;
  }
  const int64_t rows_per_segment = static_cast<int64_t>(window) * groups;
  const dim3 grid(static_cast<unsigned>(rows_per_segment), n);
  const int mode = rows::choose_stage<T>(max_length, rows_aligned<T>(table, n));
  const int64_t bytes = rows::staged_bytes<T>(mode, max_length);
  int status = LRK_OK;
  if (mode == rows::kWeights) {
    if ((status = allow_shared(stats_kernel<T, rows::kWeights>, bytes)) != LRK_OK) return status;
    stats_kernel<T, rows::kWeights><<<grid, rows::kLanes, bytes, stream>>>(table, qpos, groups, scale, stats,
                                                                           visible, s0, rows_per_segment, 0, stash);
  } else if (mode == rows::kBits) {
    if ((status = allow_shared(stats_kernel<T, rows::kBits>, bytes)) != LRK_OK) return status;
    stats_kernel<T, rows::kBits><<<grid, rows::kLanes, bytes, stream>>>(table, qpos, groups, scale, stats, visible,
                                                                        s0, rows_per_segment, 0, stash);
  } else if (mode == rows::kPacked) {
    if constexpr (sizeof(T) == 2) {
      if ((status = allow_shared(stats_kernel<T, rows::kPacked>, bytes)) != LRK_OK) return status;
      // Two waves of 3 CTAs per SM ahead.
      const int64_t ahead = 6 * static_cast<int64_t>(sm_count());
      stats_kernel<T, rows::kPacked><<<grid, rows::kLanes, bytes, stream>>>(table, qpos, groups, scale, stats,
                                                                            visible, s0, rows_per_segment, ahead,
                                                                            stash);
    }
  } else {
    stats_kernel<T, rows::kStream><<<grid, rows::kLanes, 0, stream>>>(table, qpos, groups, scale, stats, visible,
                                                                      s0, rows_per_segment, 0, stash);
  }
  return launch_status("lrk_temporal_scores statistics");
}

__device__ __forceinline__ double softplus64(double value) { return value > 20.0 ? value : log1p(exp(value)); }

// csrc/scoring.cu:68-75, same operation order.
__device__ __forceinline__ double risk64(double margin, double probability, double base_softplus, float drop) {
  const double compared = __dsub_rn(margin, static_cast<double>(drop));
  const double kl = __dadd_rn(__dsub_rn(__dmul_rn(probability, __dsub_rn(margin, compared)), base_softplus),
                              softplus64(compared));
  return fmax(0.0, kl);
}

// Number of queries per chunk of a segment's running maximum.
__device__ __forceinline__ int chunk_queries(const lrk_score_segment &seg, int window) {
  return seg.query_chunk > 0 && seg.query_chunk < window ? static_cast<int>(seg.query_chunk) : window;
}

// Margin terms shared by every chunk score: m, sigmoid(m), softplus(m).
struct MarginTerms {
  double m, probability, base_softplus;
};
__device__ __forceinline__ MarginTerms margin_terms(const float *margin) {
  const double m = static_cast<double>(margin[0]);
  return {m, 1.0 / (1.0 + exp(-m)), softplus64(m)};
}

// One chunk's score from its drop range (csrc/scoring.cu:68-128): NaN when a
// drop was not finite, else max(R(min), R(max)) rounded to float.
__device__ __forceinline__ float chunk_score(const MarginTerms &t, bool nonfinite, float minimum, float maximum) {
  if (nonfinite) return NAN;
  return static_cast<float>(fmax(risk64(t.m, t.probability, t.base_softplus, minimum),
                                 risk64(t.m, t.probability, t.base_softplus, maximum)));
}

// Order-preserving int image of a float (for float min / max through integer
// atomics): non-negative floats keep their bits, negative ones flip the
// magnitude bits, so signed comparison of the images orders the floats.  NaN
// never reaches it (a non-finite drop is flagged instead).
__device__ __forceinline__ int ordered_key(float f) {
  const int bits = __float_as_int(f);
  return bits >= 0 ? bits : bits ^ 0x7fffffff;
}
__device__ __forceinline__ float from_ordered_key(int key) {
  return __int_as_float(key >= 0 ? key : key ^ 0x7fffffff);
}

// Query chunks one pass of risk_vec_kernel folds in shared memory, and the
// candidates of one of its CTAs (16: a layer's ~2k candidates per head give
// ~1k CTAs, enough to fill every SM).
constexpr int kRiskChunks = 8;
constexpr int kRiskTile = 16;

// The running maximum over chunks, torch.maximum's semantics (NaN wins).
__device__ __forceinline__ float running_max(float a, float b) { return isnan(a) || isnan(b) ? NAN : fmaxf(a, b); }

// A CTA covers 32 consecutive candidate columns (one warp row, 64-byte bf16
// reads per logits row) with kQueryLanes query lanes: lane y walks queries
// y, y + kQueryLanes, ...  The lanes' min / max / non-finite flags meet in
// shared memory (min and max are order-free), then lane 0 computes the risk.
template <typename T, int G>
__global__ void __launch_bounds__(kRiskThreads) risk_kernel(ScoreTableParam table, const int64_t *__restrict__ qpos,
                                                            int window, int groups, float scale,
                                                            const float3 *__restrict__ stats,
                                                            int64_t segment_base, const float *__restrict__ margin,
                                                            float epsilon) {
  using D = rows::Dtype<T>;
  extern __shared__ float4 shared_stats[];  // [window * groups] (max, denominator, projection, query position)
  __shared__ float lane_min[kQueryLanes][33], lane_max[kQueryLanes][33];
  __shared__ int lane_bad[kQueryLanes][33];
  const int si = blockIdx.y;
  const lrk_score_segment &seg = table.segment[si];
  const int ng = G > 0 ? G : groups;
  const int tid = threadIdx.y * 32 + threadIdx.x;
  for (int i = tid; i < window * ng; i += kRiskThreads) {
    const float3 st = stats[(segment_base + si) * window * ng + i];
    shared_stats[i] = make_float4(st.x, st.y, st.z, static_cast<float>(qpos[i / ng]));
  }
  __syncthreads();
  const int64_t count = seg.last - seg.first;
  const int64_t candidate = static_cast<int64_t>(blockIdx.x) * 32 + threadIdx.x;
  const bool active = candidate < count;
  const int64_t column = seg.first + (active ? candidate : 0);
  const int64_t stride = seg.logits_stride;
  const float key_position = active ? __ldg(seg.key_positions + column) : 0.0f;
  float pv[G > 0 ? G : kMaxGroups];
#pragma unroll
  for (int g = 0; g < (G > 0 ? G : kMaxGroups); ++g)
    pv[g] = active && g < ng ? __ldg(seg.projected_values + g * seg.projected_stride + column) : 0.0f;
  const typename D::Bits *base = static_cast<const typename D::Bits *>(seg.logits) + column;
  const int chunk = chunk_queries(seg, window);
  const bool leader = threadIdx.y == 0 && active;
  MarginTerms terms{};
  if (leader) terms = margin_terms(margin);
  float result = 0.0f;
  for (int c0 = 0; c0 < window; c0 += chunk) {
    const int c1 = min(window, c0 + chunk);
    float minimum = INFINITY, maximum = -INFINITY;
    int nonfinite = 0;
    if (active) {
#pragma unroll 2
      for (int q = c0 + threadIdx.y; q < c1; q += kQueryLanes) {
        float drop = 0.0f;
#pragma unroll
        for (int g = 0; g < (G > 0 ? G : kMaxGroups); ++g) {
          if (g < ng) {
            const float4 st = shared_stats[q * ng + g];
            const float rounded = D::to_float(
                D::round(D::to_float(__ldg(base + (static_cast<int64_t>(q) * ng + g) * stride)), scale));
            const float x = key_position <= st.w ? rounded : -INFINITY;
            const float probability = __fdiv_rn(expf(__fsub_rn(x, st.x)), st.y);
            const float ratio = __fdiv_rn(probability, fmaxf(__fsub_rn(1.0f, probability), epsilon));
            drop = __fadd_rn(drop, __fmul_rn(ratio, __fsub_rn(pv[g], st.z)));
          }
        }
        nonfinite |= !isfinite(drop);
        minimum = fminf(minimum, drop);
        maximum = fmaxf(maximum, drop);
      }
    }
    lane_min[threadIdx.y][threadIdx.x] = minimum;
    lane_max[threadIdx.y][threadIdx.x] = maximum;
    lane_bad[threadIdx.y][threadIdx.x] = nonfinite;
    __syncthreads();
    if (leader) {
      for (int y = 1; y < kQueryLanes; ++y) {
        minimum = fminf(minimum, lane_min[y][threadIdx.x]);
        maximum = fmaxf(maximum, lane_max[y][threadIdx.x]);
        nonfinite |= lane_bad[y][threadIdx.x];
      }
      const float score = chunk_score(terms, nonfinite != 0, minimum, maximum);
      result = c0 == 0 ? score : running_max(result, score);
    }
    __syncthreads();
  }
  if (leader) seg.scores[candidate] = result;
}

// Vectorised risk for 16-bit logits in 16-byte aligned rows.  A CTA covers
// kRiskTile consecutive candidate columns from a 16-byte boundary; thread (tx, ty)
// owns C consecutive candidates (one C * 2-byte load per logits row, C = 8, 4
// or 2) and
// walks queries ty, ty + TY, ..., with the next query's rows loaded while the
// current one computes.  Candidates in pairs share every per-row operand, so
// the elementwise steps run as float2 operations, and the first division uses
// the row's correctly rounded reciprocal (rows::divide2).  Per candidate the
// operations and their order are those of risk_kernel.
// Four CTAs per SM (64 registers, a few bytes of spills): the kernel waits on
// its logits loads, and the fourth CTA hides more of that than the spills cost
// (measured: 483 instead of 489 us per configs[1] layer call with three).
template <typename T, int G, int C>
__global__ void __launch_bounds__(kRiskThreads, 4) risk_vec_kernel(ScoreTableParam table,
                                                                const int64_t *__restrict__ qpos, int window,
                                                                float scale, const float3 *__restrict__ stats,
                                                                int64_t segment_base,
                                                                const float *__restrict__ margin, float epsilon) {
  using D = rows::Dtype<T>;
  using P = rows::Packed<T>;
  using Bits = typename D::Bits;
  using Vec = typename std::conditional<C == 8, uint4, typename std::conditional<C == 4, uint2, uint32_t>::type>::type;
  constexpr int TX = kRiskTile / C, TY = kRiskThreads / TX;
  constexpr int kTile = kRiskTile;
  extern __shared__ float4 shared_stats[];  // [window * G] (max, denominator, projection, query position)
  float *reciprocal = reinterpret_cast<float *>(shared_stats + window * G);  // [window * G]
  // Per (chunk of this pass, candidate): order-preserving keys of the drop
  // range and a non-finite flag, folded with integer atomics (order-free).
  __shared__ int cell_min[kRiskChunks][kTile], cell_max[kRiskChunks][kTile];
  __shared__ int cell_bad[kRiskChunks][kTile];
  const lrk_score_segment &seg = table.segment[blockIdx.y];
  const int64_t tile = (seg.first & ~int64_t{7}) + static_cast<int64_t>(blockIdx.x) * kTile;
  if (tile >= seg.last) return;  // the whole CTA: nothing of this segment here
  for (int i = threadIdx.x; i < window * G; i += kRiskThreads) {
    const float3 st = stats[(segment_base + blockIdx.y) * window * G + i];
    shared_stats[i] = make_float4(st.x, st.y, st.z, static_cast<float>(qpos[i / G]));
    reciprocal[i] = __frcp_rn(st.y);
  }
  __syncthreads();
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
  const int64_t col0 = tile + tx * C;
  const bool full = col0 + C <= seg.length;
  float key_position[C], pv[G][C];
#pragma unroll
  for (int j = 0; j < C; ++j) {
    const bool inside = col0 + j < seg.length;
    key_position[j] = inside ? __ldg(seg.key_positions + col0 + j) : INFINITY;
#pragma unroll
    for (int g = 0; g < G; ++g)
      pv[g][j] = inside ? __ldg(seg.projected_values + g * seg.projected_stride + col0 + j) : 0.0f;
  }
  const Bits *base = static_cast<const Bits *>(seg.logits) + col0;
  auto load = [&](int q, int g) -> Vec {
    const Bits *row = base + (static_cast<int64_t>(q) * G + g) * seg.logits_stride;
    if (full) return __ldg(reinterpret_cast<const Vec *>(row));
    uint32_t w[C / 2];
#pragma unroll
    for (int i = 0; i < C / 2; ++i) {
      const uint32_t a = col0 + 2 * i < seg.length ? row[2 * i] : 0u;
      const uint32_t b = col0 + 2 * i + 1 < seg.length ? row[2 * i + 1] : 0u;
      w[i] = a | (b << 16);
    }
    if constexpr (C == 8) return make_uint4(w[0], w[1], w[2], w[3]);
    else if constexpr (C == 4) return make_uint2(w[0], w[1]);
    else return w[0];
  };
  auto word_of = [](const Vec &v, int i) -> uint32_t {
    if constexpr (C == 8) return rows::word(v, i);
    else if constexpr (C == 4) return i == 0 ? v.x : v.y;
    else return v;
  };
  const float2 scale2 = make_float2(scale, scale), one2 = make_float2(1.0f, 1.0f);
  const int chunk = chunk_queries(seg, window);
  const int chunks = (window + chunk - 1) / chunk;
  const bool leader = threadIdx.x < kTile;
  float result = 0.0f;
  // Passes of up to kRiskChunks chunks: each thread walks its queries of the
  // pass, folding its candidates' drop range into the chunk's cells whenever
  // it leaves a chunk; one barrier, then the leaders score the pass's chunks.
  for (int c_first = 0; c_first < chunks; c_first += kRiskChunks) {
    const int c_last = min(chunks, c_first + kRiskChunks);
    for (int i = threadIdx.x; i < (c_last - c_first) * kTile; i += kRiskThreads) {
      cell_min[i / kTile][i % kTile] = ordered_key(INFINITY);
      cell_max[i / kTile][i % kTile] = ordered_key(-INFINITY);
      cell_bad[i / kTile][i % kTile] = 0;
    }
    __syncthreads();
    const int q_begin = c_first * chunk, q_end = min(window, c_last * chunk);
    float lo[C], hi[C];
    uint32_t bad = 0;
#pragma unroll
    for (int j = 0; j < C; ++j) {
      lo[j] = INFINITY;
      hi[j] = -INFINITY;
    }
    auto flush = [&](int c) {
#pragma unroll
      for (int j = 0; j < C; ++j) {
        atomicMin(&cell_min[c - c_first][tx * C + j], ordered_key(lo[j]));
        atomicMax(&cell_max[c - c_first][tx * C + j], ordered_key(hi[j]));
        lo[j] = INFINITY;
        hi[j] = -INFINITY;
      }
      if (bad) {
#pragma unroll
        for (int j = 0; j < C; ++j)
          if ((bad >> j) & 1u) cell_bad[c - c_first][tx * C + j] = 1;
      }
      bad = 0;
    };
    int current_chunk = -1;
    Vec current[G], next[G];
    if (q_begin + ty < q_end) {
#pragma unroll
      for (int g = 0; g < G; ++g) current[g] = load(q_begin + ty, g);
    }
    for (int q = q_begin + ty; q < q_end; q += TY) {
      if (q + TY < q_end) {
#pragma unroll
        for (int g = 0; g < G; ++g) next[g] = load(q + TY, g);
      }
      const int c = q / chunk;
      if (c != current_chunk) {
        if (current_chunk >= 0) flush(current_chunk);
        current_chunk = c;
      }
      const float query_position = shared_stats[q * G].w;
      float drop[C];
#pragma unroll
      for (int j = 0; j < C; ++j) drop[j] = 0.0f;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 st = shared_stats[q * G + g];
        rows::Divider divider;
        divider.b = st.y;
        divider.y = reciprocal[q * G + g];
        divider.fast = st.y >= 1.0f && st.y <= 4294967296.0f;
        const float2 minus_max = make_float2(-st.x, -st.x), minus_projection = make_float2(-st.z, -st.z);
#pragma unroll
        for (int i = 0; i < C / 2; ++i) {
          float2 x = P::unpack(P::round(rows::mul2_rn(P::unpack(word_of(current[g], i)), scale2)));
          if (!(key_position[2 * i] <= query_position)) x.x = -INFINITY;
          if (!(key_position[2 * i + 1] <= query_position)) x.y = -INFINITY;
          const float2 d = rows::add2_rn(x, minus_max);
          const float2 probability = rows::divide2(divider, make_float2(expf(d.x), expf(d.y)));
          const float2 rest = rows::add2_rn(one2, make_float2(-probability.x, -probability.y));
          const float2 ratio = make_float2(__fdiv_rn(probability.x, fmaxf(rest.x, epsilon)),
                                           __fdiv_rn(probability.y, fmaxf(rest.y, epsilon)));
          const float2 term = rows::mul2_rn(ratio, rows::add2_rn(make_float2(pv[g][2 * i], pv[g][2 * i + 1]),
                                                               minus_projection));
          // Scalar sums: a packed product feeding a packed sum may be fused.
          drop[2 * i] = __fadd_rn(drop[2 * i], term.x);
          drop[2 * i + 1] = __fadd_rn(drop[2 * i + 1], term.y);
        }
      }
#pragma unroll
      for (int j = 0; j < C; ++j) {
        bad |= static_cast<uint32_t>(!isfinite(drop[j])) << j;
        lo[j] = fminf(lo[j], drop[j]);
        hi[j] = fmaxf(hi[j], drop[j]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) current[g] = next[g];
    }
    if (current_chunk >= 0) flush(current_chunk);
    __syncthreads();
    if (leader) {
      const MarginTerms terms = margin_terms(margin);
      for (int c = c_first; c < c_last; ++c) {
        const float score = chunk_score(terms, cell_bad[c - c_first][threadIdx.x] != 0,
                                        from_ordered_key(cell_min[c - c_first][threadIdx.x]),
                                        from_ordered_key(cell_max[c - c_first][threadIdx.x]));
        result = c == 0 ? score : running_max(result, score);
      }
    }
    __syncthreads();  // cells free for the next pass
  }
  if (!leader) return;
  const int64_t column = tile + threadIdx.x;
  if (column < seg.first || column >= seg.last) return;
  seg.scores[column - seg.first] = result;
}

// Risk from stashed probabilities (the row statistics' pass C stored the
// probability of every candidate column of every row).  Per candidate and
// query, drop = sum over g, in order, of ratio * (pv[g] - projection[q, g])
// with ratio = p / max(1 - p, epsilon) -- the reference's drop
// (csrc/scoring.cu:68-128) from the same p its probabilities kernel produced
// -- then the drop range of each query chunk, its fp64 risk and the running
// maximum, exactly as risk_vec_kernel folds them.  This skips risk_vec's
// logits load, scale, rounding, mask, expf and first division per element.
// A CTA covers TILE candidates; thread (tx, ty) owns C consecutive
// candidates (one 4C-byte copy per stashed row; C = 4, or 2 for 8 groups to
// keep the registers in check) and walks queries ty, ty + TY, ...  Each
// thread streams its rows through its own kStashStages-slot ring in shared
// memory with cp.async, kStashStages - 1 queries ahead of the one it
// computes: the copies in flight hold no registers, so a CTA keeps
// 3 x 64 bytes per thread on the way from HBM (one query ahead in registers
// covered about one memory latency and left the kernel latency-bound); 2 x 64
// for 8 groups, whose projections take twice the shared memory, so that
// 3 CTAs still fit an SM at a 250-query window.  The launch picks TILE (32,
// 16 or 8) for the fewest waves of CTAs weighted by their length.
template <int G>
__host__ __device__ constexpr int stash_stages() {
  return G >= 8 ? 3 : 4;
}

template <int BYTES>
__device__ __forceinline__ void stage_async(void *dst, const void *src) {
  const auto to = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  if constexpr (BYTES == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(to), "l"(src) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(to), "l"(src), "n"(BYTES) : "memory");
}
__device__ __forceinline__ void stage_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int PENDING>
__device__ __forceinline__ void stage_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(PENDING) : "memory");
}

template <int G, int C>
__host__ __device__ constexpr size_t stash_ring_bytes() {
  return static_cast<size_t>(stash_stages<G>()) * G * kRiskThreads * C * sizeof(float);
}

template <int G, int C, int TILE>
__global__ void __launch_bounds__(kRiskThreads, 3) risk_stash_kernel(ScoreTableParam table,
                                                                  const float *__restrict__ stash, int window,
                                                                  const float3 *__restrict__ stats,
                                                                  int64_t segment_base,
                                                                  const float *__restrict__ margin,
                                                                  float epsilon) {
  using Vec = typename std::conditional<C == 4, float4, float2>::type;
  constexpr int TX = TILE / C, TY = kRiskThreads / TX, kStashStages = stash_stages<G>();
  // [kStashStages][G][kRiskThreads] vectors, then the projections [window * G].
  extern __shared__ __align__(16) unsigned char risk_shared[];
  Vec *ring = reinterpret_cast<Vec *>(risk_shared);
  float *projection = reinterpret_cast<float *>(risk_shared + stash_ring_bytes<G, C>());
  __shared__ int cell_min[kRiskChunks][TILE], cell_max[kRiskChunks][TILE];
  __shared__ int cell_bad[kRiskChunks][TILE];
  __shared__ float cell_risk[kRiskChunks][TILE][2];
  const lrk_score_segment &seg = table.segment[blockIdx.y];
  const int64_t count = seg.last - seg.first;
  const int64_t tile = static_cast<int64_t>(blockIdx.x) * TILE;
  if (tile >= count) return;  // the whole CTA: nothing of this segment here
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
  const int64_t col0 = tile + tx * C;  // candidate index of this thread's first candidate
  const int64_t stride = stash_stride(count);
  // Rows are padded to `stride` floats (a multiple of 32 >= the last tile's
  // end), so a vector past the last candidate stays inside the row (its
  // lanes are never scored).
  const float *base = stash + table.stash_offset[blockIdx.y] + col0;
  Vec *mine = ring + threadIdx.x;  // slot (s, g) at mine[(s * G + g) * kRiskThreads]
  const int chunk = chunk_queries(seg, window);
  const int chunks = (window + chunk - 1) / chunk;
  const bool leader = threadIdx.x < TILE;
  // A pass folds up to kRiskChunks query chunks; this thread walks its
  // queries q_first, q_first + TY, ... of the pass, `steps` of them.  One
  // commit group per step (empty past the last one), so group i is complete
  // once at most kStashStages - 2 later groups are pending.
  int q_first = 0, steps = 0;
  auto issue = [&](int step) {
    if (step < steps) {
      const int64_t row = static_cast<int64_t>(q_first + step * TY) * G;
      Vec *slot = mine + (step % kStashStages) * G * kRiskThreads;
#pragma unroll
      for (int g = 0; g < G; ++g) stage_async<sizeof(Vec)>(slot + g * kRiskThreads, base + (row + g) * stride);
    }
    stage_commit();
  };
  // The pass's first copies and its cells; the caller synchronises.
  auto start_pass = [&](int c_first) {
    const int c_last = min(chunks, c_first + kRiskChunks);
    const int q_end = min(window, c_last * chunk);
    q_first = c_first * chunk + ty;
    steps = q_first < q_end ? (q_end - q_first + TY - 1) / TY : 0;
#pragma unroll
    for (int s = 0; s < kStashStages - 1; ++s) issue(s);
    for (int i = threadIdx.x; i < (c_last - c_first) * TILE; i += kRiskThreads) {
      cell_min[i / TILE][i % TILE] = ordered_key(INFINITY);
      cell_max[i / TILE][i % TILE] = ordered_key(-INFINITY);
      cell_bad[i / TILE][i % TILE] = 0;
    }
  };
  // The first pass's copies are on their way while the projections and this
  // thread's projected values load.
  start_pass(0);
  float pv[G][C];
#pragma unroll
  for (int j = 0; j < C; ++j) {
#pragma unroll
    for (int g = 0; g < G; ++g)
      pv[g][j] = col0 + j < count ? __ldg(seg.projected_values + g * seg.projected_stride + seg.first + col0 + j)
                                  : 0.0f;
  }
  for (int i = threadIdx.x; i < window * G; i += kRiskThreads)
    projection[i] = stats[(segment_base + blockIdx.y) * window * G + i].z;
  __syncthreads();
  float result = 0.0f;
  for (int c_first = 0; c_first < chunks; c_first += kRiskChunks) {
    const int c_last = min(chunks, c_first + kRiskChunks);
    if (c_first > 0) {
      start_pass(c_first);
      __syncthreads();
    }
    float lo[C], hi[C];
    uint32_t bad = 0;
#pragma unroll
    for (int j = 0; j < C; ++j) {
      lo[j] = INFINITY;
      hi[j] = -INFINITY;
    }
    auto flush = [&](int c) {
#pragma unroll
      for (int j = 0; j < C; ++j) {
        atomicMin(&cell_min[c - c_first][tx * C + j], ordered_key(lo[j]));
        atomicMax(&cell_max[c - c_first][tx * C + j], ordered_key(hi[j]));
        lo[j] = INFINITY;
        hi[j] = -INFINITY;
      }
      if (bad) {
#pragma unroll
        for (int j = 0; j < C; ++j)
          if ((bad >> j) & 1u) cell_bad[c - c_first][tx * C + j] = 1;
      }
      bad = 0;
    };
    int current_chunk = -1;
    for (int step = 0; step < steps; ++step) {
      stage_wait<kStashStages - 2>();
      // A thread reads only the slots its own copies filled; the slot the
      // next issue refills was read (and its values used) one step earlier.
      const Vec *slot = mine + (step % kStashStages) * G * kRiskThreads;
      Vec current[G];
#pragma unroll
      for (int g = 0; g < G; ++g) current[g] = slot[g * kRiskThreads];
      issue(step + kStashStages - 1);
      const int q = q_first + step * TY;
      const int c = q / chunk;
      if (c != current_chunk) {
        if (current_chunk >= 0) flush(current_chunk);
        current_chunk = c;
      }
      float drop[C];
#pragma unroll
      for (int j = 0; j < C; ++j) drop[j] = 0.0f;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float op = projection[q * G + g];
        const float *p = reinterpret_cast<const float *>(&current[g]);
#pragma unroll
        for (int j = 0; j < C; ++j) {
          const float ratio = __fdiv_rn(p[j], fmaxf(__fsub_rn(1.0f, p[j]), epsilon));
          drop[j] = __fadd_rn(drop[j], __fmul_rn(ratio, __fsub_rn(pv[g][j], op)));
        }
      }
#pragma unroll
      for (int j = 0; j < C; ++j) {
        bad |= static_cast<uint32_t>(!isfinite(drop[j])) << j;
        lo[j] = fminf(lo[j], drop[j]);
        hi[j] = fmaxf(hi[j], drop[j]);
      }
    }
    if (current_chunk >= 0) flush(current_chunk);
    __syncthreads();
    // The fp64 risk of each end of each (chunk, candidate) drop range on its
    // own thread, rounded to float: rounding is monotonic, so the larger of
    // the two rounded risks is chunk_score's rounded larger risk.
    const int jobs = (c_last - c_first) * TILE * 2;
    if (threadIdx.x < jobs) {
      const MarginTerms terms = margin_terms(margin);
      for (int i = threadIdx.x; i < jobs; i += kRiskThreads) {
        const int c = i / (2 * TILE), k = (i >> 1) % TILE;
        const int key = (i & 1) ? cell_max[c][k] : cell_min[c][k];
        cell_risk[c][k][i & 1] =
            static_cast<float>(risk64(terms.m, terms.probability, terms.base_softplus, from_ordered_key(key)));
      }
    }
    __syncthreads();
    if (leader) {
      for (int c = c_first; c < c_last; ++c) {
        const float score = cell_bad[c - c_first][threadIdx.x] != 0
                                ? NAN
                                : fmaxf(cell_risk[c - c_first][threadIdx.x][0], cell_risk[c - c_first][threadIdx.x][1]);
        result = c == 0 ? score : running_max(result, score);
      }
    }
    if (c_last < chunks) __syncthreads();  // cells free for the next pass
  }
  if (!leader) return;
  const int64_t candidate = tile + threadIdx.x;
  if (candidate < count) seg.scores[candidate] = result;
}

template <int G, int TILE>
int launch_risk_stash_tile(const ScoreTableParam &table, int n, const float *stash, int window, const float3 *stats,
                           int64_t s0, const float *margin, float epsilon, int64_t max_candidates,
                           cudaStream_t stream) {
  constexpr int C = G >= 8 ? 2 : 4;
  const size_t shared = stash_ring_bytes<G, C>() + static_cast<size_t>(window) * G * sizeof(float);
  auto kernel = risk_stash_kernel<G, C, TILE>;
  if (shared > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
    if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  }
  const dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, ceil_div(max_candidates, TILE))), n);
  kernel<<<grid, kRiskThreads, shared, stream>>>(table, stash, window, stats, s0, margin, epsilon);
  return launch_status("lrk_temporal_scores risk from stashed probabilities");
}

// Candidates per CTA: a CTA's length grows with its tile plus a fixed part
// (the projections it stages, the cells, the fp64 scores of its leaders),
// taken as 8 candidates' worth; the tile with the fewest waves x length wins
// (3 CTAs per SM).  A configs[1] layer (8 x 2080 candidates) takes 16: 3
// waves of 1040 CTAs instead of 2 of 520 with the second one 17 % full.
inline int stash_tile(int64_t max_candidates, int n) {
#ifdef LRK_STASH_TILE
  return LRK_STASH_TILE;
#endif
  const int64_t slots = 3 * static_cast<int64_t>(sm_count());
  int best = 32;
  int64_t best_cost = INT64_MAX;
  for (int tile : {32, 16, 8}) {
    const int64_t waves = ceil_div(ceil_div(max_candidates, tile) * n, slots);
    const int64_t cost = waves * (tile + 8);
    if (cost < best_cost) best = tile, best_cost = cost;
  }
  return best;
}

template <int G>
int launch_risk_stash(const ScoreTableParam &table, int n, const float *stash, int window, const float3 *stats,
                      int64_t s0, const float *margin, float epsilon, int64_t max_candidates, cudaStream_t stream) {
  switch (stash_tile(max_candidates, n)) {
    case 8: return launch_risk_stash_tile<G, 8>(table, n, stash, window, stats, s0, margin, epsilon, max_candidates,
                                                stream);
    case 16: return launch_risk_stash_tile<G, 16>(table, n, stash, window, stats, s0, margin, epsilon, max_candidates,
                                                  stream);
    default: return launch_risk_stash_tile<G, 32>(table, n, stash, window, stats, s0, margin, epsilon,
                                                  max_candidates, stream);
  }
}

template <typename T, int G, int C>
int launch_risk_vec(const ScoreTableParam &table, int n, const int64_t *qpos, int window, float scale,
                    const float3 *stats, int64_t s0, const float *margin, float epsilon, int64_t max_span,
                    cudaStream_t stream) {
  const size_t shared = static_cast<size_t>(window) * G * (sizeof(float4) + sizeof(float));
  auto kernel = risk_vec_kernel<T, G, C>;
  if (shared > 16 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
    if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  }
  const dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, ceil_div(max_span, kRiskTile))), n);
  kernel<<<grid, kRiskThreads, shared, stream>>>(table, qpos, window, scale, stats, s0, margin, epsilon);
  return launch_status("lrk_temporal_scores");
}

// The risk kernels of one table of segments (row statistics already in
// stats[(s0 + segment) * window * groups + row]).
template <typename T>
int launch_risk(const ScoreTableParam &table, int n, const int64_t *qpos, int window, int groups, float scale,
                const float *margin, float epsilon, const float3 *stats, int64_t s0, cudaStream_t stream) {
  int64_t max_candidates = 0, max_span = 0;
  for (int i = 0; i < n; ++i) {
    max_candidates = std::max<int64_t>(max_candidates, table.segment[i].last - table.segment[i].first);
    max_span = std::max<int64_t>(max_span, table.segment[i].last - (table.segment[i].first & ~int64_t{7}));
  }
  if constexpr (sizeof(T) == 2) {
    if (rows_aligned<T>(table, n) && window * groups * 20 <= 200 * 1024 &&
        (groups == 1 || groups == 2 || groups == 4 || groups == 8)) {
      const auto args = std::make_tuple(table, n, qpos, window, scale, stats, s0, margin, epsilon, max_span, stream);
      // Candidates per thread: G * C <= 16 keeps the per-thread state near 64 registers.
      return groups == 1   ? std::apply(launch_risk_vec<T, 1, 8>, args)
             : groups == 2 ? std::apply(launch_risk_vec<T, 2, 4>, args)
             : groups == 4 ? std::apply(launch_risk_vec<T, 4, 4>, args)
                           : std::apply(launch_risk_vec<T, 8, 2>, args);
    }
  }
  const size_t shared = static_cast<size_t>(window) * groups * sizeof(float4);
  const dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, ceil_div(max_candidates, 32))), n);
  const dim3 block(32, kQueryLanes);
  if (shared > 48 * 1024) {
    auto set = [&](auto kernel) {
      return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
    };
    cudaError_t e = groups == 4 ? set(risk_kernel<T, 4>) : groups == 8 ? set(risk_kernel<T, 8>) : set(risk_kernel<T, 0>);
    if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  }
  if (groups == 4)
    risk_kernel<T, 4><<<grid, block, shared, stream>>>(table, qpos, window, groups, scale, stats, s0, margin, epsilon);
  else if (groups == 8)
    risk_kernel<T, 8><<<grid, block, shared, stream>>>(table, qpos, window, groups, scale, stats, s0, margin, epsilon);
  else
    risk_kernel<T, 0><<<grid, block, shared, stream>>>(table, qpos, window, groups, scale, stats, s0, margin, epsilon);
  return launch_status("lrk_temporal_scores");
}

ScoreTableParam make_table(const lrk_score_segment *segments, int64_t s0, int n) {
  ScoreTableParam table;
  table.count = n;
  for (int i = 0; i < n; ++i) {
    table.segment[i] = segments[s0 + i];
    table.stash_offset[i] = 0;
  }
  return table;
}

// Floats of the probability stash for segments [s0, s0 + n): per segment,
// its rows x stash_stride(candidates); fills table.stash_offset.
int64_t stash_layout(ScoreTableParam &table, int n, int64_t rows_per_segment) {
  int64_t total = 0;
  for (int i = 0; i < n; ++i) {
    table.stash_offset[i] = total;
    total += rows_per_segment * stash_stride(table.segment[i].last - table.segment[i].first);
  }
  return total;
}

// The stash path serves 1, 2, 4 or 8 groups, with the risk kernel's ring
// and projections within 200 KB of shared memory.
bool stash_supported(int groups, int window) {
  const size_t ring = groups == 1   ? stash_ring_bytes<1, 4>()
                      : groups == 2 ? stash_ring_bytes<2, 4>()
                      : groups == 4 ? stash_ring_bytes<4, 4>()
                                    : stash_ring_bytes<8, 2>();
  return (groups == 1 || groups == 2 || groups == 4 || groups == 8) &&
         ring + static_cast<size_t>(window) * groups * sizeof(float) <= 200 * 1024;
}

template <typename T>
int launch_scores(const lrk_score_segment *segments, int64_t count, const int64_t *qpos, int window, int groups,
                  float scale, const float *margin, float epsilon, float3 *stats, int32_t *visible, float *stash,
                  cudaStream_t stream) {
  for (int64_t s0 = 0; s0 < count; s0 += kMaxScoreSegments) {
    const int n = static_cast<int>(std::min<int64_t>(kMaxScoreSegments, count - s0));
    ScoreTableParam table = make_table(segments, s0, n);
    int64_t max_length = 0, max_candidates = 0;
    for (int i = 0; i < n; ++i) {
      max_length = std::max<int64_t>(max_length, table.segment[i].length);
      max_candidates = std::max<int64_t>(max_candidates, table.segment[i].last - table.segment[i].first);
    }
    float *table_stash = stash != nullptr && stash_supported(groups, window) ? stash : nullptr;
    if (table_stash != nullptr) stash_layout(table, n, static_cast<int64_t>(window) * groups);
    int status = launch_stats<T>(table, n, qpos, window, groups, scale, stats, visible, s0, max_length, table_stash,
                                 stream);
    if (status != LRK_OK) return status;
    if (table_stash != nullptr) {
      const auto args = std::make_tuple(table, n, table_stash, window, static_cast<const float3 *>(stats), s0, margin,
                                        epsilon, max_candidates, stream);
      status = groups == 1   ? std::apply(launch_risk_stash<1>, args)
               : groups == 2 ? std::apply(launch_risk_stash<2>, args)
               : groups == 4 ? std::apply(launch_risk_stash<4>, args)
                             : std::apply(launch_risk_stash<8>, args);
    } else {
      status = launch_risk<T>(table, n, qpos, window, groups, scale, margin, epsilon, stats, s0, stream);
    }
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
}

// Bytes of the probability stash for a call: the largest 48-segment table's
// rows x padded candidates (tables run one after another on one stream, so
// they share it).
size_t stash_bytes(const lrk_score_segment *segments, int64_t count, int64_t window, int64_t groups) {
  int64_t most = 0;
  for (int64_t s0 = 0; s0 < count; s0 += kMaxScoreSegments) {
    const int n = static_cast<int>(std::min<int64_t>(kMaxScoreSegments, count - s0));
    int64_t total = 0;
    for (int i = 0; i < n; ++i)
      total += window * groups * stash_stride(segments[s0 + i].last - segments[s0 + i].first);
    most = std::max(most, total);
  }
  return static_cast<size_t>(most) * sizeof(float);
}

// Scratch of lrk_temporal_scores_static: the per-row statistics of up to
// LRK_STATIC_SCORE_ROWS rows.  Every device that loads liblrk holds one copy
// until the process exits.  Host code must not pass this name to a kernel (on
// the host it is a stand-in, not a device address); static_scratch() looks up
// the device address with cudaGetSymbolAddress.
__device__ __align__(256) float3 g_static_row_stats[LRK_STATIC_SCORE_ROWS];

// The array's device address belongs to one CUDA context (the module is loaded
// per context), so the looked-up addresses are kept per context, keyed by the
// context's unique ID (cuCtxGetId: never reused within a process, unlike the
// context handle).  A context created later -- after cudaDeviceReset, or by a
// host that makes its own driver contexts -- gets its own lookup.
using CtxGetCurrent = CUresult (*)(CUcontext *);
using CtxGetId = CUresult (*)(CUcontext, unsigned long long *);

struct StaticEntry {
  unsigned long long context;
  float3 *address;
};
constexpr int kStaticEntries = 64;
std::mutex g_static_mutex;
StaticEntry g_static_entries[kStaticEntries] = {};
int g_static_used = 0, g_static_next = 0;

template <typename F>
F driver_function(const char *name) {
  void *function = nullptr;
  cudaDriverEntryPointQueryResult found;
  if (cudaGetDriverEntryPoint(name, &function, cudaEnableDefault, &found) != cudaSuccess ||
      found != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return reinterpret_cast<F>(function);
}

int lookup_static_address(float3 **address) {
  void *found = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&found, g_static_row_stats);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaGetSymbolAddress(g_static_row_stats): %s", cudaGetErrorString(e));
    return LRK_ERR_CUDA;
  }
  *address = static_cast<float3 *>(found);
  return LRK_OK;
}

// Device address of g_static_row_stats in the calling thread's current
// context; the first call in a context looks it up (cudaGetSymbolAddress,
// which also makes the device's primary context current when none is).
int static_scratch(float3 **address) {
  static const CtxGetCurrent get_current = driver_function<CtxGetCurrent>("cuCtxGetCurrent");
  static const CtxGetId get_id = driver_function<CtxGetId>("cuCtxGetId");
  if (get_current == nullptr || get_id == nullptr) return fail(LRK_ERR_CUDA, "cuCtxGetCurrent/cuCtxGetId unavailable");
  CUcontext context = nullptr;
  if (get_current(&context) != CUDA_SUCCESS) return fail(LRK_ERR_CUDA, "cuCtxGetCurrent failed");
  float3 *fresh = nullptr;
  if (context == nullptr) {
    // No context yet on this thread: the lookup binds the primary context.
    const int status = lookup_static_address(&fresh);
    if (status != LRK_OK) return status;
    if (get_current(&context) != CUDA_SUCCESS || context == nullptr) return fail(LRK_ERR_CUDA, "no CUDA context");
  }
  unsigned long long id = 0;
  if (get_id(context, &id) != CUDA_SUCCESS) return fail(LRK_ERR_CUDA, "cuCtxGetId failed");
  std::lock_guard<std::mutex> lock(g_static_mutex);
  for (int i = 0; i < g_static_used; ++i) {
    if (g_static_entries[i].context == id) {
      *address = g_static_entries[i].address;
      return LRK_OK;
    }
  }
  if (fresh == nullptr) {
    const int status = lookup_static_address(&fresh);
    if (status != LRK_OK) return status;
  }
  const int slot = g_static_used < kStaticEntries ? g_static_used++ : (g_static_next++ % kStaticEntries);
  g_static_entries[slot] = StaticEntry{id, fresh};
  *address = fresh;
  return LRK_OK;
}

int check_score_call(const lrk_score_segment *segments, int64_t count, int64_t window, int64_t groups,
                     float epsilon, const int64_t *query_positions, const float *margin) {
  LRK_REQUIRE(count >= 0 && window > 0 && groups > 0 && epsilon > 0, "invalid score sizes");
  LRK_REQUIRE(groups <= kMaxGroups, "fused scoring supports at most 8 query heads per KV head");
  LRK_REQUIRE(window <= 65535 && window * groups * static_cast<int64_t>(sizeof(float4)) <= 200 * 1024,
              "window * groups too large for one CTA's statistics");
  if (count == 0) return LRK_OK;
  LRK_REQUIRE(segments && query_positions && margin, "null pointer");
  for (int64_t s = 0; s < count; ++s) {
    const lrk_score_segment &seg = segments[s];
    LRK_REQUIRE(seg.logits && seg.projected_values && seg.key_positions && seg.scores, "null segment pointer");
    LRK_REQUIRE(seg.length > 0 && seg.first >= 0 && seg.last > seg.first && seg.last <= seg.length,
                "Invalid risk interval");
    LRK_REQUIRE(seg.projected_stride >= seg.length, "projected_stride shorter than the segment");
    LRK_REQUIRE(seg.logits_stride >= seg.length, "logits_stride shorter than the segment");
    LRK_REQUIRE(seg.query_chunk >= 0, "query_chunk must be >= 0");
  }
  return LRK_OK;
}

int dispatch_scores(const lrk_score_segment *segments, int64_t count, int logits_dtype, const int64_t *qpos,
                    int64_t window, int64_t groups, float scale, const float *margin, float epsilon, float3 *stats,
                    int32_t *visible, float *stash, lrk_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int w = static_cast<int>(window), g = static_cast<int>(groups);
  switch (logits_dtype) {
    case LRK_BF16:
      return launch_scores<__nv_bfloat16>(segments, count, qpos, w, g, scale, margin, epsilon, stats, visible, stash,
                                          s);
    case LRK_F16:
      return launch_scores<__half>(segments, count, qpos, w, g, scale, margin, epsilon, stats, visible, stash, s);
    case LRK_F32:
      return launch_scores<float>(segments, count, qpos, w, g, scale, margin, epsilon, stats, visible, stash, s);
    default: return fail(LRK_ERR_UNSUPPORTED, "Only FP32/FP16/BF16 scores are supported");
  }
}

}  // namespace

int score_visibility(const lrk_score_segment *segments, int64_t count, const int64_t *qpos, int window,
                     int32_t *visible, cudaStream_t stream) {
  for (int64_t s0 = 0; s0 < count; s0 += kMaxScoreSegments) {
    const int n = static_cast<int>(std::min<int64_t>(kMaxScoreSegments, count - s0));
    visibility_kernel<<<n, kVisibilityThreads, 0, stream>>>(make_table(segments, s0, n), qpos, window, visible, s0);
    const int status = launch_status("lrk_scores_from_keys visibility");
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
}

int score_risk_bf16(const lrk_score_segment *segments, int64_t count, const int64_t *qpos, int window, int groups,
                    float scale, const float *margin, float epsilon, const float3 *stats, cudaStream_t stream) {
  for (int64_t s0 = 0; s0 < count; s0 += kMaxScoreSegments) {
    const int n = static_cast<int>(std::min<int64_t>(kMaxScoreSegments, count - s0));
    const int status = launch_risk<__nv_bfloat16>(make_table(segments, s0, n), n, qpos, window, groups, scale, margin,
                                                  epsilon, stats, s0, stream);
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
}

}  // namespace lrk

using namespace lrk;

// Workspace: the row statistics (float3 per row), then the visible-prefix
// lengths (int32 per segment and query); optionally, after them, the
// probability stash (lrk_temporal_scores_stash_bytes).
extern "C" size_t lrk_temporal_scores_workspace_bytes(int64_t segments, int64_t window, int64_t groups) {
  if (segments < 0 || window < 0 || groups < 0) return 0;
  return static_cast<size_t>(segments) * window * groups * sizeof(float3) +
         static_cast<size_t>(segments) * window * sizeof(int32_t) + 256;
}

extern "C" size_t lrk_temporal_scores_stash_bytes(const lrk_score_segment *segments, int64_t count, int64_t window,
                                                  int64_t groups) {
  if (segments == nullptr || count <= 0 || window <= 0 || groups <= 0) return 0;
  for (int64_t i = 0; i < count; ++i)
    if (segments[i].last < segments[i].first) return 0;
  return stash_bytes(segments, count, window, groups) + 256;
}

extern "C" int lrk_temporal_scores(const lrk_score_segment *segments, int64_t count, int logits_dtype,
                                   const int64_t *query_positions, int64_t window, int64_t groups, float scale,
                                   const float *margin, float epsilon, void *workspace, size_t workspace_bytes,
                                   lrk_stream_t stream) {
  clear_error();
  int status = check_score_call(segments, count, window, groups, epsilon, query_positions, margin);
  if (status != LRK_OK || count == 0) return status;
  const size_t need = lrk_temporal_scores_workspace_bytes(count, window, groups);
  if (workspace == nullptr || workspace_bytes < need) return fail(LRK_ERR_WORKSPACE, "score workspace too small");
  float3 *stats = reinterpret_cast<float3 *>((reinterpret_cast<uintptr_t>(workspace) + 15) & ~uintptr_t{15});
  int32_t *visible = reinterpret_cast<int32_t *>(stats + count * window * groups);
  // With room for the probability stash after the base workspace, the risk
  // reads the candidates' probabilities the statistics pass stored instead of
  // recomputing them from the logits.
  float *stash = nullptr;
  const size_t extra = lrk_temporal_scores_stash_bytes(segments, count, window, groups);
  if (extra > 0 && workspace_bytes >= need + extra) {
    const uintptr_t at = reinterpret_cast<uintptr_t>(workspace) + need;
    stash = reinterpret_cast<float *>((at + 255) & ~uintptr_t{255});
  }
  return dispatch_scores(segments, count, logits_dtype, query_positions, window, groups, scale, margin, epsilon, stats,
                         visible, stash, stream);
}

extern "C" int lrk_temporal_scores_static(const lrk_score_segment *segments, int64_t count, int logits_dtype,
                                          const int64_t *query_positions, int64_t window, int64_t groups,
                                          float scale, const float *margin, float epsilon, lrk_stream_t stream) {
  clear_error();
  int status = check_score_call(segments, count, window, groups, epsilon, query_positions, margin);
  if (status != LRK_OK || count == 0) return status;
  if (count * window * groups > LRK_STATIC_SCORE_ROWS) {
    set_error("lrk_temporal_scores_static: %lld segments x %lld queries x %lld groups exceeds the static scratch of "
              "%d row statistics (LRK_STATIC_SCORE_ROWS); split the call or use lrk_temporal_scores",
              static_cast<long long>(count), static_cast<long long>(window), static_cast<long long>(groups),
              LRK_STATIC_SCORE_ROWS);
    return LRK_ERR_INVALID;
  }
  float3 *stats = nullptr;
  status = static_scratch(&stats);
  if (status != LRK_OK) return status;
  // No visible-prefix table and no probability stash here: every row
  // compares key positions and the risk recomputes its probabilities.
  return dispatch_scores(segments, count, logits_dtype, query_positions, window, groups, scale, margin, epsilon, stats,
                         nullptr, nullptr, stream);
}
