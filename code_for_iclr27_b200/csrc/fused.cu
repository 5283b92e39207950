// Fused temporal scoring of liblrk: candidate risk straight from logits.
//
// The reference scores one head per call in two operators
// (csrc/scoring.cu:32-128): temporal_probabilities writes every fp32
// probability of a [window, groups, length] chunk, temporal_risk reads the
// candidate columns back.  Here the probabilities never reach HBM:
//
//   stats kernel   one CTA per (segment, query): for each group row an online
//                  softmax pass over the bf16 logits (16-byte loads) gives the
//                  row max m, the denominator d = sum exp(x - m) and the value
//                  projection op = sum p * pv, written to a small workspace.
//   risk kernel    one CTA per (segment, tile of 256 candidates): each thread
//                  owns one candidate column, walks every query and group,
//                  recomputes p = exp(x - m) / d for its column only, folds the
//                  margin drop sum_g p/max(1-p,eps) * (pv - op) into a running
//                  min / max / non-finite flag, and ends with the float64 risk.
//
// x is the reference's dtype-rounded, causally masked scaled logit
// (csrc/scoring.cu:44-46).  Sums run in a different order than the
// reference's 256-lane tree, so results agree with it to ~1e-6 relative
// rather than bit for bit; the drop-in operators remain the bit-exact path.
// Many (layer, head) segments go in one launch: their descriptors travel as
// a kernel parameter (up to kMaxScoreSegments per launch).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"

namespace lrk {
namespace {

constexpr int kMaxScoreSegments = 48;
constexpr int kStatsThreads = 256;
constexpr int kRiskThreads = 256;
constexpr int kMaxGroups = 8;
constexpr float kLog2e = 1.4426950408889634f;

struct ScoreTableParam {
  lrk_score_segment segment[kMaxScoreSegments];
  int count;
};

template <typename T> struct Logits;
template <> struct Logits<__nv_bfloat16> {
  using Vec = uint4;  // 8 values
  static constexpr int kPerVec = 8;
  static __device__ __forceinline__ float round_scaled(float x, float s) {
    return __bfloat162float(__float2bfloat16_rn(x * s));
  }
  static __device__ __forceinline__ float at(const __nv_bfloat16 *p) {
    return __bfloat162float(__ushort_as_bfloat16(__ldg(reinterpret_cast<const unsigned short *>(p))));
  }
  static __device__ __forceinline__ void unpack(const Vec &v, float *out) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      out[2 * i] = __uint_as_float(w[i] << 16);
      out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Logits<__half> {
  using Vec = uint4;
  static constexpr int kPerVec = 8;
  static __device__ __forceinline__ float round_scaled(float x, float s) { return __half2float(__float2half_rn(x * s)); }
  static __device__ __forceinline__ float at(const __half *p) {
    return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short *>(p))));
  }
  static __device__ __forceinline__ void unpack(const Vec &v, float *out) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
      out[2 * i] = __low2float(h);
      out[2 * i + 1] = __high2float(h);
    }
  }
};
template <> struct Logits<float> {
  using Vec = uint4;  // 4 values
  static constexpr int kPerVec = 4;
  static __device__ __forceinline__ float round_scaled(float x, float s) { return x * s; }
  static __device__ __forceinline__ float at(const float *p) { return __ldg(p); }
  static __device__ __forceinline__ void unpack(const Vec &v, float *out) {
    out[0] = __uint_as_float(v.x);
    out[1] = __uint_as_float(v.y);
    out[2] = __uint_as_float(v.z);
    out[3] = __uint_as_float(v.w);
  }
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Running softmax state of one thread: max m, sum d of exp(x - m), and
// n = sum exp(x - m) * pv.
struct Online {
  float m = -INFINITY, d = 0.0f, n = 0.0f;
  __device__ __forceinline__ void rescale_to(float new_max) {
    const float s = fast_exp2((m - new_max) * kLog2e);
    d *= s;
    n *= s;
    m = new_max;
  }
  __device__ __forceinline__ void merge(float om, float od, float on) {
    if (om == -INFINITY) return;
    if (m == -INFINITY) {
      m = om, d = od, n = on;
      return;
    }
    const float big = fmaxf(m, om);
    const float a = fast_exp2((m - big) * kLog2e), b = fast_exp2((om - big) * kLog2e);
    d = d * a + od * b;
    n = n * a + on * b;
    m = big;
  }
};

template <typename T, int N>
__device__ __forceinline__ void absorb(Online &s, const float (&x)[N], const float (&pv)[N]) {
  float vmax = x[0];
#pragma unroll
  for (int j = 1; j < N; ++j) vmax = fmaxf(vmax, x[j]);
  if (vmax == -INFINITY) return;
  if (vmax > s.m) s.rescale_to(vmax);
  const float shift = -s.m * kLog2e;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const float w = fast_exp2(fmaf(x[j], kLog2e, shift));
    s.d += w;
    s.n = fmaf(w, pv[j], s.n);
  }
}

// stats[(segment * window + q) * groups + g] = (m, d, op).
template <typename T>
__global__ void __launch_bounds__(kStatsThreads) stats_kernel(ScoreTableParam table, const int64_t *__restrict__ qpos,
                                                              int window, int groups, float scale,
                                                              float3 *__restrict__ stats, int64_t segment_base) {
  using L = Logits<T>;
  constexpr int V = L::kPerVec;
  __shared__ float shared[3][kStatsThreads / 32];
  const int q = blockIdx.x;
  const int si = blockIdx.y;
  const lrk_score_segment &seg = table.segment[si];
  const int64_t length = seg.length;
  const float query_position = static_cast<float>(qpos[q]);
  const float *kpos = seg.key_positions;
  for (int g = 0; g < groups; ++g) {
    const T *row = static_cast<const T *>(seg.logits) + (static_cast<int64_t>(q) * groups + g) * length;
    const float *pv = seg.projected_values + g * seg.projected_stride;
    // Elements before the first 16-byte boundary, the vector body, the tail.
    const int64_t lead = lmin(length, static_cast<int64_t>(((16 - (reinterpret_cast<uintptr_t>(row) & 15)) & 15) /
                                                          sizeof(T)));
    const int64_t vectors = (length - lead) / V;
    const int64_t tail_start = lead + vectors * V;
    Online s;
    auto scalar = [&](int64_t p) {
      float x[1] = {L::round_scaled(L::at(row + p), scale)};
      x[0] = __ldg(kpos + p) <= query_position ? x[0] : -INFINITY;
      const float pvv[1] = {__ldg(pv + p)};
      absorb<T, 1>(s, x, pvv);
    };
    if (threadIdx.x < lead) scalar(threadIdx.x);
    const typename L::Vec *body = reinterpret_cast<const typename L::Vec *>(row + lead);
#pragma unroll 2
    for (int64_t v = threadIdx.x; v < vectors; v += kStatsThreads) {
      const typename L::Vec raw = __ldg(body + v);
      float x[V], pvv[V];
      L::unpack(raw, x);
      const int64_t p0 = lead + v * V;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float rounded = L::round_scaled(x[j], scale);
        x[j] = __ldg(kpos + p0 + j) <= query_position ? rounded : -INFINITY;
        pvv[j] = __ldg(pv + p0 + j);
      }
      absorb<T, V>(s, x, pvv);
    }
    for (int64_t p = tail_start + threadIdx.x; p < length; p += kStatsThreads) scalar(p);
    // Block reduction of (m, d, n).
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, s.m, o);
      const float od = __shfl_xor_sync(0xffffffffu, s.d, o);
      const float on = __shfl_xor_sync(0xffffffffu, s.n, o);
      s.merge(om, od, on);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
      shared[0][warp] = s.m;
      shared[1][warp] = s.d;
      shared[2][warp] = s.n;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      Online total;
      for (int w = 0; w < kStatsThreads / 32; ++w) total.merge(shared[0][w], shared[1][w], shared[2][w]);
      stats[((segment_base + si) * window + q) * groups + g] =
          make_float3(total.m, total.d, total.n / total.d);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ double softplus64(double value) { return value > 20.0 ? value : log1p(exp(value)); }

__device__ __forceinline__ double risk64(double margin, double probability, double base_softplus, float drop) {
  const double compared = margin - static_cast<double>(drop);
  return fmax(0.0, probability * (margin - compared) - base_softplus + softplus64(compared));
}

template <typename T, int G>
__global__ void __launch_bounds__(kRiskThreads) risk_kernel(ScoreTableParam table, const int64_t *__restrict__ qpos,
                                                            int window, int groups, float scale,
                                                            const float3 *__restrict__ stats,
                                                            int64_t segment_base, const float *__restrict__ margin,
                                                            float epsilon) {
  using L = Logits<T>;
  extern __shared__ float4 shared_stats[];  // [window * groups] (m, 1/d-free d, op, qpos)
  const int si = blockIdx.y;
  const lrk_score_segment &seg = table.segment[si];
  const int ng = G > 0 ? G : groups;
  for (int i = threadIdx.x; i < window * ng; i += kRiskThreads) {
    const float3 st = stats[(segment_base + si) * window * ng + i];
    shared_stats[i] = make_float4(st.x, st.y, st.z, static_cast<float>(qpos[i / ng]));
  }
  __syncthreads();
  const int64_t count = seg.last - seg.first;
  const int64_t candidate = static_cast<int64_t>(blockIdx.x) * kRiskThreads + threadIdx.x;
  if (candidate >= count) return;
  const int64_t column = seg.first + candidate;
  const int64_t length = seg.length;
  const float key_position = __ldg(seg.key_positions + column);
  float pv[G > 0 ? G : kMaxGroups];
#pragma unroll
  for (int g = 0; g < (G > 0 ? G : kMaxGroups); ++g)
    pv[g] = g < ng ? __ldg(seg.projected_values + g * seg.projected_stride + column) : 0.0f;
  const T *base = static_cast<const T *>(seg.logits) + column;
  float minimum = INFINITY, maximum = -INFINITY;
  bool nonfinite = false;
#pragma unroll 4
  for (int q = 0; q < window; ++q) {
    float drop = 0.0f;
#pragma unroll
    for (int g = 0; g < (G > 0 ? G : kMaxGroups); ++g) {
      if (g < ng) {
        const float4 st = shared_stats[q * ng + g];
        const float rounded = L::round_scaled(L::at(base + (static_cast<int64_t>(q) * ng + g) * length), scale);
        const float x = key_position <= st.w ? rounded : -INFINITY;
        const float probability = expf(x - st.x) / st.y;
        const float ratio = probability / fmaxf(1.0f - probability, epsilon);
        drop += ratio * (pv[g] - st.z);
      }
    }
    nonfinite |= !isfinite(drop);
    minimum = fminf(minimum, drop);
    maximum = fmaxf(maximum, drop);
  }
  float result;
  if (nonfinite) {
    result = NAN;
  } else {
    const double m = static_cast<double>(margin[0]);
    const double probability = 1.0 / (1.0 + exp(-m));
    const double base_sp = softplus64(m);
    result = static_cast<float>(fmax(risk64(m, probability, base_sp, minimum), risk64(m, probability, base_sp, maximum)));
  }
  seg.scores[candidate] = result;
}

template <typename T>
int launch_scores(const lrk_score_segment *segments, int64_t count, const int64_t *qpos, int window, int groups,
                  float scale, const float *margin, float epsilon, float3 *stats, cudaStream_t stream) {
  for (int64_t s0 = 0; s0 < count; s0 += kMaxScoreSegments) {
    const int n = static_cast<int>(std::min<int64_t>(kMaxScoreSegments, count - s0));
    ScoreTableParam table;
    table.count = n;
    int64_t max_candidates = 0;
    for (int i = 0; i < n; ++i) {
      table.segment[i] = segments[s0 + i];
      max_candidates = std::max<int64_t>(max_candidates, segments[s0 + i].last - segments[s0 + i].first);
    }
    stats_kernel<T><<<dim3(window, n), kStatsThreads, 0, stream>>>(table, qpos, window, groups, scale, stats, s0);
    const size_t shared = static_cast<size_t>(window) * groups * sizeof(float4);
    const dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, ceil_div(max_candidates, kRiskThreads))), n);
    if (shared > 48 * 1024) {
      auto set = [&](auto kernel) {
        return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
      };
      cudaError_t e = groups == 4 ? set(risk_kernel<T, 4>) : groups == 8 ? set(risk_kernel<T, 8>) : set(risk_kernel<T, 0>);
      if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
    }
    if (groups == 4)
      risk_kernel<T, 4><<<grid, kRiskThreads, shared, stream>>>(table, qpos, window, groups, scale, stats, s0, margin,
                                                                 epsilon);
    else if (groups == 8)
      risk_kernel<T, 8><<<grid, kRiskThreads, shared, stream>>>(table, qpos, window, groups, scale, stats, s0, margin,
                                                                 epsilon);
    else
      risk_kernel<T, 0><<<grid, kRiskThreads, shared, stream>>>(table, qpos, window, groups, scale, stats, s0, margin,
                                                                 epsilon);
    const int status = launch_status("lrk_temporal_scores");
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
}

}  // namespace
}  // namespace lrk

using namespace lrk;

extern "C" size_t lrk_temporal_scores_workspace_bytes(int64_t segments, int64_t window, int64_t groups) {
  if (segments < 0 || window < 0 || groups < 0) return 0;
  return static_cast<size_t>(segments) * window * groups * sizeof(float3) + 256;
}

extern "C" int lrk_temporal_scores(const lrk_score_segment *segments, int64_t count, int logits_dtype,
                                   const int64_t *query_positions, int64_t window, int64_t groups, float scale,
                                   const float *margin, float epsilon, void *workspace, size_t workspace_bytes,
                                   lrk_stream_t stream) {
  clear_error();
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
  }
  const size_t need = lrk_temporal_scores_workspace_bytes(count, window, groups);
  if (workspace == nullptr || workspace_bytes < need) return fail(LRK_ERR_WORKSPACE, "score workspace too small");
  float3 *stats = reinterpret_cast<float3 *>((reinterpret_cast<uintptr_t>(workspace) + 15) & ~uintptr_t{15});
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int w = static_cast<int>(window), g = static_cast<int>(groups);
  switch (logits_dtype) {
    case LRK_BF16: return launch_scores<__nv_bfloat16>(segments, count, query_positions, w, g, scale, margin, epsilon, stats, s);
    case LRK_F16: return launch_scores<__half>(segments, count, query_positions, w, g, scale, margin, epsilon, stats, s);
    case LRK_F32: return launch_scores<float>(segments, count, query_positions, w, g, scale, margin, epsilon, stats, s);
    default: return fail(LRK_ERR_UNSUPPORTED, "Only FP32/FP16/BF16 scores are supported");
  }
}
