// Scoring kernels of liblrk: temporal probabilities, temporal risk, Pool7 and
// the legacy single-query decision risk.  Compiled with --fmad=false, and the
// order-sensitive arithmetic is written with explicit round-to-nearest
// intrinsics, so every value matches the reference operator bit for bit:
//
// * A softmax row's denominator and value projection are sums.  The
//   reference (csrc/scoring.cu:32-66) forms them as 256 per-thread sequential
//   sums over positions t, t+256, t+512, ... followed by a 256-wide tree
//   (csrc/scoring.cu:15-30).  Here the same 256 "lanes" and the same tree are
//   kept, but the row is read from HBM once: it is staged in shared memory and
//   every element-wise step (scale/round/mask, exp, divide, product) runs on all
//   threads in parallel, so only the 256 cheap sequential add chains remain.
// * Max and min reductions are order-free and use warp shuffles.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "rows.cuh"

namespace lrk {
namespace {

constexpr int kLanes = rows::kLanes;  // the reference's reduction width

// One CTA per (query, group) row (csrc/scoring.cu:32-66): the row's exact
// statistics (rows.cuh), its probabilities written out, its value projection.
template <typename T, int MODE>
__global__ void __launch_bounds__(kLanes) probabilities_kernel(
    const T *__restrict__ logits, const float *__restrict__ projected_values,
    const int64_t *__restrict__ query_positions, const float *__restrict__ key_positions,
    float *__restrict__ probabilities, float *__restrict__ output_projection, int groups, int64_t length,
    float scale) {
  extern __shared__ __align__(16) unsigned char stage[];
  __shared__ float scratch[kLanes];
  const int64_t row = blockIdx.x;
  const int group = static_cast<int>(row % groups);
  const int64_t query = row / groups;
  const rows::RowResult result = rows::row_statistics<T, MODE>(
      logits + row * length, length, rows::Visibility{key_positions, static_cast<float>(query_positions[query]), -1},
      projected_values + static_cast<int64_t>(group) * length, scale, probabilities + row * length, stage, scratch);
  if (threadIdx.x == 0) output_projection[row] = result.projection;
}

__device__ __forceinline__ double softplus64(double value) {
  return value > 20.0 ? value : log1p(exp(value));
}

// max(0, p*(m - c) - softplus(m) + softplus(c)) with c = m - drop
// (csrc/scoring.cu:68-75), evaluated in the same operation order.
__device__ __forceinline__ double risk64(double margin, double probability, double base_softplus, float drop) {
  const double compared = __dsub_rn(margin, static_cast<double>(drop));
  const double kl = __dadd_rn(__dsub_rn(__dmul_rn(probability, __dsub_rn(margin, compared)), base_softplus),
                              softplus64(compared));
  return fmax(0.0, kl);
}

// One warp row = 32 consecutive candidates; `split` query lanes per candidate
// (blockDim.y), each taking queries lane, lane + split, ...  G <= MAXG keeps
// the candidate's projected values in registers.
template <int MAXG>
__global__ void __launch_bounds__(1024) risk_kernel(
    const float *__restrict__ probabilities, const float *__restrict__ output_projection,
    const float *__restrict__ projected_values, const float *__restrict__ margin, float *__restrict__ result,
    int window, int groups, int64_t length, int64_t first, int64_t count, float epsilon) {
  __shared__ float minimums[32][33];
  __shared__ float maximums[32][33];
  __shared__ int bad[32][33];
  const int lane = threadIdx.x;
  const int split = blockDim.y;
  const int64_t candidate = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const int64_t position = first + candidate;
  const bool active = candidate < count;
  float minimum = INFINITY, maximum = -INFINITY;
  int nonfinite = 0;
  if (active) {
    float pv[MAXG > 0 ? MAXG : 1];
    if (MAXG > 0) {
#pragma unroll
      for (int g = 0; g < MAXG; ++g) pv[g] = g < groups ? projected_values[g * length + position] : 0.0f;
    }
#pragma unroll 2
    for (int query = threadIdx.y; query < window; query += split) {
      float drop = 0.0f;
      const float *column = probabilities + static_cast<int64_t>(query) * groups * length + position;
      const float *op = output_projection + static_cast<int64_t>(query) * groups;
      if (MAXG > 0) {
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
          if (g < groups) {
            const float probability = __ldcs(column + g * length);
            const float ratio = __fdiv_rn(probability, fmaxf(__fsub_rn(1.0f, probability), epsilon));
            drop = __fadd_rn(drop, __fmul_rn(ratio, __fsub_rn(pv[g], op[g])));
          }
        }
      } else {
        for (int g = 0; g < groups; ++g) {
          const float probability = __ldcs(column + g * length);
          const float ratio = __fdiv_rn(probability, fmaxf(__fsub_rn(1.0f, probability), epsilon));
          drop = __fadd_rn(drop, __fmul_rn(ratio, __fsub_rn(projected_values[g * length + position], op[g])));
        }
      }
      if (!isfinite(drop)) nonfinite = 1;
      minimum = fminf(minimum, drop);
      maximum = fmaxf(maximum, drop);
    }
  }
  minimums[threadIdx.y][lane] = minimum;
  maximums[threadIdx.y][lane] = maximum;
  bad[threadIdx.y][lane] = nonfinite;
  __syncthreads();
  if (threadIdx.y == 0 && active) {
    for (int y = 1; y < split; ++y) {
      minimum = fminf(minimum, minimums[y][lane]);
      maximum = fmaxf(maximum, maximums[y][lane]);
      nonfinite |= bad[y][lane];
    }
    if (nonfinite) {
      result[candidate] = NAN;
    } else {
      const double m = static_cast<double>(margin[0]);
      const double probability = 1.0 / (1.0 + exp(-m));
      const double base = softplus64(m);
      result[candidate] = static_cast<float>(fmax(risk64(m, probability, base, minimum),
                                                  risk64(m, probability, base, maximum)));
    }
  }
}

// Pool over aligned tiles.  A CTA owns one tile of one segment: the 128
// 4-element quads that start at A + 512 x, A = the segment's first index
// rounded down to a multiple of 4.  It stages the tile plus a halo on each
// side in shared memory with 16-byte loads (quads that cross the array's ends
// are read element by element); each thread then takes its quad's window of
// elements into registers, replaces those outside the segment by -inf, and
// folds each output's window with fmaxf in ascending index order from -inf.
// Folding an extra -inf changes nothing (fmaxf(v, -inf) == v, and the
// running value is never NaN), so this equals the reference's clipped window
// (csrc/scoring.cu:190-203).  Outputs are stored as 16-byte vectors, element
// by element where a quad crosses the segment's ends.  HALF > 0 fixes the
// half-width at compile time (Pool7: 3); HALF = 0 reads it from `half`.
constexpr int kPoolThreads = 128;
constexpr int kPoolTile = 4 * kPoolThreads;  // elements per tile: one quad per thread
constexpr int kPoolHalo = 32;                // largest half-width the tiled kernel serves

template <int HALF>
__global__ void __launch_bounds__(kPoolThreads) pool_tile_kernel(const float *__restrict__ scores, int64_t n,
                                                                 const int64_t *__restrict__ bounds,
                                                                 int64_t segments, int half_runtime,
                                                                 float *__restrict__ out) {
  __shared__ __align__(16) float tile[kPoolTile + 2 * kPoolHalo];
  const int half = HALF > 0 ? HALF : half_runtime;
  const int halo = (half + 3) & ~3;
  for (int64_t segment = blockIdx.y; segment < segments; segment += gridDim.y) {
    const int64_t begin = lmax(0, bounds[segment]);
    const int64_t end = lmin(n, bounds[segment + 1]);
    const int64_t first = begin & ~int64_t{3};
    for (int64_t base = first + static_cast<int64_t>(blockIdx.x) * kPoolTile; base < end;
         base += static_cast<int64_t>(gridDim.x) * kPoolTile) {
      __syncthreads();  // the previous tile's reads are done
      const int quads = (kPoolTile + 2 * halo) / 4;
      for (int q = threadIdx.x; q < quads; q += kPoolThreads) {
        const int64_t g = base - halo + 4 * q;
        float4 v;
        if (g >= 0 && g + 3 < n) {
          v = __ldcs(reinterpret_cast<const float4 *>(scores + g));
        } else {
          v.x = (g >= 0 && g < n) ? scores[g] : 0.0f;
          v.y = (g + 1 >= 0 && g + 1 < n) ? scores[g + 1] : 0.0f;
          v.z = (g + 2 >= 0 && g + 2 < n) ? scores[g + 2] : 0.0f;
          v.w = (g + 3 >= 0 && g + 3 < n) ? scores[g + 3] : 0.0f;
        }
        *reinterpret_cast<float4 *>(tile + 4 * q) = v;
      }
      __syncthreads();
      const int64_t g = base + 4 * threadIdx.x;
      if (g >= end) continue;
      // Segment bounds relative to the quad's first element (small ints).
      const int lo = static_cast<int>(lmax(begin - g, -(kPoolHalo + 4)));
      const int hi = static_cast<int>(lmin(end - g, kPoolHalo + 8));
      const float *at = tile + halo + 4 * threadIdx.x;  // element g
      float r[4];
      if (HALF > 0) {
        // Elements g - H4 .. g + 3 + H4 in registers, H4 = HALF rounded up to 4.
        constexpr int H4 = (HALF + 3) & ~3;
        float w[4 + 2 * H4];
#pragma unroll
        for (int j = 0; j < 4 + 2 * H4; j += 4) {
          const float4 v = *reinterpret_cast<const float4 *>(at - H4 + j);
          w[j] = v.x;
          w[j + 1] = v.y;
          w[j + 2] = v.z;
          w[j + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < 4 + 2 * H4; ++j) {
          const int offset = j - H4;
          if (offset < lo || offset >= hi) w[j] = -INFINITY;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float value = -INFINITY;
#pragma unroll
          for (int o = -HALF; o <= HALF; ++o) value = fmaxf(value, w[H4 + e + o]);
          r[e] = value;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float value = -INFINITY;
          const int from = max(lo, e - half), to = min(hi - 1, e + half);
          for (int j = from; j <= to; ++j) value = fmaxf(value, at[j]);
          r[e] = value;
        }
      }
      if (g >= begin && g + 3 < end) {
        __stcs(reinterpret_cast<float4 *>(out + g), make_float4(r[0], r[1], r[2], r[3]));
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (g + e >= begin && g + e < end) out[g + e] = r[e];
      }
    }
  }
}

// Pool: out[i] = max of scores over [i - w/2, i + w/2] clipped to i's segment.
// Element-per-thread form for unaligned pointers and windows wider than the
// tiled kernel's halo.
__global__ void pool_kernel(const float *__restrict__ scores, int64_t n, const int64_t *__restrict__ bounds,
                            int64_t segments, int half, float *__restrict__ out) {
  for (int64_t segment = blockIdx.y; segment < segments; segment += gridDim.y) {
    const int64_t begin = lmax(0, bounds[segment]);
    const int64_t end = lmin(n, bounds[segment + 1]);
    for (int64_t i = begin + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < end;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      float value = -INFINITY;
      const int64_t lo = lmax(begin, i - half), hi = lmin(end - 1, i + half);
      for (int64_t j = lo; j <= hi; ++j) value = fmaxf(value, scores[j]);
      out[i] = value;
    }
  }
}

template <typename T> __device__ __forceinline__ float to_float(T v);
template <> __device__ __forceinline__ float to_float(float v) { return v; }
template <> __device__ __forceinline__ float to_float(double v) { return static_cast<float>(v); }
template <> __device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ double stable_sigmoid(double value) {
  if (value >= 0.0) return 1.0 / (1.0 + exp(-value));
  const double e = exp(value);
  return e / (1.0 + e);
}
__device__ double stable_softplus(double value) {
  if (value > 20.0) return __dadd_rn(value, log1p(exp(-value)));
  return log1p(exp(value));
}

// Legacy decision risk (csrc/cache_legacy.cu:81-135): 256 threads per
// candidate, term index t, t + 256, ... over (group, channel), then a tree.
template <typename T>
__global__ void __launch_bounds__(kLanes) decision_risk_kernel(
    float *__restrict__ scores, const float *__restrict__ probabilities, const T *__restrict__ values,
    const float *__restrict__ head_outputs, const float *__restrict__ gradients, int groups, int64_t candidates,
    int dimension, double base_margin, float epsilon) {
  __shared__ float tree[kLanes];
  const int64_t candidate = blockIdx.x;
  float partial = 0.0f;
  const int terms = groups * dimension;
  for (int index = threadIdx.x; index < terms; index += kLanes) {
    const int group = index / dimension;
    const int channel = index % dimension;
    const float alpha = probabilities[group * candidates + candidate];
    const float denominator = fmaxf(__fsub_rn(1.0f, alpha), epsilon);
    const float value = to_float(values[candidate * dimension + channel]);
    const float local_delta =
        __fmul_rn(__fdiv_rn(alpha, denominator), __fsub_rn(value, head_outputs[group * dimension + channel]));
    partial = __fadd_rn(partial, __fmul_rn(gradients[group * dimension + channel], local_delta));
  }
  const float total = rows::tree_sum(partial, tree);
  if (threadIdx.x == 0) {
    const double compared = __dsub_rn(base_margin, static_cast<double>(total));
    const double probability = stable_sigmoid(base_margin);
    double kl = __dadd_rn(__dsub_rn(__dmul_rn(probability, __dsub_rn(base_margin, compared)),
                                    stable_softplus(base_margin)),
                          stable_softplus(compared));
    if (kl < 0.0) kl = 0.0;
    scores[candidate] = static_cast<float>(kl);
  }
}

template <typename K>
int allow_shared(K kernel, int64_t bytes) {
  if (bytes <= 48 * 1024) return LRK_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  return e == cudaSuccess ? LRK_OK : fail(LRK_ERR_CUDA, cudaGetErrorString(e));
}

template <typename T>
int launch_probabilities(const void *logits, const float *pv, const int64_t *qpos, const float *kpos, float *probs,
                         float *op, int64_t rows, int groups, int64_t length, float scale, cudaStream_t stream) {
  const T *in = static_cast<const T *>(logits);
  const bool aligned_rows = aligned(logits, 16) && (length * static_cast<int64_t>(sizeof(T))) % 16 == 0;
  const int mode = rows::choose_stage<T>(length, aligned_rows);
  const int64_t bytes = rows::staged_bytes<T>(mode, length);
  const unsigned grid = static_cast<unsigned>(rows);
  int status = LRK_OK;
  if (mode == rows::kWeights) {
    if ((status = allow_shared(probabilities_kernel<T, rows::kWeights>, bytes)) != LRK_OK) return status;
    probabilities_kernel<T, rows::kWeights><<<grid, kLanes, bytes, stream>>>(in, pv, qpos, kpos, probs, op, groups,
                                                                             length, scale);
  } else if (mode == rows::kBits) {
    if ((status = allow_shared(probabilities_kernel<T, rows::kBits>, bytes)) != LRK_OK) return status;
    probabilities_kernel<T, rows::kBits><<<grid, kLanes, bytes, stream>>>(in, pv, qpos, kpos, probs, op, groups,
                                                                          length, scale);
  } else if (mode == rows::kPacked) {
    if constexpr (sizeof(T) == 2) {
      if ((status = allow_shared(probabilities_kernel<T, rows::kPacked>, bytes)) != LRK_OK) return status;
      probabilities_kernel<T, rows::kPacked><<<grid, kLanes, bytes, stream>>>(in, pv, qpos, kpos, probs, op, groups,
                                                                              length, scale);
    }
  } else {
    probabilities_kernel<T, rows::kStream><<<grid, kLanes, 0, stream>>>(in, pv, qpos, kpos, probs, op, groups, length,
                                                                        scale);
  }
  return launch_status("lrk_temporal_probabilities");
}

// rows::divide against __fdiv_rn over count pseudo-random (a, b) pairs: a any
// float in [0, 1], b in [1, 2^32) with a random significand, plus every 1024th
// a in [1/4, 1) and every 4096th b with a significand of trailing ones (the
// hard cases of reciprocal rounding).  Counts the pairs whose bits differ.
__global__ void divider_check_kernel(uint64_t count, uint64_t seed, unsigned long long *mismatches) {
  unsigned long long local = 0;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    uint64_t x = (i + 1) * 0x9e3779b97f4a7c15ull ^ seed;
    x ^= x >> 31;
    x *= 0xbf58476d1ce4e5b9ull;
    x ^= x >> 29;
    x *= 0x94d049bb133111ebull;
    x ^= x >> 32;
    const uint32_t u = static_cast<uint32_t>(x), v = static_cast<uint32_t>(x >> 32);
    float a = __uint_as_float(u % 0x3f800001u);
    float b = __uint_as_float(0x3f800000u + (v % (32u << 23)));
    if ((i & 1023) == 0) a = __uint_as_float((u & 0x007fffffu) | ((v & 1u) ? 0x3f000000u : 0x3e800000u));
    if ((i & 4095) == 1) b = __uint_as_float((__float_as_uint(b) & 0xff800000u) | 0x007ff000u | (v & 0xfffu));
    const rows::Divider divider = rows::make_divider(b);
    const float expected = __fdiv_rn(a, b);
    if (__float_as_uint(rows::divide(divider, a)) != __float_as_uint(expected)) ++local;
    // The pair form, with a second numerator from the other half of the draw.
    const float a2 = __uint_as_float(static_cast<uint32_t>(x >> 7) % 0x3f800001u);
    const float2 pair = rows::divide2(divider, make_float2(a, a2));
    if (__float_as_uint(pair.x) != __float_as_uint(expected) ||
        __float_as_uint(pair.y) != __float_as_uint(__fdiv_rn(a2, b)))
      ++local;
  }
  if (local) atomicAdd(mismatches, local);
}

}  // namespace
}  // namespace lrk

using namespace lrk;

// Test hook: number of (a, b) pairs out of `count` on which the row
// statistics' division differs from IEEE division (expected 0).
extern "C" int lrk_check_division(uint64_t count, uint64_t seed, unsigned long long *mismatches_device,
                                  lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(mismatches_device != nullptr, "null pointer");
  divider_check_kernel<<<sm_count() * 8, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(count, seed,
                                                                                         mismatches_device);
  return launch_status("lrk_check_division");
}

extern "C" int lrk_temporal_probabilities(const void *logits, int logits_dtype, const float *projected_values,
                                          const int64_t *query_positions, const float *key_positions,
                                          float *probabilities, float *output_projection, int64_t window,
                                          int64_t groups, int64_t length, float scale, lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(window > 0 && groups > 0 && length > 0, "Empty attention dimensions");
  LRK_REQUIRE(length <= INT32_MAX && groups <= INT32_MAX && window * groups <= INT32_MAX, "attention too large");
  LRK_REQUIRE(logits && projected_values && query_positions && key_positions && probabilities && output_projection,
              "null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t rows = window * groups;
  switch (logits_dtype) {
    case LRK_BF16:
      return launch_probabilities<__nv_bfloat16>(logits, projected_values, query_positions, key_positions,
                                                 probabilities, output_projection, rows, static_cast<int>(groups),
                                                 length, scale, s);
    case LRK_F16:
      return launch_probabilities<__half>(logits, projected_values, query_positions, key_positions, probabilities,
                                          output_projection, rows, static_cast<int>(groups), length, scale, s);
    case LRK_F32:
      return launch_probabilities<float>(logits, projected_values, query_positions, key_positions, probabilities,
                                         output_projection, rows, static_cast<int>(groups), length, scale, s);
    default:
      return fail(LRK_ERR_UNSUPPORTED, "Only FP32/FP16/BF16 scores are supported");
  }
}

extern "C" int lrk_temporal_risk(const float *probabilities, const float *output_projection,
                                 const float *projected_values, const float *margin, float *scores, int64_t window,
                                 int64_t groups, int64_t length, int64_t first, int64_t last, float epsilon,
                                 lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(window > 0 && groups > 0 && first >= 0 && last > first && last <= length && epsilon > 0,
              "Invalid risk interval");
  LRK_REQUIRE(window <= INT32_MAX && groups <= INT32_MAX, "risk too large");
  LRK_REQUIRE(probabilities && output_projection && projected_values && margin && scores, "null pointer");
  const int64_t count = last - first;
  const int64_t blocks = ceil_div(count, 32);
  LRK_REQUIRE(blocks <= INT32_MAX, "too many candidates");
  const int sms = sm_count();
  int split = 8;
  if (blocks < 2 * sms) split = 16;
  if (blocks < sms) split = 32;
  split = static_cast<int>(std::min<int64_t>(split, std::max<int64_t>(1, window)));
  dim3 block(32, split);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int g = static_cast<int>(groups);
  if (g <= 4)
    risk_kernel<4><<<static_cast<unsigned>(blocks), block, 0, s>>>(probabilities, output_projection, projected_values,
                                                                    margin, scores, static_cast<int>(window), g,
                                                                    length, first, count, epsilon);
  else if (g <= 8)
    risk_kernel<8><<<static_cast<unsigned>(blocks), block, 0, s>>>(probabilities, output_projection, projected_values,
                                                                    margin, scores, static_cast<int>(window), g,
                                                                    length, first, count, epsilon);
  else
    risk_kernel<0><<<static_cast<unsigned>(blocks), block, 0, s>>>(probabilities, output_projection, projected_values,
                                                                    margin, scores, static_cast<int>(window), g,
                                                                    length, first, count, epsilon);
  return launch_status("lrk_temporal_risk");
}

extern "C" int lrk_pool(const float *scores, int64_t n, const int64_t *bounds, int64_t segments,
                        int64_t maximum_count, int64_t width, float *out, lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(width > 0 && width % 2 == 1 && maximum_count > 0, "Invalid pool configuration");
  LRK_REQUIRE(segments >= 1 && n >= 0, "Invalid pool layout");
  if (n == 0) return LRK_OK;
  LRK_REQUIRE(scores && bounds && out, "null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (width / 2 <= kPoolHalo && aligned(scores, 16) && aligned(out, 16)) {
    // Tiles per segment: the longest segment plus its leading misalignment.
    const int64_t tiles = std::max<int64_t>(1, std::min<int64_t>(ceil_div(maximum_count + 3, kPoolTile), 65535));
    dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(std::min<int64_t>(segments, 65535)));
    const int half = static_cast<int>(width / 2);
    if (half == 3)
      pool_tile_kernel<3><<<grid, kPoolThreads, 0, s>>>(scores, n, bounds, segments, half, out);
    else
      pool_tile_kernel<0><<<grid, kPoolThreads, 0, s>>>(scores, n, bounds, segments, half, out);
    return launch_status("lrk_pool");
  }
  const int threads = 256;
  const int64_t tiles = std::max<int64_t>(1, std::min<int64_t>(ceil_div(maximum_count, threads), 65535));
  dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(std::min<int64_t>(segments, 65535)));
  const int half = static_cast<int>(std::min<int64_t>(width / 2, INT32_MAX));
  pool_kernel<<<grid, threads, 0, s>>>(scores, n, bounds, segments, half, out);
  return launch_status("lrk_pool");
}

extern "C" int lrk_decision_risk(const float *probabilities, const void *values, int values_dtype,
                                 const float *head_outputs, const float *gradients, int64_t groups,
                                 int64_t candidates, int64_t dimension, double base_margin, float epsilon,
                                 float *scores, lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(groups >= 0 && candidates >= 0 && dimension >= 0, "invalid sizes");
  LRK_REQUIRE(epsilon > 0.0f && epsilon < 1.0f, "denominator_epsilon must be in (0,1)");
  if (candidates == 0) return LRK_OK;
  LRK_REQUIRE(groups * dimension <= INT32_MAX && candidates <= INT32_MAX, "too large");
  LRK_REQUIRE(probabilities && values && head_outputs && gradients && scores, "null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(candidates);
  const int g = static_cast<int>(groups), d = static_cast<int>(dimension);
  switch (values_dtype) {
    case LRK_F32:
      decision_risk_kernel<float><<<grid, kLanes, 0, s>>>(scores, probabilities, static_cast<const float *>(values),
                                                          head_outputs, gradients, g, candidates, d, base_margin,
                                                          epsilon);
      break;
    case LRK_F64:
      decision_risk_kernel<double><<<grid, kLanes, 0, s>>>(scores, probabilities, static_cast<const double *>(values),
                                                           head_outputs, gradients, g, candidates, d, base_margin,
                                                           epsilon);
      break;
    case LRK_F16:
      decision_risk_kernel<__half><<<grid, kLanes, 0, s>>>(scores, probabilities, static_cast<const __half *>(values),
                                                           head_outputs, gradients, g, candidates, d, base_margin,
                                                           epsilon);
      break;
    case LRK_BF16:
      decision_risk_kernel<__nv_bfloat16><<<grid, kLanes, 0, s>>>(
          scores, probabilities, static_cast<const __nv_bfloat16 *>(values), head_outputs, gradients, g, candidates,
          d, base_margin, epsilon);
      break;
    default:
      return fail(LRK_ERR_UNSUPPORTED, "unsupported values dtype");
  }
  return launch_status("lrk_decision_risk");
}
