// Projected values of a layer for the audit (scoring.py:175): each packed row
// against its own KV head's query-head margin gradients.
//
// The reference forms g V^T per head with a float32 GEMM after converting V to
// float32 (a [G, D] x [D, L] product per head).  Here one pass reads the bf16
// V rows once: a warp owns a row, its lanes stride over the row's channels,
// the G partial dot products are folded with warp shuffles, and the head's
// gradients sit in shared memory.  Float32 accumulation; the order of the
// per-row sums is this kernel's own.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"

namespace lrk {
namespace {

constexpr int kProjectThreads = 256;
constexpr int kMaxProjectGroups = 8;
constexpr int kMaxProjectHeads = 64;
constexpr int kRowsPerWarp = 4;

template <typename T> __device__ __forceinline__ float as_float(T v);
template <> __device__ __forceinline__ float as_float(float v) { return v; }
template <> __device__ __forceinline__ float as_float(double v) { return static_cast<float>(v); }
template <> __device__ __forceinline__ float as_float(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float as_float(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T, int G>
__global__ void __launch_bounds__(kProjectThreads) project_kernel(const T *__restrict__ values, int64_t rows, int dim,
                                                                   const float *__restrict__ gradients,
                                                                   const int32_t *__restrict__ cumulative, int heads,
                                                                   float *__restrict__ out) {
  extern __shared__ float shared_gradients[];  // [heads * G * dim]
  __shared__ int32_t bounds[kMaxProjectHeads + 1];
  for (int i = threadIdx.x; i < heads * G * dim; i += kProjectThreads) shared_gradients[i] = gradients[i];
  for (int i = threadIdx.x; i <= heads; i += kProjectThreads) bounds[i] = cumulative[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kProjectThreads / 32);
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * (kProjectThreads / 32) + (threadIdx.x >> 5);
  for (int64_t base = warp * kRowsPerWarp; base < rows; base += warps * kRowsPerWarp) {
#pragma unroll
    for (int u = 0; u < kRowsPerWarp; ++u) {
      const int64_t r = base + u;
      if (r >= rows) break;
      int lo = 0, hi = heads;  // head h with bounds[h] <= r < bounds[h + 1]
      while (hi - lo > 1) {
        const int mid = (lo + hi) / 2;
        if (bounds[mid] <= r) lo = mid; else hi = mid;
      }
      if (r < bounds[0] || r >= bounds[heads]) continue;
      const float *g = shared_gradients + static_cast<int64_t>(lo) * G * dim;
      float acc[G];
#pragma unroll
      for (int j = 0; j < G; ++j) acc[j] = 0.0f;
      const T *row = values + r * dim;
      for (int d = lane; d < dim; d += 32) {
        const float v = as_float(__ldg(row + d));
#pragma unroll
        for (int j = 0; j < G; ++j) acc[j] = fmaf(g[j * dim + d], v, acc[j]);
      }
#pragma unroll
      for (int j = 0; j < G; ++j) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
      }
      if (lane < G) {
        float mine = acc[0];
#pragma unroll
        for (int j = 1; j < G; ++j) if (lane == j) mine = acc[j];
        out[static_cast<int64_t>(lane) * rows + r] = mine;
      }
    }
  }
}

template <typename T, int G>
int launch_project(const void *values, int64_t rows, int dim, const float *gradients, const int32_t *cumulative,
                   int heads, float *out, cudaStream_t stream) {
  const size_t shared = static_cast<size_t>(heads) * G * dim * sizeof(float);
  auto kernel = project_kernel<T, G>;
  if (shared > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
    if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  }
  const int64_t warps_needed = ceil_div(rows, kRowsPerWarp);
  const int grid = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(ceil_div(warps_needed, kProjectThreads / 32), static_cast<int64_t>(sm_count()) * 8)));
  kernel<<<grid, kProjectThreads, shared, stream>>>(static_cast<const T *>(values), rows, dim, gradients, cumulative,
                                                    heads, out);
  return launch_status("lrk_project_values");
}

template <typename T>
int dispatch_groups(const void *values, int64_t rows, int dim, const float *gradients, const int32_t *cumulative,
                    int heads, int groups, float *out, cudaStream_t stream) {
  switch (groups) {
    case 1: return launch_project<T, 1>(values, rows, dim, gradients, cumulative, heads, out, stream);
    case 2: return launch_project<T, 2>(values, rows, dim, gradients, cumulative, heads, out, stream);
    case 4: return launch_project<T, 4>(values, rows, dim, gradients, cumulative, heads, out, stream);
    case 8: return launch_project<T, 8>(values, rows, dim, gradients, cumulative, heads, out, stream);
    default: return fail(LRK_ERR_UNSUPPORTED, "project_values supports 1, 2, 4 or 8 query heads per KV head");
  }
}

}  // namespace
}  // namespace lrk

using namespace lrk;

extern "C" int lrk_project_values(const void *values, int values_dtype, int64_t rows, int64_t dimension,
                                  const float *gradients, const int32_t *cumulative, int64_t heads, int64_t groups,
                                  float *out, lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(rows >= 0 && dimension > 0 && heads > 0 && groups > 0, "invalid projection sizes");
  LRK_REQUIRE(heads <= kMaxProjectHeads && groups <= kMaxProjectGroups, "too many heads or groups");
  LRK_REQUIRE(heads * groups * dimension * 4 <= 200 * 1024, "gradients exceed one CTA's shared memory");
  if (rows == 0) return LRK_OK;
  LRK_REQUIRE(values && gradients && cumulative && out, "null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int d = static_cast<int>(dimension), h = static_cast<int>(heads), g = static_cast<int>(groups);
  switch (values_dtype) {
    case LRK_BF16: return dispatch_groups<__nv_bfloat16>(values, rows, d, gradients, cumulative, h, g, out, s);
    case LRK_F16: return dispatch_groups<__half>(values, rows, d, gradients, cumulative, h, g, out, s);
    case LRK_F32: return dispatch_groups<float>(values, rows, d, gradients, cumulative, h, g, out, s);
    case LRK_F64: return dispatch_groups<double>(values, rows, d, gradients, cumulative, h, g, out, s);
    default: return fail(LRK_ERR_UNSUPPORTED, "unsupported values dtype");
  }
}
