// Projected values of a layer for the audit (scoring.py:175): each packed row
// against its own KV head's query-head margin gradients.
//
// The reference forms g V^T per head with a float32 GEMM after converting V to
// float32 (a [G, D] x [D, L] product per head); at the audit's head sizes that
// GEMM accumulates each dot product in channel order with one fused
// multiply-add per channel.  sequential_dim_kernel (16-bit values in 16-byte
// aligned rows, D = 64 or 128) and sequential_kernel (any other D, or
// unaligned rows) keep that order: a thread per row, G accumulators, the
// gradients transposed in shared memory so that one read serves the G
// products of a channel.  project_kernel (a warp per row) serves other group
// counts, and rows_kernel (lanes sharing a row, butterfly reduce-scatter) is a
// build option (LRK_PROJECT_LANES); both sum in their own order.
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

template <typename T> __device__ __forceinline__ float2 unpack_pair(uint32_t w);
template <> __device__ __forceinline__ float2 unpack_pair<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack_pair<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

constexpr int kRowsBatch = 4;  // row groups whose loads are in flight together

// LPR = D / 8 lanes per row (G <= LPR), 32 / LPR rows per warp step.  Warp w
// owns rows [w * chunk, (w + 1) * chunk).
template <typename T, int G, int LPR>
__global__ void __launch_bounds__(kProjectThreads) rows_kernel(const T *__restrict__ values, int64_t rows,
                                                               const float *__restrict__ gradients,
                                                               const int32_t *__restrict__ cumulative, int heads,
                                                               int64_t chunk, float *__restrict__ out) {
  constexpr int kDim = LPR * 8;
  constexpr int kRowsPerStep = 32 / LPR;
  constexpr int kSteps = LPR == 1 ? 0 : LPR == 2 ? 1 : LPR == 4 ? 2 : LPR == 8 ? 3 : LPR == 16 ? 4 : 5;
  constexpr int kHalvings = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
  static_assert(G <= LPR, "each lane keeps at least one group after the halvings");
  __shared__ int32_t bounds[kMaxProjectHeads + 1];
  for (int i = threadIdx.x; i <= heads; i += kProjectThreads) bounds[i] = cumulative[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;       // which 8 channels
  const int slot = lane / LPR;      // which row of the step
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * (kProjectThreads / 32) + (threadIdx.x >> 5);
  const int64_t begin = warp * chunk, end = lmin(rows, begin + chunk);
  const int64_t first = bounds[0], past = bounds[heads];
  // The group this lane writes after the reduce-scatter, and whether it writes.
  int my_group = 0;
#pragma unroll
  for (int s = 0; s < kHalvings; ++s)
    if (sub & (LPR >> (s + 1))) my_group += G >> (s + 1);
  const bool writer = (sub & ((LPR >> kHalvings) - 1)) == 0;

  int head = -1;
  int64_t head_end = 0;
  float grad[G][8];
  const uint4 *base = reinterpret_cast<const uint4 *>(values);
  for (int64_t r0 = begin; r0 < end; r0 += kRowsPerStep * kRowsBatch) {
    uint4 raw[kRowsBatch];
#pragma unroll
    for (int b = 0; b < kRowsBatch; ++b) {
      const int64_t r = r0 + b * kRowsPerStep + slot;
      raw[b] = r < end ? __ldcs(base + r * LPR + sub) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int b = 0; b < kRowsBatch; ++b) {
      const int64_t r = r0 + b * kRowsPerStep + slot;
      const bool live = r < end && r >= first && r < past;
      if (live && (head < 0 || r >= head_end || r < bounds[head])) {
        int lo = 0, hi = heads;  // head h with bounds[h] <= r < bounds[h + 1]
        while (hi - lo > 1) {
          const int mid = (lo + hi) / 2;
          if (bounds[mid] <= r) lo = mid; else hi = mid;
        }
        head = lo;
        head_end = bounds[lo + 1];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 *src = reinterpret_cast<const float4 *>(gradients + (static_cast<int64_t>(head) * G + g) * kDim +
                                                               sub * 8);
          const float4 a = __ldg(src), c = __ldg(src + 1);
          grad[g][0] = a.x; grad[g][1] = a.y; grad[g][2] = a.z; grad[g][3] = a.w;
          grad[g][4] = c.x; grad[g][5] = c.y; grad[g][6] = c.z; grad[g][7] = c.w;
        }
      }
      float acc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 x = unpack_pair<T>(word_of(raw[b], i));
#pragma unroll
        for (int g = 0; g < G; ++g) {
          acc[g] = fmaf(grad[g][2 * i], x.x, acc[g]);
          acc[g] = fmaf(grad[g][2 * i + 1], x.y, acc[g]);
        }
      }
      // Butterfly reduce-scatter across the LPR lanes of the row: while a lane
      // holds n >= 2 partial sums it keeps one half and sends the other.
#pragma unroll
      for (int s = 0; s < kSteps; ++s) {
        const int offset = LPR >> (s + 1);
        const int n = G >> s;
        if (n >= 2) {
          const bool upper = (sub & offset) != 0;
#pragma unroll
          for (int i = 0; i < n / 2; ++i) {
            const float send = upper ? acc[i] : acc[i + n / 2];
            const float keep = upper ? acc[i + n / 2] : acc[i];
            acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, offset);
          }
        } else {
          acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], offset);
        }
      }
      if (live && writer) out[static_cast<int64_t>(my_group) * rows + r] = acc[0];
    }
  }
}

// Thread per row, each of the G dot products accumulated in channel order
// with one fused multiply-add per channel from 0: acc = fma(g[d], v[d], acc),
// d = 0 .. D-1.  Gradients sit in shared memory transposed to [head][d][g],
// so one broadcast read serves the G products of a channel.
template <typename T, int G>
__global__ void __launch_bounds__(kProjectThreads) sequential_kernel(const T *__restrict__ values, int64_t rows,
                                                                     int dim, const float *__restrict__ gradients,
                                                                     const int32_t *__restrict__ cumulative,
                                                                     int heads, bool vector_rows,
                                                                     float *__restrict__ out) {
  extern __shared__ float transposed[];  // [heads][dim][G]
  __shared__ int32_t bounds[kMaxProjectHeads + 1];
  for (int i = threadIdx.x; i < heads * G * dim; i += kProjectThreads) {
    const int h = i / (G * dim), g = (i / dim) % G, d = i % dim;
    transposed[(h * dim + d) * G + g] = gradients[i];
  }
  for (int i = threadIdx.x; i <= heads; i += kProjectThreads) bounds[i] = cumulative[i];
  __syncthreads();
  const int64_t first = bounds[0], past = bounds[heads];
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kProjectThreads + threadIdx.x; r < rows;
       r += static_cast<int64_t>(gridDim.x) * kProjectThreads) {
    if (r < first || r >= past) continue;
    int lo = 0, hi = heads;  // head h with bounds[h] <= r < bounds[h + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) / 2;
      if (bounds[mid] <= r) lo = mid; else hi = mid;
    }
    const float *grad = transposed + static_cast<int64_t>(lo) * dim * G;
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.0f;
    auto channel = [&](int d, float x) {
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = __fmaf_rn(grad[d * G + g], x, acc[g]);
    };
    const T *row = values + r * dim;
    if constexpr (sizeof(T) == 2) {
      if (vector_rows) {
        const uint4 *vec = reinterpret_cast<const uint4 *>(row);
        for (int c = 0; c < dim / 8; ++c) {
          const uint4 raw = __ldg(vec + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 x = unpack_pair<T>(word_of(raw, i));
            channel(c * 8 + 2 * i, x.x);
            channel(c * 8 + 2 * i + 1, x.y);
          }
        }
      } else {
        for (int d = 0; d < dim; ++d) channel(d, as_float(__ldg(row + d)));
      }
    } else {
      for (int d = 0; d < dim; ++d) channel(d, as_float(__ldg(row + d)));
    }
#pragma unroll
    for (int g = 0; g < G; ++g) out[static_cast<int64_t>(g) * rows + r] = acc[g];
  }
}

// sequential_kernel for 16-bit rows of DIM channels in 16-byte aligned rows:
// the same per-channel FMA order, with the loops unrolled at compile time.
// A CTA stages tiles of 256 consecutive rows (one contiguous block of
// 256 * DIM * 2 bytes) in shared memory with coalesced 16-byte loads, 16-byte
// chunk c of row r at chunk c ^ (r & 7) of the row (so the 8 threads of a
// quarter-warp, each reading the same chunk of its own row, touch 8
// distinct bank groups); then each thread takes one row of the tile.  A
// channel's G gradients are one vector read from shared memory.
constexpr int kTileRows = kProjectThreads;

template <int DIM>
__host__ __device__ constexpr size_t sequential_tile_bytes() {
  return static_cast<size_t>(kTileRows) * DIM * 2;
}

template <typename T, int G, int DIM>
__global__ void __launch_bounds__(kProjectThreads, 2) sequential_dim_kernel(const T *__restrict__ values, int64_t rows,
                                                                           const float *__restrict__ gradients,
                                                                           const int32_t *__restrict__ cumulative,
                                                                           int heads, float *__restrict__ out) {
  static_assert(DIM % 64 == 0, "at least 8 16-byte chunks per row");
  constexpr int kChunks = DIM / 8;
  extern __shared__ __align__(16) unsigned char project_shared[];
  uint4 *tile = reinterpret_cast<uint4 *>(project_shared);                                  // [kTileRows][kChunks]
  float *transposed = reinterpret_cast<float *>(project_shared + sequential_tile_bytes<DIM>());  // [heads][DIM][G]
  __shared__ int32_t bounds[kMaxProjectHeads + 1];
  for (int i = threadIdx.x; i < heads * G * DIM; i += kProjectThreads) {
    const int h = i / (G * DIM), g = (i / DIM) % G, d = i % DIM;
    transposed[(h * DIM + d) * G + g] = gradients[i];
  }
  for (int i = threadIdx.x; i <= heads; i += kProjectThreads) bounds[i] = cumulative[i];
  const uint4 *source = reinterpret_cast<const uint4 *>(values);
  const int64_t tiles = (rows + kTileRows - 1) / kTileRows;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t r0 = t * kTileRows;
    const int in_tile = static_cast<int>(lmin(kTileRows, rows - r0));
    __syncthreads();  // the previous tile's reads (and the set-up above) are done
    const uint4 *block = source + r0 * kChunks;
    if (in_tile == kTileRows) {
      // All of the thread's kChunks loads in flight at once, then the stores.
      uint4 staged[kChunks];
#pragma unroll
      for (int u = 0; u < kChunks; ++u) staged[u] = __ldcs(block + threadIdx.x + u * kProjectThreads);
#pragma unroll
      for (int u = 0; u < kChunks; ++u) {
        const int v = threadIdx.x + u * kProjectThreads, row = v / kChunks, c = v % kChunks;
        tile[row * kChunks + (c ^ (row & 7))] = staged[u];
      }
    } else {
      for (int v = threadIdx.x; v < in_tile * kChunks; v += kProjectThreads) {
        const int row = v / kChunks, c = v % kChunks;
        tile[row * kChunks + (c ^ (row & 7))] = __ldcs(block + v);
      }
    }
    __syncthreads();
    const int64_t r = r0 + threadIdx.x;
    if (threadIdx.x >= in_tile || r < bounds[0] || r >= bounds[heads]) continue;
    uint4 raw[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) raw[c] = tile[threadIdx.x * kChunks + (c ^ (threadIdx.x & 7))];
    int lo = 0, hi = heads;  // head h with bounds[h] <= r < bounds[h + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) / 2;
      if (bounds[mid] <= r) lo = mid; else hi = mid;
    }
    const float *grad = transposed + lo * DIM * G;
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.0f;
#pragma unroll
    for (int d = 0; d < DIM; ++d) {
      const float2 pair = unpack_pair<T>(word_of(raw[d / 8], (d % 8) / 2));
      const float x = d % 2 ? pair.y : pair.x;
      float w[G];
      if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g = 0; g < G; g += 4) {
          const float4 q = *reinterpret_cast<const float4 *>(grad + d * G + g);
          w[g] = q.x, w[g + 1] = q.y, w[g + 2] = q.z, w[g + 3] = q.w;
        }
      } else if constexpr (G == 2) {
        const float2 q = *reinterpret_cast<const float2 *>(grad + d * G);
        w[0] = q.x, w[1] = q.y;
      } else {
        w[0] = grad[d];
      }
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = __fmaf_rn(w[g], x, acc[g]);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) out[static_cast<int64_t>(g) * rows + r] = acc[g];
  }
}

template <typename T, int G, int DIM>
int launch_sequential_dim(const void *values, int64_t rows, const float *gradients, const int32_t *cumulative,
                          int heads, float *out, cudaStream_t stream) {
  const size_t shared = sequential_tile_bytes<DIM>() + static_cast<size_t>(heads) * G * DIM * sizeof(float);
  auto kernel = sequential_dim_kernel<T, G, DIM>;
  if (shared > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
    if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  }
  const int grid = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(ceil_div(rows, kTileRows), static_cast<int64_t>(sm_count()) * 2)));
  kernel<<<grid, kProjectThreads, shared, stream>>>(static_cast<const T *>(values), rows, gradients, cumulative, heads,
                                                    out);
  return launch_status("lrk_project_values");
}

template <typename T, int G>
int launch_sequential(const void *values, int64_t rows, int dim, const float *gradients, const int32_t *cumulative,
                      int heads, float *out, cudaStream_t stream) {
  if constexpr (sizeof(T) == 2) {
    // The staged tile and the gradients must fit one CTA's shared memory.
    const bool fits = static_cast<size_t>(heads) * G * dim * sizeof(float) + kTileRows * dim * 2 <= 200 * 1024;
    if (aligned(values, 16) && fits) {
      if (dim == 128) return launch_sequential_dim<T, G, 128>(values, rows, gradients, cumulative, heads, out, stream);
      if (dim == 64) return launch_sequential_dim<T, G, 64>(values, rows, gradients, cumulative, heads, out, stream);
    }
  }
  const size_t shared = static_cast<size_t>(heads) * G * dim * sizeof(float);
  auto kernel = sequential_kernel<T, G>;
  if (shared > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
    if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  }
  const bool vector_rows = sizeof(T) == 2 && dim % 8 == 0 && aligned(values, 16);
  const int grid = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(ceil_div(rows, kProjectThreads), static_cast<int64_t>(sm_count()) * 8)));
  kernel<<<grid, kProjectThreads, shared, stream>>>(static_cast<const T *>(values), rows, dim, gradients, cumulative,
                                                    heads, vector_rows, out);
  return launch_status("lrk_project_values");
}

template <typename T, int G>
int launch_rows(const void *values, int64_t rows, int dim, const float *gradients, const int32_t *cumulative,
                int heads, float *out, cudaStream_t stream) {
  const int64_t warps = static_cast<int64_t>(sm_count()) * (2048 / 32);
  const int lpr = dim / 8;
  const int64_t step = (32 / lpr) * kRowsBatch;
  const int64_t chunk = ceil_div(ceil_div(rows, warps), step) * step;
  const int grid = static_cast<int>(ceil_div(ceil_div(rows, chunk), kProjectThreads / 32));
  const T *v = static_cast<const T *>(values);
  switch (lpr) {
    case 8: rows_kernel<T, G, 8><<<grid, kProjectThreads, 0, stream>>>(v, rows, gradients, cumulative, heads, chunk, out); break;
    case 16: rows_kernel<T, G, 16><<<grid, kProjectThreads, 0, stream>>>(v, rows, gradients, cumulative, heads, chunk, out); break;
    case 32: rows_kernel<T, G, 32><<<grid, kProjectThreads, 0, stream>>>(v, rows, gradients, cumulative, heads, chunk, out); break;
    default: return fail(LRK_ERR_UNSUPPORTED, "rows_kernel: unsupported dimension");
  }
  return launch_status("lrk_project_values");
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
#ifdef LRK_PROJECT_LANES
  if constexpr (sizeof(T) == 2) {
    // 16-byte rows of 8-channel lane slices; gradients read as float4.
    const bool fast = (dim == 64 || dim == 128 || dim == 256) && groups <= dim / 8 && aligned(values, 16) &&
                      aligned(gradients, 16);
    if (fast) {
      switch (groups) {
        case 1: return launch_rows<T, 1>(values, rows, dim, gradients, cumulative, heads, out, stream);
        case 2: return launch_rows<T, 2>(values, rows, dim, gradients, cumulative, heads, out, stream);
        case 4: return launch_rows<T, 4>(values, rows, dim, gradients, cumulative, heads, out, stream);
        case 8: return launch_rows<T, 8>(values, rows, dim, gradients, cumulative, heads, out, stream);
        default: break;
      }
    }
  }
#endif
  switch (groups) {
    case 1: return launch_sequential<T, 1>(values, rows, dim, gradients, cumulative, heads, out, stream);
    case 2: return launch_sequential<T, 2>(values, rows, dim, gradients, cumulative, heads, out, stream);
    case 4: return launch_sequential<T, 4>(values, rows, dim, gradients, cumulative, heads, out, stream);
    case 8: return launch_sequential<T, 8>(values, rows, dim, gradients, cumulative, heads, out, stream);
    default: break;
  }
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
