// Q K^T logits of one head in the accumulation order of the bf16 GEMM that
// torch.matmul runs for it (src/lazy_recall/scoring.py:184), written as rows
// padded to a 16-byte multiple for the scoring kernels.
//
// cuBLAS accumulates each 128-term product in float32 over tensor-core steps
// in increasing k and rounds the sum to bf16.  For an odd key count it runs a
// kernel built on mma m16n8k8 (eight-term steps); otherwise its kernels take
// sixteen-term steps, and the two differ in the last bit of some logits.  This
// kernel issues mma m16n8k8 or m16n8k16 steps (KSTEP) in the same order, so
// its logits equal torch.matmul's bit for bit (checked by the GPU tests).
//
// A CTA keeps 128 query rows in shared memory and walks a contiguous range of
// 64-key tiles, double-buffered with cp.async; 8 warps of 32 x 32 outputs;
// fragments through ldmatrix with the k loop unrolled (DIM is a template
// parameter); each thread stores its bf16 pairs straight from registers.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"

namespace lrk {
namespace {

constexpr int kTileM = 128, kTileN = 64;
constexpr int kThreads = 256;

template <int DIM>
struct Layout {
  static constexpr int kPitch = DIM + 8;  // bf16 per staged row: conflict-free ldmatrix
  static constexpr size_t kSharedBytes =
      (static_cast<size_t>(kTileM) * kPitch + 2 * static_cast<size_t>(kTileN) * kPitch) * 2;
};

__device__ __forceinline__ uint32_t shared_address(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16 bytes global -> shared, zero-filled when !valid.
__device__ __forceinline__ void copy16(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(shared_address(dst)), "l"(src),
               "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void copy_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void copy_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

template <int KSTEP, int DIM>
__global__ void __launch_bounds__(kThreads, 3) logits_kernel(const __nv_bfloat16 *__restrict__ queries,
                                                             int64_t rows, const __nv_bfloat16 *__restrict__ keys,
                                                             int64_t count, __nv_bfloat16 *__restrict__ out,
                                                             int64_t out_stride, int tiles_per_cta) {
  constexpr int kPitch = Layout<DIM>::kPitch;
  constexpr int dim = DIM;
  extern __shared__ __align__(16) __nv_bfloat16 smem[];
  __nv_bfloat16 *q_s = smem;                              // [kTileM][kPitch]
  __nv_bfloat16 *k_s = q_s + kTileM * kPitch;             // [2][kTileN][kPitch]
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kTileM;
  const int64_t key_tiles = (count + kTileN - 1) / kTileN;
  const int64_t t_begin = static_cast<int64_t>(blockIdx.x) * tiles_per_cta;
  const int64_t t_end = lmin(key_tiles, t_begin + tiles_per_cta);
  if (t_begin >= t_end) return;
  constexpr int pieces = dim / 8;                 // 16-byte pieces per row
  constexpr int rows_per_pass = kThreads / pieces;  // rows one pass of the CTA's copies covers
  // This thread's piece within every row it copies.
  const int copy_row = threadIdx.x / pieces, copy_piece = threadIdx.x % pieces;
  for (int r = copy_row; r < kTileM; r += rows_per_pass) {
    const bool valid = m0 + r < rows;
    copy16(q_s + r * kPitch + copy_piece * 8, queries + (valid ? (m0 + r) * dim + copy_piece * 8 : 0), valid);
  }
  const __nv_bfloat16 *key_piece = keys + static_cast<int64_t>(copy_row) * dim + copy_piece * 8;
  auto load_keys = [&](int64_t tile, int buffer) {
    __nv_bfloat16 *dst = k_s + buffer * kTileN * kPitch + copy_row * kPitch + copy_piece * 8;
    const int64_t n0 = tile * kTileN;
    const __nv_bfloat16 *src = key_piece + n0 * dim;
    if (n0 + kTileN <= count) {
#pragma unroll
      for (int u = 0; u < kTileN / rows_per_pass; ++u)
        copy16(dst + u * rows_per_pass * kPitch, src + u * rows_per_pass * dim, true);
    } else {
#pragma unroll
      for (int u = 0; u < kTileN / rows_per_pass; ++u) {
        const bool valid = n0 + copy_row + u * rows_per_pass < count;
        copy16(dst + u * rows_per_pass * kPitch, valid ? src + u * rows_per_pass * dim : keys, valid);
      }
    }
  };
  load_keys(t_begin, 0);
  copy_commit();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;  // warp tile origin in the CTA tile
  const int group = lane >> 2, pair = (lane & 3) * 2;
  // Shared addresses of this lane's fragment rows (k offsets are constants).
  uint32_t a_base[2], b_base[2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
    a_base[i] = shared_address(q_s + (wm + i * 16 + (lane & 15)) * kPitch + (KSTEP == 16 ? (lane >> 4) * 8 : 0));
#pragma unroll
  for (int buffer = 0; buffer < 2; ++buffer) {
    const __nv_bfloat16 *kb = k_s + buffer * kTileN * kPitch;
    b_base[buffer] = KSTEP == 8 ? shared_address(kb + (wn + lane) * kPitch)
                                : shared_address(kb + (wn + (lane & 7) + ((lane >> 4) << 3)) * kPitch +
                                                 ((lane >> 3) & 1) * 8);
  }
  // Output rows of this thread: wm + i * 16 + group (+ 8 for the second half).
  __nv_bfloat16 *row_out[2][2];
  bool row_live[2][2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t r = m0 + wm + i * 16 + group + h * 8;
      row_live[i][h] = r < rows;
      row_out[i][h] = out + (row_live[i][h] ? r : 0) * out_stride + wn + pair;
    }
  const bool full_rows = m0 + kTileM <= rows;

  for (int64_t t = t_begin; t < t_end; ++t) {
    const int buffer = static_cast<int>((t - t_begin) & 1);
    copy_wait_all();
    __syncthreads();  // tile t (and the query rows) visible; the other buffer is free
    if (t + 1 < t_end) load_keys(t + 1, buffer ^ 1);
    copy_commit();
    const uint32_t b_tile = buffer ? b_base[1] : b_base[0];
    float acc[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < dim; k0 += KSTEP) {
      if constexpr (KSTEP == 8) {
        uint32_t a[2][2], b[4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
          asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];\n"
                       : "=r"(a[i][0]), "=r"(a[i][1])
                       : "r"(a_base[i] + k0 * 2));
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                     : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                     : "r"(b_tile + k0 * 2));
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            asm("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, "
                "{%0, %1, %2, %3};\n"
                : "+f"(acc[i][j][0]), "+f"(acc[i][j][1]), "+f"(acc[i][j][2]), "+f"(acc[i][j][3])
                : "r"(a[i][0]), "r"(a[i][1]), "r"(b[j]));
      } else {
        uint32_t a[2][4], b[4][2];
#pragma unroll
        for (int i = 0; i < 2; ++i)
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                       : "=r"(a[i][0]), "=r"(a[i][1]), "=r"(a[i][2]), "=r"(a[i][3])
                       : "r"(a_base[i] + k0 * 2));
#pragma unroll
        for (int j = 0; j < 4; j += 2)
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                       : "=r"(b[j][0]), "=r"(b[j][1]), "=r"(b[j + 1][0]), "=r"(b[j + 1][1])
                       : "r"(b_tile + (j * 8 * kPitch + k0) * 2));
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                "{%8, %9}, {%0, %1, %2, %3};\n"
                : "+f"(acc[i][j][0]), "+f"(acc[i][j][1]), "+f"(acc[i][j][2]), "+f"(acc[i][j][3])
                : "r"(a[i][0]), "r"(a[i][1]), "r"(a[i][2]), "r"(a[i][3]), "r"(b[j][0]), "r"(b[j][1]));
      }
    }
    // bf16 pairs straight to global memory: a quarter-warp writes 16
    // contiguous bytes of each of 8 rows; columns at or past `count` are the
    // row's padding (out_stride rounds count up to 8).
    const int64_t n0 = t * kTileN;
    if (full_rows && n0 + kTileN <= count) {
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          __nv_bfloat16 *row = row_out[i][h] + n0;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<__nv_bfloat162 *>(row + j * 8) =
                __floats2bfloat162_rn(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
        }
    } else {
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          __nv_bfloat16 *row = row_out[i][h] + n0;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (row_live[i][h] && n0 + wn + j * 8 + pair < count)
              *reinterpret_cast<__nv_bfloat162 *>(row + j * 8) =
                  __floats2bfloat162_rn(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
        }
    }
  }
}

}  // namespace
}  // namespace lrk

namespace lrk {
int launch_logits_tc(const void *queries, int64_t rows, const void *keys, int64_t count, int64_t dim, bool eight,
                     void *out, int64_t out_stride, cudaStream_t stream);
int launch_logits_heads(const lrk_logits_head *heads, int64_t head_count, int64_t rows, int64_t dim,
                        cudaStream_t stream);

namespace {
// The argument rules of one head (lrk_logits, lrk_logits_heads).
int check_logits_head(const void *queries, int64_t rows, const void *keys, int64_t count, int64_t dim,
                      int64_t k_step, const void *out, int64_t out_stride) {
  LRK_REQUIRE(rows >= 0 && count >= 0 && dim > 0, "invalid logits sizes");
  LRK_REQUIRE(k_step == 8 || k_step == 16, "k_step must be 8 or 16");
  LRK_REQUIRE(dim == 64 || dim == 128, "lrk_logits takes head dimension 64 or 128");
  LRK_REQUIRE(out_stride >= (count + 7) / 8 * 8 && out_stride % 8 == 0,
              "out_stride must be a multiple of 8 covering the keys rounded up to 8");
  if (rows == 0 || count == 0) return LRK_OK;
  LRK_REQUIRE(queries && keys && out, "null pointer");
  LRK_REQUIRE(aligned(queries, 16) && aligned(keys, 16) && aligned(out, 16), "logits operands must be 16-byte aligned");
  return LRK_OK;
}
}  // namespace
}  // namespace lrk

using namespace lrk;

extern "C" int lrk_logits_heads(const lrk_logits_head *heads, int64_t head_count, int64_t rows, int64_t dim,
                                lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(head_count >= 0 && rows >= 0, "invalid logits sizes");
  LRK_REQUIRE(head_count == 0 || heads != nullptr, "null pointer");
  bool work = false;
  for (int64_t i = 0; i < head_count; ++i) {
    const lrk_logits_head &h = heads[i];
    const int status = check_logits_head(h.queries, rows, h.keys, h.count, dim, h.k_step, h.out, h.out_stride);
    if (status != LRK_OK) return status;
    work = work || h.count > 0;
  }
  if (rows == 0 || !work) return LRK_OK;
#ifndef LRK_LOGITS_MMA_SYNC
  return launch_logits_heads(heads, head_count, rows, dim, reinterpret_cast<cudaStream_t>(stream));
#else
  for (int64_t i = 0; i < head_count; ++i) {
    const lrk_logits_head &h = heads[i];
    const int status = lrk_logits(h.queries, rows, h.keys, h.count, dim, h.k_step, h.out, h.out_stride, stream);
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
#endif
}

extern "C" int lrk_logits(const void *queries, int64_t rows, const void *keys, int64_t count, int64_t dim,
                          int64_t k_step, void *out, int64_t out_stride, lrk_stream_t stream) {
  clear_error();
  const int status = check_logits_head(queries, rows, keys, count, dim, k_step, out, out_stride);
  if (status != LRK_OK) return status;
  if (rows == 0 || count == 0) return LRK_OK;
#ifndef LRK_LOGITS_MMA_SYNC
  // Tensor-core (tcgen05) path; the mma.sync kernel below is its reference.
  return launch_logits_tc(queries, rows, keys, count, dim, k_step == 8, out, out_stride,
                          reinterpret_cast<cudaStream_t>(stream));
#endif
  decltype(&logits_kernel<8, 128>) kernel = nullptr;
  size_t shared = 0;
  if (dim == 128) {
    kernel = k_step == 8 ? logits_kernel<8, 128> : logits_kernel<16, 128>;
    shared = Layout<128>::kSharedBytes;
  } else if (dim == 64) {
    kernel = k_step == 8 ? logits_kernel<8, 64> : logits_kernel<16, 64>;
    shared = Layout<64>::kSharedBytes;
  } else {
    return fail(LRK_ERR_UNSUPPORTED, "lrk_logits takes head dimension 64 or 128");
  }
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
  if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  // About three CTAs per SM over the whole grid, each on a contiguous key range.
  const int64_t m_tiles = ceil_div(rows, kTileM), key_tiles = ceil_div(count, kTileN);
  const int64_t splits = std::max<int64_t>(1, std::min<int64_t>(key_tiles, ceil_div(3 * sm_count(), m_tiles)));
  const int64_t per = ceil_div(key_tiles, splits);
  const dim3 grid(static_cast<unsigned>(ceil_div(key_tiles, per)), static_cast<unsigned>(m_tiles));
  kernel<<<grid, kThreads, shared, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16 *>(queries), rows, static_cast<const __nv_bfloat16 *>(keys), count,
      static_cast<__nv_bfloat16 *>(out), out_stride, static_cast<int>(per));
  return launch_status("lrk_logits");
}
