// Q K^T logits of one head on the 5th-generation tensor cores (tcgen05), in
// the accumulation order of the bf16 GEMM torch.matmul runs for the same
// product (src/lazy_recall/scoring.py:184).
//
// cuBLAS accumulates each product in float32 over K/16 sixteen-term tensor-core
// steps in increasing k when the key count is even, and over K/8 eight-term
// steps when it is odd.  A sixteen-term step whose upper or lower eight terms
// are zero in A (and finite in B) gives exactly the eight-term step's result
// (measured on B200 against torch.matmul at every tested shape, configs[1]
// heads included), so both orders run as UMMA
// (tcgen05.mma kind::f16, M = 128, N = 128, K = 16):
//   sixteen-term order   A = the query tile, B = the key tile, as usual;
//   eight-term order     step j reads the key tile's 32-byte pair of
//                        chunks that holds chunk j (the sixteen-term order's
//                        pairs, each read twice), and A (built in shared
//                        memory) holds query chunk j in the half of the step
//                        that meets key chunk j and zeros in the other, so
//                        the step multiplies query chunk j by key chunk j
//                        alone.
// Operands are K-major with 128-byte swizzling (8 rows x 128 B atoms, what a
// 64-element x 128-row TMA box writes); step j starts inside its atom at
// 32-byte offsets.
//
// One CTA (1 per SM) owns 128 query rows and a contiguous range of 128-key
// tiles; warp-specialised:
//   warp 9, one thread   TMA loads of key tiles into a ring of stages
//                        (full/empty mbarriers);
//   warp 8, one thread   the UMMAs of each tile into one of four TMEM
//                        accumulators (all 512 columns), committed to the
//                        accumulator's and the stage's mbarriers -- it never
//                        waits for its own MMAs, so several tiles stay queued;
//   warps 0-7            build the query tile once; then two warpgroups
//                        draining alternate tiles:
//                        tcgen05.ld of the warp's 32 TMEM lanes (= query rows),
//                        release, round to bf16 into the group's 128B-swizzled
//                        staging tile, TMA store (which clips columns past
//                        `count` and rows past `rows`).
//
// Every mbarrier wait is bounded (polls and one second of %globaltimer); a
// timeout raises a CTA-wide abort flag, the roles stop, the issuer waits
// (bounded) for its own TMA loads and MMAs in flight, TMEM is freed and the
// CTA returns; g_logits_timeouts counts such CTAs.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace lrk {

__device__ unsigned int g_logits_timeouts = 0;

namespace {

using namespace tc;

constexpr int kEpilogueGroups = 2;                  // warpgroups draining alternate tiles
constexpr int kEpilogueWarps = 4 * kEpilogueGroups;  // warps 0-7
constexpr int kIssuerWarp = kEpilogueWarps;          // warp 8: UMMA issue
constexpr int kLoaderWarp = kEpilogueWarps + 1;      // warp 9: TMA loads
constexpr int kThreadsTc = (kEpilogueWarps + 2) * 32;
constexpr uint32_t kOutTile = kRows * kKeys * 2;  // one bf16 output tile (two 64-column halves)
constexpr int kAccumulators = 4;                       // fp32 accumulators in TMEM
constexpr uint32_t kTmemColumns = kAccumulators * kKeys;

template <int DIM, bool EIGHT>
struct TcLayout {
  static constexpr int kChunks = DIM / 8;                        // 8-element chunks per row
  static constexpr int kSteps = EIGHT ? kChunks : kChunks / 2;   // UMMA K=16 steps per tile
  static constexpr int kAAtoms = EIGHT ? DIM / 32 : DIM / 64;    // query tile (interleaved for EIGHT)
  static constexpr int kBAtoms = DIM / 64;
  static constexpr int kStages = EIGHT ? 3 : 4;
  static constexpr uint32_t kOut = 0;                             // 2 staging tiles
  static constexpr uint32_t kA = kOut + 2 * kOutTile;
  static constexpr uint32_t kB = kA + kAAtoms * kAtom;
  static constexpr uint32_t kStage = kBAtoms * kAtom;
  static constexpr uint32_t kBarriers = kB + kStages * kStage;   // full[S] empty[S] acc_full[4] acc_empty[4]
  static constexpr uint32_t kTmemSlot = kBarriers + 128;
  static constexpr uint32_t kAbort = kTmemSlot + 8;
  static constexpr uint32_t kCounters = kAbort + 8;                // tiles consumed by MMAs, tiles loaded
  static constexpr uint32_t kBytes = kCounters + 8 + 1024;         // + alignment slack
};

template <int DIM, bool EIGHT>
__global__ void __launch_bounds__(kThreadsTc, 1)
    logits_tc_kernel(const __nv_bfloat16 *__restrict__ queries, const __grid_constant__ CUtensorMap key_map,
                     const __grid_constant__ CUtensorMap out_map, int64_t rows, int64_t count, int tiles_per_cta) {
  using L = TcLayout<DIM, EIGHT>;
  constexpr int S = L::kStages;
  extern __shared__ unsigned char smem_raw[];
  // Swizzled atoms and TMA destinations: 1024-byte aligned base.
  const uint32_t raw = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char *smem = smem_raw + (base - raw);
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kRows;
  const int64_t key_tiles = (count + kKeys - 1) / kKeys;
  const int64_t t_begin = static_cast<int64_t>(blockIdx.x) * tiles_per_cta;
  const int tiles = static_cast<int>(lmin(key_tiles, t_begin + tiles_per_cta) - t_begin);
  if (tiles <= 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t bar = base + L::kBarriers;
  auto full = [&](int s) { return bar + 8 * s; };
  auto empty = [&](int s) { return bar + 8 * (S + s); };
  auto acc_full = [&](int a) { return bar + 8 * (2 * S + a); };
  auto acc_empty = [&](int a) { return bar + 8 * (2 * S + kAccumulators + a); };
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::kAbort);
  // The CTAs of the query tiles that share a key range start at different
  // tiles of it, so they do not all ask L2 for the same key tile at once.
  const int rotation = tiles > 1 ? static_cast<int>((blockIdx.y * static_cast<int64_t>(tiles)) / gridDim.y) % tiles : 0;
  auto rotated = [&](int t) { return (t + rotation) % tiles; };

  if (warp < kEpilogueWarps) {
    // The query tile, swizzled; for EIGHT step j's 32-byte window holds query
    // chunk j in the half that meets key chunk j and zeros in the other
    // (A-chunks 2j, 2j + 1 = (q_j, 0) for even j, (0, q_j) for odd j).
    constexpr int kQChunks = DIM / 8;
    for (int i = threadIdx.x; i < kRows * kQChunks; i += kEpilogueWarps * 32) {
      const int r = i / kQChunks, j = i % kQChunks;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (m0 + r < rows) v = __ldg(reinterpret_cast<const uint4 *>(queries + (m0 + r) * DIM) + j);
      const int a = EIGHT ? 2 * j + (j & 1) : j;  // chunk index in the A tile
      *reinterpret_cast<uint4 *>(smem + L::kA + (a >> 3) * kAtom + swizzled(r, a & 7)) = v;
      if (EIGHT) {
        const int z = 2 * j + 1 - (j & 1);
        *reinterpret_cast<uint4 *>(smem + L::kA + (z >> 3) * kAtom + swizzled(r, z & 7)) = make_uint4(0, 0, 0, 0);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic writes -> tensor-core reads
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(full(s)) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(empty(s)) : "memory");
    }
    for (int a = 0; a < kAccumulators; ++a) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(acc_full(a)) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;\n" ::"r"(acc_empty(a)) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    *abort = 0;
    reinterpret_cast<volatile int *>(smem + L::kCounters)[0] = 0;
    reinterpret_cast<volatile int *>(smem + L::kCounters)[1] = 0;
  }
  if (warp == kIssuerWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(base + L::kTmemSlot),
                 "r"(kTmemColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + L::kTmemSlot);

  volatile int *counters = reinterpret_cast<volatile int *>(smem + L::kCounters);
  if (warp == kLoaderWarp) {
    if (lane == 0) {
      // ------------------------------------------------------- TMA loads
      // Stage t % S takes tile t once the MMAs of tile t - S are done.
      int loaded = 0;
      for (int t = 0; t < tiles; ++t) {
        const int s = t % S;
        if (t >= S && !wait_phase(empty(s), ((t / S) - 1) & 1, abort)) break;
        expect_bytes(full(s), L::kStage);
        const int y = static_cast<int>((t_begin + rotated(t)) * kKeys);
        const uint32_t dst = base + L::kB + s * L::kStage;
#pragma unroll
        for (int b = 0; b < L::kBAtoms; ++b) tma_box(dst + b * kAtom, &key_map, 64 * b, y, full(s));
        loaded = t + 1;
      }
      counters[1] = loaded;
    }
  } else if (warp == kIssuerWarp) {
    if (lane == 0) {
      // ------------------------------------------------------- MMA issue
      // Never waits on its own MMAs inside the loop: the tensor pipe keeps
      // up to kAccumulators tiles queued.
      int issued = 0;  // tiles whose MMAs were issued
      bool ok = true;
      for (int t = 0; t < tiles; ++t) {
        const int s = t % S, a = t % kAccumulators;
        if (!wait_phase(full(s), (t / S) & 1, abort)) { ok = false; break; }
        if (t >= kAccumulators && !wait_phase(acc_empty(a), ((t / kAccumulators) - 1) & 1, abort)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint32_t A = base + L::kA, B = base + L::kB + s * L::kStage;
        const uint32_t d = tmem + a * kKeys;
#pragma unroll
        for (int j = 0; j < L::kSteps; ++j) {
          // A: 32 bytes per step through its atoms (EIGHT: query chunk j and zeros).
          const uint32_t a_addr = A + (j >> 2) * kAtom + (j & 3) * 32;
          // B: the 32-byte pair of key chunks holding chunk j (EIGHT) or 2j, 2j + 1.
          const int pair = EIGHT ? j >> 1 : j;
          const uint32_t b_addr = B + (pair >> 2) * kAtom + (pair & 3) * 32;
          umma(d, smem_descriptor(a_addr), smem_descriptor(b_addr), j > 0);
        }
        umma_commit(acc_full(a));
        umma_commit(empty(s));
        issued = t + 1;
      }
      // Before the CTA may exit, every arrival this thread set in motion must
      // have landed (bounded waits, whatever the abort flag says).
      for (int t = issued > S ? issued - S : 0; t < issued; ++t) wait_phase(empty(t % S), (t / S) & 1, nullptr);
      if (!ok) {
        for (int t = issued > kAccumulators ? issued - kAccumulators : 0; t < issued; ++t)
          wait_phase(acc_full(t % kAccumulators), (t / kAccumulators) & 1, nullptr);
        *abort = 1;
      }
      counters[0] = issued;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warpgroup g drains the tiles t = g, g + 2, ... (accumulator t % 4).
    // Thread = query row r (its TMEM lane).  Each 64-column half of the bf16
    // tile is staged as 128 rows x 128 B with 128B swizzling (16-byte chunk c
    // of row r at chunk c ^ (r % 8): a quarter-warp's 8 rows hit 8 distinct
    // bank groups) and leaves with one TMA store, which clips the columns
    // past `count` and the rows past `rows`.
    const int group = warp >> 2, r = (warp & 3) * 32 + lane;
    const uint32_t named = 1 + group;  // this warpgroup's named barrier
    const bool issuer = (threadIdx.x & 127) == 0;
    const uint32_t stage_out = base + L::kOut + group * kOutTile;
    for (int t = group; t < tiles; t += kEpilogueGroups) {
      const int a = t % kAccumulators;
      // The group's 128 threads leave together or not at all (they meet in
      // named barriers below): AND of every thread's wait.
      const uint32_t got = wait_phase(acc_full(a), (t / kAccumulators) & 1, abort) ? 1u : 0u;
      uint32_t all_got;
      asm volatile(
          "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
          : "=r"(all_got)
          : "r"(got), "r"(named)
          : "memory");
      if (!all_got) {
        *abort = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      uint32_t v[kKeys];
#pragma unroll
      for (int part = 0; part < kKeys / 32; ++part)
        tmem_load32(tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + a * kKeys + part * 32, v + part * 32);
      asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      __syncwarp();
      if (lane == 0) arrive(acc_empty(a));  // the accumulator is free for tile t + kAccumulators
      // The group's previous store has read the staging tile.
      if (issuer && t >= kEpilogueGroups) asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
      asm volatile("bar.sync %0, 128;\n" ::"r"(named) : "memory");
#pragma unroll
      for (int half = 0; half < 2; ++half)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = half * 64 + c * 8 + 2 * e;
            const __nv_bfloat162 pair = __floats2bfloat162_rn(__uint_as_float(v[col]), __uint_as_float(v[col + 1]));
            w[e] = *reinterpret_cast<const uint32_t *>(&pair);
          }
          const uint32_t dst = stage_out + half * (kOutTile / 2) + r * 128 + ((c ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                       "r"(w[3])
                       : "memory");
        }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // staging -> TMA store reads
      asm volatile("bar.sync %0, 128;\n" ::"r"(named) : "memory");
      if (issuer) {
        const int x = static_cast<int>((t_begin + rotated(t)) * kKeys), y = static_cast<int>(m0);
#pragma unroll
        for (int half = 0; half < 2; ++half)
          asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(
                           reinterpret_cast<uint64_t>(&out_map)),
                       "r"(x + half * 64), "r"(y), "r"(stage_out + half * (kOutTile / 2))
                       : "memory");
        asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
      }
    }
    if (issuer) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");  // stores complete before exit
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  // After an abort, loads the MMAs never consumed must land before the
  // shared memory is released (bounded waits).
  if (warp == kLoaderWarp && lane == 0 && *abort) {
    for (int t = counters[0]; t < counters[1]; ++t) wait_phase(full(t % S), (t / S) & 1, nullptr);
  }
  __syncthreads();
  if (warp == kIssuerWarp) {
    if (lane == 0 && *abort) atomicAdd(&g_logits_timeouts, 1u);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemColumns) : "memory");
  }
}

}  // namespace

namespace tc {

// cuTensorMapEncodeTiled, looked up once through the runtime.
static PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 function = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      function = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return function;
}

// bf16 matrix [rows_total, columns] with a row stride of `stride` elements;
// boxes of box_columns x 128 rows.
int make_map(CUtensorMap *map, const void *data, int64_t rows_total, int64_t columns, int64_t stride,
             uint32_t box_columns, CUtensorMapSwizzle swizzle) {
  auto encode = encode_tiled();
  if (encode == nullptr) return fail(LRK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t sizes[2] = {static_cast<cuuint64_t>(columns), static_cast<cuuint64_t>(rows_total)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 2};
  const cuuint32_t box[2] = {box_columns, kRows};
  const cuuint32_t element_strides[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(data), sizes, strides, box,
                            element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return LRK_ERR_CUDA;
  }
  return LRK_OK;
}

}  // namespace tc

// Tensor-core logits for dim 64 / 128 (LRK_ERR_UNSUPPORTED otherwise).
int launch_logits_tc(const void *queries, int64_t rows, const void *keys, int64_t count, int64_t dim, bool eight,
                     void *out, int64_t out_stride, cudaStream_t stream) {
  if (dim != 64 && dim != 128) return LRK_ERR_UNSUPPORTED;
  if (rows > INT32_MAX || count > INT32_MAX) return fail(LRK_ERR_UNSUPPORTED, "lrk_logits: too many rows");
  CUtensorMap key_map, out_map;
  int status = tc::make_map(&key_map, keys, count, dim, dim, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (status != LRK_OK) return status;
  if ((status = tc::make_map(&out_map, out, rows, count, out_stride, 64, CU_TENSOR_MAP_SWIZZLE_128B)) != LRK_OK)
    return status;
  auto launch = [&](auto kernel, uint32_t bytes) -> int {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
    // One CTA per SM (shared memory), each on a contiguous key range; at most
    // one wave.
    const int64_t m_tiles = ceil_div(rows, kRows), key_tiles = ceil_div(count, kKeys);
    const int64_t splits = std::max<int64_t>(1, std::min<int64_t>(key_tiles, sm_count() / m_tiles));
    const int64_t per = ceil_div(key_tiles, splits);
    const dim3 grid(static_cast<unsigned>(ceil_div(key_tiles, per)), static_cast<unsigned>(m_tiles));
    kernel<<<grid, kThreadsTc, bytes, stream>>>(static_cast<const __nv_bfloat16 *>(queries), key_map, out_map, rows,
                                                count, static_cast<int>(per));
    return launch_status("lrk_logits");
  };
  if (dim == 128)
    return eight ? launch(logits_tc_kernel<128, true>, TcLayout<128, true>::kBytes)
                 : launch(logits_tc_kernel<128, false>, TcLayout<128, false>::kBytes);
  return eight ? launch(logits_tc_kernel<64, true>, TcLayout<64, true>::kBytes)
               : launch(logits_tc_kernel<64, false>, TcLayout<64, false>::kBytes);
}

}  // namespace lrk

using namespace lrk;

extern "C" int lrk_logits_timeouts(unsigned int *count) {
  clear_error();
  LRK_REQUIRE(count != nullptr, "null pointer");
  cudaError_t e = cudaMemcpyFromSymbol(count, g_logits_timeouts, sizeof(unsigned int));
  return e == cudaSuccess ? LRK_OK : fail(LRK_ERR_CUDA, cudaGetErrorString(e));
}
