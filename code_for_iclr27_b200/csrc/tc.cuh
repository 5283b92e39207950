// 5th-generation tensor-core plumbing shared by the tcgen05 kernels
// (logits_tc.cu, scores_tc.cu): bounded mbarrier waits, TMA tile loads,
// UMMA descriptors and issue, TMEM loads, and the host-side tensor-map
// encoder.  sm_100a only.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "common.cuh"

namespace lrk {
namespace tc {

constexpr int kRows = 128;                   // UMMA M: query rows per tile
constexpr int kKeys = 128;                   // UMMA N: keys per tile
constexpr uint32_t kAtom = kRows * 128;      // one 64-element-wide 128B-swizzled atom column of 128 rows: 16 KB
constexpr uint32_t kWaitPolls = 1u << 26;
constexpr uint64_t kWaitNanoseconds = 1000000000ull;

__device__ __forceinline__ uint64_t global_nanoseconds() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the mbarrier phase of the given parity.  False on timeout
// (after which *abort is raised) or when another role raised *abort (abort
// may be null: then only the bound ends the wait).
__device__ __forceinline__ bool wait_phase(uint32_t barrier, uint32_t parity, volatile int *abort) {
  const uint64_t start = global_nanoseconds();
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(barrier), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 63) == 63) {
      if (abort != nullptr && *abort) return false;
      if (global_nanoseconds() - start > kWaitNanoseconds) break;
    }
  }
  if (abort != nullptr) *abort = 1;
  return false;
}

__device__ __forceinline__ void init_barrier(uint32_t barrier, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(barrier), "r"(count) : "memory");
}

__device__ __forceinline__ void arrive(uint32_t barrier) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(barrier) : "memory");
}

__device__ __forceinline__ void expect_bytes(uint32_t barrier, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(barrier), "r"(bytes) : "memory");
}

// TMA: a 64-element x 128-row box at (x, y), 128B-swizzled -> 16 KB.  x must
// be a multiple of 8 (16 bytes of bf16).
__device__ __forceinline__ void tma_box(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t barrier) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(barrier)
      : "memory");
}

// UMMA shared-memory descriptor, K-major, 128-byte swizzle: 8-row groups 1024
// bytes apart (stride), leading offset unused (1), version 1 (bits 46-47),
// layout SWIZZLE_128B (2, bits 61-63).
__device__ __forceinline__ uint64_t smem_descriptor(uint32_t address) {
  return static_cast<uint64_t>((address >> 4) & 0x3FFFu) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both
// K-major, N = 128, M = 128.
constexpr uint32_t kInstr = (1u << 4) | (1u << 7) | (1u << 10) | ((kKeys >> 3) << 17) | ((kRows >> 4) << 24);

__device__ __forceinline__ void umma(uint32_t tmem, uint64_t a, uint64_t b, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(a), "l"(b), "r"(kInstr), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t barrier) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(barrier)
               : "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_load32(uint32_t address, uint32_t *v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(address));
}

// Waits for this thread's TMEM loads; the 32 registers are operands, so that
// no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait_load32(uint32_t *v) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                 "+r"(v[15]), "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]),
                 "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]),
                 "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}

// 16 consecutive fp32 accumulator columns of this thread's TMEM lane, and the
// matching wait.
__device__ __forceinline__ void tmem_load16(uint32_t address, uint32_t *v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(address));
}
__device__ __forceinline__ void tmem_wait_load16(uint32_t *v) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                 "+r"(v[15])
               :
               : "memory");
}

// 16 fp32 columns of this thread's TMEM lane from registers; complete
// before a later tcgen05.ld of the same columns only after tmem_wait_store.
__device__ __forceinline__ void tmem_store16(uint32_t address, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};\n" ::"r"(address),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_store() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// The wait for every outstanding load of this thread, without operands;
// follow it with tmem_loaded16 on each register group it completes.
__device__ __forceinline__ void tmem_wait_loads() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_loaded16(uint32_t *v) {
  asm volatile(""
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                 "+r"(v[15])
               :
               : "memory");
}

// Byte offset of 16-byte chunk c (0..7) of row r inside a 128B-swizzled atom column.
__device__ __forceinline__ uint32_t swizzled(int r, int c) {
  return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Host: tensor map of a bf16 matrix [rows_total, columns] with a row stride of
// `stride` elements; boxes of box_columns x 128 rows (logits_tc.cu).
int make_map(CUtensorMap *map, const void *data, int64_t rows_total, int64_t columns, int64_t stride,
             uint32_t box_columns, CUtensorMapSwizzle swizzle);

}  // namespace tc
}  // namespace lrk
