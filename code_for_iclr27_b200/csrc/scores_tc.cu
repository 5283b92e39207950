// Row statistics of the temporal decision-risk scorer straight from the keys:
// the bf16 logits GEMM (src/lazy_recall/scoring.py:184) and the softmax row
// statistics of csrc/scoring.cu:32-66 in one tcgen05 kernel, so the logits
// never reach HBM (only the candidate columns the risk step reads are
// written).
//
// Per (segment = one KV head, M tile = 128 query rows) unit, three passes over
// the head's 128-key tiles, each running the tile's UMMAs again into one of
// two TMEM accumulators (the logits are recomputed, never stored):
//   pass 1  x = dtype(dtype(logit) * scale), masked; the row maximum; the
//           candidate columns' logits written for the risk kernel;
//   pass 2  w = expf(x - max) summed per reference lane;
//   pass 3  p = w / denominator (IEEE), p * projected value summed per lane.
// The reference's 256 lanes are the key index mod 256: a 128-key tile holds
// lanes 0-127 (even tiles) or 128-255 (odd tiles) of every row, so the
// epilogue thread of TMEM lane (row) r and column quarter c owns the
// sequential partial sums of lanes 32c .. 32c + 31 and 128 + 32c .. + 31,
// kept in TMEM columns 256 .. 511 of its lane (loaded for a tile, added to in
// key order -- the reference's per-lane order -- and stored back).  The
// pairwise tree (csrc/scoring.cu:15-30) is then level 128 inside each thread,
// levels 64 and 32 across the four threads of a row (shared memory), levels
// 16 .. 1 inside the thread of c = 0.  Every element takes
// the reference's operations (this file is compiled with --fmad=false), so
// the statistics equal lrk_temporal_scores' bit for bit on the logits
// cuBLAS would produce; the step order of the product is the one cuBLAS uses
// for the head's key count (logits_tc.cu: 16-term steps for an even count,
// 8-term steps for an odd one).
//
// Warp roles (544 threads, one CTA per SM, persistent over units):
//   warp 16, one thread  TMA loads of key tiles into a ring of stages and
//                        the UMMAs of every (unit, pass, tile) in order;
//   warps 0-15           per unit: build the query tile (A) in shared
//                        memory once the previous unit's MMAs are done;
//                        then drain every tile: warp w reads TMEM lanes
//                        32 (w % 4) .. + 31, columns 32 (w / 4) .. + 31.
// In pass 3 the epilogue stages each tile's projected values (all groups,
// zero past the head) in shared memory, one tile ahead.
// Every wait is bounded (tc::wait_phase); a timeout raises the CTA's abort
// flag, all roles stop, the issuer waits (bounded) for its work in flight,
// TMEM is freed and g_scores_tc_timeouts counts the CTA.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "rows.cuh"
#include "scoring.h"
#include "tc.cuh"

namespace lrk {

__device__ unsigned int g_scores_tc_timeouts = 0;

namespace {

using namespace tc;

constexpr int kEpilogueWarps = 16;
constexpr int kEpilogueThreads = kEpilogueWarps * 32;
constexpr int kIssuerWarp = kEpilogueWarps;
constexpr int kThreads = (kEpilogueWarps + 1) * 32;
constexpr int kAccumulators = 2;
constexpr uint32_t kPartialColumn = kAccumulators * kKeys;  // lane partial sums: columns 256 .. 511
constexpr uint32_t kTmemColumns = 512;
constexpr int kQuarter = kKeys / 4;                         // columns per epilogue thread per tile
constexpr int kMaxGroups = 8;
constexpr int kValueStride = kKeys + 4;                     // floats per staged projected-value row
constexpr int kMaxLayers = 32;
constexpr int kMaxSegments = 256;
constexpr int kEpilogueBarrier = 1;                       // named barrier of warps 0-7

// One (layer, head) segment of a launch.
struct FusedSegment {
  const __nv_bfloat16 *queries;  // row (q, g) at queries + q * query_stride + g * dim
  const float *projected;        // group g's projected values at projected + g * projected_stride
  __nv_bfloat16 *candidates;     // logits of columns [first8, first8 + candidate_stride), row-major
  float3 *stats;                 // [window * groups]
  const int32_t *visible;        // [window] visible-prefix length per query
  int64_t query_stride;
  int64_t projected_stride;
  int64_t key_row;               // the head's first row in its layer's key tensor
  int32_t length;                // keys of the head
  int32_t layer;                 // its key tensor map
  int32_t first8;                // first candidate column rounded down to 8
  int32_t candidate_stride;      // columns of the candidate buffer (multiple of 16)
  const float *key_positions;    // [length]: the mask when visible[q] < 0 (positions not sorted)
};

struct alignas(64) FusedParams {
  CUtensorMap keys[kMaxLayers];  // per layer: bf16 [rows, dim], 64 x 128 boxes, 128B swizzle
  FusedSegment segment[kMaxSegments];
  int32_t count;                 // segments
  int32_t m_tiles;               // ceil(rows / 128)
  int32_t rows;                  // window * groups
  int32_t groups;
  float scale;
  const int64_t *query_positions;  // [window]
};

template <int DIM, bool EIGHT>
struct FusedLayout {
  static constexpr int kChunks = DIM / 8;
  static constexpr int kSteps = EIGHT ? kChunks : kChunks / 2;
  static constexpr int kAAtoms = EIGHT ? DIM / 32 : DIM / 64;
  static constexpr int kBAtoms = EIGHT ? (kChunks + 6) / 7 : DIM / 64;
  static constexpr int kStages = EIGHT ? 2 : 4;
  static constexpr uint32_t kA = 0;
  static constexpr uint32_t kB = kA + kAAtoms * kAtom;
  static constexpr uint32_t kStage = kBAtoms * kAtom;
  static constexpr uint32_t kExchange = kB + kStages * kStage;          // [64][128] floats
  static constexpr uint32_t kMaxima = kExchange + 2 * kQuarter * kRows * 4;  // [4][128] maxima, [128] totals
  static constexpr uint32_t kValues = kMaxima + 5 * kRows * 4;           // 2 x [groups][kValueStride] floats
  static constexpr uint32_t kBarriers = kValues + 2 * kMaxGroups * kValueStride * 4;
  // full[S] empty[S] acc_full[4] acc_empty[4] a_ready
  static constexpr uint32_t kTmemSlot = kBarriers + 8 * (2 * kStages + 2 * kAccumulators + 1);
  static constexpr uint32_t kAbort = kTmemSlot + 8;
  static constexpr uint32_t kBytes = kAbort + 8 + 1024;  // + alignment slack
};

// The (unit, pass, tile) sequence of one CTA: units blockIdx.x, + gridDim.x,
// ...; three passes over each unit's key tiles.
struct Cursor {
  int unit, pass, tile, tiles;
  __device__ void start(const FusedParams &p) {
    unit = blockIdx.x;
    pass = 0;
    tile = 0;
    tiles = unit < p.count * p.m_tiles ? (p.segment[unit / p.m_tiles].length + kKeys - 1) / kKeys : 0;
  }
  __device__ bool valid(const FusedParams &p) const { return unit < p.count * p.m_tiles; }
  __device__ void next(const FusedParams &p) {
    if (++tile < tiles) return;
    tile = 0;
    if (++pass < 3) return;
    pass = 0;
    unit += gridDim.x;
    tiles = unit < p.count * p.m_tiles ? (p.segment[unit / p.m_tiles].length + kKeys - 1) / kKeys : 0;
  }
};

using P = rows::Packed<__nv_bfloat16>;
constexpr uint32_t kMinusInfinityLow = 0x0000ff80u, kMinusInfinityHigh = 0xff800000u;

// Which keys a row sees: a visible prefix (key positions sorted), or, when the
// pre-pass found them unsorted (visible < 0), key p with
// key_positions[p] <= the query's position (csrc/scoring.cu:43).  Keys at or
// past the head's length (the rest of the last tile) are never seen.
struct RowMask {
  int32_t visible, length;
  const float *key_positions;
  float query_position;
  __device__ __forceinline__ bool all(int p0, int n) const { return visible >= 0 && p0 + n <= visible; }
  __device__ __forceinline__ bool sees(int p) const {
    return visible >= 0 ? p < visible : (p < length && __ldg(key_positions + p) <= query_position);
  }
};

// x = bf16(bf16(logit) * scale) of 16 consecutive columns from p0 as 8 packed
// pairs (low half = the earlier column), masked to -inf; the bf16 logits too.
__device__ __forceinline__ void columns_x(const uint32_t *v, float2 scale2, const RowMask &mask, int p0,
                                          uint32_t *logit, uint32_t *x) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    logit[i] = P::round(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])));
    x[i] = P::round(rows::mul2_rn(P::unpack(logit[i]), scale2));
  }
  if (!mask.all(p0, 16)) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!mask.sees(p0 + 2 * i)) x[i] = (x[i] & 0xffff0000u) | kMinusInfinityLow;
      if (!mask.sees(p0 + 2 * i + 1)) x[i] = (x[i] & 0x0000ffffu) | kMinusInfinityHigh;
    }
  }
}

// All epilogue threads agree: true only if every one passes true.
__device__ __forceinline__ bool epilogue_all(bool value) {
  uint32_t all;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(all)
      : "r"(static_cast<uint32_t>(value)), "n"(kEpilogueBarrier), "n"(kEpilogueThreads)
      : "memory");
  return all != 0;
}

__device__ __forceinline__ void epilogue_sync() {
  asm volatile("bar.sync %0, %1;\n" ::"n"(kEpilogueBarrier), "n"(kEpilogueThreads) : "memory");
}

// The pairwise tree of csrc/scoring.cu:15-30 over one row's 256 lane sums,
// kept in TMEM at `partials` (this thread's lanes 32c + i at column i,
// 128 + 32c + i at column 32 + i, c = its column quarter).  Level 128 pairs
// columns i and 32 + i in the thread; level 64 adds quarters 2, 3 into 0, 1
// and level 32 quarter 1 into 0 through shared memory; levels 16 .. 1 run in
// the thread of quarter 0.  Returns the total to every thread of the row.
// `exchange` is [64][128] floats, `totals` [128].
__device__ __forceinline__ float row_tree(uint32_t partials, int c, int r, float *exchange, float *totals) {
  tmem_wait_store();
  float partial[kQuarter];
#pragma unroll
  for (int k = 0; k < kQuarter / 16; ++k) {
    uint32_t even[16], odd[16];
    tmem_load16(partials + 16 * k, even);
    tmem_load16(partials + kQuarter + 16 * k, odd);
    tmem_wait_loads();
    tmem_loaded16(even);
    tmem_loaded16(odd);
#pragma unroll
    for (int i = 0; i < 16; ++i) partial[16 * k + i] = __fadd_rn(__uint_as_float(even[i]), __uint_as_float(odd[i]));
  }
  if (c >= 2) {
#pragma unroll
    for (int i = 0; i < kQuarter; ++i) exchange[((c - 2) * kQuarter + i) * kRows + r] = partial[i];
  }
  epilogue_sync();
  if (c < 2) {
#pragma unroll
    for (int i = 0; i < kQuarter; ++i)
      partial[i] = __fadd_rn(partial[i], exchange[(c * kQuarter + i) * kRows + r]);  // s = 64
  }
  epilogue_sync();
  if (c == 1) {
#pragma unroll
    for (int i = 0; i < kQuarter; ++i) exchange[i * kRows + r] = partial[i];
  }
  epilogue_sync();
  if (c == 0) {
#pragma unroll
    for (int i = 0; i < kQuarter; ++i) partial[i] = __fadd_rn(partial[i], exchange[i * kRows + r]);  // s = 32
#pragma unroll
    for (int s = kQuarter / 2; s > 0; s >>= 1) {
#pragma unroll
      for (int i = 0; i < s; ++i) partial[i] = __fadd_rn(partial[i], partial[i + s]);
    }
    totals[r] = partial[0];
  }
  epilogue_sync();
  const float total = totals[r];
  epilogue_sync();  // exchange and totals free for the next use
  return total;
}

// Zeroes this thread's 64 partial-sum columns.
__device__ __forceinline__ void clear_partials(uint32_t partials) {
  uint32_t zero[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) zero[i] = 0u;
#pragma unroll
  for (int k = 0; k < 2 * kQuarter / 16; ++k) tmem_store16(partials + 16 * k, zero);
}

template <int DIM, bool EIGHT>
__global__ void __launch_bounds__(kThreads, 1) scores_tc_kernel(const __grid_constant__ FusedParams p) {
  using L = FusedLayout<DIM, EIGHT>;
  constexpr int S = L::kStages;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char *smem = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t bar = base + L::kBarriers;
  auto full = [&](int s) { return bar + 8 * s; };
  auto empty = [&](int s) { return bar + 8 * (S + s); };
  auto acc_full = [&](int a) { return bar + 8 * (2 * S + a); };
  auto acc_empty = [&](int a) { return bar + 8 * (2 * S + kAccumulators + a); };
  const uint32_t a_ready = bar + 8 * (2 * S + 2 * kAccumulators);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::kAbort);
  const int units = p.count * p.m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      init_barrier(full(s), 1);
      init_barrier(empty(s), 1);
    }
    for (int a = 0; a < kAccumulators; ++a) {
      init_barrier(acc_full(a), 1);
      init_barrier(acc_empty(a), kEpilogueWarps);
    }
    init_barrier(a_ready, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    *abort = 0;
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

  if (warp == kIssuerWarp) {
    if (lane == 0 && units > static_cast<int>(blockIdx.x)) {
      // ------------------------------------------------- TMA loads + MMA issue
      Cursor load, mma;
      load.start(p);
      mma.start(p);
      int loaded = 0, issued = 0, started = 0;
      bool ok = true;
      auto load_tile = [&](int s) {
        const FusedSegment &seg = p.segment[load.unit / p.m_tiles];
        expect_bytes(full(s), L::kStage);
        const int y = static_cast<int>(seg.key_row + static_cast<int64_t>(load.tile) * kKeys);
        const uint32_t dst = base + L::kB + s * L::kStage;
#pragma unroll
        for (int b = 0; b < L::kBAtoms; ++b)
          tma_box(dst + b * kAtom, &p.keys[seg.layer], (EIGHT ? 7 * b : 8 * b) * 8, y, full(s));
        load.next(p);
        ++loaded;
      };
      for (int s = 0; s < S && load.valid(p); ++s) load_tile(s);
      while (mma.valid(p)) {
        const int t = issued, s = t % S, a = t % kAccumulators;
        if (mma.pass == 0 && mma.tile == 0) {  // a new unit: its query tile must be in place
          if (!wait_phase(a_ready, started & 1, abort)) { ok = false; break; }
          ++started;
        }
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
          const uint32_t a_addr = A + (j >> 2) * kAtom + (j & 3) * 32;
          uint32_t b_addr;
          if constexpr (EIGHT) b_addr = B + (j / 7) * kAtom + (j % 7) * 16;  // key chunks j, j + 1
          else b_addr = B + (j >> 2) * kAtom + (j & 3) * 32;
          umma(d, smem_descriptor(a_addr), smem_descriptor(b_addr), j > 0);
        }
        umma_commit(acc_full(a));
        umma_commit(empty(s));
        issued = t + 1;
        mma.next(p);
        // Refill the stage of the previous tile once its MMAs are done.
        if (t >= 1 && load.valid(p)) {
          if (!wait_phase(empty((t - 1) % S), ((t - 1) / S) & 1, abort)) { ok = false; break; }
          load_tile((t - 1) % S);
        }
      }
      // Every arrival this thread set in motion lands before the CTA exits
      // (bounded waits, whatever the abort flag says).
      for (int t = issued > S ? issued - S : 0; t < issued; ++t) wait_phase(empty(t % S), (t / S) & 1, nullptr);
      if (!ok) {
        for (int t = issued; t < loaded; ++t) wait_phase(full(t % S), (t / S) & 1, nullptr);
        *abort = 1;
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3, c4 = warp >> 2, r = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t lanes = lane_base + c4 * kQuarter;
    const uint32_t partials = lane_base + kPartialColumn + c4 * 2 * kQuarter;
    float *exchange = reinterpret_cast<float *>(smem + L::kExchange);
    float *maxima = reinterpret_cast<float *>(smem + L::kMaxima);
    float *totals = maxima + 4 * kRows;
    float *staged = reinterpret_cast<float *>(smem + L::kValues);  // [2][groups][kValueStride]
    const float2 scale2 = make_float2(p.scale, p.scale);
    const int tid = threadIdx.x;
    int t = 0;
    bool ok = true;
    for (int unit = blockIdx.x; unit < units && ok; unit += gridDim.x) {
      const FusedSegment &seg = p.segment[unit / p.m_tiles];
      const int m = unit % p.m_tiles, row = m * kRows + r;
      const bool valid = row < p.rows;
      const int query = valid ? row / p.groups : 0, group = valid ? row % p.groups : 0;
      const int tiles = (seg.length + kKeys - 1) / kKeys;
      const RowMask mask{valid ? min(seg.visible[query], seg.length) : 0, seg.length, seg.key_positions,
                         static_cast<float>(p.query_positions[query])};
      // The query tile (A), after the previous unit's last MMA (whose
      // accumulator every epilogue warp has drained).
      {
        constexpr int kChunks = L::kChunks;
        for (int i = tid; i < kRows * kChunks; i += kEpilogueThreads) {
          const int rr = i / kChunks, j = i % kChunks, q_row = m * kRows + rr;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (q_row < p.rows) {
            const __nv_bfloat16 *src = seg.queries + static_cast<int64_t>(q_row / p.groups) * seg.query_stride +
                                       static_cast<int64_t>(q_row % p.groups) * DIM;
            v = __ldg(reinterpret_cast<const uint4 *>(src) + j);
          }
          const int a = EIGHT ? 2 * j : j;
          *reinterpret_cast<uint4 *>(smem + L::kA + (a >> 3) * kAtom + swizzled(rr, a & 7)) = v;
          if (EIGHT) {
            const int z = 2 * j + 1;
            *reinterpret_cast<uint4 *>(smem + L::kA + (z >> 3) * kAtom + swizzled(rr, z & 7)) =
                make_uint4(0, 0, 0, 0);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        epilogue_sync();
        if (tid == 0) arrive(a_ready);
      }
      // The accumulator of tile t: every epilogue thread waits, all agree.
      auto next_tile = [&]() -> bool {
        const bool got = wait_phase(acc_full(t % kAccumulators), (t / kAccumulators) & 1, abort);
        if (!epilogue_all(got)) {
          *abort = 1;
          return false;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        return true;
      };
      auto release_tile = [&]() {
        asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
        __syncwarp();
        if (lane == 0) arrive(acc_empty(t % kAccumulators));
        ++t;
      };
      // Columns 16k .. 16k + 15 of this thread's quarter of tile t.
      auto load_part = [&](int k, uint32_t *v) {
        tmem_load16(lanes + (t % kAccumulators) * kKeys + k * 16, v);
        tmem_wait_load16(v);
      };

      // Pass 1: the row maximum (order-free), and the logits of the
      // candidate columns for the risk kernel.
      uint32_t max_pair = P::kMinusInfinity;
      for (int j = 0; j < tiles; ++j) {
        if (!next_tile()) {
          ok = false;
          break;
        }
        const int tile0 = j * kKeys + c4 * kQuarter;
#pragma unroll
        for (int k = 0; k < kQuarter / 16; ++k) {
          uint32_t v[16], logit[8], x[8];
          load_part(k, v);
          if (k == kQuarter / 16 - 1) release_tile();
          const int p0 = tile0 + 16 * k;
          columns_x(v, scale2, mask, p0, logit, x);
#pragma unroll
          for (int i = 0; i < 8; ++i) max_pair = P::max(max_pair, x[i]);
          if (valid && p0 + 16 > seg.first8 && p0 < seg.first8 + seg.candidate_stride) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int column = p0 + 8 * c - seg.first8;
              if (column >= 0 && column < seg.candidate_stride)
                *reinterpret_cast<uint4 *>(seg.candidates + static_cast<int64_t>(row) * seg.candidate_stride +
                                           column) =
                    make_uint4(logit[4 * c], logit[4 * c + 1], logit[4 * c + 2], logit[4 * c + 3]);
            }
          }
        }
      }
      if (!ok) break;
      {
        const float2 pair_max = P::unpack(max_pair);
        maxima[c4 * kRows + r] = fmaxf(pair_max.x, pair_max.y);
      }
      epilogue_sync();
      const float maximum =
          fmaxf(fmaxf(maxima[r], maxima[kRows + r]), fmaxf(maxima[2 * kRows + r], maxima[3 * kRows + r]));
      const float2 minus_max = make_float2(-maximum, -maximum);

      // The 32 partial sums of this thread's lanes in the tile's parity:
      // loaded before the tile, stored back after it.  Keys past the head's
      // length add +0 (a masked weight, or a zero projected value): a lane
      // sum starts at +0 and no sum with +0 changes a value that is not -0,
      // which these sums never are, so the extra terms leave every bit.
      float sums[kQuarter];
      auto load_sums = [&](int j) {
        tmem_wait_store();
        uint32_t *bits = reinterpret_cast<uint32_t *>(sums);
#pragma unroll
        for (int k = 0; k < kQuarter / 16; ++k) tmem_load16(partials + (j & 1) * kQuarter + 16 * k, bits + 16 * k);
        tmem_wait_loads();
#pragma unroll
        for (int k = 0; k < kQuarter / 16; ++k) tmem_loaded16(bits + 16 * k);
      };
      auto store_sums = [&](int j) {
        const uint32_t *bits = reinterpret_cast<const uint32_t *>(sums);
#pragma unroll
        for (int k = 0; k < kQuarter / 16; ++k) tmem_store16(partials + (j & 1) * kQuarter + 16 * k, bits + 16 * k);
      };

      // Pass 2: per-lane sums of expf(x - max) in key order.
      clear_partials(partials);
      for (int j = 0; j < tiles; ++j) {
        if (!next_tile()) {
          ok = false;
          break;
        }
        load_sums(j);
        const int tile0 = j * kKeys + c4 * kQuarter;
#pragma unroll
        for (int k = 0; k < kQuarter / 16; ++k) {
          uint32_t v[16], logit[8], x[8];
          load_part(k, v);
          if (k == kQuarter / 16 - 1) release_tile();
          columns_x(v, scale2, mask, tile0 + 16 * k, logit, x);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 d = rows::add2_rn(P::unpack(x[i]), minus_max);
            const int c = 16 * k + 2 * i;
            sums[c] = __fadd_rn(sums[c], expf(d.x));
            sums[c + 1] = __fadd_rn(sums[c + 1], expf(d.y));
          }
        }
        store_sums(j);
      }
      if (!ok) break;
      const float denominator = row_tree(partials, c4, r, exchange, totals);

      // Pass 3: per-lane sums of (w / denominator) * projected value.  The
      // tile's projected values (every group, zero past the head) are staged
      // in shared memory one tile ahead by all epilogue threads.
      clear_partials(partials);
      const rows::Divider divider = rows::make_divider(denominator);
      constexpr int kStagedPerThread = kMaxGroups * kKeys / kEpilogueThreads;
      const int staged_count = p.groups * kKeys;
      float ahead[kStagedPerThread];
      auto fetch_values = [&](int j) {
#pragma unroll
        for (int i = 0; i < kStagedPerThread; ++i) {
          const int e = tid + i * kEpilogueThreads, g = e / kKeys, column = j * kKeys + e % kKeys;
          ahead[i] = e < staged_count && column < seg.length
                         ? __ldg(seg.projected + static_cast<int64_t>(g) * seg.projected_stride + column)
                         : 0.0f;
        }
      };
      auto stage_values = [&](int j) {
        float *buffer = staged + (j & 1) * kMaxGroups * kValueStride;
#pragma unroll
        for (int i = 0; i < kStagedPerThread; ++i) {
          const int e = tid + i * kEpilogueThreads;
          if (e < staged_count) buffer[(e / kKeys) * kValueStride + e % kKeys] = ahead[i];
        }
      };
      fetch_values(0);
      stage_values(0);  // visible after the barrier in next_tile
      for (int j = 0; j < tiles; ++j) {
        if (!next_tile()) {
          ok = false;
          break;
        }
        if (j + 1 < tiles) fetch_values(j + 1);
        load_sums(j);
        const int tile0 = j * kKeys + c4 * kQuarter;
        const float *values_row = staged + (j & 1) * kMaxGroups * kValueStride + group * kValueStride + c4 * kQuarter;
#pragma unroll
        for (int k = 0; k < kQuarter / 16; ++k) {
          uint32_t v[16], logit[8], x[8];
          load_part(k, v);
          if (k == kQuarter / 16 - 1) release_tile();
          columns_x(v, scale2, mask, tile0 + 16 * k, logit, x);
          float values[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 q = reinterpret_cast<const float4 *>(values_row + 16 * k)[i];
            values[4 * i] = q.x;
            values[4 * i + 1] = q.y;
            values[4 * i + 2] = q.z;
            values[4 * i + 3] = q.w;
          }
          // One operand test for the 16 divisions (rows::divide2_fast's range).
          const uint32_t lowest =
              P::min_nan(P::min_nan(P::min_nan(x[0], x[1]), P::min_nan(x[2], x[3])),
                         P::min_nan(P::min_nan(x[4], x[5]), P::min_nan(x[6], x[7])));
          const float2 lowest_d = rows::add2_rn(P::unpack(lowest), minus_max);
          const bool fast =
              divider.fast && lowest_d.x >= rows::kFastExponentFloor && lowest_d.y >= rows::kFastExponentFloor;
          if (fast) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float2 d = rows::add2_rn(P::unpack(x[i]), minus_max);
              const float2 probability = rows::divide2_fast(divider, make_float2(expf(d.x), expf(d.y)));
              const float2 product = rows::mul2_rn(probability, make_float2(values[2 * i], values[2 * i + 1]));
              const int c = 16 * k + 2 * i;
              sums[c] = __fadd_rn(sums[c], product.x);
              sums[c + 1] = __fadd_rn(sums[c + 1], product.y);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float2 d = rows::add2_rn(P::unpack(x[i]), minus_max);
              const float2 probability =
                  make_float2(rows::divide(divider, expf(d.x)), rows::divide(divider, expf(d.y)));
              const float2 product = rows::mul2_rn(probability, make_float2(values[2 * i], values[2 * i + 1]));
              const int c = 16 * k + 2 * i;
              sums[c] = __fadd_rn(sums[c], product.x);
              sums[c + 1] = __fadd_rn(sums[c + 1], product.y);
            }
          }
        }
        store_sums(j);
        if (j + 1 < tiles) stage_values(j + 1);  // the other buffer: its last readers passed next_tile
      }
      if (!ok) break;
      const float projection = row_tree(partials, c4, r, exchange, totals);
      if (c4 == 0 && valid) seg.stats[row] = make_float3(maximum, denominator, projection);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == kIssuerWarp) {
    if (lane == 0 && *abort) atomicAdd(&g_scores_tc_timeouts, 1u);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemColumns) : "memory");
  }
}

}  // namespace

namespace {

// Candidate columns the risk kernels read for a segment: [first8, first8 +
// width), width a multiple of 16 (their 16-column tiles start at first8).
int64_t candidate_width(const lrk_key_segment &seg) {
  const int64_t first8 = seg.first & ~int64_t{7};
  return (seg.last - first8 + 15) / 16 * 16;
}

size_t align256(size_t bytes) { return (bytes + 255) / 256 * 256; }

template <int DIM, bool EIGHT>
int launch_fused(const FusedParams &params, cudaStream_t stream) {
  auto kernel = scores_tc_kernel<DIM, EIGHT>;
  constexpr uint32_t bytes = FusedLayout<DIM, EIGHT>::kBytes;
  static_assert(bytes <= 227 * 1024, "shared memory of the fused scorer");
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  const int units = params.count * params.m_tiles;
  const int grid = std::min(units, sm_count());
  kernel<<<grid, kThreads, bytes, stream>>>(params);
  return launch_status("lrk_scores_from_keys statistics");
}

// One statistics launch per batch of same-parity segments (at most
// kMaxSegments segments over at most kMaxLayers layers).
int launch_statistics(const lrk_key_segment *segments, const std::vector<int64_t> &order, const lrk_key_layer *layers,
                      int64_t window, int64_t groups, int64_t dim, float scale, const int64_t *qpos, float3 *stats,
                      const int32_t *visible, const std::vector<__nv_bfloat16 *> &candidates, bool eight,
                      cudaStream_t stream) {
  const int64_t rows = window * groups;
  size_t i = 0;
  while (i < order.size()) {
    FusedParams params;
    std::memset(&params, 0, sizeof(params));
    std::vector<int64_t> layer_of_map;
    int n = 0;
    for (; i < order.size() && n < kMaxSegments; ++i) {
      const int64_t s = order[i];
      const lrk_key_segment &seg = segments[s];
      auto found = std::find(layer_of_map.begin(), layer_of_map.end(), seg.layer);
      int map = static_cast<int>(found - layer_of_map.begin());
      if (found == layer_of_map.end()) {
        if (static_cast<int>(layer_of_map.size()) == kMaxLayers) break;
        const lrk_key_layer &layer = layers[seg.layer];
        const int status = tc::make_map(&params.keys[map], layer.keys, layer.rows, dim, dim, 64,
                                        CU_TENSOR_MAP_SWIZZLE_128B);
        if (status != LRK_OK) return status;
        layer_of_map.push_back(seg.layer);
      }
      FusedSegment &f = params.segment[n++];
      f.queries = static_cast<const __nv_bfloat16 *>(seg.queries);
      f.projected = seg.projected_values;
      f.candidates = candidates[s];
      f.stats = stats + s * rows;
      f.visible = visible + s * window;
      f.query_stride = seg.query_stride;
      f.projected_stride = seg.projected_stride;
      f.key_row = seg.key_row;
      f.length = static_cast<int32_t>(seg.length);
      f.layer = map;
      f.first8 = static_cast<int32_t>(seg.first & ~int64_t{7});
      f.candidate_stride = static_cast<int32_t>(candidate_width(seg));
      f.key_positions = seg.key_positions;
    }
    params.count = n;
    params.m_tiles = static_cast<int32_t>(ceil_div(rows, kRows));
    params.rows = static_cast<int32_t>(rows);
    params.groups = static_cast<int32_t>(groups);
    params.scale = scale;
    params.query_positions = qpos;
    const int status = dim == 128 ? (eight ? launch_fused<128, true>(params, stream) : launch_fused<128, false>(params, stream))
                                  : (eight ? launch_fused<64, true>(params, stream) : launch_fused<64, false>(params, stream));
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
}

int check_key_call(const lrk_key_segment *segments, int64_t count, const lrk_key_layer *layers, int64_t layer_count,
                   int64_t window, int64_t groups, int64_t dim) {
  LRK_REQUIRE(dim == 64 || dim == 128, "lrk_scores_from_keys: head dimension 64 or 128");
  LRK_REQUIRE(window > 0 && groups > 0 && groups <= 8 && window <= 65535 &&
                  window * groups * static_cast<int64_t>(sizeof(float4)) <= 200 * 1024,
              "lrk_scores_from_keys: invalid window or groups (the risk step keeps window * groups row "
              "statistics in shared memory)");
  if (count == 0) return LRK_OK;
  LRK_REQUIRE(segments != nullptr && layers != nullptr && layer_count > 0, "null pointer");
  for (int64_t l = 0; l < layer_count; ++l) {
    LRK_REQUIRE(layers[l].keys != nullptr && aligned(layers[l].keys, 16) && layers[l].rows > 0 &&
                    layers[l].rows <= INT32_MAX,
                "lrk_scores_from_keys: invalid layer keys");
  }
  for (int64_t s = 0; s < count; ++s) {
    const lrk_key_segment &seg = segments[s];
    LRK_REQUIRE(seg.layer >= 0 && seg.layer < layer_count, "lrk_scores_from_keys: layer index out of range");
    LRK_REQUIRE(seg.queries && seg.projected_values && seg.key_positions && seg.scores, "null segment pointer");
    LRK_REQUIRE(aligned(seg.queries, 16) && seg.query_stride % 8 == 0 && seg.query_stride >= groups * dim,
                "lrk_scores_from_keys: queries must be 16-byte aligned rows");
    LRK_REQUIRE(seg.length > 0 && seg.length <= INT32_MAX / 2 && seg.key_row >= 0 &&
                    seg.key_row + seg.length <= layers[seg.layer].rows,
                "lrk_scores_from_keys: keys outside the layer");
    LRK_REQUIRE(seg.first >= 0 && seg.last > seg.first && seg.last <= seg.length, "Invalid risk interval");
    LRK_REQUIRE(seg.projected_stride >= seg.length, "projected_stride shorter than the segment");
    LRK_REQUIRE(seg.query_chunk >= 0, "query_chunk must be >= 0");
  }
  return LRK_OK;
}

}  // namespace
}  // namespace lrk

using namespace lrk;

// Workspace: row statistics, visible prefixes, then each segment's candidate
// logits (rows x candidate width bf16), every part 256-byte aligned.
extern "C" size_t lrk_scores_from_keys_workspace_bytes(const lrk_key_segment *segments, int64_t count, int64_t window,
                                                       int64_t groups) {
  if (count < 0 || window < 0 || groups < 0 || (count > 0 && segments == nullptr)) return 0;
  const size_t rows = static_cast<size_t>(window) * groups;
  size_t bytes = align256(count * rows * sizeof(float3)) + align256(count * window * sizeof(int32_t));
  for (int64_t s = 0; s < count; ++s) {
    if (segments[s].last <= segments[s].first) return 0;
    bytes += align256(rows * candidate_width(segments[s]) * sizeof(__nv_bfloat16));
  }
  return bytes + 256;
}

extern "C" int lrk_scores_from_keys(const lrk_key_segment *segments, int64_t count, const lrk_key_layer *layers,
                                    int64_t layer_count, const int64_t *query_positions, int64_t window,
                                    int64_t groups, int64_t dim, float scale, const float *margin, float epsilon,
                                    void *workspace, size_t workspace_bytes, lrk_stream_t stream) {
  clear_error();
  int status = check_key_call(segments, count, layers, layer_count, window, groups, dim);
  if (status != LRK_OK || count == 0) return status;
  LRK_REQUIRE(query_positions != nullptr && margin != nullptr && epsilon > 0, "invalid score arguments");
  const size_t need = lrk_scores_from_keys_workspace_bytes(segments, count, window, groups);
  if (workspace == nullptr || workspace_bytes < need) return fail(LRK_ERR_WORKSPACE, "score workspace too small");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t rows = static_cast<size_t>(window) * groups;
  uintptr_t cursor = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t{255};
  float3 *stats = reinterpret_cast<float3 *>(cursor);
  cursor += align256(count * rows * sizeof(float3));
  int32_t *visible = reinterpret_cast<int32_t *>(cursor);
  cursor += align256(count * window * sizeof(int32_t));
  std::vector<__nv_bfloat16 *> candidates(count);
  std::vector<lrk_score_segment> table(count);
  for (int64_t i = 0; i < count; ++i) {
    const lrk_key_segment &seg = segments[i];
    candidates[i] = reinterpret_cast<__nv_bfloat16 *>(cursor);
    cursor += align256(rows * candidate_width(seg) * sizeof(__nv_bfloat16));
    lrk_score_segment &t = table[i];
    // The risk kernels index logits by key column: column c of the
    // candidate buffer is key first8 + c.
    t.logits = candidates[i] - (seg.first & ~int64_t{7});
    t.logits_stride = candidate_width(seg);
    t.projected_values = seg.projected_values;
    t.projected_stride = seg.projected_stride;
    t.key_positions = seg.key_positions;
    t.length = seg.length;
    t.first = seg.first;
    t.last = seg.last;
    t.scores = seg.scores;
    t.query_chunk = seg.query_chunk;
  }
  status = score_visibility(table.data(), count, query_positions, static_cast<int>(window), visible, s);
  if (status != LRK_OK) return status;
  std::vector<int64_t> even, odd;
  for (int64_t i = 0; i < count; ++i) (segments[i].length % 2 ? odd : even).push_back(i);
  for (bool eight : {false, true}) {
    status = launch_statistics(segments, eight ? odd : even, layers, window, groups, dim, scale, query_positions,
                               stats, visible, candidates, eight, s);
    if (status != LRK_OK) return status;
  }
  return score_risk_bf16(table.data(), count, query_positions, static_cast<int>(window), static_cast<int>(groups),
                         scale, margin, epsilon, stats, s);
}

extern "C" int lrk_scores_from_keys_timeouts(unsigned int *count) {
  clear_error();
  LRK_REQUIRE(count != nullptr, "null pointer");
  cudaError_t e = cudaMemcpyFromSymbol(count, g_scores_tc_timeouts, sizeof(unsigned int));
  return e == cudaSuccess ? LRK_OK : fail(LRK_ERR_CUDA, cudaGetErrorString(e));
}
