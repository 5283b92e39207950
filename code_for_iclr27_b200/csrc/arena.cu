// Gapped per-head KV arena: zero-copy decode appends and in-place eviction.
//
// The reference's packed layer cache ([rows, D], heads back to back) is
// rebuilt whole by every append, compaction and merge (csrc/scoring.cu:264-314,
// csrc/batch_append.cu:81-93, csrc/recall.cu:68-83), so each decode step
// moves every layer's cache through HBM.  The arena gives each (layer, head)
// a fixed capacity instead: keys and values [heads_total, capacity, D], float
// positions [heads_total, capacity], and int32 lengths [heads_total] on the
// device.  A head's live rows are rows [0, length) of its slot, in the same
// order as in the packed layout, so the packed cache is the concatenation of
// the slots' live rows.  FlashAttention's cache entry point reads this layout
// directly (k_cache [heads, capacity, 1, D] with cache_seqlens = lengths).
//
// * Append: one row per head at row `length`, then length + 1 -- one launch
//   for every head of every layer, 2 D + 4 bytes per head.
// * Compaction: per touched head, the rows after its first removed row move
//   down over the removed ones, in place.  One CTA per touched head walks the
//   head in chunks of rows: it loads a chunk into registers, waits at a
//   barrier, and stores it to the rows' new places.  A row only ever moves to
//   a lower index and chunks go upward, so no store can reach a row that is
//   still to be loaded.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"

namespace lrk {
namespace {

struct ArenaParam {
  char *keys;
  char *values;
  float *positions;
  int32_t *lengths;
  int64_t heads_total, capacity, row_bytes;
};

ArenaParam param(const lrk_arena &a, int64_t element) {
  return ArenaParam{static_cast<char *>(a.keys), static_cast<char *>(a.values), a.positions, a.lengths,
                    a.heads_total, a.capacity, a.dimension * element};
}

constexpr int kAppendThreads = 256;

// One warp per head: the key and value rows (16-byte vectors), the position,
// then the length.  A head at capacity is left unchanged and flags overflow.
__global__ void __launch_bounds__(kAppendThreads) arena_append_kernel(ArenaParam a, int64_t first_head, int64_t count,
                                                                      const uint4 *__restrict__ new_keys,
                                                                      const uint4 *__restrict__ new_values,
                                                                      float position,
                                                                      unsigned int *__restrict__ overflow) {
  const int lane = threadIdx.x & 31;
  const int64_t local = (static_cast<int64_t>(blockIdx.x) * kAppendThreads + threadIdx.x) >> 5;
  if (local >= count) return;
  const int64_t head = first_head + local;
  const int32_t length = a.lengths[head];
  if (length < 0 || length >= a.capacity) {
    if (lane == 0 && overflow != nullptr) atomicOr(overflow, 1u);
    return;
  }
  const int64_t vectors = a.row_bytes / 16;
  const int64_t row = head * a.capacity + length;
  uint4 *k = reinterpret_cast<uint4 *>(a.keys + row * a.row_bytes);
  uint4 *v = reinterpret_cast<uint4 *>(a.values + row * a.row_bytes);
  for (int64_t i = lane; i < vectors; i += 32) {
    k[i] = new_keys[local * vectors + i];
    v[i] = new_values[local * vectors + i];
  }
  if (lane == 0) a.positions[row] = position;
  __syncwarp();
  if (lane == 0) a.lengths[head] = length + 1;
}

constexpr int kCompactThreads = 256;
constexpr int kCompactVectors = 8;  // 16-byte vectors per thread per chunk and tensor

// Rows per chunk: what kCompactVectors vectors per thread cover, at most one
// row per thread (each thread moves at most one position).
__host__ __device__ __forceinline__ int64_t chunk_rows_for(int64_t vectors) {
  const int64_t rows = kCompactThreads * kCompactVectors / vectors;
  return rows < kCompactThreads ? rows : kCompactThreads;
}

// How many entries of list[0 .. count) (ascending) lie below `value`.
template <typename V>
__device__ __forceinline__ int64_t count_below(const V *__restrict__ list, int64_t count, V value) {
  int64_t lo = 0, hi = count;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (__ldg(list + mid) < value) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Compaction of the touched heads, one CTA per head (grid-stride).  plan
// [touched][3] = (head, first index into the removal lists, count); heads
// with count 0 are skipped, so a dense plan over every head is allowed.
// BY_POSITION false: the list holds row indices (int64), strictly ascending,
// below the head's length.  BY_POSITION true: it holds logical positions
// (float) of rows to drop, strictly ascending, each present in the head,
// whose live positions must be ascending (as appends and position-ordered
// merges keep them); the rows are found by binary search.  A head whose list
// breaks its rule is left unchanged and sets *error.
template <bool BY_POSITION>
__global__ void __launch_bounds__(kCompactThreads) arena_compact_kernel(ArenaParam a,
                                                                        const int64_t *__restrict__ plan,
                                                                        int64_t touched,
                                                                        const void *__restrict__ removed,
                                                                        unsigned int *__restrict__ error) {
  extern __shared__ int64_t destination[];  // [rows per chunk]: new row, or -1 for a removed row
  __shared__ int64_t first_row;
  const int64_t vectors = a.row_bytes / 16;
  const int64_t chunk_rows = chunk_rows_for(vectors);
  for (int64_t t = blockIdx.x; t < touched; t += gridDim.x) {
    const int64_t head = plan[3 * t], offset = plan[3 * t + 1], count = plan[3 * t + 2];
    if (count <= 0 || head < 0 || head >= a.heads_total) continue;
    const int64_t length = a.lengths[head];
    const int64_t *rows = static_cast<const int64_t *>(removed) + offset;
    const float *logical = static_cast<const float *>(removed) + offset;
    float *positions = a.positions + head * a.capacity;
    if (threadIdx.x == 0) first_row = length;
    __syncthreads();
    int bad = 0;
    for (int64_t i = threadIdx.x; i < count; i += kCompactThreads) {
      if (BY_POSITION) {
        const float value = logical[i];
        const int64_t at = count_below(positions, length, value);
        if (at >= length || positions[at] != value || (i > 0 && !(logical[i - 1] < value))) bad = 1;
        if (i == 0) first_row = at;
      } else {
        const int64_t r = rows[i];
        if (r < 0 || r >= length || (i > 0 && rows[i - 1] >= r)) bad = 1;
        if (i == 0) first_row = r;
      }
    }
    if (__syncthreads_or(bad)) {
      if (threadIdx.x == 0 && error != nullptr) atomicOr(error, 1u);
      continue;
    }
    const int64_t first = first_row;
    char *keys = a.keys + head * a.capacity * a.row_bytes;
    char *values = a.values + head * a.capacity * a.row_bytes;
    for (int64_t base = first + 1; base < length; base += chunk_rows) {
      const int64_t rows_here = lmin(chunk_rows, length - base);
      for (int64_t i = threadIdx.x; i < rows_here; i += kCompactThreads) {
        const int64_t source = base + i;
        int64_t below;
        bool gone;
        if (BY_POSITION) {
          const float value = positions[source];
          below = count_below(logical, count, value);
          gone = below < count && __ldg(logical + below) == value;
        } else {
          below = count_below(rows, count, source);
          gone = below < count && __ldg(rows + below) == source;
        }
        destination[i] = gone ? -1 : source - below;
      }
      __syncthreads();
      // Load the chunk's kept rows ...
      uint4 k[kCompactVectors], v[kCompactVectors];
      float p = 0.0f;
#pragma unroll
      for (int j = 0; j < kCompactVectors; ++j) {
        const int64_t item = threadIdx.x + static_cast<int64_t>(j) * kCompactThreads;
        const int64_t r = item / vectors, c = item % vectors;
        if (r < rows_here && destination[r] >= 0) {
          k[j] = reinterpret_cast<const uint4 *>(keys + (base + r) * a.row_bytes)[c];
          v[j] = reinterpret_cast<const uint4 *>(values + (base + r) * a.row_bytes)[c];
        }
      }
      if (threadIdx.x < rows_here && destination[threadIdx.x] >= 0) p = positions[base + threadIdx.x];
      __syncthreads();
      // ... then store them at their new rows (all loads of the chunk are done).
#pragma unroll
      for (int j = 0; j < kCompactVectors; ++j) {
        const int64_t item = threadIdx.x + static_cast<int64_t>(j) * kCompactThreads;
        const int64_t r = item / vectors, c = item % vectors;
        if (r < rows_here && destination[r] >= 0) {
          reinterpret_cast<uint4 *>(keys + destination[r] * a.row_bytes)[c] = k[j];
          reinterpret_cast<uint4 *>(values + destination[r] * a.row_bytes)[c] = v[j];
        }
      }
      if (threadIdx.x < rows_here && destination[threadIdx.x] >= 0) positions[destination[threadIdx.x]] = p;
      __syncthreads();  // destination[] and the moved rows settle before the next chunk
    }
    if (threadIdx.x == 0) a.lengths[head] = static_cast<int32_t>(length - count);
    __syncthreads();
  }
}

int check_arena(const lrk_arena *arena, int64_t *element) {
  LRK_REQUIRE(arena != nullptr, "null arena");
  LRK_REQUIRE(arena->heads_total >= 0 && arena->capacity > 0 && arena->dimension > 0, "invalid arena sizes");
  *element = lrk_dtype_size(arena->dtype);
  if (*element == 0) return fail(LRK_ERR_UNSUPPORTED, "unsupported arena dtype");
  LRK_REQUIRE((arena->dimension * *element) % 16 == 0, "arena rows must be a multiple of 16 bytes");
  LRK_REQUIRE(arena->dimension * *element <= 16 * kCompactThreads * kCompactVectors,
              "arena rows longer than one compaction chunk");
  LRK_REQUIRE(arena->capacity <= INT32_MAX, "arena capacity beyond int32 lengths");
  LRK_REQUIRE(arena->keys && arena->values && arena->positions && arena->lengths, "null arena pointer");
  LRK_REQUIRE(aligned(arena->keys, 16) && aligned(arena->values, 16), "arena K/V must be 16-byte aligned");
  return LRK_OK;
}

}  // namespace
}  // namespace lrk

using namespace lrk;

extern "C" int lrk_arena_append(const lrk_arena *arena, int64_t first_head, int64_t count, const void *new_keys,
                                const void *new_values, float position, unsigned int *overflow,
                                lrk_stream_t stream) {
  clear_error();
  int64_t element = 0;
  int status = check_arena(arena, &element);
  if (status != LRK_OK) return status;
  LRK_REQUIRE(first_head >= 0 && count >= 0 && first_head + count <= arena->heads_total, "heads out of range");
  if (count == 0) return LRK_OK;
  LRK_REQUIRE(new_keys && new_values, "null pointer");
  LRK_REQUIRE(aligned(new_keys, 16) && aligned(new_values, 16), "new rows must be 16-byte aligned");
  const int64_t blocks = ceil_div(count * 32, kAppendThreads);
  arena_append_kernel<<<static_cast<unsigned>(blocks), kAppendThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      param(*arena, element), first_head, count, static_cast<const uint4 *>(new_keys),
      static_cast<const uint4 *>(new_values), position, overflow);
  return launch_status("lrk_arena_append");
}

template <bool BY_POSITION>
int launch_compact(const lrk_arena *arena, const int64_t *plan, int64_t touched, const void *removed,
                   unsigned int *error, lrk_stream_t stream) {
  clear_error();
  int64_t element = 0;
  int status = check_arena(arena, &element);
  if (status != LRK_OK) return status;
  LRK_REQUIRE(touched >= 0, "invalid plan size");
  if (touched == 0) return LRK_OK;
  LRK_REQUIRE(plan && removed, "null pointer");
  const int64_t chunk_rows = chunk_rows_for(arena->dimension * element / 16);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(touched, 65535));
  arena_compact_kernel<BY_POSITION><<<blocks, kCompactThreads, chunk_rows * sizeof(int64_t),
                                      reinterpret_cast<cudaStream_t>(stream)>>>(param(*arena, element), plan,
                                                                                touched, removed, error);
  return launch_status("lrk_arena_compact");
}

extern "C" int lrk_arena_compact(const lrk_arena *arena, const int64_t *plan, int64_t touched, const int64_t *removed,
                                 unsigned int *error, lrk_stream_t stream) {
  return launch_compact<false>(arena, plan, touched, removed, error, stream);
}

extern "C" int lrk_arena_compact_positions(const lrk_arena *arena, const int64_t *plan, int64_t touched,
                                           const float *removed_positions, unsigned int *error, lrk_stream_t stream) {
  return launch_compact<true>(arena, plan, touched, removed_positions, error, stream);
}
