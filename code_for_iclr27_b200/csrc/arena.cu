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

// How many entries of list[0 .. count) (ascending) lie below `value`.  The
// list may be in global or shared memory (plain generic loads).
template <typename V>
__device__ __forceinline__ int64_t count_below(const V *list, int64_t count, V value) {
  int64_t lo = 0, hi = count;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (list[mid] < value) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Removal lists a CTA keeps in shared memory (longer lists are read from
// global memory).
constexpr int kListMax = 2048;

// The chunk loop of one head's in-place compaction (all threads of the CTA):
// rows [first + 1, length) move down over the removed rows.  Each chunk's
// rows -- keys, values and positions -- are loaded with no dependence on
// which of them stay, each row's destination is found from its index
// (BY_POSITION false: the number of listed rows below it) or its position
// (BY_POSITION true: the number of listed positions below it), and after a
// barrier the kept rows are stored.  One memory latency per chunk.
template <bool BY_POSITION>
__device__ void compact_head(const ArenaParam &a, int64_t head, int64_t length, int64_t first,
                             const int64_t *__restrict__ rows_list, const float *__restrict__ position_list,
                             int64_t count, int64_t *destination) {
  const int64_t vectors = a.row_bytes / 16;
  const int64_t chunk_rows = chunk_rows_for(vectors);
  char *keys = a.keys + head * a.capacity * a.row_bytes;
  char *values = a.values + head * a.capacity * a.row_bytes;
  float *positions = a.positions + head * a.capacity;
  for (int64_t base = first + 1; base < length; base += chunk_rows) {
    const int64_t rows_here = lmin(chunk_rows, length - base);
    uint4 k[kCompactVectors], v[kCompactVectors];
#pragma unroll
    for (int j = 0; j < kCompactVectors; ++j) {
      const int64_t item = threadIdx.x + static_cast<int64_t>(j) * kCompactThreads;
      const int64_t r = item / vectors, c = item % vectors;
      if (r < rows_here) {
        k[j] = reinterpret_cast<const uint4 *>(keys + (base + r) * a.row_bytes)[c];
        v[j] = reinterpret_cast<const uint4 *>(values + (base + r) * a.row_bytes)[c];
      }
    }
    float p = 0.0f;
    if (threadIdx.x < rows_here) {
      const int64_t source = base + threadIdx.x;
      p = positions[source];
      int64_t below;
      bool gone;
      if (BY_POSITION) {
        below = count_below(position_list, count, p);
        gone = below < count && position_list[below] == p;
      } else {
        below = count_below(rows_list, count, source);
        gone = below < count && rows_list[below] == source;
      }
      destination[threadIdx.x] = gone ? -1 : source - below;
    }
    __syncthreads();  // every load of the chunk is ordered before any store
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
    __syncthreads();  // destination[] is reused by the next chunk
  }
}

// Check a head's sorted removal list and find its first row; returns false
// (after flagging) when the list is out of order or names a row / position
// the head does not hold.
template <bool BY_POSITION>
__device__ bool check_list(const ArenaParam &a, int64_t head, int64_t length, const int64_t *rows_list,
                           const float *position_list, int64_t count, int64_t *first_row, unsigned int *error) {
  const float *positions = a.positions + head * a.capacity;
  if (threadIdx.x == 0) *first_row = length;
  __syncthreads();
  int bad = 0;
  for (int64_t i = threadIdx.x; i < count; i += kCompactThreads) {
    if (BY_POSITION) {
      const float value = position_list[i];
      const int64_t at = count_below(positions, length, value);
      if (at >= length || positions[at] != value || (i > 0 && !(position_list[i - 1] < value))) bad = 1;
      if (i == 0) *first_row = at;
    } else {
      const int64_t r = rows_list[i];
      if (r < 0 || r >= length || (i > 0 && rows_list[i - 1] >= r)) bad = 1;
      if (i == 0) *first_row = r;
    }
  }
  if (__syncthreads_or(bad)) {
    if (threadIdx.x == 0 && error != nullptr) atomicOr(error, 1u);
    return false;
  }
  return true;
}

// Compaction of the heads a plan names, one CTA per plan entry (grid-stride).
// plan [touched][3] = (head, first index into the removal lists, count);
// entries with count 0 are skipped, so a dense plan over every head works.
// BY_POSITION false: int64 rows, strictly ascending, below the head's length.
// BY_POSITION true: float logical positions, strictly ascending, each present
// in the head, whose live positions must be ascending (as appends and
// position-ordered merges keep them).  A head whose list breaks its rule is
// left unchanged and sets *error.  Heads must be distinct.
template <bool BY_POSITION>
__global__ void __launch_bounds__(kCompactThreads, 2) arena_compact_kernel(ArenaParam a,
                                                                        const int64_t *__restrict__ plan,
                                                                        int64_t touched,
                                                                        const void *__restrict__ removed,
                                                                        unsigned int *__restrict__ error) {
  __shared__ int64_t destination[kCompactThreads];
  __shared__ __align__(8) unsigned char list_bytes[kListMax * sizeof(int64_t)];
  __shared__ int64_t first_row;
  for (int64_t t = blockIdx.x; t < touched; t += gridDim.x) {
    const int64_t head = plan[3 * t], offset = plan[3 * t + 1], count = plan[3 * t + 2];
    if (count <= 0 || head < 0 || head >= a.heads_total) continue;
    const int64_t length = a.lengths[head];
    // The list, in shared memory when it fits.
    const int64_t *rows_list = static_cast<const int64_t *>(removed) + offset;
    const float *position_list = static_cast<const float *>(removed) + offset;
    if (count <= kListMax) {
      for (int64_t i = threadIdx.x; i < count; i += kCompactThreads) {
        if (BY_POSITION) reinterpret_cast<float *>(list_bytes)[i] = position_list[i];
        else reinterpret_cast<int64_t *>(list_bytes)[i] = rows_list[i];
      }
      rows_list = reinterpret_cast<const int64_t *>(list_bytes);
      position_list = reinterpret_cast<const float *>(list_bytes);
    }
    if (check_list<BY_POSITION>(a, head, length, rows_list, position_list, count, &first_row, error)) {
      compact_head<BY_POSITION>(a, head, length, first_row, rows_list, position_list, count, destination);
      if (threadIdx.x == 0) a.lengths[head] = static_cast<int32_t>(length - count);
    }
    __syncthreads();
  }
}

// Eviction of an unsorted batch of (head, logical position) references, one
// CTA per head (grid-stride over every head): the CTA collects its head's
// entries from the batch, sorts them in shared memory (bitonic), and
// compacts the head as arena_compact_kernel<true> does.  A head with more
// than kListMax entries, a duplicate or a position it does not hold is left
// unchanged and sets *error.
__global__ void __launch_bounds__(kCompactThreads, 2) arena_evict_kernel(ArenaParam a,
                                                                      const int64_t *__restrict__ heads,
                                                                      const float *__restrict__ positions_in,
                                                                      int64_t n, unsigned int *__restrict__ error) {
  __shared__ int64_t destination[kCompactThreads];
  __shared__ float list[kListMax];
  __shared__ int count_shared;
  __shared__ int64_t first_row;
  for (int64_t head = blockIdx.x; head < a.heads_total; head += gridDim.x) {
    if (threadIdx.x == 0) count_shared = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n; i += kCompactThreads) {
      if (heads[i] == head) {
        const int slot = atomicAdd(&count_shared, 1);
        if (slot < kListMax) list[slot] = positions_in[i];
      }
    }
    __syncthreads();
    const int count = count_shared;
    __syncthreads();  // every thread has read the count before the next reset
    if (count == 0) continue;  // uniform: every thread read the same count
    if (count > kListMax) {
      if (threadIdx.x == 0 && error != nullptr) atomicOr(error, 1u);
      continue;
    }
    // Bitonic sort of list[0 .. size), padded with +inf.
    int size = 1;
    while (size < count) size <<= 1;
    for (int i = count + threadIdx.x; i < size; i += kCompactThreads) list[i] = INFINITY;
    __syncthreads();
    for (int k = 2; k <= size; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < size; i += kCompactThreads) {
          const int partner = i ^ j;
          if (partner > i) {
            const bool up = (i & k) == 0;
            const float x = list[i], y = list[partner];
            if ((x > y) == up) {
              list[i] = y;
              list[partner] = x;
            }
          }
        }
        __syncthreads();
      }
    }
    const int64_t length = a.lengths[head];
    if (check_list<true>(a, head, length, nullptr, list, count, &first_row, error)) {
      compact_head<true>(a, head, length, first_row, nullptr, list, count, destination);
      if (threadIdx.x == 0) a.lengths[head] = static_cast<int32_t>(length - count);
    }
    __syncthreads();
  }
}

// Recall reinsertion in place (lrk_arena_insert).  One CTA per touched head.
// The head's recalled entries (ascending positions, at most kInsertMax) sit
// in shared memory.  CHECK: only flags (1: a position recalled twice or
// recalled while resident; 2: resident positions not ascending; 4: the head
// would pass its capacity; 8: more than kInsertMax entries).  Otherwise a
// resident row i moves up by k(i) = the entries below its position, which
// never decreases with i: chunks of rows go from the top of the head down
// (loads, barrier, stores), so no store reaches a row still to be loaded and
// no chunk writes where a higher chunk wrote; only the rows above the first
// entry's place move.  Then entry e lands in row e + (resident rows below
// it), a slot the moves have emptied, and the length grows by the count.
constexpr int kInsertMax = 2048;

template <bool CHECK>
__global__ void __launch_bounds__(kCompactThreads) arena_insert_kernel(ArenaParam a, const int64_t *__restrict__ plan,
                                                                       int64_t touched,
                                                                       const char *__restrict__ recalled,
                                                                       const float *__restrict__ recalled_positions,
                                                                       unsigned int *__restrict__ flag) {
  __shared__ float entries[kInsertMax];
  __shared__ int32_t landing[kInsertMax];
  __shared__ int32_t shift[kCompactThreads];
  const int64_t vectors = a.row_bytes / 16;
  const int64_t chunk_rows = chunk_rows_for(vectors);
  for (int64_t t = blockIdx.x; t < touched; t += gridDim.x) {
    const int64_t head = plan[3 * t], first = plan[3 * t + 1], count = plan[3 * t + 2];
    if (head < 0 || head >= a.heads_total || count <= 0) continue;
    const int64_t length = a.lengths[head];
    char *keys = a.keys + head * a.capacity * a.row_bytes;
    char *values = a.values + head * a.capacity * a.row_bytes;
    float *positions = a.positions + head * a.capacity;
    const float *wanted = recalled_positions + first;
    if (CHECK) {
      if (threadIdx.x == 0) {
        if (length < 0 || length + count > a.capacity) atomicOr(flag, 4u);
        if (count > kInsertMax) atomicOr(flag, 8u);
      }
      const int64_t rows = lmin(lmax(length, 0), a.capacity);
      for (int64_t i = threadIdx.x; i < rows; i += kCompactThreads) {
        const float p = positions[i];
        if (i > 0 && !(positions[i - 1] < p)) atomicOr(flag, 2u);
        const int64_t k = count_below(wanted, count, p);
        if (k < count && wanted[k] == p) atomicOr(flag, 1u);
      }
      for (int64_t e = threadIdx.x; e < count; e += kCompactThreads)
        if (e > 0 && !(wanted[e - 1] < wanted[e])) atomicOr(flag, 1u);
      continue;
    }
    if (length < 0 || length + count > a.capacity || count > kInsertMax) {  // the check refused it
      if (threadIdx.x == 0) atomicOr(flag, 4u);
      continue;
    }
    __syncthreads();  // the previous head's shared arrays are free
    for (int64_t e = threadIdx.x; e < count; e += kCompactThreads) {
      entries[e] = wanted[e];
      landing[e] = static_cast<int32_t>(e + count_below(positions, length, wanted[e]));
    }
    __syncthreads();
    const int64_t lowest = landing[0];  // resident rows below the first entry stay
    for (int64_t end = length; end > lowest;) {
      const int64_t start = lmax(lowest, end - chunk_rows), rows_here = end - start;
      uint4 k[kCompactVectors], v[kCompactVectors];
#pragma unroll
      for (int j = 0; j < kCompactVectors; ++j) {
        const int64_t item = threadIdx.x + static_cast<int64_t>(j) * kCompactThreads;
        const int64_t r = item / vectors, c = item % vectors;
        if (r < rows_here) {
          k[j] = reinterpret_cast<const uint4 *>(keys + (start + r) * a.row_bytes)[c];
          v[j] = reinterpret_cast<const uint4 *>(values + (start + r) * a.row_bytes)[c];
        }
      }
      float p = 0.0f;
      if (threadIdx.x < rows_here) {
        p = positions[start + threadIdx.x];
        shift[threadIdx.x] = static_cast<int32_t>(count_below(entries, count, p));
      }
      __syncthreads();
#pragma unroll
      for (int j = 0; j < kCompactVectors; ++j) {
        const int64_t item = threadIdx.x + static_cast<int64_t>(j) * kCompactThreads;
        const int64_t r = item / vectors, c = item % vectors;
        if (r < rows_here) {
          const int64_t to = start + r + shift[r];
          reinterpret_cast<uint4 *>(keys + to * a.row_bytes)[c] = k[j];
          reinterpret_cast<uint4 *>(values + to * a.row_bytes)[c] = v[j];
        }
      }
      if (threadIdx.x < rows_here) positions[start + threadIdx.x + shift[threadIdx.x]] = p;
      __syncthreads();  // shift[] and this chunk's stores before the next chunk
      end = start;
    }
    const char *rows = recalled + first * 2 * a.row_bytes;
    for (int64_t item = threadIdx.x; item < count * vectors; item += kCompactThreads) {
      const int64_t e = item / vectors, c = item % vectors, to = landing[e];
      reinterpret_cast<uint4 *>(keys + to * a.row_bytes)[c] =
          reinterpret_cast<const uint4 *>(rows + 2 * e * a.row_bytes)[c];
      reinterpret_cast<uint4 *>(values + to * a.row_bytes)[c] =
          reinterpret_cast<const uint4 *>(rows + (2 * e + 1) * a.row_bytes)[c];
    }
    for (int64_t e = threadIdx.x; e < count; e += kCompactThreads) positions[landing[e]] = entries[e];
    if (threadIdx.x == 0) a.lengths[head] = static_cast<int32_t>(length + count);
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
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(touched, 65535));
  arena_compact_kernel<BY_POSITION><<<blocks, kCompactThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      param(*arena, element), plan, touched, removed, error);
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

extern "C" int lrk_arena_evict(const lrk_arena *arena, const int64_t *heads, const float *removed_positions,
                               int64_t count, unsigned int *error, lrk_stream_t stream) {
  clear_error();
  int64_t element = 0;
  int status = check_arena(arena, &element);
  if (status != LRK_OK) return status;
  LRK_REQUIRE(count >= 0, "invalid batch size");
  if (count == 0 || arena->heads_total == 0) return LRK_OK;
  LRK_REQUIRE(heads && removed_positions, "null pointer");
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(arena->heads_total, 65535));
  arena_evict_kernel<<<blocks, kCompactThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      param(*arena, element), heads, removed_positions, count, error);
  return launch_status("lrk_arena_evict");
}

extern "C" int lrk_arena_insert(const lrk_arena *arena, const int64_t *plan, int64_t touched, const void *recalled,
                                const float *recalled_positions, int check, unsigned int *flag, lrk_stream_t stream) {
  clear_error();
  int64_t element = 0;
  int status = check_arena(arena, &element);
  if (status != LRK_OK) return status;
  LRK_REQUIRE(touched >= 0, "invalid plan size");
  if (touched == 0) return LRK_OK;
  LRK_REQUIRE(plan && recalled && recalled_positions && flag, "null pointer");
  LRK_REQUIRE(aligned(recalled, 16), "recalled rows must be 16-byte aligned");
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(touched, 65535));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (check)
    arena_insert_kernel<true><<<blocks, kCompactThreads, 0, s>>>(param(*arena, element), plan, touched,
                                                                 static_cast<const char *>(recalled),
                                                                 recalled_positions, flag);
  else
    arena_insert_kernel<false><<<blocks, kCompactThreads, 0, s>>>(param(*arena, element), plan, touched,
                                                                  static_cast<const char *>(recalled),
                                                                  recalled_positions, flag);
  return launch_status("lrk_arena_insert");
}
