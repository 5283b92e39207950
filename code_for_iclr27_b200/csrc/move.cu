// Cache data-movement kernels of liblrk: compact, append, batch_append, merge,
// pack, and the two legacy flattened-cache ops.
//
// All of them are row gathers: every output row is a copy of one source row
// (or is left unwritten when its source is out of range).  One engine serves
// them all.  A CTA owns a tile of consecutive output rows; it first resolves
// each row's source (K pointer, V pointer, position) into shared memory with an
// operator-specific "plan", then copies the tile with the widest vector the
// pointers allow (16 B normally), all loads of a chunk issued before its
// stores, with streaming cache hints since each byte is touched once.
// The output of a tile is contiguous, so stores are fully coalesced; reads are
// coalesced within each source row (128-256 B for bf16 D=64/128).
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "tc.cuh"

namespace lrk {
namespace {

constexpr int kThreads = 256;

struct RowSource {
  const char *k;  // nullptr: row skipped (source out of range)
  const char *v;
  float position;
};

// n / d for n * d < 2^32 (n < 2^24 here): one multiply-high.
struct FastDiv {
  uint32_t d, magic;
  __host__ void init(uint32_t divisor) {
    d = divisor;
    magic = divisor == 1 ? 0u : static_cast<uint32_t>(((1ull << 32) + divisor - 1) / divisor);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return d == 1 ? n : __umulhi(n, magic);
  }
};

struct GatherOut {
  char *k;
  char *v;          // nullptr for single-tensor ops
  float *position;  // nullptr when the op has no position rows
  int64_t k_stride;  // bytes between consecutive output rows
  int64_t v_stride;
  int64_t rows;
  int64_t row_bytes;
  FastDiv units;  // vectors per row
};

template <int VB>
__device__ __forceinline__ typename Bits<VB>::type load_stream(const char *p) {
  using V = typename Bits<VB>::type;
  return __ldcs(reinterpret_cast<const V *>(p));
}
template <int VB>
__device__ __forceinline__ void store_stream(char *p, typename Bits<VB>::type value) {
  using V = typename Bits<VB>::type;
  __stcs(reinterpret_cast<V *>(p), value);
}

// Copy rows [0, nrows) of the tile whose sources are in `sources`.
template <int VB>
__device__ __forceinline__ void copy_tile(const RowSource *sources, int nrows, int64_t first_row,
                                          const GatherOut &out) {
  using V = typename Bits<VB>::type;
  constexpr int kChunk = 4;
  const int upr = static_cast<int>(out.units.d);
  const int items = nrows * upr;
  for (int base = 0; base < items; base += kThreads * kChunk) {
    V kb[kChunk], vb[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const int item = base + j * kThreads + threadIdx.x;
      if (item < items) {
        const int row = static_cast<int>(out.units.div(static_cast<uint32_t>(item)));
        const int unit = item - row * upr;
        const RowSource s = sources[row];
        if (s.k != nullptr) {
          kb[j] = load_stream<VB>(s.k + unit * VB);
          if (out.v != nullptr) vb[j] = load_stream<VB>(s.v + unit * VB);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const int item = base + j * kThreads + threadIdx.x;
      if (item < items) {
        const int row = static_cast<int>(out.units.div(static_cast<uint32_t>(item)));
        const int unit = item - row * upr;
        if (sources[row].k != nullptr) {
          const int64_t r = first_row + row;
          store_stream<VB>(out.k + r * out.k_stride + unit * VB, kb[j]);
          if (out.v != nullptr) store_stream<VB>(out.v + r * out.v_stride + unit * VB, vb[j]);
        }
      }
    }
  }
  if (out.position != nullptr) {
    for (int row = threadIdx.x; row < nrows; row += kThreads)
      if (sources[row].k != nullptr) out.position[first_row + row] = sources[row].position;
  }
}

template <int VB, int TR, class Plan>
__global__ void __launch_bounds__(kThreads) gather_kernel(Plan plan, GatherOut out) {
  __shared__ RowSource sources[TR];
  __shared__ typename Plan::Shared shared;
  plan.prologue(shared);
  for (int64_t tile = blockIdx.x; tile * TR < out.rows; tile += gridDim.x) {
    const int64_t first = tile * TR;
    const int nrows = static_cast<int>(lmin(TR, out.rows - first));
    __syncthreads();  // previous tile's sources fully consumed
    plan.template fill<TR>(first, nrows, sources, shared);
    __syncthreads();
    copy_tile<VB>(sources, nrows, first, out);
  }
}

// ------------------------------------------------------------------ plans

struct NoShared {};

// _C.compact: output row r comes from source row r + lower(r), where
// lower(r) = #{m : removed[m] - m <= r} (removed sorted ascending, unique).
// Per tile: two binary searches bound the removed entries that land in the
// tile; a shared histogram of their (removed[m] - m) values and a scan give
// lower(r) for every row of the tile, so each removed entry is visited once.
struct CompactPlan {
  const char *k, *v;
  const float *positions;
  int64_t rows, row_bytes;
  const int64_t *removed;
  int64_t removed_count;
  struct Shared {
    int64_t bounds[2];
    int counts[256];
    int warp_totals[kThreads / 32];
  };
  __device__ void prologue(Shared &) const {}

  // #{m : removed[m] - m <= r}
  __device__ int64_t lower(int64_t r) const {
    int64_t lo = 0, hi = removed_count;
    while (lo < hi) {
      const int64_t mid = lo + (hi - lo) / 2;
      if (removed[mid] - mid <= r) lo = mid + 1; else hi = mid;
    }
    return lo;
  }

  template <int TR>
  __device__ void fill(int64_t first, int nrows, RowSource *sources, Shared &s) const {
    static_assert(TR <= kThreads, "one scan element per thread");
    if (threadIdx.x == 0) s.bounds[0] = first == 0 ? 0 : lower(first - 1);
    if (threadIdx.x == 32) s.bounds[1] = lower(first + nrows - 1);
    for (int i = threadIdx.x; i < TR; i += kThreads) s.counts[i] = 0;
    __syncthreads();
    const int64_t begin = s.bounds[0], end = s.bounds[1];
    for (int64_t m = begin + threadIdx.x; m < end; m += kThreads) {
      const int64_t key = removed[m] - m - first;  // in [0, nrows) by construction
      if (key >= 0 && key < nrows) atomicAdd(&s.counts[key], 1);
    }
    __syncthreads();
    // Inclusive scan of counts[0..TR) across the block.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int value = threadIdx.x < TR ? s.counts[threadIdx.x] : 0;
#pragma unroll
    for (int offset = 1; offset < 32; offset <<= 1) {
      const int other = __shfl_up_sync(0xffffffffu, value, offset);
      if (lane >= offset) value += other;
    }
    if (lane == 31) s.warp_totals[warp] = value;
    __syncthreads();
    int carry = 0;
    for (int w = 0; w < warp; ++w) carry += s.warp_totals[w];
    if (threadIdx.x < nrows) {
      const int64_t source = first + threadIdx.x + begin + value + carry;
      RowSource out;
      if (source >= 0 && source < rows) {
        out.k = k + source * row_bytes;
        out.v = v + source * row_bytes;
        out.position = positions[source];
      } else {
        out.k = out.v = nullptr;
        out.position = 0.0f;
      }
      sources[threadIdx.x] = out;
    }
  }
};

// Head-segmented append shared by _C.append and _legacy_C.append_flattened_cache.
// Output head h starts at start[h] = cumulative[h] + h * added and holds
// old_length[h] existing rows followed by `added` new rows.
constexpr int kMaxSharedHeads = 1024;

struct AppendPlan {
  const char *k, *v;           // existing rows (v may be null)
  const float *positions;      // null for the legacy op
  int64_t rows, row_bytes;
  const char *new_k, *new_v;   // [heads, added, row]
  const int32_t *cumulative;   // [heads + 1]
  const int32_t *head_lens;    // legacy: explicit old lengths; null: from cumulative
  int64_t heads, added, logical_start;
  int32_t *out_cumulative, *out_lengths;  // written by CTA 0 when non-null
  struct Shared {
    int64_t start[kMaxSharedHeads + 1];
  };
  __device__ int64_t old_length(int64_t h) const {
    return head_lens != nullptr ? head_lens[h]
                                : static_cast<int64_t>(cumulative[h + 1]) - cumulative[h];
  }
  __device__ int64_t start_of(const Shared &s, int64_t h) const {
    return heads <= kMaxSharedHeads ? s.start[h] : cumulative[h] + h * added;
  }
  __device__ void prologue(Shared &s) const {
    if (heads <= kMaxSharedHeads)
      for (int64_t h = threadIdx.x; h <= heads; h += kThreads) s.start[h] = cumulative[h] + h * added;
    if (blockIdx.x == 0 && out_cumulative != nullptr) {
      for (int64_t h = threadIdx.x; h < heads; h += kThreads) {
        out_cumulative[h] = static_cast<int32_t>(cumulative[h] + h * added);
        out_lengths[h] = static_cast<int32_t>(old_length(h) + added);
      }
      if (threadIdx.x == 0) out_cumulative[heads] = static_cast<int32_t>(cumulative[heads] + heads * added);
    }
    __syncthreads();
  }
  // Last head whose start is <= o.
  __device__ int64_t head_of(int64_t o, const Shared &s) const {
    int64_t lo = 0, hi = heads;  // answer in [0, heads)
    while (hi - lo > 1) {
      const int64_t mid = (lo + hi) / 2;
      if (start_of(s, mid) <= o) lo = mid; else hi = mid;
    }
    return lo;
  }
  __device__ RowSource source(int64_t o, const Shared &s) const {
    const int64_t h = head_of(o, s);
    const int64_t local = o - start_of(s, h);
    const int64_t old = old_length(h);
    RowSource out{nullptr, nullptr, 0.0f};
    if (local >= 0 && local < old) {
      const int64_t source = cumulative[h] + local;
      if (source >= 0 && source < rows) {
        out.k = k + source * row_bytes;
        out.v = v != nullptr ? v + source * row_bytes : nullptr;
        out.position = positions != nullptr ? positions[source] : 0.0f;
      }
    } else if (local >= old && local < old + added) {
      const int64_t j = local - old;
      const int64_t source = h * added + j;
      out.k = new_k + source * row_bytes;
      out.v = new_v != nullptr ? new_v + source * row_bytes : nullptr;
      out.position = static_cast<float>(logical_start + j);
    }
    return out;
  }
  template <int TR>
  __device__ void fill(int64_t first, int nrows, RowSource *sources, Shared &s) const {
    for (int i = threadIdx.x; i < nrows; i += kThreads) sources[i] = source(first + i, s);
  }
};

// _C.merge: mapping[o] >= 0 takes existing row mapping[o]; otherwise recalled
// row j = -mapping[o] - 1, whose K is recalled[j, 0] and V recalled[j, 1].
struct MergePlan {
  const char *k, *v;
  const float *positions;
  int64_t rows, row_bytes;
  const char *recalled;
  const float *recalled_positions;
  int64_t recalled_rows;
  const int64_t *mapping;
  using Shared = NoShared;
  __device__ void prologue(Shared &) const {}
  template <int TR>
  __device__ void fill(int64_t first, int nrows, RowSource *sources, Shared &) const {
    for (int i = threadIdx.x; i < nrows; i += kThreads) {
      const int64_t m = mapping[first + i];
      RowSource out{nullptr, nullptr, 0.0f};
      if (m >= 0) {
        if (m < rows) {
          out.k = k + m * row_bytes;
          out.v = v + m * row_bytes;
          out.position = positions[m];
        }
      } else {
        const int64_t j = -m - 1;
        if (j < recalled_rows) {
          out.k = recalled + (2 * j) * row_bytes;
          out.v = recalled + (2 * j + 1) * row_bytes;
          out.position = recalled_positions[j];
        }
      }
      sources[i] = out;
    }
  }
};

// lrk_merge_layers: MergePlan over several layers whose outputs are
// concatenated (layer i's rows start at out_first[i]); each output row finds
// its layer by binary search over the (<= kMaxMergeLayers) first rows.
constexpr int kMaxMergeLayers = 64;
struct MergeLayer {
  const char *k, *v;
  const float *positions;
  int64_t rows;
  const char *recalled;
  const float *recalled_positions;
  int64_t recalled_rows;
  const int64_t *mapping;
  int64_t out_first;
};
struct MergeLayersPlan {
  MergeLayer layer[kMaxMergeLayers];
  int count;
  int64_t row_bytes;
  using Shared = NoShared;
  __device__ void prologue(Shared &) const {}
  template <int TR>
  __device__ void fill(int64_t first, int nrows, RowSource *sources, Shared &) const {
    for (int i = threadIdx.x; i < nrows; i += kThreads) {
      const int64_t o = first + i;
      int lo = 0, hi = count - 1;  // last layer with out_first <= o
      while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (layer[mid].out_first <= o) lo = mid; else hi = mid - 1;
      }
      const MergeLayer &L = layer[lo];
      const int64_t m = L.mapping[o - L.out_first];
      RowSource out{nullptr, nullptr, 0.0f};
      if (m >= 0) {
        if (m < L.rows) {
          out.k = L.k + m * row_bytes;
          out.v = L.v + m * row_bytes;
          out.position = L.positions[m];
        }
      } else {
        const int64_t j = -m - 1;
        if (j < L.recalled_rows) {
          out.k = L.recalled + (2 * j) * row_bytes;
          out.v = L.recalled + (2 * j + 1) * row_bytes;
          out.position = L.recalled_positions[j];
        }
      }
      sources[i] = out;
    }
  }
};

// Index gather: _C.pack (with metadata) and _legacy_C.compact_flattened_kv.
struct IndexPlan {
  const char *k, *v;
  const float *positions;  // pack only
  int64_t rows, row_bytes;
  const int64_t *indices;
  const int64_t *heads;    // pack only
  int64_t *metadata;       // pack only: [count, 3]
  int64_t layer;
  using Shared = NoShared;
  __device__ void prologue(Shared &) const {}
  template <int TR>
  __device__ void fill(int64_t first, int nrows, RowSource *sources, Shared &) const {
    for (int i = threadIdx.x; i < nrows; i += kThreads) {
      const int64_t o = first + i;
      const int64_t source = indices[o];
      RowSource out{nullptr, nullptr, 0.0f};
      if (source >= 0 && source < rows) {
        out.k = k + source * row_bytes;
        out.v = v + source * row_bytes;
        if (metadata != nullptr) {
          metadata[o * 3] = layer;
          metadata[o * 3 + 1] = heads[o];
          metadata[o * 3 + 2] = static_cast<int64_t>(positions[source]);
        }
      }
      sources[i] = out;
    }
  }
};

// Plain row gather out of one table: dst row i <- src row indices[i].
struct RowsPlan {
  const char *src;
  int64_t rows, row_bytes;
  const int64_t *indices;
  using Shared = NoShared;
  __device__ void prologue(Shared &) const {}
  template <int TR>
  __device__ void fill(int64_t first, int nrows, RowSource *sources, Shared &) const {
    for (int i = threadIdx.x; i < nrows; i += kThreads) {
      const int64_t source = indices[first + i];
      RowSource out{nullptr, nullptr, 0.0f};
      if (source >= 0 && source < rows) out.k = src + source * row_bytes;
      sources[i] = out;
    }
  }
};

// _C.batch_append: segments (request-major, head-minor) passed by value.
constexpr int kMaxSegmentsPerLaunch = 64;

struct BatchTable {
  lrk_segment segment[kMaxSegmentsPerLaunch];
  int count;
};

struct BatchAppendPlan {
  BatchTable table;
  const char *new_k, *new_v;  // row s of this launch's first segment is at segment_base
  int64_t segment_base;
  int64_t row_bytes;
  using Shared = NoShared;
  __device__ void prologue(Shared &) const {}
  // Last segment whose destination is <= o.
  __device__ int segment_of(int64_t o) const {
    int lo = 0, hi = table.count;
    while (hi - lo > 1) {
      const int mid = (lo + hi) / 2;
      if (table.segment[mid].destination_row <= o) lo = mid; else hi = mid;
    }
    return lo;
  }
  __device__ RowSource source(int64_t o) const {
    const int lo = segment_of(o);
    const lrk_segment &seg = table.segment[lo];
    const int64_t local = o - seg.destination_row;
    RowSource out{nullptr, nullptr, 0.0f};
    if (local >= 0 && local < seg.length) {
      const int64_t source = seg.source_row + local;
      out.k = static_cast<const char *>(seg.keys) + source * row_bytes;
      out.v = static_cast<const char *>(seg.values) + source * row_bytes;
      out.position = seg.positions[source];
    } else if (local == seg.length) {
      out.k = new_k + (segment_base + lo) * row_bytes;
      out.v = new_v + (segment_base + lo) * row_bytes;
      out.position = static_cast<float>(seg.logical_position);
    }
    return out;
  }
  template <int TR>
  __device__ void fill(int64_t first, int nrows, RowSource *sources, Shared &) const {
    for (int i = threadIdx.x; i < nrows; i += kThreads) sources[i] = source(first + i);
  }
};

// ------------------------------------------------------------ dispatch

// Widest vector (bytes) that divides the row and every pointer's alignment.
template <class Pointers>
int widest_vector(int64_t row_bytes, const Pointers &pointers, std::initializer_list<int64_t> strides) {
  for (int vb : {16, 8, 4, 2}) {
    if (row_bytes % vb) continue;
    bool ok = true;
    for (const void *p : pointers) ok = ok && (p == nullptr || aligned(p, vb));
    for (int64_t s : strides) ok = ok && (s % vb == 0);
    if (ok) return vb;
  }
  return 0;
}
int pick_vector(int64_t row_bytes, std::initializer_list<const void *> pointers,
                std::initializer_list<int64_t> strides) {
  return widest_vector(row_bytes, pointers, strides);
}
int pick_vector(int64_t row_bytes, const std::vector<const void *> &pointers,
                std::initializer_list<int64_t> strides) {
  return widest_vector(row_bytes, pointers, strides);
}

template <class Plan>
int launch_gather(const Plan &plan, GatherOut out, int vb, cudaStream_t stream, const char *what) {
  if (out.rows <= 0) return LRK_OK;
  const int64_t units = out.row_bytes / vb;
  if (units <= 0 || units > 1024) return fail(LRK_ERR_UNSUPPORTED, "row too wide for the gather engine");
  out.units.init(static_cast<uint32_t>(units));
  // Tile height: 256 rows for narrow rows; 64 normally; 16 when 64-row tiles
  // would leave SMs idle, 4 when even 16-row tiles would (small outputs such
  // as an archive pack: more CTAs keep more row reads in flight).
  const int sms = sm_count();
  const bool narrow = out.row_bytes < 64;
  const bool tiny = !narrow && ceil_div(out.rows, 16) < 2 * sms;
  const bool small = !narrow && !tiny && ceil_div(out.rows, 64) < 2 * sms;
  const int64_t tile_rows = narrow ? 256 : tiny ? 4 : small ? 16 : 64;
  const int64_t tiles = ceil_div(out.rows, tile_rows);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, static_cast<int64_t>(sms) * 16));
#define LRK_GATHER_CASE(VB)                                                              \
  case VB:                                                                               \
    if (narrow) gather_kernel<VB, 256, Plan><<<grid, kThreads, 0, stream>>>(plan, out);     \
    else if (tiny) gather_kernel<VB, 4, Plan><<<grid, kThreads, 0, stream>>>(plan, out);    \
    else if (small) gather_kernel<VB, 16, Plan><<<grid, kThreads, 0, stream>>>(plan, out);  \
    else gather_kernel<VB, 64, Plan><<<grid, kThreads, 0, stream>>>(plan, out);          \
    break;
  switch (vb) {
    LRK_GATHER_CASE(16)
    LRK_GATHER_CASE(8)
    LRK_GATHER_CASE(4)
    LRK_GATHER_CASE(2)
    default:
      return fail(LRK_ERR_UNSUPPORTED, "no vector width fits the row size and alignment");
  }
#undef LRK_GATHER_CASE
  return launch_status(what);
}

// Bulk-copy engine for the operators whose output tiles are a few runs of
// consecutive source rows (compaction, append, batch append), for 16-byte
// aligned rows of 16-byte multiples up to 512 bytes.  A CTA owns kBulkRows
// output rows.  Thread 0 walks the tile's runs twice (Runs::walk): first to
// check each against the sizes it knows, then to move each with one
// `cp.async.bulk` load per tensor (K and V) into shared memory, completing on
// an mbarrier; the other threads copy the positions meanwhile.  The tile then
// leaves with one bulk store per tensor.  A tile with an invalid run, or whose
// loads do not land within the bounded wait (the wait is then repeated, also
// bounded, for the copies in flight), is copied row by row with 16-byte
// vectors (Runs::source), rows without a valid source skipped as in
// gather_kernel.  A generic version (any gather plan's fill, then one thread
// merging the filled rows into runs) measured 2.7 times slower than the
// vector engine and was not kept.
constexpr int kBulkRows = 64;
constexpr int kBulkThreads = 128;
constexpr int64_t kBulkMaxRowBytes = 512;

// Runs of lrk_compact: output row o comes from o + lower(o), so a run ends
// where the next removed row lands.
struct CompactRuns {
  CompactPlan plan;
  struct Shared {};
  __device__ void setup(Shared &) const {}
  template <class Issue>
  __device__ bool walk(int64_t o0, int n, const Shared &, Issue issue) const {
    const int64_t rb = plan.row_bytes;
    for (int64_t o = o0; o < o0 + n;) {
      const int64_t c = plan.lower(o);
      const int64_t end = c < plan.removed_count ? lmin(o0 + n, plan.removed[c] - c) : o0 + n;
      if (!(end > o && o + c >= 0 && end + c <= plan.rows)) return false;
      issue(o, plan.k + (o + c) * rb, plan.v + (o + c) * rb, end - o);
      o = end;
    }
    return true;
  }
  __device__ RowSource source(int64_t o, const Shared &) const {
    const int64_t source = o + plan.lower(o);
    if (source < 0 || source >= plan.rows) return {nullptr, nullptr, 0.0f};
    return {plan.k + source * plan.row_bytes, plan.v + source * plan.row_bytes, plan.positions[source]};
  }
};

// Runs of lrk_append: per head the tile overlaps, its cache rows, then its
// new rows (new_keys is [heads, added, row]).  CTA 0 also writes the new
// cumulative lengths.
struct AppendRuns {
  AppendPlan plan;
  using Shared = AppendPlan::Shared;
  __device__ void setup(Shared &s) const {
    if (plan.heads <= kMaxSharedHeads)
      for (int64_t h = threadIdx.x; h <= plan.heads; h += kBulkThreads) s.start[h] = plan.cumulative[h] + h * plan.added;
    if (blockIdx.x == 0 && plan.out_cumulative != nullptr) {
      for (int64_t h = threadIdx.x; h < plan.heads; h += kBulkThreads) {
        plan.out_cumulative[h] = static_cast<int32_t>(plan.cumulative[h] + h * plan.added);
        plan.out_lengths[h] = static_cast<int32_t>(plan.old_length(h) + plan.added);
      }
      if (threadIdx.x == 0)
        plan.out_cumulative[plan.heads] = static_cast<int32_t>(plan.cumulative[plan.heads] + plan.heads * plan.added);
    }
  }
  template <class Issue>
  __device__ bool walk(int64_t o0, int n, const Shared &s, Issue issue) const {
    const int64_t rb = plan.row_bytes;
    int64_t h = plan.head_of(o0, s), o = o0;
    while (o < o0 + n) {
      if (h >= plan.heads) return false;
      const int64_t start = plan.start_of(s, h), old = plan.old_length(h), local = o - start;
      if (local >= 0 && local < old) {
        const int64_t end = lmin(o0 + n, start + old), source = plan.cumulative[h] + local;
        if (source < 0 || source + (end - o) > plan.rows) return false;
        issue(o, plan.k + source * rb, plan.v + source * rb, end - o);
        o = end;
      } else if (local >= old && local < old + plan.added) {
        const int64_t end = lmin(o0 + n, start + old + plan.added), source = h * plan.added + (local - old);
        issue(o, plan.new_k + source * rb, plan.new_v + source * rb, end - o);
        o = end;
      } else {
        if (local < 0) return false;
        ++h;  // past this head
      }
    }
    return true;
  }
  __device__ RowSource source(int64_t o, const Shared &s) const { return plan.source(o, s); }
};

// Runs of lrk_batch_append: per (request, head) segment the tile overlaps,
// its cache rows, then its one new row.
struct BatchAppendRuns {
  BatchAppendPlan plan;
  struct Shared {};
  __device__ void setup(Shared &) const {}
  template <class Issue>
  __device__ bool walk(int64_t o0, int n, const Shared &, Issue issue) const {
    const int64_t rb = plan.row_bytes;
    int i = plan.segment_of(o0);
    for (int64_t o = o0; o < o0 + n;) {
      if (i >= plan.table.count) return false;
      const lrk_segment &seg = plan.table.segment[i];
      const int64_t local = o - seg.destination_row;
      if (local >= 0 && local < seg.length) {
        const int64_t end = lmin(o0 + n, seg.destination_row + seg.length), source = seg.source_row + local;
        issue(o, static_cast<const char *>(seg.keys) + source * rb, static_cast<const char *>(seg.values) + source * rb,
              end - o);
        o = end;
      } else if (local == seg.length) {
        issue(o, plan.new_k + (plan.segment_base + i) * rb, plan.new_v + (plan.segment_base + i) * rb, 1);
        o += 1;
      } else {
        if (local < 0) return false;
        ++i;
      }
    }
    return true;
  }
  __device__ RowSource source(int64_t o, const Shared &) const { return plan.source(o); }
};

template <class Runs>
__global__ void __launch_bounds__(kBulkThreads) bulk_kernel(Runs runs, char *__restrict__ out_k,
                                                          char *__restrict__ out_v, float *__restrict__ out_positions,
                                                          int64_t out_rows, int64_t rb) {
  extern __shared__ __align__(128) unsigned char bulk_stage[];  // K rows, then V rows
  __shared__ typename Runs::Shared shared;
  __shared__ __align__(8) uint64_t loaded_storage;
  __shared__ int landed;
  runs.setup(shared);
  const int64_t o0 = static_cast<int64_t>(blockIdx.x) * kBulkRows;
  const int n = static_cast<int>(lmin(kBulkRows, out_rows - o0));
  const uint32_t loaded = static_cast<uint32_t>(__cvta_generic_to_shared(&loaded_storage));
  const uint32_t stage_k = static_cast<uint32_t>(__cvta_generic_to_shared(bulk_stage));
  const uint32_t stage_v = stage_k + static_cast<uint32_t>(kBulkRows * rb);
  __syncthreads();  // setup's shared state
  if (threadIdx.x == 0) {
    tc::init_barrier(loaded, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    const bool ok = runs.walk(o0, n, shared, [](int64_t, const char *, const char *, int64_t) {});
    if (ok) {
      tc::expect_bytes(loaded, static_cast<uint32_t>(2 * n * rb));
      runs.walk(o0, n, shared, [&](int64_t o, const char *k_src, const char *v_src, int64_t len) {
        const uint32_t size = static_cast<uint32_t>(len * rb), offset = static_cast<uint32_t>((o - o0) * rb);
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                         stage_k + offset),
                     "l"(k_src), "r"(size), "r"(loaded)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                         stage_v + offset),
                     "l"(v_src), "r"(size), "r"(loaded)
                     : "memory");
      });
    }
    landed = ok;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += kBulkThreads) {
    const RowSource src = runs.source(o0 + i, shared);
    if (src.k != nullptr) out_positions[o0 + i] = src.position;
  }
  if (threadIdx.x == 0 && landed) {
    if (tc::wait_phase(loaded, 0, nullptr)) {
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      const uint32_t size = static_cast<uint32_t>(n * rb);
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(out_k + o0 * rb),
                   "r"(stage_k), "r"(size)
                   : "memory");
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(out_v + o0 * rb),
                   "r"(stage_v), "r"(size)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
    } else {
      tc::wait_phase(loaded, 0, nullptr);  // the copies in flight, bounded once more
      landed = 0;
    }
  }
  __syncthreads();
  if (landed) return;
  const int units = static_cast<int>(rb / 16);
  for (int item = threadIdx.x; item < n * units; item += kBulkThreads) {
    const int row = item / units, unit = item - row * units;
    const RowSource src = runs.source(o0 + row, shared);
    if (src.k == nullptr) continue;
    __stcs(reinterpret_cast<uint4 *>(out_k + (o0 + row) * rb) + unit,
           __ldcs(reinterpret_cast<const uint4 *>(src.k) + unit));
    __stcs(reinterpret_cast<uint4 *>(out_v + (o0 + row) * rb) + unit,
           __ldcs(reinterpret_cast<const uint4 *>(src.v) + unit));
  }
}

// Launches bulk_kernel when the rows qualify (vb: the common vector width of
// every source and output pointer; breaks: how many places the output's runs
// can end, at most one per tile on average, since a tile of many short runs
// issues many small copies: an audit of configs[0] or [4] that evicts half or
// more of the rows takes the vector engine); returns LRK_ERR_UNSUPPORTED
// otherwise.
template <class Runs>
int launch_bulk(const Runs &runs, int vb, int64_t rb, char *out_k, char *out_v, float *out_positions,
                int64_t out_rows, int64_t breaks, cudaStream_t stream, const char *what) {
  const int64_t tiles = ceil_div(out_rows, kBulkRows);
  if (vb != 16 || rb % 16 != 0 || rb > kBulkMaxRowBytes || tiles < 2 * sm_count() || breaks > tiles)
    return LRK_ERR_UNSUPPORTED;
  const int shared = static_cast<int>(2 * kBulkRows * rb);
  auto kernel = bulk_kernel<Runs>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, shared);
  if (e != cudaSuccess) return fail(LRK_ERR_CUDA, cudaGetErrorString(e));
  kernel<<<static_cast<unsigned>(tiles), kBulkThreads, shared, stream>>>(runs, out_k, out_v, out_positions, out_rows,
                                                                       rb);
  return launch_status(what);
}

int element_bytes(int dtype) { return lrk_dtype_size(dtype); }

}  // namespace
}  // namespace lrk

using namespace lrk;

extern "C" int lrk_compact(const void *keys, const void *values, const float *positions, int64_t rows,
                           int64_t dimension, int dtype, const int64_t *removed, int64_t removed_count,
                           void *out_keys, void *out_values, float *out_positions, lrk_stream_t stream) {
  clear_error();
  const int eb = element_bytes(dtype);
  LRK_REQUIRE(eb > 0, "unknown dtype");
  LRK_REQUIRE(rows >= 0 && dimension > 0 && removed_count >= 0 && removed_count <= rows, "invalid compaction sizes");
  const int64_t out_rows = rows - removed_count;
  if (out_rows == 0) return LRK_OK;
  LRK_REQUIRE(keys && values && positions && out_keys && out_values && out_positions, "null pointer");
  LRK_REQUIRE(removed_count == 0 || removed != nullptr, "null removed indices");
  const int64_t rb = dimension * eb;
  const int vb = pick_vector(rb, {keys, values, out_keys, out_values}, {});
  CompactPlan plan{static_cast<const char *>(keys), static_cast<const char *>(values), positions, rows, rb,
                   removed, removed_count};
  const int bulk = launch_bulk(CompactRuns{plan}, vb, rb, static_cast<char *>(out_keys), static_cast<char *>(out_values),
                               out_positions, out_rows, removed_count, reinterpret_cast<cudaStream_t>(stream),
                               "lrk_compact");
  if (bulk != LRK_ERR_UNSUPPORTED) return bulk;
  GatherOut out{static_cast<char *>(out_keys), static_cast<char *>(out_values), out_positions, rb, rb,
                out_rows, rb, {}};
  return launch_gather(plan, out, vb, reinterpret_cast<cudaStream_t>(stream), "lrk_compact");
}

extern "C" int lrk_append(const void *keys, const void *values, const float *positions, int64_t rows,
                          const void *new_keys, const void *new_values, const int32_t *cumulative,
                          int64_t heads, int64_t added, int64_t dimension, int dtype, int64_t logical_start,
                          void *out_keys, void *out_values, float *out_positions, int32_t *out_cumulative,
                          int32_t *out_lengths, lrk_stream_t stream) {
  clear_error();
  const int eb = element_bytes(dtype);
  LRK_REQUIRE(eb > 0, "unknown dtype");
  LRK_REQUIRE(rows >= 0 && heads > 0 && added > 0 && dimension > 0, "invalid append sizes");
  LRK_REQUIRE(new_keys && new_values && cumulative && out_keys && out_values && out_positions && out_cumulative &&
                  out_lengths,
              "null pointer");
  LRK_REQUIRE(rows == 0 || (keys && values && positions), "null cache pointer");
  const int64_t rb = dimension * eb;
  const int vb = pick_vector(rb, {keys, values, new_keys, new_values, out_keys, out_values}, {});
  AppendPlan plan{static_cast<const char *>(keys), static_cast<const char *>(values), positions, rows, rb,
                  static_cast<const char *>(new_keys), static_cast<const char *>(new_values), cumulative,
                  nullptr, heads, added, logical_start, out_cumulative, out_lengths};
  const int64_t out_rows = rows + heads * added;
  if (rows > 0) {
    const int bulk = launch_bulk(AppendRuns{plan}, vb, rb, static_cast<char *>(out_keys),
                                 static_cast<char *>(out_values), out_positions, out_rows, 2 * heads,
                                 reinterpret_cast<cudaStream_t>(stream), "lrk_append");
    if (bulk != LRK_ERR_UNSUPPORTED) return bulk;
  }
  GatherOut out{static_cast<char *>(out_keys), static_cast<char *>(out_values), out_positions, rb, rb,
                out_rows, rb, {}};
  return launch_gather(plan, out, vb, reinterpret_cast<cudaStream_t>(stream), "lrk_append");
}

extern "C" int lrk_append_flattened(const void *cache, int64_t rows, const void *states, int64_t total_heads,
                                    int64_t new_length, int64_t dimension, int dtype, const int32_t *head_lens,
                                    const int32_t *cu_head_lens, void *out, int64_t out_rows,
                                    lrk_stream_t stream) {
  clear_error();
  const int eb = element_bytes(dtype);
  LRK_REQUIRE(eb > 0, "unknown dtype");
  LRK_REQUIRE(rows >= 0 && total_heads >= 0 && new_length >= 0 && dimension > 0 && out_rows >= 0,
              "invalid append sizes");
  if (out_rows == 0 || total_heads == 0) return LRK_OK;
  LRK_REQUIRE(head_lens && cu_head_lens && out, "null pointer");
  LRK_REQUIRE(new_length == 0 || states, "null states");
  LRK_REQUIRE(rows == 0 || cache, "null cache");
  const int64_t rb = dimension * eb;
  const int vb = pick_vector(rb, {cache, states, out}, {});
  AppendPlan plan{static_cast<const char *>(cache), nullptr, nullptr, rows, rb,
                  static_cast<const char *>(states), nullptr, cu_head_lens, head_lens, total_heads, new_length,
                  0, nullptr, nullptr};
  GatherOut g{static_cast<char *>(out), nullptr, nullptr, rb, rb, out_rows, rb, {}};
  return launch_gather(plan, g, vb, reinterpret_cast<cudaStream_t>(stream), "lrk_append_flattened");
}

extern "C" int lrk_merge(const void *keys, const void *values, const float *positions, int64_t rows,
                         const void *recalled, const float *recalled_positions, int64_t recalled_rows,
                         const int64_t *mapping, int64_t out_rows, int64_t dimension, int dtype, void *out_keys,
                         void *out_values, float *out_positions, lrk_stream_t stream) {
  clear_error();
  const int eb = element_bytes(dtype);
  LRK_REQUIRE(eb > 0, "unknown dtype");
  LRK_REQUIRE(rows >= 0 && recalled_rows >= 0 && out_rows >= 0 && dimension > 0, "invalid merge sizes");
  if (out_rows == 0) return LRK_OK;
  LRK_REQUIRE(mapping && out_keys && out_values && out_positions, "null pointer");
  const int64_t rb = dimension * eb;
  const int vb = pick_vector(rb, {keys, values, recalled, out_keys, out_values}, {});
  MergePlan plan{static_cast<const char *>(keys), static_cast<const char *>(values), positions, rows, rb,
                 static_cast<const char *>(recalled), recalled_positions, recalled_rows, mapping};
  GatherOut out{static_cast<char *>(out_keys), static_cast<char *>(out_values), out_positions, rb, rb,
                out_rows, rb, {}};
  return launch_gather(plan, out, vb, reinterpret_cast<cudaStream_t>(stream), "lrk_merge");
}

extern "C" int lrk_merge_layers(const lrk_merge_layer *layers, int64_t count, int64_t dimension, int dtype,
                                void *out_keys, void *out_values, float *out_positions, lrk_stream_t stream) {
  clear_error();
  const int eb = element_bytes(dtype);
  LRK_REQUIRE(eb > 0, "unknown dtype");
  LRK_REQUIRE(count >= 0 && dimension > 0, "invalid merge sizes");
  if (count == 0) return LRK_OK;
  LRK_REQUIRE(layers && out_keys && out_values && out_positions, "null pointer");
  const int64_t rb = dimension * eb;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int64_t written = 0;
  for (int64_t first = 0; first < count; first += kMaxMergeLayers) {
    const int n = static_cast<int>(std::min<int64_t>(kMaxMergeLayers, count - first));
    MergeLayersPlan plan{};
    plan.count = 0;
    plan.row_bytes = rb;
    std::vector<const void *> pointers{static_cast<char *>(out_keys) + written * rb,
                                       static_cast<char *>(out_values) + written * rb};
    int64_t rows_out = 0;
    for (int i = 0; i < n; ++i) {
      const lrk_merge_layer &l = layers[first + i];
      LRK_REQUIRE(l.rows >= 0 && l.recalled_rows >= 0 && l.out_rows >= 0, "invalid merge sizes");
      LRK_REQUIRE(l.out_rows == 0 || l.mapping != nullptr, "null pointer");
      if (l.out_rows == 0) continue;
      plan.layer[plan.count++] = {static_cast<const char *>(l.keys), static_cast<const char *>(l.values), l.positions,
                                  l.rows, static_cast<const char *>(l.recalled), l.recalled_positions, l.recalled_rows,
                                  l.mapping, rows_out};
      pointers.push_back(l.keys);
      pointers.push_back(l.values);
      pointers.push_back(l.recalled);
      rows_out += l.out_rows;
    }
    if (rows_out == 0) continue;
    const int vb = pick_vector(rb, pointers, {});
    GatherOut out{static_cast<char *>(out_keys) + written * rb, static_cast<char *>(out_values) + written * rb,
                  out_positions + written, rb, rb, rows_out, rb, {}};
    const int status = launch_gather(plan, out, vb, s, "lrk_merge_layers");
    if (status != LRK_OK) return status;
    written += rows_out;
  }
  return LRK_OK;
}

extern "C" int lrk_pack(const void *keys, const void *values, const float *positions, int64_t rows,
                        int64_t dimension, int dtype, const int64_t *indices, const int64_t *heads, int64_t count,
                        int64_t layer, void *payload, int64_t *metadata, lrk_stream_t stream) {
  clear_error();
  const int eb = element_bytes(dtype);
  LRK_REQUIRE(eb > 0, "unknown dtype");
  LRK_REQUIRE(rows >= 0 && count >= 0 && dimension > 0, "invalid pack sizes");
  if (count == 0) return LRK_OK;
  LRK_REQUIRE(keys && values && positions && indices && heads && payload && metadata, "null pointer");
  const int64_t rb = dimension * eb;
  char *base = static_cast<char *>(payload);
  const int vb = pick_vector(rb, {keys, values, payload}, {2 * rb});
  IndexPlan plan{static_cast<const char *>(keys), static_cast<const char *>(values), positions, rows, rb,
                 indices, heads, metadata, layer};
  GatherOut out{base, base + rb, nullptr, 2 * rb, 2 * rb, count, rb, {}};
  return launch_gather(plan, out, vb, reinterpret_cast<cudaStream_t>(stream), "lrk_pack");
}

extern "C" int lrk_compact_flattened(const void *keys, const void *values, int64_t rows, int64_t dimension,
                                     int dtype, const int64_t *keep, int64_t keep_count, void *out_keys,
                                     void *out_values, lrk_stream_t stream) {
  clear_error();
  const int eb = element_bytes(dtype);
  LRK_REQUIRE(eb > 0, "unknown dtype");
  LRK_REQUIRE(rows >= 0 && keep_count >= 0 && dimension > 0, "invalid compaction sizes");
  if (keep_count == 0) return LRK_OK;
  LRK_REQUIRE(keys && values && keep && out_keys && out_values, "null pointer");
  const int64_t rb = dimension * eb;
  const int vb = pick_vector(rb, {keys, values, out_keys, out_values}, {});
  IndexPlan plan{static_cast<const char *>(keys), static_cast<const char *>(values), nullptr, rows, rb, keep,
                 nullptr, nullptr, 0};
  GatherOut out{static_cast<char *>(out_keys), static_cast<char *>(out_values), nullptr, rb, rb, keep_count, rb,
                {}};
  return launch_gather(plan, out, vb, reinterpret_cast<cudaStream_t>(stream), "lrk_compact_flattened");
}

extern "C" int lrk_batch_append(const lrk_segment *segments, int64_t segment_count, const void *new_keys,
                                const void *new_values, int64_t dimension, int dtype, void *out_keys,
                                void *out_values, float *out_positions, int64_t out_rows, lrk_stream_t stream) {
  clear_error();
  const int eb = element_bytes(dtype);
  LRK_REQUIRE(eb > 0, "unknown dtype");
  LRK_REQUIRE(segment_count >= 0 && dimension > 0 && out_rows >= 0, "invalid batch sizes");
  if (segment_count == 0 || out_rows == 0) return LRK_OK;
  LRK_REQUIRE(segments && new_keys && new_values && out_keys && out_values && out_positions, "null pointer");
  const int64_t rb = dimension * eb;
  // Host-side validation: destinations ascending and inside the output.
  int64_t expected = segments[0].destination_row;
  LRK_REQUIRE(expected == 0, "first segment must start at output row 0");
  for (int64_t s = 0; s < segment_count; ++s) {
    const lrk_segment &seg = segments[s];
    LRK_REQUIRE(seg.length >= 0 && seg.source_row >= 0, "invalid segment");
    LRK_REQUIRE(seg.destination_row == expected, "segments must be contiguous in the output");
    LRK_REQUIRE(seg.length == 0 || (seg.keys && seg.values && seg.positions), "null segment pointer");
    expected += seg.length + 1;
  }
  LRK_REQUIRE(expected == out_rows, "segments do not cover the output rows");
  int vb = 16;
  for (int64_t s = 0; s < segment_count; ++s)
    vb = std::min(vb, pick_vector(rb, {segments[s].keys, segments[s].values, new_keys, new_values, out_keys,
                                       out_values},
                                  {}));
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  for (int64_t s0 = 0; s0 < segment_count; s0 += kMaxSegmentsPerLaunch) {
    const int n = static_cast<int>(std::min<int64_t>(kMaxSegmentsPerLaunch, segment_count - s0));
    BatchAppendPlan plan;
    plan.table.count = n;
    for (int i = 0; i < n; ++i) plan.table.segment[i] = segments[s0 + i];
    const int64_t first = segments[s0].destination_row;
    const int64_t last = segments[s0 + n - 1].destination_row + segments[s0 + n - 1].length + 1;
    // Shift destinations so the launch's output view starts at row 0.
    for (int i = 0; i < n; ++i) plan.table.segment[i].destination_row -= first;
    plan.new_k = static_cast<const char *>(new_keys);
    plan.new_v = static_cast<const char *>(new_values);
    plan.segment_base = s0;
    plan.row_bytes = rb;
    int status = launch_bulk(BatchAppendRuns{plan}, vb, rb, static_cast<char *>(out_keys) + first * rb,
                             static_cast<char *>(out_values) + first * rb, out_positions + first, last - first, 2 * n,
                             cs, "lrk_batch_append");
    if (status == LRK_ERR_UNSUPPORTED) {
      GatherOut out{static_cast<char *>(out_keys) + first * rb, static_cast<char *>(out_values) + first * rb,
                    out_positions + first, rb, rb, last - first, rb, {}};
      status = launch_gather(plan, out, vb, cs, "lrk_batch_append");
    }
    if (status != LRK_OK) return status;
  }
  return LRK_OK;
}

extern "C" int lrk_gather_rows(const void *src, int64_t src_rows, int64_t row_bytes, const int64_t *indices,
                               int64_t count, void *dst, lrk_stream_t stream) {
  clear_error();
  LRK_REQUIRE(src_rows >= 0 && row_bytes > 0 && count >= 0, "invalid gather sizes");
  if (count == 0) return LRK_OK;
  LRK_REQUIRE(src && indices && dst, "null pointer");
  const int vb = pick_vector(row_bytes, {src, dst}, {});
  RowsPlan plan{static_cast<const char *>(src), src_rows, row_bytes, indices};
  GatherOut out{static_cast<char *>(dst), nullptr, nullptr, row_bytes, row_bytes, count, row_bytes, {}};
  return launch_gather(plan, out, vb, reinterpret_cast<cudaStream_t>(stream), "lrk_gather_rows");
}
