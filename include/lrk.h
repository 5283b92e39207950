/*
 * lrk.h — C ABI of liblrk, the sm_100a KV-management kernels behind the
 * LazyRecall operator modules (lazy_recall._C, lazy_recall._legacy_C,
 * lazy_recall._host).
 *
 * Every entry point takes plain device pointers, element counts and the CUDA
 * stream to launch on; none allocates device memory, synchronises the stream
 * or touches torch.  Each returns LRK_OK (0) or an error code, and on error
 * lrk_last_error() gives a message for the calling thread.  Arguments are
 * validated on the host before anything is launched; device code additionally
 * skips (never performs) an access whose index falls outside the sizes given
 * here, so inconsistent metadata cannot read or write out of bounds.
 *
 * Reference citations name the operator each entry point replaces, by the
 * file path inside the reference project (wrnwwrnw/code_for_iclr27).
 */
#ifndef LRK_H
#define LRK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; a null value means the legacy default stream. */
typedef struct CUstream_st *lrk_stream_t;

enum lrk_status {
  LRK_OK = 0,
  LRK_ERR_INVALID = 1,     /* an argument was rejected before any launch */
  LRK_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  LRK_ERR_UNSUPPORTED = 3, /* dtype / size combination not implemented */
  LRK_ERR_WORKSPACE = 4    /* the caller's workspace is too small */
};

/* Element types, as the reference's AT_DISPATCH_FLOATING_TYPES_AND2(Half, BFloat16). */
enum lrk_dtype { LRK_F32 = 0, LRK_F64 = 1, LRK_F16 = 2, LRK_BF16 = 3 };

/* Message for the last failed call on this host thread ("" if none). */
const char *lrk_last_error(void);
/* 100 * major + minor of this library. */
int lrk_version(void);
/* Size in bytes of one element of an lrk_dtype, or 0 for an unknown code. */
int lrk_dtype_size(int dtype);

/* ---------------------------------------------------------------- scoring */

/* Masked causal softmax of one query chunk + value projection.
 * Replaces _C.temporal_probabilities (csrc/scoring.cu:205-233, kernel :32-66;
 * bound at csrc/bindings.cpp:21).
 * logits [window, groups, length] of logits_dtype (F32/F16/BF16);
 * projected_values [groups, length] f32; query_positions [window] i64;
 * key_positions [length] f32 -> probabilities [window, groups, length] f32,
 * output_projection [window, groups] f32.  Each scaled logit is rounded to
 * logits_dtype before the softmax, exactly as the reference. */
int lrk_temporal_probabilities(const void *logits, int logits_dtype, const float *projected_values,
                               const int64_t *query_positions, const float *key_positions,
                               float *probabilities, float *output_projection, int64_t window,
                               int64_t groups, int64_t length, float scale, lrk_stream_t stream);

/* Temporal decision risk of candidates [first, last) of one head.
 * Replaces _C.temporal_risk (csrc/scoring.cu:235-255, kernel :68-128; bound at
 * csrc/bindings.cpp:22).  margin is a device pointer to one f32.
 * scores [last - first] f32. */
int lrk_temporal_risk(const float *probabilities, const float *output_projection,
                      const float *projected_values, const float *margin, float *scores,
                      int64_t window, int64_t groups, int64_t length, int64_t first, int64_t last,
                      float epsilon, lrk_stream_t stream);

/* Per-segment sliding max of odd width (Pool7).
 * Replaces _C.pool (csrc/scoring.cu:316-329, kernel :190-203; bound at
 * csrc/bindings.cpp:25).  scores [n] f32, bounds [segments + 1] i64 (device).
 * maximum_count is validated (> 0) like the reference; every position of every
 * segment is written whatever its value. */
int lrk_pool(const float *scores, int64_t n, const int64_t *bounds, int64_t segments,
             int64_t maximum_count, int64_t width, float *out, lrk_stream_t stream);

/* Frozen single-query decision-risk scores (legacy v0 scorer).
 * Replaces _legacy_C.decision_risk_scores (csrc/cache_legacy.cu:244-302,
 * kernel :81-135).  probabilities [groups, candidates] f32; values
 * [candidates, dimension] of values_dtype; head_outputs, gradients
 * [groups, dimension] f32 -> scores [candidates] f32. */
int lrk_decision_risk(const float *probabilities, const void *values, int values_dtype,
                      const float *head_outputs, const float *gradients, int64_t groups,
                      int64_t candidates, int64_t dimension, double base_margin, float epsilon,
                      float *scores, lrk_stream_t stream);

/* One (layer, KV head) segment of a fused scoring call. */
typedef struct lrk_score_segment {
  const void *logits;              /* [window, groups, length] of the call's logits dtype */
  const float *projected_values;   /* row g at projected_values + g * projected_stride, [length] each */
  int64_t projected_stride;        /* elements between the groups' projected-value rows (>= length) */
  const float *key_positions;      /* [length] */
  int64_t length;                  /* rows of this head */
  int64_t first;                   /* candidate interval [first, last) */
  int64_t last;
  float *scores;                   /* [last - first] output */
  int64_t logits_stride;           /* elements between consecutive (query, group) rows of logits (>= length) */
  int64_t query_chunk;             /* queries per chunk of the running maximum; 0: one chunk of all queries */
} lrk_score_segment;

/* Workspace bytes for lrk_temporal_scores. */
size_t lrk_temporal_scores_workspace_bytes(int64_t segments, int64_t window, int64_t groups);

/* Temporal decision risk of every segment's candidates over all `window`
 * queries, straight from logits: the composition temporal_probabilities ->
 * temporal_risk -> running maximum over query chunks that
 * src/lazy_recall/scoring.py:179-195 performs per head, without writing the
 * probabilities.  Many heads per call (segments is a HOST array).  With each
 * segment's query_chunk set to the composition's chunk size (scoring.py:177-178)
 * the scores are bit-identical to the composition on the same logits and
 * projected values.
 * No counterpart operator in the reference (new entry point). */
int lrk_temporal_scores(const lrk_score_segment *segments, int64_t count, int logits_dtype,
                        const int64_t *query_positions, int64_t window, int64_t groups, float scale,
                        const float *margin, float epsilon, void *workspace, size_t workspace_bytes,
                        lrk_stream_t stream);

/* Extra workspace bytes for the probability stash of an lrk_temporal_scores
 * call (0 for an invalid call): with a workspace of
 * lrk_temporal_scores_workspace_bytes(...) + this many bytes, the row
 * statistics store the probability p of every candidate column of every row,
 * and the risk step (csrc/scoring.cu:68-128) reads p instead of recomputing
 * it from the logits (scale, round, mask, expf, division).  The scores are
 * the same bit for bit either way.  Per segment: window x groups rows of the
 * candidate count rounded up to 32 floats. */
size_t lrk_temporal_scores_stash_bytes(const lrk_score_segment *segments, int64_t count, int64_t window,
                                       int64_t groups);

/* Largest segments x window x groups one lrk_temporal_scores_static call takes
 * (one configs[1] audit: 256 heads x 250 queries x 4 groups = 256000). */
#define LRK_STATIC_SCORE_ROWS 262144

/* lrk_temporal_scores without a workspace argument, for callers that cannot
 * allocate device memory: a host whose device memory is all handed out by
 * another allocator (an inference engine that reserves the GPU's memory up
 * front and forbids further cudaMalloc), or a plain C host (cgo, JNI) with no
 * device allocator of its own.  It allocates nothing: its scratch is a
 * file-scope device array of LRK_STATIC_SCORE_ROWS row statistics (3 MiB),
 * which every GPU that loads liblrk holds until the process exits.  Calls with
 * segments x window x groups above LRK_STATIC_SCORE_ROWS are rejected with
 * LRK_ERR_INVALID before anything is launched.  The first call in each CUDA
 * context (normally once per device: the runtime's primary context) looks up
 * the array's device address (cudaGetSymbolAddress); the address is cached
 * per context ID, so a context made after cudaDeviceReset looks it up again.
 * Make that first call before any stream capture in that context.  All calls share the
 * one array: calls whose work overlaps on the GPU (other streams, other host
 * threads) race and must be serialised by the caller.  Nothing in the array
 * needs clearing between calls: each call writes every entry it reads first.
 * Same results as lrk_temporal_scores.
 * No counterpart in the reference (new entry point). */
int lrk_temporal_scores_static(const lrk_score_segment *segments, int64_t count, int logits_dtype,
                               const int64_t *query_positions, int64_t window, int64_t groups, float scale,
                               const float *margin, float epsilon, lrk_stream_t stream);

/* Projected values of one layer for the audit: out[g, r] = sum_d
 * gradients[head(r) * groups + g, d] * float(values[r, d]) for every row r of
 * the packed layer, head(r) the KV head whose segment (cumulative, int32
 * [heads + 1], device) holds r -- each head's rows against its own query
 * heads' margin gradients, the product src/lazy_recall/scoring.py:175 forms
 * per head.  Each dot product is accumulated in channel order with one fused
 * multiply-add per channel from zero, the order of the float32 GEMM that
 * torch.matmul runs for that product (equal bit for bit on B200, checked by
 * the tests).  values [rows, dimension] of values_dtype; gradients
 * [heads * groups, dimension] f32; out [groups, rows] f32.  Reads V once.
 * No counterpart operator in the reference (new entry point). */
int lrk_project_values(const void *values, int values_dtype, int64_t rows, int64_t dimension,
                       const float *gradients, const int32_t *cumulative, int64_t heads, int64_t groups,
                       float *out, lrk_stream_t stream);

/* Test hook: counts, into *mismatches_device (device, zeroed by the caller),
 * the pairs among `count` pseudo-random (a, b) -- a in [0, 1], b in [1, 2^20],
 * the row-statistics domain -- on which the scoring kernels' division differs
 * in any bit from IEEE round-to-nearest division.  Expected 0.
 * No counterpart in the reference. */
int lrk_check_division(uint64_t count, uint64_t seed, unsigned long long *mismatches_device, lrk_stream_t stream);

/* bf16 logits out[r, n] = sum_d queries[r, d] * keys[n, d] for r < rows,
 * n < count, accumulated in float32 as k_step-term tensor-core steps (mma
 * m16n8k8 for k_step 8, m16n8k16 for 16) in increasing d and rounded to bf16.
 * torch.matmul's bf16 GEMM (src/lazy_recall/scoring.py:184) takes eight-term
 * steps for an odd key count and sixteen-term steps otherwise; with the
 * matching k_step the logits equal its output bit for bit, written as rows of
 * out_stride elements (a multiple of 8, >= count rounded up to 8) for the
 * scoring kernels.  queries [rows, dim], keys [count, dim] bf16 row-major,
 * 16-byte aligned, dim 64 or 128.
 * No counterpart operator in the reference (new entry point). */
int lrk_logits(const void *queries, int64_t rows, const void *keys, int64_t count, int64_t dim, int64_t k_step,
               void *out, int64_t out_stride, lrk_stream_t stream);

/* One head of lrk_logits_heads: the arguments of one lrk_logits call. */
typedef struct lrk_logits_head {
  const void *queries; /* bf16 [rows, dim], row-major, 16-byte aligned */
  const void *keys;    /* bf16 [count, dim], row-major, 16-byte aligned */
  int64_t count;
  int64_t k_step;      /* 8 or 16 */
  void *out;           /* bf16 [rows, out_stride], 16-byte aligned */
  int64_t out_stride;  /* a multiple of 8, >= count rounded up to 8 */
} lrk_logits_head;

/* lrk_logits for every head of a layer in one pass over the GPU (the heads
 * share rows and dim; each has its own keys, step order and output).  The
 * per-head GEMMs of src/lazy_recall/scoring.py:184 for one layer; results
 * equal head_count lrk_logits calls bit for bit.
 * No counterpart operator in the reference (new entry point). */
int lrk_logits_heads(const lrk_logits_head *heads, int64_t head_count, int64_t rows, int64_t dim,
                     lrk_stream_t stream);

/* Number of lrk_logits / lrk_logits_heads CTAs (since the library loaded, on the current device)
 * whose bounded wait for their tensor-core steps ran out; 0 in a healthy run.
 * Synchronous.  No counterpart in the reference. */
int lrk_logits_timeouts(unsigned int *count);

/* ---------------------------------------------- scores straight from keys */

/* One layer's keys: bf16 [rows, dim], contiguous, 16-byte aligned. */
typedef struct lrk_key_layer {
  const void *keys;
  int64_t rows;
} lrk_key_layer;

/* One KV head of an audit, scored from its queries and keys. */
typedef struct lrk_key_segment {
  int64_t layer;                  /* index into the call's layers */
  const void *queries;            /* bf16: query q, group g at queries + q * query_stride + g * dim */
  int64_t query_stride;           /* elements (multiple of 8, >= groups * dim); 16-byte aligned rows */
  const float *projected_values;  /* group g at projected_values + g * projected_stride, [length] */
  int64_t projected_stride;
  const float *key_positions;     /* [length] */
  int64_t key_row;                /* the head's first row in its layer's keys */
  int64_t length;                 /* keys of the head */
  int64_t first;                  /* candidate interval [first, last) */
  int64_t last;
  float *scores;                  /* [last - first] output */
  int64_t query_chunk;            /* queries per chunk of the running maximum; 0: one chunk */
} lrk_key_segment;

/* Workspace bytes lrk_scores_from_keys needs for these segments (0 for an
 * invalid table). */
size_t lrk_scores_from_keys_workspace_bytes(const lrk_key_segment *segments, int64_t count, int64_t window,
                                            int64_t groups);

/* lrk_temporal_scores from the queries and keys instead of the logits: the
 * bf16 logits GEMM of src/lazy_recall/scoring.py:184 (16-term tensor-core
 * steps for an even key count, 8-term steps for an odd one, as cuBLAS runs
 * them) and the row statistics run as one tcgen05 kernel whose logits never
 * reach memory (only each segment's candidate columns, for the risk step).
 * The scores are bit-identical to lrk_temporal_scores on the logits
 * torch.matmul produces for the same queries and keys.  Many heads of many
 * layers per call (segments and layers are HOST arrays).  dim 64 or 128,
 * groups <= 8.  Every wait inside the kernel is bounded; a CTA that gave up
 * is counted by lrk_scores_from_keys_timeouts (its scores are then invalid).
 * No counterpart operator in the reference (new entry point). */
int lrk_scores_from_keys(const lrk_key_segment *segments, int64_t count, const lrk_key_layer *layers,
                         int64_t layer_count, const int64_t *query_positions, int64_t window, int64_t groups,
                         int64_t dim, float scale, const float *margin, float epsilon, void *workspace,
                         size_t workspace_bytes, lrk_stream_t stream);

/* CTAs of lrk_scores_from_keys that gave up a wait since the library loaded. */
int lrk_scores_from_keys_timeouts(unsigned int *count);

/* ------------------------------------------------- cache data movement */

/* Append `added` rows to each head segment of a packed layer.
 * Replaces _C.append (csrc/scoring.cu:264-292, kernel :130-162; bound at
 * csrc/bindings.cpp:23).  keys/values [rows, dimension], positions [rows];
 * new_keys/new_values [heads, added, dimension]; cumulative [heads + 1] i32
 * (device) -> out_* [rows + heads * added, ...], out_cumulative [heads + 1],
 * out_lengths [heads] (i32).  New rows get position float(logical_start + i). */
int lrk_append(const void *keys, const void *values, const float *positions, int64_t rows,
               const void *new_keys, const void *new_values, const int32_t *cumulative,
               int64_t heads, int64_t added, int64_t dimension, int dtype, int64_t logical_start,
               void *out_keys, void *out_values, float *out_positions, int32_t *out_cumulative,
               int32_t *out_lengths, lrk_stream_t stream);

/* Drop sorted, unique row indices from packed K/V/positions.
 * Replaces _C.compact (csrc/scoring.cu:294-314, kernel :164-188; bound at
 * csrc/bindings.cpp:24).  removed [removed_count] i64 sorted ascending ->
 * out_* [rows - removed_count, ...]. */
int lrk_compact(const void *keys, const void *values, const float *positions, int64_t rows,
                int64_t dimension, int dtype, const int64_t *removed, int64_t removed_count,
                void *out_keys, void *out_values, float *out_positions, lrk_stream_t stream);

/* Two-source gather of recalled rows into a layer.
 * Replaces _C.merge (csrc/recall.cu:54-84, kernel :7-28; bound at
 * csrc/bindings.cpp:26).  recalled [recalled_rows, 2, dimension] (K then V);
 * mapping [out_rows] i64: m >= 0 takes existing row m, m < 0 takes recalled
 * row -m-1. */
int lrk_merge(const void *keys, const void *values, const float *positions, int64_t rows,
              const void *recalled, const float *recalled_positions, int64_t recalled_rows,
              const int64_t *mapping, int64_t out_rows, int64_t dimension, int dtype,
              void *out_keys, void *out_values, float *out_positions, lrk_stream_t stream);

/* One layer of lrk_merge_layers: lrk_merge's inputs, and out_rows output rows. */
typedef struct lrk_merge_layer {
  const void *keys;                /* [rows, dimension] */
  const void *values;
  const float *positions;          /* [rows] */
  int64_t rows;
  const void *recalled;            /* [recalled_rows, 2, dimension] (K then V) */
  const float *recalled_positions; /* [recalled_rows] */
  int64_t recalled_rows;
  const int64_t *mapping;          /* [out_rows], as lrk_merge's */
  int64_t out_rows;
} lrk_merge_layer;

/* lrk_merge of several layers in one launch: layer i's output rows follow
 * those of layers 0 .. i-1 in out_keys / out_values / out_positions (one
 * allocation for every touched layer of a recall event).  Same rows as one
 * lrk_merge per layer.  No counterpart in the reference (new entry point). */
int lrk_merge_layers(const lrk_merge_layer *layers, int64_t count, int64_t dimension, int dtype, void *out_keys,
                     void *out_values, float *out_positions, lrk_stream_t stream);

/* Gather evicted rows into an archive payload.
 * Replaces _C.pack (csrc/recall.cu:86-111, kernel :30-47; bound at
 * csrc/bindings.cpp:27).  payload [count, 2, dimension], metadata [count, 3]
 * i64 = (layer, heads[i], int64(positions[indices[i]])). */
int lrk_pack(const void *keys, const void *values, const float *positions, int64_t rows,
             int64_t dimension, int dtype, const int64_t *indices, const int64_t *heads,
             int64_t count, int64_t layer, void *payload, int64_t *metadata, lrk_stream_t stream);

/* One (request, head) segment of a static-batch append.  Same fields, in the
 * same order, as the reference's 7-wide descriptor rows
 * (csrc/batch_append.cu:179-186). */
typedef struct lrk_segment {
  const void *keys;         /* request's packed K [*, dimension] (device) */
  const void *values;       /* request's packed V */
  const float *positions;   /* request's positions */
  int64_t source_row;       /* first row of this head in the request's cache */
  int64_t length;           /* rows of this head before the append */
  int64_t destination_row;  /* first row of this head in the output */
  int64_t logical_position; /* position value of the appended token */
} lrk_segment;

/* Multi-request one-token append into one packed output.
 * Replaces _C.batch_append (csrc/batch_append.cu:36-94, kernel :8-34; bound at
 * csrc/bindings.cpp:28).  segments is a HOST array (request-major, head-minor);
 * it is passed to the kernels by value, so no descriptor copy or device
 * allocation happens.  new_keys/new_values [segment_count, dimension]. */
int lrk_batch_append(const lrk_segment *segments, int64_t segment_count, const void *new_keys,
                     const void *new_values, int64_t dimension, int dtype, void *out_keys,
                     void *out_values, float *out_positions, int64_t out_rows,
                     lrk_stream_t stream);

/* Append new_length states per head to one flattened cache tensor.
 * Replaces _legacy_C.append_flattened_cache (csrc/cache_legacy.cu:145-197,
 * kernel :13-40).  states [total_heads, new_length, dimension]; head_lens
 * [total_heads], cu_head_lens [total_heads + 1] i32 (device). */
int lrk_append_flattened(const void *cache, int64_t rows, const void *states, int64_t total_heads,
                         int64_t new_length, int64_t dimension, int dtype, const int32_t *head_lens,
                         const int32_t *cu_head_lens, void *out, int64_t out_rows,
                         lrk_stream_t stream);

/* Gather kept rows of K and V.
 * Replaces _legacy_C.compact_flattened_kv (csrc/cache_legacy.cu:199-242,
 * kernel :42-61). */
int lrk_compact_flattened(const void *keys, const void *values, int64_t rows, int64_t dimension,
                          int dtype, const int64_t *keep, int64_t keep_count, void *out_keys,
                          void *out_values, lrk_stream_t stream);

/* ------------------------------------------------------------ selection */

/* Workspace bytes lrk_refine needs for n scores in `segments` segments. */
size_t lrk_refine_workspace_bytes(int64_t n, int64_t segments);

/* Allocation-preserving refinement: the global bottom-`count` of raw scores,
 * per-segment quotas, each segment's bottom-quota of pooled scores, and the
 * transplant of those refined positions into the raw-score slots.
 * Replaces the torch.topk + numpy body of refine_arrays
 * (src/lazy_recall/selection.py:52-88, transplant :42-49); the ordering
 * reproduces torch.topk(largest=False, sorted=True) on CUDA, ties included.
 * raw, pooled [n] f32; segment_ends, position_starts [segments] i64 (device).
 * Outputs (device): values [count] f32 (raw scores, ascending),
 * segment_ids [count] i64, positions [count] i64, stats [2] i64 =
 * (changed identities, changed heads). */
int lrk_refine(const float *raw, const float *pooled, int64_t n, const int64_t *segment_ends,
               const int64_t *position_starts, int64_t segments, int64_t count, void *workspace,
               size_t workspace_bytes, float *values, int64_t *segment_ids, int64_t *positions,
               int64_t *stats, lrk_stream_t stream);

/* Workspace bytes lrk_topk_smallest needs for n scores. */
size_t lrk_topk_workspace_bytes(int64_t n);

/* torch.topk(x, k, largest=False, sorted=True) of one 1-D f32 slice, with the
 * same choice and order of tied elements as PyTorch's CUDA implementation.
 * values [k] f32, indices [k] i64 (device). */
int lrk_topk_smallest(const float *x, int64_t n, int64_t k, void *workspace,
                      size_t workspace_bytes, float *values, int64_t *indices, lrk_stream_t stream);

/* One layer of a recall merge plan (lrk_merge_plan). */
typedef struct lrk_plan_layer {
  const float *positions;          /* [rows] the layer's positions, heads back to back */
  const int32_t *head_starts;      /* [heads + 1] the heads' row bounds (the layer's cu_seqlens) */
  const float *recalled_positions; /* [recalled] sorted by (head, position) */
  const int64_t *recalled_index;   /* [recalled] each one's index among the layer's recalled rows
                                      (NULL: entry e is recalled row e) */
  const int32_t *recalled_starts;  /* [heads + 1] each head's first entry in the two arrays above */
  int64_t rows, recalled;
  int64_t *mapping;                /* [rows + recalled] out: row i of the merged layer comes from
                                      resident row mapping[i], or recalled row -mapping[i] - 1 */
} lrk_plan_layer;

/* The recall merge plan of every touched layer on the device: the mapping
 * recall/planning.py:34-52 builds on the host after copying the positions
 * back (src/lazy_recall/cache.py:216-217), for lrk_merge / lrk_merge_layers.
 * Resident rows keep their order and recalled rows go in position order
 * (the stable argsort of the combined positions, given that each head's
 * resident positions ascend).  *flag (device, the caller zeroes it) gets bit 1
 * if a position is recalled twice or recalled while resident (the reference
 * refuses the merge) and bit 2 if a head's resident positions do not ascend
 * (the host plan is then needed), bit 4 if head_starts / recalled_starts do
 * not ascend from 0 to rows / recalled (reads and writes stay inside the
 * layer's arrays all the same); read it before adopting the merged cache.
 * All pointers device memory except `layers`. */
int lrk_merge_plan(const lrk_plan_layer *layers, int64_t count, int64_t heads, unsigned int *flag,
                   lrk_stream_t stream);

/* ---------------------------------------------------------- KV arena */

/* A gapped per-head KV arena: every (layer, head) owns a slot of `capacity`
 * rows; its live rows are rows [0, lengths[h]) of the slot, in the packed
 * layout's order (the packed cache is the concatenation of the slots' live
 * rows).  keys, values [heads_total, capacity, dimension] (dtype);
 * positions [heads_total, capacity] f32; lengths [heads_total] i32; all
 * device memory.  FlashAttention's cache entry point consumes it directly
 * (k_cache [heads, capacity, 1, D], cache_seqlens = lengths).
 * No counterpart in the reference: its cache is packed and every append,
 * compaction and merge rebuilds whole layers (csrc/scoring.cu:264-314). */
typedef struct lrk_arena {
  void *keys;
  void *values;
  float *positions;
  int32_t *lengths;
  int64_t heads_total; /* layers x heads */
  int64_t capacity;    /* rows per head slot */
  int64_t dimension;
  int dtype;           /* rows of dimension x dtype bytes, a multiple of 16 */
} lrk_arena;

/* Decode append without copying the cache: one row per head h in [first_head,
 * first_head + count) at row lengths[h] of its slot (new_keys, new_values
 * [count, dimension], device), position `position`, then lengths[h] += 1 --
 * what _C.append does per layer (csrc/scoring.cu:130-162), for any number of
 * layers in one launch.  A head at capacity is left unchanged and sets
 * *overflow (device flag, may be null); callers track lengths and grow first. */
int lrk_arena_append(const lrk_arena *arena, int64_t first_head, int64_t count, const void *new_keys,
                     const void *new_values, float position, unsigned int *overflow, lrk_stream_t stream);

/* Eviction in place: for each touched head, plan[t] = (head, offset, count)
 * (i64 [touched][3], device), the head's rows removed[offset .. offset+count)
 * (i64, device, strictly ascending, below the head's length) are dropped and
 * the later rows move down -- the packed result of _C.compact
 * (csrc/scoring.cu:164-188) restricted to the touched heads, with no other
 * head moved.  Heads must be distinct; a head whose list is out of order or
 * out of range is left unchanged and sets *error (device flag, may be null).
 * Plan entries with count 0 are skipped (a dense plan over all heads is fine). */
int lrk_arena_compact(const lrk_arena *arena, const int64_t *plan, int64_t touched, const int64_t *removed,
                      unsigned int *error, lrk_stream_t stream);

/* lrk_arena_compact with each head's rows named by their logical position:
 * removed_positions (f32, device) holds, per plan entry, positions present in
 * the head, strictly ascending; the head's live positions must be ascending
 * (appends and position-ordered merges keep them so).  This is how a lazy
 * eviction batch finds its rows with no host round trip: a queued reference's
 * row at audit time, shifted down by the rows removed from its head since
 * (src/lazy_recall/controller.py:57-70), is the row that now holds the
 * position it held at the audit. */
int lrk_arena_compact_positions(const lrk_arena *arena, const int64_t *plan, int64_t touched,
                                const float *removed_positions, unsigned int *error, lrk_stream_t stream);

/* Recall reinsertion into the arena in place: no reference counterpart (the
 * reference rebuilds every touched layer, src/lazy_recall/cache.py:201-253,
 * csrc/recall.cu:54-84; the rows and positions that result are the same as
 * that merge's for each head).  plan [touched, 3] i64 = (head, first entry,
 * count), device memory; recalled [entries, 2, dimension] (K then V, 16-byte
 * aligned) and recalled_positions [entries] (f32), each head's entries in
 * ascending position order.  check != 0 only sets *flag: bit 1 a position
 * recalled twice or recalled while resident, bit 2 resident positions that
 * do not ascend, bit 4 a head that would pass its capacity, bit 8 more than
 * 2048 entries for one head; nothing changes.  check == 0 merges: a head's
 * rows above its first entry's place move up in place and the entries land
 * in position order; lengths[head] += count.  Run the check first and merge
 * only when *flag is 0. */
int lrk_arena_insert(const lrk_arena *arena, const int64_t *plan, int64_t touched, const void *recalled,
                     const float *recalled_positions, int check, unsigned int *flag, lrk_stream_t stream);

/* A lazy eviction batch as it leaves the queue: heads [count] (i64: layer x
 * heads + head) and removed_positions [count] (f32 logical positions), in any
 * order, device memory.  Each head collects, sorts and removes its own
 * entries in one launch (up to 2048 per head; more, a duplicate or a position
 * the head does not hold leave that head unchanged and set *error). */
int lrk_arena_evict(const lrk_arena *arena, const int64_t *heads, const float *removed_positions, int64_t count,
                    unsigned int *error, lrk_stream_t stream);

/* ---------------------------------------------- layer-group selection */

/* The request-wide "k smallest raw scores" when one request's layers are
 * split over ranks (GPUs): the selection refine_arrays starts from
 * (src/lazy_recall/selection.py:52-88, torch.topk(largest=False) over the
 * whole score table), with ties taken in score-table order, which is
 * layer-major (src/lazy_recall/scoring.py:218-287), so ranks holding
 * consecutive layer groups in rank order take ties in rank order.  A rank's
 * share of the k smallest is its local bottom-(share) by (key, index).
 *
 * Three radix rounds (12, 12, 8 bits of the order-preserving key, NaN last).
 * Per round: lrk_select_histogram on every rank, an all-gather of the
 * histograms by the caller (NCCL), lrk_select_pick on every rank.  The state
 * stays on the device between rounds; after round 2, state[SHARE] is this
 * rank's share and state[TOTAL] the request-wide score count.  No counterpart
 * operator in the reference (its selection runs on one GPU). */
#define LRK_SELECT_BINS 4096
#define LRK_SELECT_ROUNDS 3
#define LRK_SELECT_MAX_QUESTIONS 4
#define LRK_SELECT_MAX_REQUESTS 64
/* Fields of one (request, question) state: int64 [LRK_SELECT_STATE_FIELDS].
 * The caller zeroes a state and sets K before round 0. */
#define LRK_SELECT_STATE_FIELDS 8
#define LRK_SELECT_K 0           /* the k asked for (clamped to TOTAL) */
#define LRK_SELECT_PREFIX 1      /* key bits fixed so far */
#define LRK_SELECT_NEED 2        /* rank of the k-th key among the keys in play */
#define LRK_SELECT_BELOW 3       /* request-wide keys below the keys in play */
#define LRK_SELECT_LOCAL_BELOW 4 /* this rank's keys below the keys in play */
#define LRK_SELECT_TOTAL 5       /* request-wide key count (set in round 0) */
#define LRK_SELECT_SHARE 6       /* result: this rank's share of the k smallest
                                  * (-1: the ranks' histograms were inconsistent) */

/* One round's histograms of this rank's keys: scores[r] / counts[r] is
 * request r's score table on this rank (device f32, HOST pointer array);
 * states [requests][questions][FIELDS] i64 (device); histograms
 * [requests][questions][LRK_SELECT_BINS] u32 (device), cleared here first. */
int lrk_select_histogram(const float *const *scores, const int64_t *counts, int64_t requests,
                         int64_t questions, int round, const int64_t *states, uint32_t *histograms,
                         lrk_stream_t stream);

/* Advance every state by one round from the all-gathered histograms:
 * gathered [world][requests][questions][LRK_SELECT_BINS] u32 (device), rank
 * this rank's index in gather order (= its layer group's order). */
int lrk_select_pick(const uint32_t *gathered, int64_t world, int64_t rank, int64_t requests,
                    int64_t questions, int round, int64_t *states, lrk_stream_t stream);

/* Gather rows of one table: dst row i = src row indices[i] (row_bytes each);
 * out-of-range indices leave their destination row unwritten.  src may be
 * device memory or pinned host memory mapped for the device
 * (lrk_host_device_pointer): the GPU then reads the recalled rows over the host
 * link itself, with no CPU gather and no staging copy.  Replaces, for recall,
 * the CPU worker's gather into a shared-memory result slot and the slot's
 * cudaMemcpyAsync (src/lazy_recall/recall/cpu_worker.py:161-166,
 * recall/transport.py:221-229); no counterpart operator in the reference. */
int lrk_gather_rows(const void *src, int64_t src_rows, int64_t row_bytes, const int64_t *indices, int64_t count,
                    void *dst, lrk_stream_t stream);

/* ------------------------------------------------------------------ host */

/* Page-lock a host range for async DMA (cudaHostRegisterDefault).
 * Replaces _host.register_host (csrc/host.cpp:5-8). */
int lrk_register_host(void *address, size_t bytes);
/* Replaces _host.unregister_host (csrc/host.cpp:10-13). */
int lrk_unregister_host(void *address);
/* Device address of registered (page-locked, mapped) host memory; fails with
 * LRK_ERR_INVALID for memory that is not registered.  No counterpart in the
 * reference. */
int lrk_host_device_pointer(void *host, void **device);

#ifdef __cplusplus
}
#endif

#endif /* LRK_H */
