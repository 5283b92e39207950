"""One LazyRecall audit pass on the GPU: score -> pool -> select -> evict.

Mirrors the KV side of LazyController.run_audit (controller.py:140-160):
compute_score_table (scoring.py:198-308) with temporal_head_scores'
GPU branch (scoring.py:152-195), pool_score_table (scoring.py:322-335),
refine_arrays (selection.py:52-88) and the eviction of the immediate prefix
(controller.py:154-158 -> cache.remove_positions).  The model-side inputs of
an audit -- per-layer query history [W, query_heads, D], query positions
[W], and the per-layer margin gradient projected to the head inputs
[query_heads, D] -- are passed in.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List

import numpy as np

from . import operators, upload
from .selection import ArrayReferences, fetch_references, refine_arrays, refine_device


@dataclass(frozen=True)
class ScoreSegment:
    """One physical head's candidate range (_core/scoring.py:198-203)."""
    layer: int
    head: int
    position_start: int
    count: int


@dataclass
class ScoreTable:
    scores: "object"
    segments: List[ScoreSegment]
    cumulative_ends: List[int]


def temporal_head_scores(queries, query_positions, keys, key_positions, values, candidate_start, candidate_end,
                         margin_gradient, base_margin, denominator_epsilon, query_chunk_size):
    """scoring.py:152-195 on the new operators: pv = g V^T, then per chunk of
    queries bf16 logits = Q K^T, temporal_probabilities, temporal_risk, and a
    running maximum."""
    import torch

    C = operators()
    projected_values = torch.matmul(margin_gradient.float(), values.float().transpose(0, 1)).contiguous()
    key_positions = key_positions.to(dtype=torch.float32).contiguous()
    query_positions = query_positions.to(dtype=torch.int64).contiguous()
    margin = base_margin.to(device=keys.device, dtype=torch.float32).reshape(1).contiguous()
    chunk_size = query_chunk(query_chunk_size, queries.shape[1], keys.shape[0], keys.element_size())
    result = None
    for start in range(0, queries.shape[0], chunk_size):
        end = min(start + chunk_size, queries.shape[0])
        # A contiguous [chunk, G, D] block folds into one [chunk*G, D] x [D, L]
        # GEMM; the permuted query-history view of scoring.py:260-262 does not,
        # and torch.matmul then runs `chunk` batched [G, D] x [D, L] products.
        logits = torch.matmul(queries[start:end].to(keys.dtype).contiguous(), keys.transpose(0, 1))
        probabilities, output_projection = C.temporal_probabilities(
            logits.contiguous(), projected_values, query_positions[start:end], key_positions,
            1.0 / math.sqrt(keys.shape[-1]))
        scores = C.temporal_risk(probabilities, output_projection, projected_values, margin, candidate_start,
                                 candidate_end, denominator_epsilon)
        result = scores if result is None else torch.maximum(result, scores)
    return result


def score_table(cache, queries, query_positions, gradients, base_margin, protect_recent=32,
                denominator_epsilon=1e-6, query_chunk_size=250) -> ScoreTable:
    """compute_score_table (scoring.py:198-308): every eligible generation row
    of every (layer, KV head), prompt protected, the last protect_recent rows
    protected.  queries[layer] [W, query_heads, D]; gradients[layer]
    [query_heads, D] float32."""
    import torch

    parts, segments, ends, running = [], [], [], 0
    for layer_index, layer in enumerate(cache.layers):
        heads = len(layer.head_lens)
        groups = queries[layer_index].shape[1] // heads
        bounds = layer.bounds()
        positions = layer.positions.reshape(-1)
        for head in range(heads):
            start, end = int(bounds[head]), int(bounds[head + 1])
            candidate_start = int(layer.prompt_lens[head])
            candidate_end = max(candidate_start, end - start - protect_recent)
            if candidate_end <= candidate_start:
                continue
            mapped = queries[layer_index][:, head * groups:(head + 1) * groups]
            scores = temporal_head_scores(mapped, query_positions, layer.keys[start:end], positions[start:end],
                                          layer.values[start:end], candidate_start, candidate_end,
                                          gradients[layer_index][head * groups:(head + 1) * groups], base_margin,
                                          denominator_epsilon, query_chunk_size)
            count = candidate_end - candidate_start
            parts.append(scores)
            segments.append(ScoreSegment(layer_index, head, candidate_start, count))
            running += count
            ends.append(running)
    if not parts:
        raise RuntimeError("No eligible KV remains after prompt/recent protection")
    return ScoreTable(torch.cat(parts), segments, ends)


def head_logits(per_head_queries, keys, start: int, end: int, chunk: int):
    """bf16 logits [W, G, L] of one head, equal bit for bit to the logits the
    reference computes per query chunk with torch.matmul (scoring.py:184), as
    a view of rows padded to a 16-byte multiple where possible.

    cuBLAS accumulates each product in tensor-core steps of 16 terms for an
    even key count -- the GEMM over the 8-aligned key block, which cuBLAS runs
    about 5x faster, gives the same bits -- and of 8 terms for an odd one,
    which lrk_logits reproduces (k_step 8).  An odd key count outside
    lrk_logits' shapes takes the reference's own chunked GEMM."""
    import torch

    window, groups, dim = per_head_queries.shape
    length = end - start
    flat = per_head_queries.contiguous().view(window * groups, dim)
    if length % 2 == 0:
        aligned = _aligned_keys(keys, start, end)
        return torch.matmul(flat, aligned.transpose(0, 1)).view(window, groups, -1)[:, :, :length]
    if keys.dtype == torch.bfloat16 and dim in (64, 128):
        padded = operators().logits(flat, keys[start:end], 8, (length + 7) // 8 * 8)
        return padded.view(window, groups, -1)[:, :, :length]
    head_keys = keys[start:end]
    return torch.cat([torch.matmul(per_head_queries[a:a + chunk], head_keys.transpose(0, 1))
                      for a in range(0, window, chunk)])


def _aligned_keys(keys, start, end, multiple=8):
    """Keys of one head extended to a multiple of 8 rows.  cuBLAS runs the
    [W*G, D] x [D, L] logits GEMM about 5x faster when L is a multiple of 8
    (B200: 20 vs 110 us at L ~ 35k); the extra columns are never read.  The
    view reaches into the next head's rows, or is a zero-padded copy at the
    end of the layer."""
    import torch

    padded = -(-(end - start) // multiple) * multiple
    if start + padded <= keys.shape[0]:
        return keys[start:start + padded]
    return torch.cat([keys[start:end], keys.new_zeros(padded - (end - start), keys.shape[1])])


def query_chunk(query_chunk_size: int, groups: int, keys: int, element_size: int) -> int:
    """Queries per chunk of temporal_head_scores' running maximum
    (scoring.py:177-178): at most query_chunk_size, and at most 64 MiB of
    logits plus probabilities per chunk."""
    bytes_per_query = groups * keys * (element_size + 4)
    return min(query_chunk_size, max(1, (64 * 1024 ** 2) // bytes_per_query))


_STREAMS = {}


def _audit_streams(device):
    """Per device: a stream for the audit's GEMM work and a high-priority
    stream for its scoring (whose CTAs the block scheduler then takes first
    when both have work queued)."""
    import torch

    key = torch.device(device).index
    if key not in _STREAMS:
        highest = torch.cuda.Stream.priority_range()[1] if hasattr(torch.cuda.Stream, "priority_range") else -1
        _STREAMS[key] = (torch.cuda.Stream(device=device), torch.cuda.Stream(device=device, priority=highest))
    return _STREAMS[key]


def score_table_fused(cache, queries, query_positions, gradients, base_margin, protect_recent=32,
                      denominator_epsilon=1e-6, query_chunk_size=250) -> ScoreTable:
    """compute_score_table with the fused scorer.  Per layer: one
    lrk_project_values call (g V^T for every head, scoring.py:175, in the
    float32 GEMM's accumulation order), one bf16 Q K^T GEMM per head
    (scoring.py:184), then one lrk_temporal_scores call over all of the
    layer's heads -- the probabilities never reach HBM.  Each head keeps the
    composition's query chunks for its running maximum, so the scores are
    bit-identical to score_table (the temporal_probabilities + temporal_risk
    composition)."""
    import torch

    C = operators()
    device = cache.layers[0].keys.device
    margin = base_margin.to(device=device, dtype=torch.float32).reshape(1).contiguous()
    qpos = query_positions.to(dtype=torch.int64).contiguous()
    parts, segments, ends, running = [], [], [], 0
    # Layer l + 1's projection and logits GEMMs run on a side stream while
    # layer l is scored on a high-priority stream (at most one layer ahead);
    # the caller's stream waits for both at the end.
    main = torch.cuda.current_stream(device)
    side, scoring = _audit_streams(device)
    side.wait_stream(main)
    scoring.wait_stream(main)
    scored = []
    # Each layer's GEMM outputs stay referenced until the side stream has
    # queued its wait for that layer's scoring, so the caching allocator
    # reuses their blocks on the side stream only after the last read
    # (no record_stream, whose deferred frees make the pool grow).
    held = []
    for layer_index, layer in enumerate(cache.layers):
        heads = len(layer.head_lens)
        layer_queries = queries[layer_index]
        groups = layer_queries.shape[1] // heads
        scale = 1.0 / math.sqrt(layer.keys.shape[-1])
        bounds = layer.bounds()
        positions = layer.positions.reshape(-1)
        window, dim = layer_queries.shape[0], layer_queries.shape[-1]
        if layer_index >= 2:
            side.wait_event(scored[layer_index - 2])
            held.pop(0)
        heads_kept = []
        with torch.cuda.stream(side):
            projected = C.project_values(layer.values, gradients[layer_index].float().contiguous(), layer.cumulative,
                                         groups)
            # [heads, window * groups, D]: each head's queries one contiguous GEMM operand.
            per_head = layer_queries.to(layer.keys.dtype).reshape(window, heads, groups, dim).transpose(0, 1)
            per_head = per_head.contiguous()
            logits = []
            for head in range(heads):
                start, end = int(bounds[head]), int(bounds[head + 1])
                candidate_start = int(layer.prompt_lens[head])
                candidate_end = max(candidate_start, end - start - protect_recent)
                if candidate_end <= candidate_start:
                    continue
                chunk = query_chunk(query_chunk_size, groups, end - start, layer.keys.element_size())
                logits.append(head_logits(per_head[head], layer.keys, start, end, chunk))
                heads_kept.append((head, start, end, candidate_start, candidate_end, chunk))
            ready = torch.cuda.Event()
            ready.record(side)
        scoring.wait_event(ready)
        held.append((projected, per_head, logits))
        pvs, kpos, firsts, lasts, chunks = [], [], [], [], []
        for head, start, end, candidate_start, candidate_end, chunk in heads_kept:
            pvs.append(projected[:, start:end])
            kpos.append(positions[start:end])
            firsts.append(candidate_start)
            lasts.append(candidate_end)
            chunks.append(chunk)
            segments.append(ScoreSegment(layer_index, head, candidate_start, candidate_end - candidate_start))
            running += candidate_end - candidate_start
            ends.append(running)
        if logits:
            with torch.cuda.stream(scoring):
                part = C.temporal_scores(logits, pvs, kpos, firsts, lasts, qpos, margin, scale, denominator_epsilon,
                                         chunks)
            part.record_stream(main)
            parts.append(part)
        done = torch.cuda.Event()
        done.record(scoring)
        scored.append(done)
    main.wait_stream(side)
    main.wait_stream(scoring)
    # The next work on the side stream (the next call) waits for the caller's
    # stream, which now waits for every layer's scoring: releasing is safe.
    held.clear()
    if not parts:
        raise RuntimeError("No eligible KV remains after prompt/recent protection")
    return ScoreTable(torch.cat(parts), segments, ends)


def keys_scoring_supported(cache, queries) -> bool:
    """score_table_from_keys' shapes: bf16 keys and queries, head dimension
    64 or 128, at most 8 query heads per KV head, contiguous query blocks."""
    import torch

    layer = cache.layers[0]
    heads = len(layer.head_lens)
    first = queries[0]
    return (layer.keys.dtype == torch.bfloat16 and layer.keys.shape[-1] in (64, 128) and first.dim() == 3
            and first.shape[1] % heads == 0 and first.shape[1] // heads <= 8
            and all(q.dtype == torch.bfloat16 and q.is_contiguous() for q in queries))


def score_table_from_keys(cache, queries, query_positions, gradients, base_margin, protect_recent=32,
                          denominator_epsilon=1e-6, query_chunk_size=250) -> ScoreTable:
    """compute_score_table with the logits never written: one
    lrk_project_values call per layer (g V^T, scoring.py:175), then a single
    lrk_scores_from_keys call for every head of every layer, which runs the
    bf16 Q K^T GEMM (scoring.py:184, cuBLAS's step order for the head's key
    count) and the row statistics as one tensor-core kernel and writes only
    the candidate columns' logits for the risk step.  Bit-identical to
    score_table_fused and score_table."""
    import torch

    C = operators()
    device = cache.layers[0].keys.device
    margin = base_margin.to(device=device, dtype=torch.float32).reshape(1).contiguous()
    qpos = query_positions.to(dtype=torch.int64).contiguous()
    keys, layer_queries, projected, positions = [], [], [], []
    table, segments, ends, running = [], [], [], 0
    groups = None
    for layer_index, layer in enumerate(cache.layers):
        heads = len(layer.head_lens)
        groups = queries[layer_index].shape[1] // heads
        bounds = layer.bounds()
        keys.append(layer.keys)
        layer_queries.append(queries[layer_index])
        positions.append(layer.positions.reshape(-1))
        projected.append(C.project_values(layer.values, gradients[layer_index].float().contiguous(),
                                          layer.cumulative, groups))
        for head in range(heads):
            start, end = int(bounds[head]), int(bounds[head + 1])
            candidate_start = int(layer.prompt_lens[head])
            candidate_end = max(candidate_start, end - start - protect_recent)
            if candidate_end <= candidate_start:
                continue
            chunk = query_chunk(query_chunk_size, groups, end - start, layer.keys.element_size())
            table.append((layer_index, head, start, end - start, candidate_start, candidate_end, chunk))
            segments.append(ScoreSegment(layer_index, head, candidate_start, candidate_end - candidate_start))
            running += candidate_end - candidate_start
            ends.append(running)
    if not table:
        raise RuntimeError("No eligible KV remains after prompt/recent protection")
    scale = 1.0 / math.sqrt(cache.layers[0].keys.shape[-1])
    scores = C.scores_from_keys(keys, layer_queries, projected, positions, table, groups, qpos, margin, scale,
                                denominator_epsilon)
    return ScoreTable(scores, segments, ends)


def pool_table(table: ScoreTable, kernel_size: int = 7) -> ScoreTable:
    """pool_score_table (scoring.py:322-335)."""
    import torch

    bounds = upload(np.asarray([0] + list(table.cumulative_ends), dtype=np.int64), table.scores.device)
    pooled = operators().pool(table.scores.contiguous(), bounds, max(s.count for s in table.segments), kernel_size)
    return ScoreTable(pooled, list(table.segments), list(table.cumulative_ends))


@dataclass
class AuditResult:
    table: ScoreTable
    references: ArrayReferences
    changed: int
    changed_heads: int
    evicted: int


def audit_pass(cache, queries, query_positions, gradients, base_margin, immediate: int, queued: int,
               protect_recent=32, denominator_epsilon=1e-6, query_chunk_size=250, pool_kernel=7,
               fused=True, from_keys=False) -> AuditResult:
    """Score, pool, select immediate + queued references, evict the immediate
    prefix.  Returns the queue (references[immediate:] is the lazy queue).
    fused=False scores through the drop-in operators exactly as the reference
    composes them; fused=True uses lrk_scores_from_keys (from_keys, where the
    shapes allow) or lrk_temporal_scores.  All three give the same scores bit
    for bit."""
    if fused and from_keys and keys_scoring_supported(cache, queries):
        table = score_table_from_keys(cache, queries, query_positions, gradients, base_margin, protect_recent,
                                      denominator_epsilon, query_chunk_size)
    elif fused:
        table = score_table_fused(cache, queries, query_positions, gradients, base_margin, protect_recent,
                                  denominator_epsilon, query_chunk_size)
    else:
        table = score_table(cache, queries, query_positions, gradients, base_margin, protect_recent,
                            denominator_epsilon, query_chunk_size)
    pooled = pool_table(table, pool_kernel)
    # The segment table is built while the device is still scoring.
    segments = cache.segment_table([(segment.layer, segment.head) for segment in table.segments])
    queue = refine_device(table, pooled, immediate + queued)
    if queue.count < immediate:
        raise RuntimeError("Not enough unprotected candidates to enforce the budget")
    # The queue leaves the device before the compactions are queued and is
    # unpacked on the host while they run.
    pending = fetch_references(queue)
    evicted = 0
    if immediate:
        evicted = cache.remove_selected(queue.coordinates, queue.segment_ids[:immediate],
                                        queue.positions[:immediate], segments)
    references, changed, changed_heads = pending.result()
    return AuditResult(table, references, changed, changed_heads, evicted)


def evict_prefix(cache, queue: ArrayReferences, removed_at_audit: dict, count: int):
    """Lazy eviction (controller.py:57-70): pop `count` queued references,
    shifting their audit-time positions by the rows already removed from the
    same head since the audit.  Returns (remaining queue, updated removed map)."""
    removals, updates = {}, {}
    for segment, positions in queue[:count].groups().items():
        removed = np.asarray(removed_at_audit.get(segment, ()), dtype=np.int64)
        removals[segment] = positions - np.searchsorted(removed, positions)
        updates[segment] = np.union1d(removed, positions)
    cache.remove_positions(removals)
    removed_at_audit = dict(removed_at_audit)
    removed_at_audit.update(updates)
    return queue[count:], removed_at_audit
