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
        # As scoring.py:184: on the permuted query-history view
        # (reference_query_view) torch.matmul runs `chunk` batched
        # [G, D] x [D, L] products; a contiguous block would fold into one
        # [chunk*G, D] x [D, L] GEMM, which cuBLAS may order differently.
        logits = torch.matmul(queries[start:end].to(keys.dtype), keys.transpose(0, 1))
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
        spans = layer.spans()
        positions = layer.positions.reshape(-1)
        for head in range(heads):
            start, end = spans[head]
            candidate_start = int(layer.prompt_lens[head])
            candidate_end = max(candidate_start, end - start - protect_recent)
            if candidate_end <= candidate_start:
                continue
            mapped = reference_query_view(queries[layer_index][:, head * groups:(head + 1) * groups])
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


def reference_query_view(head_queries):
    """[W, G, D] queries of one KV head laid out as the reference's
    mapped_queries (scoring.py:260: query_history[0, q0:q1].permute(1, 0, 2)
    of a contiguous [1, heads * G, W, D] history, i.e. strides (D, W*D, 1)).
    torch.matmul cannot fold such a view into one matrix, so it runs the
    batched GEMM the reference runs: one [G, D] x [D, L] product per query.
    The [G, W, D] copy is always made: .contiguous() would skip it when torch
    already counts the permuted tensor as contiguous (one group: a size-1
    dimension's stride is not checked), and the view would then fold."""
    import torch

    window, groups, dim = head_queries.shape
    history = torch.empty((groups, window, dim), dtype=head_queries.dtype, device=head_queries.device)
    history.copy_(head_queries.permute(1, 0, 2))
    return history.permute(1, 0, 2)


# Queries per cuBLAS call (the batch of the reference's batched GEMM) at which
# torch.matmul took an order other than lrk_logits' for some odd key count in
# a sweep on B200 (every batch size 1 .. 250, odd key counts 1025 .. 65537):
# batch 1 everywhere; at 2 groups also scattered sizes, kept here as whole
# ranges; at 4 groups one isolated size (5, at 24,577 keys).
_ODD_ORDER_EXCEPTIONS = {
    2: frozenset([1, *range(12, 26), *range(178, 250)]),
    4: frozenset([1, 5]),
    8: frozenset([1, 2]),
}


def tensor_core_order_matches(length: int, window: int, groups: int, chunk: int) -> bool:
    """Whether the reference's logits GEMM for a head -- torch.matmul of
    reference_query_view(queries)[a:a + chunk] and the head's keys, one
    batched GEMM of [groups, D] x [D, length] products per query chunk
    (scoring.py:184) -- takes the tensor-core step order lrk_logits
    reproduces: 16 terms for an even key count, 8 for an odd one.  Measured on
    B200: with one query row per product (groups 1) cuBLAS runs other kernels
    at almost every odd count; with 2, 4 or 8 rows every even count matches,
    odd counts below 1024 keys often do not, and from 1024 keys on the odd
    counts match unless a call's batch is one of _ODD_ORDER_EXCEPTIONS.
    Group counts outside the sweep take the reference's GEMM for odd counts.
    The other heads take the reference's own GEMM."""
    if groups < 2:
        return False
    if length % 2 == 0:
        return True
    exceptions = _ODD_ORDER_EXCEPTIONS.get(groups)
    if exceptions is None or length < 1024:
        return False
    batches = {min(chunk, window - a) for a in range(0, window, chunk)}
    return not (batches & exceptions)


# Runtime check of the step-order rule: the first head of each (groups, key
# count parity, window, query chunk) class this process scores through
# lrk_logits is also computed by the reference's GEMM and compared bit for
# bit.  A class that differs (a cuBLAS whose heuristics moved) takes the
# reference's GEMM from then on, and that head's logits are replaced by the
# reference's.  (The key is cheap to form: the audit asks it for every head.)
_ORDER_VERIFIED = {}


def _order_class(length: int, window: int, groups: int, chunk: int):
    return groups, length % 2, window, chunk


def order_verified(length: int, window: int, groups: int, chunk: int) -> bool:
    """False once the class of this head failed the runtime check."""
    return _ORDER_VERIFIED.get(_order_class(length, window, groups, chunk), True)


def _reference_head_logits(per_head_queries, keys, start: int, end: int, chunk: int):
    import torch

    window = per_head_queries.shape[0]
    mapped = reference_query_view(per_head_queries)
    head_keys = keys[start:end]
    return torch.cat([torch.matmul(mapped[a:a + chunk].to(keys.dtype), head_keys.transpose(0, 1))
                      for a in range(0, window, chunk)])


def _check_order(per_head_queries, keys, start: int, end: int, chunk: int, logits):
    """The runtime check for one head computed by lrk_logits: returns the
    logits to use (the reference's when the class fails)."""
    import torch

    window, groups, _ = per_head_queries.shape
    key = _order_class(end - start, window, groups, chunk)
    if key in _ORDER_VERIFIED:
        return logits
    reference = _reference_head_logits(per_head_queries, keys, start, end, chunk)
    same = bool(torch.equal(reference.view(torch.int16), logits.contiguous().view(torch.int16)))
    _ORDER_VERIFIED[key] = same
    if not same:
        import warnings

        warnings.warn(f"lrk_logits' step order differs from this cuBLAS for groups={groups}, "
                      f"{'odd' if (end - start) % 2 else 'even'} key counts, window {window}, query chunk {chunk}: "
                      "those heads take the reference's GEMM")
        return reference
    return logits


def head_logits(per_head_queries, keys, start: int, end: int, chunk: int):
    """bf16 logits [W, G, L] of one head, equal bit for bit to the logits the
    reference computes per query chunk with torch.matmul (scoring.py:184), as
    a view of rows padded to a 16-byte multiple where lrk_logits computes
    them (tensor_core_order_matches); otherwise the reference's own chunked
    GEMM on reference_query_view."""
    import torch

    window, groups, dim = per_head_queries.shape
    length = end - start
    if (keys.dtype == torch.bfloat16 and per_head_queries.dtype == torch.bfloat16 and dim in (64, 128)
            and tensor_core_order_matches(length, window, groups, chunk)
            and order_verified(length, window, groups, chunk)):
        flat = per_head_queries.contiguous().view(window * groups, dim)
        padded = operators().logits(flat, keys[start:end], 8 if length % 2 else 16, (length + 7) // 8 * 8)
        return _check_order(per_head_queries, keys, start, end, chunk,
                            padded.view(window, groups, -1)[:, :, :length])
    return _reference_head_logits(per_head_queries, keys, start, end, chunk)


def layer_logits(per_head, keys, spans, window: int, groups: int, reference_stream=None):
    """bf16 logits [W, G, L] of several heads of one layer, each equal bit for
    bit to head_logits.  per_head: [heads, W * G, D] queries; spans: (head,
    start, end, chunk) per entry.  The heads whose order lrk_logits
    reproduces run in one lrk_logits_heads launch (both step orders, one pass
    over the GPU); the others take the reference's GEMM (head_logits), on
    reference_stream when given (the caller's stream, where the reference
    issues them)."""
    import torch

    dim = per_head.shape[-1]
    out = [None] * len(spans)
    fast, slow = [], []
    for i, (head, start, end, chunk) in enumerate(spans):
        if (keys.dtype == torch.bfloat16 and dim in (64, 128) and per_head.dtype == torch.bfloat16
                and tensor_core_order_matches(end - start, window, groups, chunk)
                and order_verified(end - start, window, groups, chunk)):
            fast.append(i)
        else:
            slow.append(i)
    if slow:
        current = torch.cuda.current_stream(per_head.device)
        stream = reference_stream if reference_stream is not None else current
        stream.wait_stream(current)
        with torch.cuda.stream(stream):
            for i in slow:
                head, start, end, chunk = spans[i]
                out[i] = head_logits(per_head[head].view(window, groups, dim), keys, start, end, chunk)
        current.wait_stream(stream)
    if fast:
        heads = [spans[i][0] for i in fast]
        starts = [spans[i][1] for i in fast]
        ends = [spans[i][2] for i in fast]
        steps = [8 if (e - b) % 2 else 16 for b, e in zip(starts, ends)]
        views = operators().logits_heads(per_head, keys, heads, starts, ends, steps, groups)
        for i, view, b, e in zip(fast, views, starts, ends):
            head, _, _, chunk = spans[i]
            out[i] = view  # [window, groups, e - b]
            if _order_class(e - b, window, groups, chunk) not in _ORDER_VERIFIED:
                out[i] = _check_order(per_head[head].view(window, groups, dim), keys, b, e, chunk, out[i])
    return out


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


def _head_pieces(spans, total: int):
    """Split sizes that cut [0, total) at every head's (start, end) -- heads
    ascending and disjoint, with or without gaps between them -- and each
    head's piece index."""
    pieces, at, cursor = [], [], 0
    for start, end in spans:
        if start > cursor:
            pieces.append(start - cursor)
        at.append(len(pieces))
        pieces.append(end - start)
        cursor = end
    if cursor < total:
        pieces.append(total - cursor)
    return pieces, at


def score_table_fused(cache, queries, query_positions, gradients, base_margin, protect_recent=32,
                      denominator_epsilon=1e-6, query_chunk_size=250) -> ScoreTable:
    """compute_score_table with the fused scorer.  Per layer: one
    lrk_project_values call (g V^T for every head, scoring.py:175, in the
    float32 GEMM's accumulation order), the bf16 Q K^T GEMMs of all heads
    (scoring.py:184) in one lrk_logits_heads launch (layer_logits), then one
    lrk_temporal_scores call over all of the
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
        spans = layer.spans()
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
            for head in range(heads):
                start, end = spans[head]
                candidate_start = int(layer.prompt_lens[head])
                candidate_end = max(candidate_start, end - start - protect_recent)
                if candidate_end <= candidate_start:
                    continue
                chunk = query_chunk(query_chunk_size, groups, end - start, layer.keys.element_size())
                heads_kept.append((head, start, end, candidate_start, candidate_end, chunk))
            logits = layer_logits(per_head.view(heads, window * groups, dim), layer.keys,
                                  [(h, b, e, c) for h, b, e, _, _, c in heads_kept], window, groups,
                                  reference_stream=main)
            ready = torch.cuda.Event()
            ready.record(side)
        scoring.wait_event(ready)
        held.append((projected, per_head, logits))
        pvs, kpos, firsts, lasts, chunks = [], [], [], [], []
        # Every head's projected values and positions as views, two calls per
        # layer (the pieces between heads of a gapped layout are split off too).
        pieces, at = _head_pieces(spans, positions.shape[0])
        pv_views, kpos_views = projected.split(pieces, dim=1), positions.split(pieces)
        for head, start, end, candidate_start, candidate_end, chunk in heads_kept:
            pvs.append(pv_views[at[head]])
            kpos.append(kpos_views[at[head]])
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
    the candidate columns' logits for the risk step.  Heads whose GEMM cuBLAS
    runs in another order (tensor_core_order_matches false) are scored as in
    score_table_fused instead.  Bit-identical to score_table_fused and
    score_table."""
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
        spans = layer.spans()
        keys.append(layer.keys)
        layer_queries.append(queries[layer_index])
        positions.append(layer.positions.reshape(-1))
        projected.append(C.project_values(layer.values, gradients[layer_index].float().contiguous(),
                                          layer.cumulative, groups))
        for head in range(heads):
            start, end = spans[head]
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
    window = qpos.shape[0]
    direct = [i for i, entry in enumerate(table) if tensor_core_order_matches(entry[3], window, groups, entry[6])]
    if len(direct) == len(table):
        scores = C.scores_from_keys(keys, layer_queries, projected, positions, table, groups, qpos, margin, scale,
                                    denominator_epsilon)
        return ScoreTable(scores, segments, ends)
    parts = [None] * len(table)
    if direct:
        scores = C.scores_from_keys(keys, layer_queries, projected, positions, [table[i] for i in direct], groups,
                                    qpos, margin, scale, denominator_epsilon)
        for i, part in zip(direct, torch.split(scores, [table[i][5] - table[i][4] for i in direct])):
            parts[i] = part
    for i in sorted(set(range(len(table))) - set(direct)):
        layer_index, head, start, length, first, last, chunk = table[i]
        head_queries = layer_queries[layer_index][:, head * groups:(head + 1) * groups]
        logits = head_logits(head_queries, keys[layer_index], start, start + length, chunk)
        parts[i] = C.temporal_scores([logits], [projected[layer_index][:, start:start + length]],
                                     [positions[layer_index][start:start + length]], [first], [last], qpos, margin,
                                     scale, denominator_epsilon, [chunk])
    return ScoreTable(torch.cat(parts), segments, ends)


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
    # For caches that evict lazy batches on the device (arena.ArenaCache):
    # every queue slot's (flat head, logical position), taken before the
    # immediate eviction.
    lazy: tuple = None


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
    lazy = None
    if hasattr(cache, "queue_positions") and queue.count:
        lazy = cache.queue_positions(segments, queue.segment_ids, queue.positions)
    evicted = 0
    if immediate:
        evicted = cache.remove_selected(queue.coordinates, queue.segment_ids[:immediate],
                                        queue.positions[:immediate], segments)
    references, changed, changed_heads = pending.result()
    return AuditResult(table, references, changed, changed_heads, evicted, lazy)


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
