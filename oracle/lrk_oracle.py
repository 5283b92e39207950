"""numpy restatement of the LazyRecall KV-management operators (test oracle).

TEST INFRASTRUCTURE ONLY -- see oracle/__init__.py.  Each function names the
reference code it restates (paths inside the reference project).  bf16 and
fp16 data travel as uint16 / float16 arrays; positions are float32; indices
int64.  Byte-moving operators are exact.  Scoring operators follow the
reference CUDA kernels' operation order (including the 256-lane reduction
order and the rounding of scaled logits to the logits dtype); numpy's float32
exp/log can differ from CUDA's by an ulp, so their outputs are compared with a
relative tolerance, never bit for bit.
"""
from __future__ import annotations

import numpy as np

LANES = 256
BITONIC_MAX = 32

# --------------------------------------------------------------- dtypes


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit pattern (NaN -> canonical NaN)."""
    x = np.asarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    bias = 0x7FFF + ((bits >> 16) & 1)
    rounded = ((bits + bias) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), rounded)


def to_f32(array: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_to_f32(array)
    return np.asarray(array).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> dtype -> float32 (the reference's static_cast round trip)."""
    if dtype == "bf16":
        return bf16_to_f32(f32_to_bf16(x))
    if dtype == "f16":
        return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(x, np.float32)


# ------------------------------------------------------------ reductions


def lane_sum(values: np.ndarray) -> np.ndarray:
    """Sum over the last axis in the reference's order: 256 lanes each add
    elements lane, lane+256, ... sequentially from 0.0f, then a pairwise tree
    partial[t] += partial[t+s] for s = 128 .. 1 (csrc/scoring.cu:15-30, :51-64)."""
    values = np.asarray(values, dtype=np.float32)
    length = values.shape[-1]
    rounds = -(-length // LANES)
    padded = np.zeros(values.shape[:-1] + (rounds * LANES,), dtype=np.float32)
    padded[..., :length] = values
    blocks = padded.reshape(values.shape[:-1] + (rounds, LANES))
    acc = np.zeros(values.shape[:-1] + (LANES,), dtype=np.float32)
    for r in range(rounds):
        acc = (acc + blocks[..., r, :]).astype(np.float32)
    stride = LANES // 2
    while stride:
        acc[..., :stride] = acc[..., :stride] + acc[..., stride:2 * stride]
        stride //= 2
    return acc[..., 0].copy()


# --------------------------------------------------------------- scoring


def temporal_probabilities(logits, logits_dtype, projected_values, query_positions, key_positions, scale):
    """_C.temporal_probabilities -- csrc/scoring.cu:32-66, host :205-233.

    Per (query, group) row: x = dtype(float(logit) * scale); x = -inf where
    key_position > query_position; softmax by max, exp, 256-lane sum, divide;
    output_projection = 256-lane sum of p * projected_values[group]."""
    x = to_f32(logits, logits_dtype)
    window, groups, length = x.shape
    scaled = round_to((x * np.float32(scale)).astype(np.float32), logits_dtype)
    qpos = np.asarray(query_positions, dtype=np.int64).astype(np.float32)
    kpos = np.asarray(key_positions, dtype=np.float32)
    mask = kpos[None, None, :] <= qpos[:, None, None]
    value = np.where(mask, scaled, np.float32(-np.inf)).astype(np.float32)
    maximum = np.fmax.reduce(value, axis=-1)
    with np.errstate(invalid="ignore", over="ignore"):
        weights = np.exp((value - maximum[..., None]).astype(np.float32)).astype(np.float32)
        denominator = lane_sum(weights)
        probabilities = (weights / denominator[..., None]).astype(np.float32)
        products = (probabilities * np.asarray(projected_values, np.float32)[None, :, :]).astype(np.float32)
    return probabilities, lane_sum(products)


def _softplus64(value):
    value = np.asarray(value, dtype=np.float64)
    with np.errstate(over="ignore"):
        return np.where(value > 20.0, value, np.log1p(np.exp(np.minimum(value, 20.0))))


def _risk64(margin: float, probability: float, base_softplus: float, drop):
    """csrc/scoring.cu:68-75 (and scoring.py:61-72): KL of the Bernoulli
    decision before/after a margin drop, clamped at 0, in float64."""
    compared = margin - np.asarray(drop, dtype=np.float32).astype(np.float64)
    kl = (probability * (margin - compared) - base_softplus) + _softplus64(compared)
    return np.fmax(0.0, kl)


def temporal_risk(probabilities, output_projection, projected_values, margin, first, last, epsilon):
    """_C.temporal_risk -- csrc/scoring.cu:77-128, host :235-255.

    drop[q, c] = sum over g, in order, of p/max(1-p, eps) * (pv[g,c] - op[q,g]);
    any non-finite drop makes the candidate NaN; otherwise
    risk = max(R(min_q drop), R(max_q drop))."""
    p = np.asarray(probabilities, np.float32)[:, :, first:last]
    op = np.asarray(output_projection, np.float32).reshape(p.shape[0], p.shape[1])
    pv = np.asarray(projected_values, np.float32).reshape(p.shape[1], -1)[:, first:last]
    eps = np.float32(epsilon)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        ratio = (p / np.fmax(np.float32(1.0) - p, eps)).astype(np.float32)
        drop = np.zeros((p.shape[0], p.shape[2]), dtype=np.float32)
        for g in range(p.shape[1]):
            drop = (drop + (ratio[:, g, :] * (pv[g][None, :] - op[:, g][:, None]).astype(np.float32))).astype(
                np.float32)
    bad = ~np.isfinite(drop).all(axis=0)
    safe = np.where(np.isfinite(drop), drop, np.float32(0))
    m = float(np.float32(np.asarray(margin).reshape(-1)[0]))
    probability = 1.0 / (1.0 + np.exp(-m))
    base = float(_softplus64(m))
    risk = np.fmax(_risk64(m, probability, base, safe.min(axis=0)), _risk64(m, probability, base, safe.max(axis=0)))
    return np.where(bad, np.float32(np.nan), risk.astype(np.float32)).astype(np.float32)


def temporal_head_scores_gpu_path(queries, query_positions, keys, key_positions, values, candidate_start,
                                  candidate_end, margin_gradient, base_margin, denominator_epsilon,
                                  query_chunk_size, kv_dtype="bf16"):
    """The GPU branch of temporal_head_scores (scoring.py:152-195): pv = g V^T,
    chunked logits = Q K^T in the KV dtype, then temporal_probabilities and
    temporal_risk per chunk, combined by maximum.  keys/values/queries are
    float32 arrays of values already representable in kv_dtype."""
    keys = np.asarray(keys, np.float32)
    values = np.asarray(values, np.float32)
    queries = np.asarray(queries, np.float32)
    groups = queries.shape[1]
    pv = (np.asarray(margin_gradient, np.float32) @ values.T).astype(np.float32)
    bytes_per_query = groups * keys.shape[0] * (2 + 4)
    chunk = min(query_chunk_size, max(1, (64 * 1024 ** 2) // bytes_per_query))
    scale = np.float32(1.0 / np.sqrt(keys.shape[-1]))
    result = None
    for start in range(0, queries.shape[0], chunk):
        end = min(start + chunk, queries.shape[0])
        q = round_to(queries[start:end], kv_dtype)
        # Q K^T comes out of the GEMM in the KV dtype; the kernel then rounds
        # logit * scale to that dtype again.
        logits = round_to((q.reshape(-1, q.shape[-1]) @ keys.T).reshape(q.shape[0], q.shape[1], -1), kv_dtype)
        stored = f32_to_bf16(logits) if kv_dtype == "bf16" else logits
        probs, op = temporal_probabilities(stored, kv_dtype, pv, query_positions[start:end], key_positions, scale)
        scores = temporal_risk(probs, op, pv, np.float32(base_margin), candidate_start, candidate_end,
                               denominator_epsilon)
        result = scores if result is None else np.fmax(result, scores)
    return result


def temporal_head_scores_cpu_path(queries, query_positions, keys, key_positions, values, candidate_start,
                                  candidate_end, margin_gradient, base_margin, denominator_epsilon,
                                  query_chunk_size, kv_dtype="bf16"):
    """temporal_head_scores_reference (scoring.py:75-149), the reference's CPU
    math path: logits = (Q K^T) / sqrt(D) in the KV dtype, causal mask,
    float32 softmax, output_gradient = P @ (g V^T), local margin drop per
    candidate summed over groups, min/max over queries, float64 risk."""
    keys = np.asarray(keys, np.float32)
    values = np.asarray(values, np.float32)
    queries = np.asarray(queries, np.float32)
    pv = (np.asarray(margin_gradient, np.float32) @ values.T).astype(np.float32)
    vg = pv[:, candidate_start:candidate_end]
    count = candidate_end - candidate_start
    minimum = np.full(count, np.inf, np.float32)
    maximum = np.full(count, -np.inf, np.float32)
    kpos = np.asarray(key_positions, np.float32)
    qpos_all = np.asarray(query_positions)
    sqrt_d = np.float32(np.sqrt(keys.shape[-1]))
    for start in range(0, queries.shape[0], query_chunk_size):
        end = min(start + query_chunk_size, queries.shape[0])
        q = round_to(queries[start:end], kv_dtype)
        logits = round_to((q.reshape(-1, q.shape[-1]) @ keys.T).reshape(q.shape[0], q.shape[1], -1), kv_dtype)
        logits = round_to((logits / sqrt_d).astype(np.float32), kv_dtype)
        causal = kpos[None, None, :] <= qpos_all[start:end].reshape(-1, 1, 1)
        logits = np.where(causal, logits, np.float32(-np.inf))
        shifted = logits - logits.max(axis=-1, keepdims=True)
        weights = np.exp(shifted).astype(np.float32)
        probs = (weights / weights.sum(axis=-1, keepdims=True)).astype(np.float32)
        og = (probs * pv[None]).sum(axis=-1, dtype=np.float32)
        cand = probs[:, :, candidate_start:candidate_end]
        ratio = cand / np.maximum(np.float32(1.0) - cand, np.float32(denominator_epsilon))
        drop = (ratio * (vg[None] - og[..., None])).sum(axis=1).astype(np.float32)
        minimum = np.minimum(minimum, drop.min(axis=0))
        maximum = np.maximum(maximum, drop.max(axis=0))
    m = float(np.asarray(base_margin, np.float64).reshape(-1)[0])
    probability = 1.0 / (1.0 + np.exp(-m))
    base = float(_softplus64(m))
    return np.maximum(_risk64(m, probability, base, minimum), _risk64(m, probability, base, maximum)).astype(
        np.float32)


def pool(scores, bounds, width):
    """_C.pool -- csrc/scoring.cu:190-203 (CPU twin: F.max_pool1d per segment,
    scoring.py:336-353): out[i] = max over [i - w/2, i + w/2] within i's
    segment, NaN-ignoring like fmaxf.  Positions outside every segment are
    left as NaN here (the operator leaves them unwritten)."""
    scores = np.asarray(scores, np.float32)
    out = np.full_like(scores, np.nan)
    half = width // 2
    bounds = np.asarray(bounds, np.int64)
    for s in range(len(bounds) - 1):
        begin, end = int(bounds[s]), int(bounds[s + 1])
        if end <= begin:
            continue
        segment = scores[begin:end]
        padded = np.concatenate([np.full(half, -np.inf, np.float32), segment, np.full(half, -np.inf, np.float32)])
        acc = np.full(end - begin, -np.inf, np.float32)
        for offset in range(width):
            acc = np.fmax(acc, padded[offset:offset + end - begin])
        out[begin:end] = acc
    return out


def decision_risk(probabilities, values, values_dtype, head_outputs, gradients, base_margin, epsilon):
    """_legacy_C.decision_risk_scores -- csrc/cache_legacy.cu:81-135 (CPU twin
    decision_risk_scores_pytorch, _core/cuda_ops.py:228-273).  Per candidate:
    256-lane sum over (group, channel) of g * (a / max(1-a, eps)) * (v - o),
    then a clamped Bernoulli KL in float64 with stable sigmoid/softplus."""
    probabilities = np.asarray(probabilities, np.float32)
    groups, candidates = probabilities.shape
    v = to_f32(values, values_dtype).reshape(candidates, -1)
    dimension = v.shape[1]
    eps = np.float32(epsilon)
    with np.errstate(invalid="ignore", divide="ignore"):
        alpha = probabilities[:, :, None]  # [G, C, 1]
        denominator = np.fmax(np.float32(1.0) - alpha, eps)
        delta = ((alpha / denominator).astype(np.float32)
                 * (v[None, :, :] - np.asarray(head_outputs, np.float32)[:, None, :]).astype(np.float32))
        terms = (np.asarray(gradients, np.float32)[:, None, :] * delta.astype(np.float32)).astype(np.float32)
    # term index = group * D + channel, per candidate
    terms = np.transpose(terms, (1, 0, 2)).reshape(candidates, groups * dimension)
    total = lane_sum(terms).astype(np.float64)
    m = float(base_margin)
    compared = m - total
    probability = 1.0 / (1.0 + np.exp(-m)) if m >= 0 else np.exp(m) / (1.0 + np.exp(m))

    def stable_softplus(x):
        x = np.asarray(x, np.float64)
        with np.errstate(over="ignore"):
            return np.where(x > 20.0, x + np.log1p(np.exp(-np.abs(x))), np.log1p(np.exp(np.minimum(x, 20.0))))

    kl = (probability * (m - compared) - stable_softplus(m)) + stable_softplus(compared)
    return np.where(kl < 0.0, 0.0, kl).astype(np.float32)


# ----------------------------------------------------------- data movement


def append(keys, values, positions, new_keys, new_values, cumulative, logical_start):
    """_C.append -- csrc/scoring.cu:130-162, host :264-292.  new_* [1, H, A, D];
    returns (keys, values, positions [R', 1], cumulative, lengths)."""
    cumulative = np.asarray(cumulative, np.int64)
    heads, added = new_keys.shape[1], new_keys.shape[2]
    positions = np.asarray(positions, np.float32).reshape(-1)
    k_parts, v_parts, p_parts = [], [], []
    for h in range(heads):
        a, b = int(cumulative[h]), int(cumulative[h + 1])
        k_parts += [keys[a:b], new_keys[0, h]]
        v_parts += [values[a:b], new_values[0, h]]
        p_parts += [positions[a:b], (np.int64(logical_start) + np.arange(added, dtype=np.int64)).astype(np.float32)]
    out_cumulative = (cumulative + np.arange(heads + 1, dtype=np.int64) * added).astype(np.int32)
    lengths = (np.diff(cumulative) + added).astype(np.int32)
    return (np.concatenate(k_parts), np.concatenate(v_parts), np.concatenate(p_parts).reshape(-1, 1),
            out_cumulative, lengths)


def compact(keys, values, positions, removed):
    """_C.compact -- csrc/scoring.cu:164-188 (CPU twin index_select,
    cache.py:162-167): drop the sorted, unique removed rows."""
    removed = np.asarray(removed, np.int64)
    keep = np.setdiff1d(np.arange(keys.shape[0]), removed, assume_unique=False)
    positions = np.asarray(positions, np.float32).reshape(-1)
    return keys[keep], values[keep], positions[keep].reshape(-1, 1)


def merge(keys, values, positions, recalled, recalled_positions, mapping):
    """_C.merge -- csrc/recall.cu:7-28 (CPU twin cache.py:240-245)."""
    mapping = np.asarray(mapping, np.int64)
    positions = np.asarray(positions, np.float32).reshape(-1)
    recalled_positions = np.asarray(recalled_positions, np.float32).reshape(-1)
    k = np.empty((len(mapping),) + keys.shape[1:], keys.dtype)
    v = np.empty_like(k)
    p = np.empty(len(mapping), np.float32)
    existing = mapping >= 0
    k[existing], v[existing], p[existing] = keys[mapping[existing]], values[mapping[existing]], \
        positions[mapping[existing]]
    rows = -mapping[~existing] - 1
    k[~existing], v[~existing], p[~existing] = recalled[rows, 0], recalled[rows, 1], recalled_positions[rows]
    return k, v, p.reshape(-1, 1)


def pack(keys, values, positions, indices, heads, layer):
    """_C.pack -- csrc/recall.cu:30-47: payload [N, 2, D] and metadata
    [N, 3] = (layer, head, int64(position)) (float -> int truncation)."""
    indices = np.asarray(indices, np.int64)
    positions = np.asarray(positions, np.float32).reshape(-1)
    payload = np.stack([keys[indices], values[indices]], axis=1)
    metadata = np.stack([np.full(len(indices), layer, np.int64), np.asarray(heads, np.int64),
                         np.trunc(positions[indices]).astype(np.int64)], axis=1)
    return payload, metadata


def batch_append(keys_list, values_list, positions_list, new_keys, new_values, lengths, logical):
    """_C.batch_append -- csrc/batch_append.cu:8-94 (CPU twin append_reference,
    batch_attention.py:30-38): request-major, head-minor; each head = its old
    rows then the new token at position float(logical[request])."""
    k_parts, v_parts, p_parts = [], [], []
    for r, (k, v, p) in enumerate(zip(keys_list, values_list, positions_list)):
        p = np.asarray(p, np.float32).reshape(-1)
        source = 0
        for h, length in enumerate(lengths[r]):
            k_parts += [k[source:source + length], np.asarray(new_keys[r, h]).reshape(1, -1)]
            v_parts += [v[source:source + length], np.asarray(new_values[r, h]).reshape(1, -1)]
            p_parts += [p[source:source + length], np.asarray([logical[r]], np.float32)]
            source += length
    return np.concatenate(k_parts), np.concatenate(v_parts), np.concatenate(p_parts).reshape(-1, 1)


def append_flattened(cache, states, head_lens, cu_head_lens):
    """_legacy_C.append_flattened_cache -- csrc/cache_legacy.cu:13-40 (CPU twin
    append_flattened_cache_pytorch, _core/cuda_ops.py:38-62)."""
    b, h, n, d = states.shape
    parts = []
    for flat in range(b * h):
        start, length = int(cu_head_lens[flat]), int(head_lens[flat])
        parts += [cache[start:start + length], states[flat // h, flat % h]]
    return np.concatenate(parts).reshape(-1, d)


def compact_flattened(keys, values, keep):
    """_legacy_C.compact_flattened_kv -- csrc/cache_legacy.cu:42-61."""
    keep = np.asarray(keep, np.int64)
    return keys[keep], values[keep]


# -------------------------------------------------------------- selection


def radix_key(x) -> np.ndarray:
    """PyTorch's order-preserving float32 -> uint32 map used by its CUDA radix
    select (TopKTypeConfig<float>::convert); NaN -> 0xffffffff."""
    x = np.asarray(x, np.float32)
    bits = x.view(np.uint32)
    mask = np.where(bits & np.uint32(0x80000000), np.uint32(0xFFFFFFFF), np.uint32(0x80000000))
    return np.where(np.isnan(x), np.uint32(0xFFFFFFFF), bits ^ mask).astype(np.uint32)


def _nan_last_less(a: float, b: float) -> bool:
    return (np.isnan(b) and not np.isnan(a)) or bool(a < b)


def bitonic_order(keys, values):
    """PyTorch's 16-thread, 32-slot bitonic key/value network (SortUtils.cuh
    bitonicSortKVInPlace / bitonicSort with LTOp<float, true>) applied to at
    most 32 entries; unused slots are invalid and sort to the end."""
    n = len(keys)
    k = [float(x) for x in keys] + [0.0] * (BITONIC_MAX - n)
    v = list(values) + [0] * (BITONIC_MAX - n)
    valid = [True] * n + [False] * (BITONIC_MAX - n)

    def swap_step(pos, stride, direction):
        a, b = pos, pos + stride
        swap = (_nan_last_less(k[a], k[b]) and valid[a]) or not valid[b]
        if swap == direction:
            k[a], k[b] = k[b], k[a]
            v[a], v[b] = v[b], v[a]
            valid[a], valid[b] = valid[b], valid[a]

    size = 2
    while size < BITONIC_MAX:
        stride = size // 2
        while stride > 0:
            for t in range(BITONIC_MAX // 2):
                swap_step(2 * t - (t & (stride - 1)), stride, (t & (size // 2)) != 0)
            stride //= 2
        size *= 2
    stride = BITONIC_MAX // 2
    while stride > 0:
        for t in range(BITONIC_MAX // 2):
            swap_step(2 * t - (t & (stride - 1)), stride, False)
        stride //= 2
    return np.asarray(v[:n], dtype=np.int64)


def topk_smallest(x, k):
    """torch.topk(x, k, largest=False, sorted=True) for a 1-D float32 CUDA
    slice (PyTorch 2.11.0, pinned by the reference's pyproject.toml:10 and
    environment.txt:1; used at selection.py:69 and :77).

    Chosen set: the k smallest by (radix key, index).  Order: (radix key,
    index), except for 2 <= k <= 32, where the gathered order (below-kth keys
    by index, then kth-key ties by index) goes through the bitonic network --
    at every slice length (measured against torch 2.11 on B200).
    Returns (values, indices)."""
    x = np.asarray(x, np.float32)
    if k == 0:
        return x[:0].copy(), np.zeros(0, np.int64)
    keys = radix_key(x)
    order = np.lexsort((np.arange(len(x)), keys))[:k]
    if 2 <= k <= BITONIC_MAX:
        kth = keys[order[-1]]
        below = np.sort(order[keys[order] < kth])
        ties = np.sort(order[keys[order] == kth])
        gathered = np.concatenate([below, ties])
        order = gathered[bitonic_order(x[gathered], np.arange(len(gathered)))]
    return x[order], order.astype(np.int64)


def transplant(segment_ids, local_positions):
    """selection.py:42-49: each head's sorted local picks fill that head's slots
    in global order (stable argsort by segment)."""
    order = np.argsort(np.asarray(segment_ids), kind="stable")
    result = np.empty(len(segment_ids), dtype=np.int64)
    result[order] = local_positions
    return result


def refine(raw, pooled, ends, position_starts, count, topk=None):
    """refine_arrays -- selection.py:52-88, numeric part: global bottom-count of
    raw scores, quotas per segment, each segment's bottom-quota of pooled
    scores, transplant, and the changed-identity statistics.  ``topk(x, k)``
    returns (values, indices) of the k smallest (default: topk_smallest, the
    restatement of torch.topk on CUDA).
    Returns (values, segment_ids, positions, changed, changed_heads)."""
    topk = topk or topk_smallest
    raw = np.asarray(raw, np.float32)
    pooled = np.asarray(pooled, np.float32)
    ends = np.asarray(ends, np.int64)
    starts = np.concatenate(([0], ends[:-1]))
    count = min(max(0, int(count)), raw.size)
    if not count:
        return raw[:0].copy(), np.zeros(0, np.int64), np.zeros(0, np.int64), 0, 0
    values, indices = topk(raw, count)
    segment_ids = np.searchsorted(ends, indices, side="right")
    quotas = np.bincount(segment_ids, minlength=len(ends))
    selected, selected_segments = [], []
    for s, (start, end, quota) in enumerate(zip(starts, ends, quotas)):
        if quota:
            selected.append(np.asarray(topk(pooled[start:end], int(quota))[1], np.int64))
            selected_segments += [s] * int(quota)
    selected_local = np.concatenate(selected)
    selected_segments = np.asarray(selected_segments, np.int64)
    positions = transplant(segment_ids, selected_local + np.asarray(position_starts, np.int64)[selected_segments])
    refined_global = selected_local + starts[selected_segments]
    changed = ~np.isin(refined_global, indices, assume_unique=True)
    return (values, segment_ids.astype(np.int64), positions, int(changed.sum()),
            int(np.unique(selected_segments[changed]).size))


# ------------------------------------------------------------ recall planning


def merge_plan(old_positions, head_lengths, recalled_metadata):
    """recall/planning.py:34-52: per head, the stable chronological merge of
    existing positions and recalled ones; mapping >= 0 is an old row,
    -j-1 the j-th recalled row."""
    old_positions = np.asarray(old_positions, np.int64).reshape(-1)
    recalled_metadata = np.asarray(recalled_metadata, np.int64).reshape(-1, 3)
    mapping, lengths, start = [], [], 0
    for head, length in enumerate(head_lengths):
        existing = old_positions[start:start + length]
        chosen = np.flatnonzero(recalled_metadata[:, 1] == head)
        combined = np.concatenate((existing, recalled_metadata[chosen, 2]))
        if len(np.unique(combined)) != len(combined):
            raise ValueError("Cannot merge duplicate physical KV identities")
        sources = np.concatenate((np.arange(start, start + length), -chosen - 1))
        mapping.extend(sources[np.argsort(combined, kind="stable")])
        lengths.append(len(combined))
        start += length
    return np.asarray(mapping, np.int64), lengths
