"""Layer-group sharding of one request's eviction selection across ranks.

When one request's cache is split by layers over several GPUs (each rank
scores and compacts its own contiguous group of layers), the selection of
refine_arrays (selection.py:52-88) still needs the request-wide bottom-`count`
of raw scores.  The only data that crosses ranks is a few histograms:

  1. Each rank maps its scores to order-preserving 32-bit keys (the map
     PyTorch's radix select uses; NaN last).
  2. Radix rounds of 12, 12 and 8 bits: every rank histograms the digit of
     the keys still in play (lrk_select_histogram), the histograms are
     all-gathered (one NCCL all-gather per round over NVLink), and every rank
     sums them and fixes the bin holding the k-th key (lrk_select_pick).  The
     search state stays on the device from round to round; one copy of the
     final shares comes back to the host.
  3. Ties at the k-th key are taken in global flat-index order (layer-major,
     the order compute_score_table concatenates heads in, scoring.py:218-287),
     which is torch.topk's choice: ranks own increasing index ranges, and the
     last round's gathered histograms hold every rank's tie count, so each
     rank takes the first ties it holds after the ties of lower ranks with no
     further exchange.

A rank's share of the request-wide set is exactly its local bottom-(share) by
(key, index), so a local refine_arrays with that count gives the single-GPU
quotas, refined positions and queue order for its layers.  Queue prefixes
(the immediate eviction) are smaller "k smallest" questions over the same
keys and run in the same rounds.  Many requests go through one set of rounds.

On CPU tensors (gloo process groups, the multi-process tests) the same rounds
run as torch operations (_histogram_host, _pick_host): a restatement of the
two kernels, so the state machine is exercised without a GPU.
"""
from __future__ import annotations

from typing import Sequence

import torch
import torch.distributed as dist

DIGITS = (12, 12, 8)
BINS = 4096
# State fields (LRK_SELECT_* in include/lrk.h).
K, PREFIX, NEED, BELOW, LOCAL_BELOW, TOTAL, SHARE = range(7)
FIELDS = 8


def radix_keys(scores: torch.Tensor) -> torch.Tensor:
    """Order-preserving uint32 image of float32 scores, held in int64."""
    bits = scores.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    negative = (bits & 0x80000000) != 0
    keys = torch.where(negative, bits ^ 0xFFFFFFFF, bits ^ 0x80000000)
    return torch.where(torch.isnan(scores), torch.full_like(keys, 0xFFFFFFFF), keys)


def _all_gather_counts(local: torch.Tensor, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    gathered = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(gathered, local, group=group)
    return torch.stack(gathered)


def _histogram_host(tables: Sequence[torch.Tensor], states: torch.Tensor, round_index: int) -> torch.Tensor:
    """lrk_select_histogram restated in torch (CPU tensors): per (request,
    question) the histogram of this round's digit over the keys whose higher
    bits equal the question's prefix (all keys in round 0)."""
    requests, questions = states.shape[:2]
    shift = 32 - sum(DIGITS[:round_index + 1])
    width = DIGITS[round_index]
    out = torch.zeros(requests, questions, BINS, dtype=torch.int32)
    for r, scores in enumerate(tables):
        keys = radix_keys(scores)
        digit = (keys >> shift) & ((1 << width) - 1)
        for q in range(questions):
            if round_index == 0:
                picked = digit
            elif int(states[r, q, NEED]) > 0:
                picked = digit[(keys >> (shift + width)) == int(states[r, q, PREFIX])]
            else:
                continue
            out[r, q] = torch.bincount(picked, minlength=BINS).to(torch.int32)
    return out


def _pick_host(gathered: torch.Tensor, rank: int, states: torch.Tensor, round_index: int) -> None:
    """lrk_select_pick restated in torch (CPU tensors), in place on states."""
    requests, questions = states.shape[:2]
    width = DIGITS[round_index]
    for r in range(requests):
        for q in range(questions):
            state = states[r, q]
            counts = gathered[:, r, q, :1 << width].to(torch.int64)  # [world, bins]
            total = counts.sum(0)
            if round_index == 0:
                state[TOTAL] = int(total.sum())
                state[NEED] = max(0, min(int(state[K]), int(state[TOTAL])))
            need = int(state[NEED])
            if need <= 0:
                if round_index == len(DIGITS) - 1 and need == 0:
                    state[SHARE] = 0
                continue
            cumulative = total.cumsum(0)
            bin_index = int(torch.searchsorted(cumulative, torch.tensor([need])).item())
            if bin_index >= total.numel():
                state[NEED] = -1
                state[SHARE] = -1
                continue
            before = int(cumulative[bin_index] - total[bin_index])
            state[PREFIX] = (int(state[PREFIX]) << width) | bin_index
            state[BELOW] += before
            state[LOCAL_BELOW] += int(counts[rank, :bin_index].sum())
            state[NEED] = need - before
            if round_index == len(DIGITS) - 1:
                ties = counts[:, bin_index]
                take = max(0, min(need - before - int(ties[:rank].sum()), int(ties[rank])))
                state[SHARE] = int(state[LOCAL_BELOW]) + take


def select_shares(tables: Sequence[torch.Tensor], ks: Sequence[Sequence[int]], group=None, timings=None):
    """This rank's share of each request's request-wide k smallest scores.

    tables[r]: this rank's score table of request r (1-D float32; ranks hold
    consecutive layer groups in rank order); ks[r]: the k of each question for
    request r (the same number of questions for every request).  Returns
    (shares [requests, questions], totals [requests]) as numpy int64: the
    count of this rank's rows in each request-wide bottom-k by (key, global
    index), and each request's request-wide score count (k larger than it is
    clamped).  Every rank calls this with the same ks.  On CUDA tensors: three
    rounds of lrk_select_histogram, one NCCL all-gather and lrk_select_pick,
    with one device-to-host copy at the end; `timings`, a list, receives a
    (start, end) CUDA event pair around each all-gather."""
    import numpy as np

    requests = len(tables)
    questions = len(ks[0]) if requests else 0
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if not requests:
        return np.zeros((0, questions), np.int64), np.zeros(0, np.int64)
    host_states = torch.zeros(requests, questions, FIELDS, dtype=torch.int64)
    host_states[:, :, K] = torch.as_tensor(np.asarray(ks, dtype=np.int64).reshape(requests, questions))
    device = tables[0].device
    if device.type == "cuda":
        from . import operators, upload

        C = operators()
        states = upload(host_states.numpy(), device)
        gathered = torch.empty(world, requests, questions, BINS, dtype=torch.int32, device=device)
        tables = [t.float().contiguous() for t in tables]
        for round_index in range(len(DIGITS)):
            histograms = C.select_histogram(tables, states, round_index)
            if timings is not None:
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
            dist.all_gather_into_tensor(gathered, histograms, group=group)
            if timings is not None:
                end.record()
                timings.append((start, end))
            C.select_pick(gathered, rank, states, round_index)
        final = states[:, :, [SHARE, TOTAL]].cpu().numpy()
    else:
        states = host_states
        for round_index in range(len(DIGITS)):
            histograms = _histogram_host(tables, states, round_index)
            gathered = _all_gather_counts(histograms, group)
            _pick_host(gathered, rank, states, round_index)
        final = states[:, :, [SHARE, TOTAL]].numpy()
    shares = final[:, :, 0].astype(np.int64)
    if (shares < 0).any():
        raise RuntimeError("layer-group selection: the ranks' histograms disagree (inconsistent score tables)")
    return shares, final[:, 0, 1].astype(np.int64)


def local_smallest(scores: torch.Tensor, count: int) -> torch.Tensor:
    """Mask of the `count` smallest local scores by (key, index)."""
    mask = torch.zeros(scores.numel(), dtype=torch.bool, device=scores.device)
    if count > 0:
        keys = radix_keys(scores)
        index = torch.arange(scores.numel(), device=scores.device)
        order = torch.argsort(keys * (scores.numel() + 1) + index, stable=True)
        mask[order[:count]] = True
    return mask


def select_smallest(scores: torch.Tensor, k: int, group=None) -> torch.Tensor:
    """Boolean mask of this rank's share of the request-wide k smallest
    scores, ties broken by global flat index (ranks in index order)."""
    shares, _ = select_shares([scores], [[max(0, int(k))]], group)
    return local_smallest(scores, int(shares[0, 0]))


def queue_order(scores: torch.Tensor, chosen: torch.Tensor) -> torch.Tensor:
    """Local indices of this rank's chosen rows in queue order: ascending
    (key, index), the order of torch.topk(sorted=True) for more than 32 picks."""
    index = torch.nonzero(chosen, as_tuple=False).reshape(-1)
    keys = radix_keys(scores[index])
    order = torch.argsort(keys * (index.numel() + 1) + torch.arange(index.numel(), device=keys.device), stable=True)
    return index[order]


def prefix_split(scores: torch.Tensor, chosen: torch.Tensor, prefix: int, group=None) -> torch.Tensor:
    """Mask of this rank's chosen rows that fall in the first `prefix` slots of
    the request-wide queue (an immediate or lazy eviction batch): with prefix
    no larger than the chosen count, that is the request-wide bottom-prefix."""
    return select_smallest(scores, prefix, group) & chosen


def lazy_prefix_share(queue_scores, count: int, group=None) -> int:
    """This rank's share of the next `count` slots of a request's lazy queue
    when the request's layers are split over ranks (controller.py:57-70: each
    lazy batch evicts the next `count` queued references).  queue_scores:
    this rank's remaining queue slots' scores in queue order (ascending raw
    score, ties by score-table index), ranks holding consecutive layer groups
    in rank order -- so the request-wide queue is the merge of the ranks'
    queues by (score, rank, slot).  Every rank gathers each rank's first
    `count` scores and takes the same first `count` of that merge.  Returns 0
    on every rank while the request-wide queue holds fewer than `count`
    slots (the batch waits, as on one GPU).  One all-gather of the queue
    lengths and one of `count` scores per call, on every rank."""
    import numpy as np

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    device = (torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl"
              else torch.device("cpu"))
    lengths = _all_gather_counts(torch.tensor([len(queue_scores)], dtype=torch.int64, device=device),
                                 group).reshape(-1)
    if int(lengths.sum().item()) < count or count <= 0:
        return 0
    n = min(count, len(queue_scores))
    scores = torch.zeros(count, dtype=torch.float32, device=device)
    if n:
        scores[:n] = torch.as_tensor(np.asarray(queue_scores[:n], dtype=np.float32), device=device)
    keys = radix_keys(_all_gather_counts(scores, group))  # [world, count]
    slots = torch.arange(count, device=device)
    valid = slots[None, :] < torch.clamp(lengths, max=count)[:, None]
    keys = torch.where(valid, keys, torch.full_like(keys, 1 << 32))
    ranks = torch.arange(world, device=device)[:, None]
    merged = (keys * (world * count) + ranks * count + slots[None, :]).reshape(-1)
    first = torch.topk(merged, count, largest=False).indices
    return int(((first // count) == rank).sum().item())


def layer_group_audit_requests(requests, query_positions, base_margin, immediate: int, queued: int, group=None,
                               protect_recent=32, denominator_epsilon=1e-6, query_chunk_size=250, pool_kernel=7,
                               timings=None):
    """audit_pass (score, Pool7, select, evict the immediate prefix) for this
    rank's contiguous layer group of each request: requests is a list of
    (cache, queries, gradients) holding this rank's layers only, ranks in
    layer order, the same requests in the same order on every rank.

    Scoring, pooling, refinement and compaction are layer-local.  The
    request-wide choices of every request come from one select_shares call
    (three histogram all-gathers in all): this rank's share of the
    bottom-(immediate + queued) raw scores and of the bottom-immediate.  A
    local refine_arrays with the first count gives the single-GPU quotas,
    refined positions and queue order for these layers; the rank then evicts
    its share of the request-wide immediate prefix, the first slots of its
    local queue.  Returns the local AuditResults (their references are this
    rank's queue slots)."""
    from .audit import AuditResult, pool_table, score_table_fused
    from .selection import fetch_references, refine_device

    tables = [score_table_fused(cache, queries, query_positions, gradients, base_margin, protect_recent,
                                denominator_epsilon, query_chunk_size) for cache, queries, gradients in requests]
    pooled = [pool_table(table, pool_kernel) for table in tables]
    shares, totals = select_shares([table.scores for table in tables],
                                   [[immediate + queued, immediate]] * len(tables), group, timings)
    if (totals < immediate).any():
        raise RuntimeError("Not enough unprotected candidates to enforce the budget")
    results = []
    for (cache, _, _), table, pool, (local_count, local_immediate) in zip(requests, tables, pooled, shares.tolist()):
        queue = refine_device(table, pool, local_count)
        pending = fetch_references(queue)
        evicted = 0
        if local_immediate:
            evicted = cache.remove_selected(queue.coordinates, queue.segment_ids[:local_immediate],
                                            queue.positions[:local_immediate])
        references, changed, changed_heads = pending.result()
        results.append(AuditResult(table, references, changed, changed_heads, evicted))
    return results


def layer_group_audit_pass(cache, queries, query_positions, gradients, base_margin, immediate: int, queued: int,
                           group=None, protect_recent=32, denominator_epsilon=1e-6, query_chunk_size=250,
                           pool_kernel=7, timings=None):
    """layer_group_audit_requests for one request."""
    return layer_group_audit_requests([(cache, queries, gradients)], query_positions, base_margin, immediate, queued,
                                      group, protect_recent, denominator_epsilon, query_chunk_size, pool_kernel,
                                      timings)[0]
