"""Layer-group sharding of one request's eviction selection across ranks.

When one request's cache is split by layers over several GPUs (each rank
scores and compacts its own contiguous group of layers), the selection of
refine_arrays (selection.py:52-88) still needs the request-wide bottom-`count`
of raw scores.  The only data that crosses ranks is a few histograms:

  1. Each rank maps its scores to order-preserving 32-bit keys (the map
     PyTorch's radix select uses; NaN last).
  2. Radix rounds of 12, 12 and 8 bits: every rank histograms the digit of
     the keys still in play, the histograms are all-gathered (NCCL over
     NVLink on GPUs, gloo on CPU), summed, and the bin holding the k-th key is
     fixed.  After the rounds every rank knows the exact k-th key and how many
     keys lie below it request-wide.
  3. Ties at the k-th key are taken in global flat-index order (layer-major,
     the order compute_score_table concatenates heads in, scoring.py:218-287),
     which is torch.topk's choice: ranks own increasing index ranges, so each
     rank takes the first ties it holds after the ties of lower ranks (one
     all-gather of per-rank tie counts).

The chosen set equals the single-GPU set exactly.  Queue prefixes (the
immediate eviction and each lazy prefix of controller.py:57-70) are again
"k smallest" questions over the chosen set and use the same rounds.
Per-segment refinement (Pool7 quotas and transplant) is layer-local, so each
rank finishes it on its own segments.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import torch
import torch.distributed as dist

DIGITS = (12, 12, 8)


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


@dataclass
class Threshold:
    key: int          # the k-th smallest key request-wide
    below: int        # keys strictly below it, request-wide
    ties_taken: int   # keys equal to it that belong to the chosen k


def global_kth_key(keys: torch.Tensor, k: int, group=None, digits: Sequence[int] = DIGITS) -> Threshold:
    """Exact k-th smallest (1 <= k <= total) of the union of every rank's keys,
    found with one histogram all-gather per radix round."""
    if sum(digits) != 32:
        raise ValueError("digit widths must cover 32 bits")
    prefix, done, need, below = 0, 0, int(k), 0
    in_play = keys
    for width in digits:
        shift = 32 - done - width
        digit = (in_play >> shift) & ((1 << width) - 1)
        local = torch.bincount(digit, minlength=1 << width).to(torch.int64)
        total = _all_gather_counts(local, group).sum(0)
        cumulative = total.cumsum(0)
        bin_index = int(torch.searchsorted(cumulative, torch.tensor([need], device=cumulative.device)).item())
        if bin_index >= total.numel():
            raise ValueError(f"k={k} exceeds the number of keys")
        skipped = int(cumulative[bin_index].item() - total[bin_index].item())
        below += skipped
        need -= skipped
        prefix = (prefix << width) | bin_index
        done += width
        in_play = in_play[digit == bin_index]
    return Threshold(key=prefix, below=below, ties_taken=need)


def select_smallest(scores: torch.Tensor, k: int, group=None, eligible: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Boolean mask of this rank's share of the request-wide k smallest
    scores, ties broken by global flat index (ranks in index order).
    `eligible` restricts the candidates (e.g. to already-chosen rows)."""
    keys = radix_keys(scores)
    if eligible is not None:
        keys = torch.where(eligible, keys, torch.full_like(keys, 1 << 32))  # beyond every real key
    if k <= 0:
        return torch.zeros_like(keys, dtype=torch.bool)
    real = keys < (1 << 32)
    threshold = global_kth_key(keys[real], k, group)
    below = keys < threshold.key
    ties = keys == threshold.key
    tie_counts = _all_gather_counts(ties.sum().reshape(1).to(torch.int64), group).reshape(-1)
    rank = dist.get_rank(group)
    before = int(tie_counts[:rank].sum().item())
    take = max(0, min(threshold.ties_taken - before, int(tie_counts[rank].item())))
    chosen = below.clone()
    if take:
        tie_index = torch.nonzero(ties, as_tuple=False).reshape(-1)[:take]
        chosen[tie_index] = True
    return chosen


def queue_order(scores: torch.Tensor, chosen: torch.Tensor) -> torch.Tensor:
    """Local indices of this rank's chosen rows in queue order: ascending
    (key, index), the order of torch.topk(sorted=True) for more than 32 picks."""
    index = torch.nonzero(chosen, as_tuple=False).reshape(-1)
    keys = radix_keys(scores[index])
    order = torch.argsort(keys * (index.numel() + 1) + torch.arange(index.numel(), device=keys.device), stable=True)
    return index[order]


def prefix_split(scores: torch.Tensor, chosen: torch.Tensor, prefix: int, group=None) -> torch.Tensor:
    """Mask of this rank's chosen rows that fall in the first `prefix` slots of
    the request-wide queue (an immediate or lazy eviction batch)."""
    return select_smallest(scores, prefix, group, eligible=chosen)


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


def layer_group_audit_pass(cache, queries, query_positions, gradients, base_margin, immediate: int, queued: int,
                           group=None, protect_recent=32, denominator_epsilon=1e-6, query_chunk_size=250,
                           pool_kernel=7):
    """audit_pass (score, Pool7, select, evict the immediate prefix) for one
    rank's contiguous group of a request's layers: `cache`, `queries` and
    `gradients` hold this rank's layers only, ranks in layer order.

    Scoring, pooling, refinement and compaction are layer-local.  The
    request-wide choices go through select_smallest / prefix_split (radix
    histograms all-gathered over `group`): this rank's share of the
    bottom-(immediate + queued) raw scores is exactly its local bottom-k for k
    = its share (ties by index on both sides), so a local refine_arrays with
    that count gives the single-GPU quotas, refined positions and queue order
    for these layers; the rank then evicts its share of the request-wide
    immediate prefix, the first slots of its local queue.  Returns the local
    AuditResult (its references are this rank's queue slots)."""
    from .audit import AuditResult, pool_table, score_table_fused
    from .selection import fetch_references, refine_device

    table = score_table_fused(cache, queries, query_positions, gradients, base_margin, protect_recent,
                              denominator_epsilon, query_chunk_size)
    pooled = pool_table(table, pool_kernel)
    total = torch.tensor([table.scores.numel()], dtype=torch.int64, device=table.scores.device)
    dist.all_reduce(total, group=group)
    count = min(immediate + queued, int(total.item()))
    if count < immediate:
        raise RuntimeError("Not enough unprotected candidates to enforce the budget")
    chosen = select_smallest(table.scores, count, group)
    head = prefix_split(table.scores, chosen, immediate, group)
    local_count, local_immediate = (int(v) for v in torch.stack([chosen.sum(), head.sum()]).tolist())
    queue = refine_device(table, pooled, local_count)
    pending = fetch_references(queue)
    evicted = 0
    if local_immediate:
        evicted = cache.remove_selected(queue.coordinates, queue.segment_ids[:local_immediate],
                                        queue.positions[:local_immediate])
    references, changed, changed_heads = pending.result()
    return AuditResult(table, references, changed, changed_heads, evicted)
