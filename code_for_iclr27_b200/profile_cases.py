"""Single-kernel workloads at configs[1] shape, for profiling one operator.

    python -m code_for_iclr27_b200.profile_cases CASE [--iters N]

CASE is one of:
  scores         lrk_temporal_scores over one layer (8 heads x [250, 4, 34880]
                 bf16 logits, 558 MB, larger than L2)
  scores_large   lrk_temporal_scores over one configs[4] layer (8 heads x
                 [250, 8, 32768] bf16 logits, 1 GB; every row but the last 32
                 a candidate, so the probability stash is 2.1 GB)
  probabilities  temporal_probabilities on one query chunk [79, 4, 35026]
  risk           temporal_risk over 2226 candidates of that chunk
  compact        compaction of one layer (279k rows of D=128 bf16) removing 64 rows
  append         one-token append to one layer
  refine         selection over 502k scores in 256 segments
  project        projected values of one layer (279k rows of D=128 bf16, 4 groups)
  logits         one head's logits, [1000, 128] x [34880, 128] bf16, 16-term steps
  logits_odd     the same with 34883 keys, 8-term steps
  logits_layer   one layer's logits in one launch (lrk_logits_heads): 8 heads of
                 34,878 .. 34,885 keys (both step orders), 1000 query rows each
  large_pass     one configs[4] audit pass of one 70B-shaped request (80 layers x
                 8 heads x 32768 rows, GQA 8; score, Pool7, select 18.6M,
                 evict 18.4M), the layer tensors put back after each pass
  arena_evict    one lazy eviction batch (2048 references over 128 heads of
                 ~34,900 rows, D=128) in a 16-layer KV arena (lrk_arena_evict),
                 the slots refilled between iterations
  select         one layer-group selection round-0 histogram over 8 requests x
                 2.6M scores (lrk_select_histogram, two questions)
Inputs are seeded and generated on the device; each iteration launches the
operator once (large_pass: one whole audit pass).
"""
from __future__ import annotations

import argparse
import math

LAYER_ROWS = 8 * 34880


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("case", choices=["scores", "scores_large", "probabilities", "risk", "compact", "append", "refine",
                                           "project", "logits", "logits_odd", "logits_layer", "from_keys",
                                           "table_fused", "large_pass", "arena_evict", "select"])
    parser.add_argument("--iters", type=int, default=3)
    args = parser.parse_args(argv)

    import torch

    from . import operators

    C = operators()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    if args.case == "scores":
        length, window, groups = 34880, 250, 4
        logits = [(torch.randn(window, groups, length, generator=g, device=dev) * 2 * math.sqrt(128)).to(torch.bfloat16)
                  for _ in range(8)]
        pv = [torch.randn(groups, length, generator=g, device=dev) for _ in range(8)]
        kpos = [torch.arange(length, dtype=torch.float32, device=dev) for _ in range(8)]
        qpos = torch.arange(length - window, length, dtype=torch.int64, device=dev)
        margin = torch.tensor([1.0], device=dev)
        run = lambda: C.temporal_scores(logits, pv, kpos, [32768] * 8, [length - 32] * 8, qpos, margin,
                                        1 / math.sqrt(128), 1e-6)
    elif args.case == "scores_large":
        length, window, groups = 32768, 250, 8
        logits = [(torch.randn(window, groups, length, generator=g, device=dev) * 2 * math.sqrt(128)).to(torch.bfloat16)
                  for _ in range(8)]
        pv = [torch.randn(groups, length, generator=g, device=dev) for _ in range(8)]
        kpos = [torch.arange(length, dtype=torch.float32, device=dev) for _ in range(8)]
        qpos = torch.arange(length - window, length, dtype=torch.int64, device=dev)
        margin = torch.tensor([1.0], device=dev)
        run = lambda: C.temporal_scores(logits, pv, kpos, [0] * 8, [length - 32] * 8, qpos, margin,
                                        1 / math.sqrt(128), 1e-6)
    elif args.case in ("probabilities", "risk"):
        window, groups, length = 79, 4, 35026
        logits = (torch.randn(window, groups, length, generator=g, device=dev) * 2 * math.sqrt(128)).to(torch.bfloat16)
        pv = torch.rand(groups, length, generator=g, device=dev)
        qpos = torch.arange(length - window, length, dtype=torch.int64, device=dev)
        kpos = torch.arange(length, dtype=torch.float32, device=dev)
        if args.case == "probabilities":
            run = lambda: C.temporal_probabilities(logits, pv, qpos, kpos, 1 / math.sqrt(128))
        else:
            probs, op = C.temporal_probabilities(logits, pv, qpos, kpos, 1 / math.sqrt(128))
            margin = torch.tensor([1.0], device=dev)
            run = lambda: C.temporal_risk(probs, op, pv, margin, length - 2258, length - 32, 1e-6)
    elif args.case in ("compact", "append"):
        keys = torch.randn(LAYER_ROWS, 128, generator=g, device=dev).to(torch.bfloat16)
        values = torch.randn(LAYER_ROWS, 128, generator=g, device=dev).to(torch.bfloat16)
        positions = torch.arange(LAYER_ROWS, dtype=torch.float32, device=dev).reshape(-1, 1)
        if args.case == "compact":
            removed = torch.randperm(LAYER_ROWS, generator=g, device=dev)[:64].sort().values
            run = lambda: C.compact(keys, values, positions, removed)
        else:
            cumulative = torch.arange(0, LAYER_ROWS + 1, 34880, dtype=torch.int32, device=dev)
            new = torch.randn(1, 8, 1, 128, generator=g, device=dev).to(torch.bfloat16)
            run = lambda: C.append(keys, values, positions, new, new, cumulative, 40000, 34880)
    elif args.case in ("logits", "logits_odd"):
        count = 34880 if args.case == "logits" else 34883
        queries = (torch.randn(1000, 128, generator=g, device=dev) * 2).to(torch.bfloat16)
        keys = torch.randn(count, 128, generator=g, device=dev).to(torch.bfloat16)
        step = 16 if args.case == "logits" else 8
        run = lambda: C.logits(queries, keys, step, (count + 7) // 8 * 8)
    elif args.case == "logits_layer":
        lens = [34880, 34881, 34883, 34878, 34885, 34880, 34879, 34882]
        bounds = [0]
        for n in lens:
            bounds.append(bounds[-1] + n)
        queries = (torch.randn(len(lens), 1000, 128, generator=g, device=dev) * 2).to(torch.bfloat16)
        keys = torch.randn(bounds[-1], 128, generator=g, device=dev).to(torch.bfloat16)
        steps = [8 if n % 2 else 16 for n in lens]
        run = lambda: C.logits_heads(queries, keys, list(range(len(lens))), bounds[:-1], bounds[1:], steps)
    elif args.case in ("from_keys", "table_fused"):
        # One configs[1] layer scored straight from its keys (lrk_scores_from_keys), or
        # through its logits (table_fused: cuBLAS / lrk_logits, then lrk_temporal_scores):
        # 8 KV heads of 34,880 / 34,881 keys (both step orders), 250 queries x 4 groups.
        from .kvcache import PackedCache

        lens = [34880, 34881] * 4
        rows = sum(lens)
        cache = PackedCache()
        keys = torch.randn(rows, 128, generator=g, device=dev).to(torch.bfloat16)
        values = torch.randn(rows, 128, generator=g, device=dev).to(torch.bfloat16)
        positions = torch.cat([torch.arange(n, dtype=torch.float32, device=dev) for n in lens])
        cache.add_layer(keys, values, positions, lens, [32768] * 8)
        queries = [(torch.randn(250, 32, 128, generator=g, device=dev) * 2).to(torch.bfloat16)]
        gradients = [torch.randn(32, 128, generator=g, device=dev) / math.sqrt(128)]
        qpos = torch.arange(34880 - 250, 34880, dtype=torch.int64, device=dev)
        margin = torch.tensor([1.0], device=dev)
        from .audit import score_table_from_keys, score_table_fused

        table = score_table_from_keys if args.case == "from_keys" else score_table_fused
        run = lambda: table(cache, queries, qpos, gradients, margin)
    elif args.case == "large_pass":
        from .audit import audit_pass
        from .workloads import LARGE_PROTECT, LARGE_ROWS, LARGE_WINDOW, _restore, _snapshot, large_counts, \
            large_request

        counts = large_counts()
        cache, queries, gradients = large_request(dev, 40)
        qpos = torch.arange(LARGE_ROWS - LARGE_WINDOW, LARGE_ROWS, dtype=torch.int64, device=dev)
        margin = torch.tensor([1.0], device=dev)

        def run():
            saved = _snapshot(cache)
            audit_pass(cache, queries, qpos, gradients, margin, counts["immediate"], counts["queued"], LARGE_PROTECT)
            _restore(cache, saved)
    elif args.case == "arena_evict":
        from .arena import ArenaCache

        layers, heads, rows = 16, 8, 34900
        arena = ArenaCache(layers, heads, 128, rows + 256, dev)
        arena.keys.normal_(generator=g)
        arena.values.normal_(generator=g)
        arena.positions.copy_(torch.arange(rows + 256, dtype=torch.float32, device=dev).expand_as(arena.positions))
        full = torch.full((layers * heads,), rows, dtype=torch.int32, device=dev)
        picks = torch.randperm(layers * heads * 2100, generator=g, device=dev)[:2048]
        flat = (picks // 2100).to(torch.int64)
        logical = (picks % 2100 + 32768).to(torch.float32)

        def run():
            arena.lengths.copy_(full)  # the removed rows come back (their positions never moved out of range)
            arena.positions.copy_(torch.arange(rows + 256, dtype=torch.float32, device=dev).expand_as(arena.positions))
            C.arena_evict(arena.keys, arena.values, arena.positions, arena.lengths, flat, logical, arena.flags[1:2])
    elif args.case == "select":
        requests, n = 8, 2_618_880
        tables = [torch.rand(n, generator=g, device=dev) for _ in range(requests)]
        states = torch.zeros(requests, 2, 8, dtype=torch.int64, device=dev)
        states[:, 0, 0], states[:, 1, 0] = 2_322_080, 2_302_080
        run = lambda: C.select_histogram(tables, states, 0)
    elif args.case == "project":
        values = torch.randn(LAYER_ROWS, 128, generator=g, device=dev).to(torch.bfloat16)
        gradients = torch.randn(8 * 4, 128, generator=g, device=dev)
        cumulative = torch.arange(0, LAYER_ROWS + 1, 34880, dtype=torch.int32, device=dev)
        run = lambda: C.project_values(values, gradients, cumulative, 4)
    else:
        n = 256 * 1962
        raw = torch.rand(n, generator=g, device=dev)
        bounds = torch.arange(0, n + 1, 1962, dtype=torch.int64, device=dev)
        pooled = C.pool(raw, bounds, 1962, 7)
        starts = torch.zeros(256, dtype=torch.int64, device=dev)
        run = lambda: C.refine(raw, pooled, bounds[1:].contiguous(), starts, 64512)
    times = []
    for _ in range(args.iters):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        run()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    times.sort()
    print(f"{args.case}: {args.iters} iterations ok, median {times[len(times) // 2]:.3f} ms (CUDA events)")


if __name__ == "__main__":
    main()
