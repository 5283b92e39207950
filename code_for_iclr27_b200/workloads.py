"""Measured workloads beside the audit pass: recall transport and
static-batch append.

Each function builds seeded synthetic inputs of the configuration's shape on
the GPU (and in host memory for recall), times the operators with CUDA events
on the current stream, and returns a JSON-ready dict.  bench.py adds them to
its line.
"""
from __future__ import annotations

import mmap
import time

import numpy as np

from . import abi, host_operators, operators


def _events():
    import torch

    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _median(values):
    values = sorted(values)
    return values[len(values) // 2]


def pinned_h2d_peak(device, megabytes: int = 256, repeats: int = 10) -> dict:
    """The host link's copy rate: `repeats` copies of one contiguous pinned
    buffer of `megabytes` MiB to the device, each timed with CUDA events.
    Returns the best rate (the peak) and the spread."""
    import torch

    host = torch.empty(megabytes << 20, dtype=torch.uint8).pin_memory()
    dest = torch.empty(megabytes << 20, dtype=torch.uint8, device=device)
    dest.copy_(host, non_blocking=True)
    torch.cuda.synchronize()
    rates = []
    for _ in range(repeats):
        a, b = _events()
        a.record()
        dest.copy_(host, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        rates.append((megabytes << 20) / (a.elapsed_time(b) / 1e3) / 1e9)
    return {"GBps": max(rates), "min_GBps": min(rates), "median_GBps": _median(rates), "copies": repeats,
            "bytes": megabytes << 20}


class _HostPool:
    """One request's archive: rows of [2, D] bf16 (K, V) in page-aligned host
    memory registered for the device (the transport's shared-memory slots,
    recall/transport.py:16-31, archive layout recall/cpu_worker.py:21-22)."""

    def __init__(self, rows: int, dim: int, seed: int):
        self.rows, self.row_bytes = rows, 2 * dim * 2
        self.buffer = mmap.mmap(-1, rows * self.row_bytes)
        self.array = np.frombuffer(self.buffer, dtype=np.uint16).reshape(rows, 2, dim)
        rng = np.random.default_rng(seed)
        # bf16 bit patterns of N(0, 1) samples
        self.array[:] = (rng.standard_normal(self.array.shape, dtype=np.float32).view(np.uint32) >> 16).astype(
            np.uint16)
        self.address = self.array.__array_interface__["data"][0]
        host_operators().register_host(self.address, rows * self.row_bytes)
        self.device_address = host_operators().device_pointer(self.address)

    def close(self):
        host_operators().unregister_host(self.address)
        del self.array
        self.buffer.close()


def measure_recall(device, requests: int = 4, pool_rows: int = 200_000, recall_rows: int = 256, layers: int = 32,
                   heads: int = 8, dim: int = 128, cache_rows_per_head: int = 2000, events: int = 20,
                   seed: int = 3) -> dict:
    """per recall event, `recall_rows` random rows of each
    request's host pool reach the GPU and are merged into its cache.

    Two transports are timed: the GPU gathering the rows from the registered
    pool itself (lrk_gather_rows over the host link), and the reference's path
    (a CPU gather into a pinned staging slot, then one cudaMemcpyAsync,
    recall/cpu_worker.py:161-166, transport.py:221-229).  A size sweep gives
    the link rate where it is not latency-bound, against the pinned-copy peak.
    The merge is timed for rows spread uniformly over (layer, head): as
    _C.merge per touched layer (one whole-layer copy each), and as one
    lrk_merge_layers launch for all of them."""
    import torch

    lib = abi.library()
    C = operators()
    stream = torch.cuda.current_stream(device).cuda_stream
    rng = np.random.default_rng(seed)
    pools = [_HostPool(pool_rows, dim, seed + r) for r in range(requests)]
    try:
        row_bytes = pools[0].row_bytes
        out = torch.empty(requests, recall_rows, 2, dim, dtype=torch.bfloat16, device=device)
        host_indices = torch.empty(requests, recall_rows, dtype=torch.int64).pin_memory()
        dev_indices = torch.empty(requests, recall_rows, dtype=torch.int64, device=device)
        staging = torch.empty(requests, recall_rows, 2, dim, dtype=torch.int16).pin_memory()
        staged_out = torch.empty(requests, recall_rows, 2, dim, dtype=torch.int16, device=device)

        # Each event's rows, drawn before the timed region (uniform, without replacement).
        chosen = [np.stack([rng.choice(pool_rows, recall_rows, replace=False) for _ in range(requests)])
                  for _ in range(events + 1)]

        def zero_copy_event(i):
            host_indices.numpy()[:] = chosen[i]
            dev_indices.copy_(host_indices, non_blocking=True)
            for r, pool in enumerate(pools):
                abi.check(lib.lrk_gather_rows(pool.device_address, pool_rows, row_bytes,
                                              dev_indices[r].data_ptr(), recall_rows, out[r].data_ptr(), stream))

        def staged_event(i):
            for r, pool in enumerate(pools):
                staging[r].numpy()[:] = pool.array[chosen[i][r]].view(np.int16)
            staged_out.copy_(staging, non_blocking=True)

        results = {}
        for name, event in (("zero_copy", zero_copy_event), ("staged", staged_event)):
            event(events)
            torch.cuda.synchronize()
            device_times, wall_times = [], []
            for i in range(events):
                a, b = _events()
                start = time.perf_counter()
                a.record()
                event(i)
                b.record()
                torch.cuda.synchronize()
                wall_times.append((time.perf_counter() - start) * 1e3)
                device_times.append(a.elapsed_time(b))
            results[name] = {"event_us": _median(wall_times) * 1e3, "device_us": _median(device_times) * 1e3}

        # Size sweep: zero-copy gather of random rows vs one contiguous pinned copy.
        # The host link's rate: the better of a copy-engine copy (256 MiB
        # pinned) and the GPU reading a registered pool itself (all of one
        # pool's rows, sequential, through lrk_gather_rows).
        link = pinned_h2d_peak(device)
        sequential = torch.arange(pool_rows, dtype=torch.int64, device=device)
        whole = torch.empty(pool_rows, 2, dim, dtype=torch.bfloat16, device=device)
        reads = []
        for attempt in range(11):
            a, b = _events()
            a.record()
            abi.check(lib.lrk_gather_rows(pools[0].device_address, pool_rows, row_bytes, sequential.data_ptr(),
                                          pool_rows, whole.data_ptr(), stream))
            b.record()
            torch.cuda.synchronize()
            if attempt:
                reads.append(pool_rows * row_bytes / (a.elapsed_time(b) / 1e3) / 1e9)
        link["zero_copy_read_GBps"] = max(reads)
        link["zero_copy_read_bytes"] = pool_rows * row_bytes
        peak = max(link["GBps"], link["zero_copy_read_GBps"])
        link["link_peak_GBps"] = peak
        sweep = []
        for size in (128 << 10, 512 << 10, 2 << 20, 8 << 20, 32 << 20):
            rows = size // row_bytes
            picks = torch.from_numpy(rng.choice(pool_rows, rows, replace=False)).to(device)
            dest = torch.empty(rows, 2, dim, dtype=torch.bfloat16, device=device)
            contiguous = torch.empty(size, dtype=torch.uint8).pin_memory()
            contiguous_dest = torch.empty(size, dtype=torch.uint8, device=device)

            def gather():
                abi.check(lib.lrk_gather_rows(pools[0].device_address, pool_rows, row_bytes, picks.data_ptr(), rows,
                                              dest.data_ptr(), stream))

            def copy():
                contiguous_dest.copy_(contiguous, non_blocking=True)

            entry = {"bytes": size}
            for label, fn in (("zero_copy_gather_GBps", gather), ("pinned_copy_GBps", copy)):
                fn()
                torch.cuda.synchronize()
                times = []
                for _ in range(10):
                    a, b = _events()
                    a.record()
                    fn()
                    b.record()
                    torch.cuda.synchronize()
                    times.append(a.elapsed_time(b))
                entry[label] = size / (_median(times) / 1e3) / 1e9
            sweep.append(entry)

        # Merge: each request's recalled rows into its cache, rows spread over
        # (layer, head); one whole-layer copy per touched layer.
        g = torch.Generator(device=device).manual_seed(seed)
        layer_rows = heads * cache_rows_per_head
        merge_us = []
        merged_bytes = 0
        keys = torch.randn(layer_rows, dim, generator=g, device=device).to(torch.bfloat16)
        values = torch.randn(layer_rows, dim, generator=g, device=device).to(torch.bfloat16)
        positions = torch.arange(layer_rows, dtype=torch.float32, device=device).reshape(-1, 1) * 4
        owners = rng.integers(0, layers * heads, recall_rows)
        plans = []
        for layer in range(layers):
            mine = np.flatnonzero(owners // heads == layer)
            if not mine.size:
                continue
            head_of = owners[mine] % heads
            mapping = []
            for h in range(heads):
                existing = np.arange(h * cache_rows_per_head, (h + 1) * cache_rows_per_head)
                recalled = np.flatnonzero(head_of == h)
                # recalled positions fall between existing ones (odd multiples of 2)
                new_pos = rng.choice(cache_rows_per_head, recalled.size, replace=False) * 4 + 2
                order = np.argsort(np.concatenate([existing * 4, h * cache_rows_per_head * 4 + new_pos]),
                                   kind="stable")
                entries = np.concatenate([existing, -(mine[recalled] + 1)])
                mapping.append(entries[order])
            plans.append((torch.from_numpy(np.concatenate(mapping)).to(device), mine.size))
        recalled_rows = out[0].contiguous()
        recalled_positions = torch.arange(recall_rows, dtype=torch.float32, device=device) * 4 + 2
        for _ in range(3):
            for mapping, _count in plans:
                C.merge(keys, values, positions, recalled_rows, recalled_positions, mapping)
        torch.cuda.synchronize()
        for _ in range(events):
            a, b = _events()
            a.record()
            for mapping, _count in plans:
                C.merge(keys, values, positions, recalled_rows, recalled_positions, mapping)
            b.record()
            torch.cuda.synchronize()
            merge_us.append(a.elapsed_time(b) * 1e3)
        for mapping, count in plans:
            merged_bytes += 2 * (layer_rows + count) * (4 * dim + 4)
        merge = _median(merge_us)
        # The same event as one lrk_merge_layers launch over every touched layer.
        n = len(plans)
        layers_args = ([keys] * n, [values] * n, [positions] * n, [recalled_rows] * n, [recalled_positions] * n,
                       [mapping for mapping, _ in plans])
        for _ in range(3):
            C.merge_layers(*layers_args)
        torch.cuda.synchronize()
        merge_layers_us = []
        for _ in range(events):
            a, b = _events()
            a.record()
            C.merge_layers(*layers_args)
            b.record()
            torch.cuda.synchronize()
            merge_layers_us.append(a.elapsed_time(b) * 1e3)
        merge_layers = _median(merge_layers_us)

        reinsert = measure_reinsert(device, layers, heads, dim, cache_rows_per_head, recall_rows, events, rng)

        link_bytes = requests * recall_rows * (4 * dim + 8)  # K, V rows + the int64 index
        zero_copy_us = results["zero_copy"]["device_us"]
        return {
            "config": f"configs[3]: {requests} requests, host pools of {pool_rows} rows x [2, {dim}] bf16, "
                      f"{recall_rows} random rows each per event; cache {cache_rows_per_head} rows/head, "
                      f"{layers} layers x {heads} heads",
            "pinned_h2d_peak_GBps": link["GBps"],
            "link_peak_GBps": peak,
            "link_peak": link,
            "event_zero_copy_us": zero_copy_us,
            "event_zero_copy_link_GBps": link_bytes / (zero_copy_us / 1e6) / 1e9,
            "event_staged_us": results["staged"]["event_us"],
            "event_staged_device_us": results["staged"]["device_us"],
            "sweep": sweep,
            # A fraction above 1.05 means the peak copy was measured low: not reported.
            "sweep_frac_of_peak_at_32MiB": (None if sweep[-1]["zero_copy_gather_GBps"] / peak > 1.05
                                            else sweep[-1]["zero_copy_gather_GBps"] / peak),
            "merge_us_per_request_event": merge,
            "merge_GBps": merged_bytes / (merge / 1e6) / 1e9,
            "merge_layers_us_per_request_event": merge_layers,
            "merge_layers_GBps": merged_bytes / (merge_layers / 1e6) / 1e9,
            "reinsert": reinsert,
        }
    finally:
        for pool in pools:
            pool.close()


def measure_reinsert(device, layers, heads, dim, rows_per_head, recall_rows, events, rng) -> dict:
    """One request's recall event end to end through PackedCache.insert_payload
    (cache.py:201-253): `recall_rows` identities spread uniformly over
    (layer, head), positions between resident ones, rows already on the GPU.
    Timed on the host clock (the call returns after its one flag read), with
    the merge plan on the device and with the host plan (the resident
    positions of the touched layers copied to the host, numpy's stable
    argsort per head, recall/planning.py:34-52); the cache is restored
    between events; and the same events into a KV arena (in place)."""
    import torch

    from .kvcache import PackedCache

    g = torch.Generator(device=device).manual_seed(7)
    cache = PackedCache()
    lens = [rows_per_head] * heads
    head_positions = torch.arange(rows_per_head, dtype=torch.float32, device=device) * 4
    for _ in range(layers):
        keys = torch.randn(heads * rows_per_head, dim, generator=g, device=device).to(torch.bfloat16)
        values = torch.randn(heads * rows_per_head, dim, generator=g, device=device).to(torch.bfloat16)
        cache.add_layer(keys, values, head_positions.repeat(heads), lens, [0] * heads)
    saved = [(layer.keys, layer.values, layer.positions, list(layer.head_lens), layer.cumulative)
             for layer in cache.layers]
    payload = torch.randn(recall_rows, 2, dim, generator=g, device=device).to(torch.bfloat16)
    plans = []
    for _ in range(events + 3):
        picks = rng.choice(layers * heads * rows_per_head, recall_rows, replace=False)
        plans.append(np.stack((picks // (heads * rows_per_head), picks // rows_per_head % heads,
                               picks % rows_per_head * 4 + 2), axis=1))
    result = {"rows": recall_rows, "layers": layers, "heads": heads, "rows_per_head": rows_per_head}
    # The same events into a KV arena holding the same rows (in place,
    # lrk_arena_insert), its tensors copied back between events.
    from .arena import ArenaCache

    arena = ArenaCache.from_packed(cache, margin=512)
    kept = (arena.keys.clone(), arena.values.clone(), arena.positions.clone(), arena.lengths.clone(),
            arena.head_lens.copy())
    times = []
    for i, metadata in enumerate(plans):
        arena.keys.copy_(kept[0]), arena.values.copy_(kept[1]), arena.positions.copy_(kept[2])
        arena.lengths.copy_(kept[3])
        arena.head_lens[:] = kept[4]
        torch.cuda.synchronize()
        start = time.perf_counter()
        arena.insert_payload(payload, metadata)
        torch.cuda.synchronize()
        if i >= 3:
            times.append((time.perf_counter() - start) * 1e6)
    result["arena_in_place_us"] = _median(times)
    del arena, kept
    for plan in ("device", "host"):
        times = []
        for i, metadata in enumerate(plans):
            for layer, state in zip(cache.layers, saved):
                layer.keys, layer.values, layer.positions, lens_copy, layer.cumulative = state
                layer.head_lens = list(lens_copy)
            torch.cuda.synchronize()
            start = time.perf_counter()
            cache.insert_payload(payload, metadata, plan=plan)
            torch.cuda.synchronize()
            if i >= 3:
                times.append((time.perf_counter() - start) * 1e6)
        result[f"{plan}_plan_us"] = _median(times)
    return result


def measure_batch_append(device, requests: int = 8, layers: int = 32, heads: int = 8, dim: int = 128,
                         generated: int = 2000, steps: int = 10, seed: int = 2) -> dict:
    """one decode step of a static batch appends one token per
    request per layer through _C.batch_append (batch_attention.py:41-64);
    prompt lengths uniform in [1024, 16384]."""
    import torch

    C = operators()
    rng = np.random.default_rng(seed)
    g = torch.Generator(device=device).manual_seed(seed)
    prompts = rng.integers(1024, 16385, requests)
    lengths = [[int(p) + generated] * heads for p in prompts]
    caches = []
    for _ in range(layers):
        ks, vs, ps = [], [], []
        for r in range(requests):
            rows = sum(lengths[r])
            ks.append(torch.randn(rows, dim, generator=g, device=device).to(torch.bfloat16))
            vs.append(torch.randn(rows, dim, generator=g, device=device).to(torch.bfloat16))
            ps.append(torch.arange(rows, dtype=torch.float32, device=device).reshape(-1, 1))
        caches.append([ks, vs, ps])
    new = torch.randn(requests, heads, 1, dim, generator=g, device=device).to(torch.bfloat16)
    logical = [int(p) + generated for p in prompts]
    total_rows = sum(sum(x) for x in lengths)

    def step():
        nonlocal lengths
        for layer in range(layers):
            ks, vs, ps = caches[layer]
            k, v, p = C.batch_append(ks, vs, ps, new, new, lengths, logical)
            # the caller keeps per-request views of the packed output (batch_attention.py:54-63)
            offsets = np.concatenate(([0], np.cumsum([sum(x) + heads for x in lengths])))
            active = len(lengths)
            caches[layer] = [[k[offsets[r]:offsets[r + 1]] for r in range(active)],
                             [v[offsets[r]:offsets[r + 1]] for r in range(active)],
                             [p[offsets[r]:offsets[r + 1]] for r in range(active)]]
        lengths = [[n + 1 for n in row] for row in lengths]

    def timed_steps():
        times, moved = [], 0
        for _ in range(steps):
            rows_before = sum(sum(x) for x in lengths)
            a, b = _events()
            a.record()
            step()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b) * 1e3)
            moved = layers * (rows_before + (rows_before + len(lengths) * heads)) * (4 * dim + 4)
        return _median(times), moved

    step()
    torch.cuda.synchronize()
    us, moved = timed_steps()
    # EOS: the request with the earliest end (EOS steps uniform in [500,
    # 8000]) retires -- batching.py:150-163 drops its cache -- and the next
    # steps append for the others only.
    eos = rng.integers(500, 8001, requests)
    leaving = int(np.argmin(eos))
    t0 = time.perf_counter()
    for layer in range(layers):
        for part in caches[layer]:
            del part[leaving]
    del lengths[leaving]
    del logical[leaving]
    new = new[[r for r in range(requests) if r != leaving]].contiguous()
    retire_us = (time.perf_counter() - t0) * 1e6
    step()
    torch.cuda.synchronize()
    us_after, moved_after = timed_steps()
    return {
        "config": f"configs[2]: {requests} requests, prompts U[1024, 16384] + {generated} generated rows per head, "
                  f"{layers} layers x {heads} heads x D{dim}",
        "rows_per_layer": total_rows,
        "us_per_step": us,
        "GBps": moved / (us / 1e6) / 1e9,
        "eos": {"retired_request": leaving, "eos_step": int(eos[leaving]), "retire_host_us": retire_us,
                "us_per_step_after": us_after, "GBps_after": moved_after / (us_after / 1e6) / 1e9,
                "requests_after": requests - 1},
    }


def measure_small(device, steps: int = 5, warmup: int = 3, seed: int = 11, peak_gbs=None) -> dict:
    """one Llama-3.2-1B-shaped request (16 layers x 8 KV heads x
    D64, GQA 4), 4096 rows per head, every row a generation row (prompt
    lengths 0), protect_recent 32; one audit pass scores the 520,192
    candidates, selects 301,312 (immediate 269,312 + 250 x 128 queued:
    controller.py:148-150 with budget 2000) and evicts the immediate ones.
    Each pass starts from the same state."""
    import torch

    from .audit import audit_pass
    from .kvcache import PackedCache

    layers, heads, groups, dim, rows, window = 16, 8, 4, 64, 4096, 250
    slots = layers * heads
    wall, staging = 2000 * slots, 8 * slots
    immediate = slots * rows - (wall - staging)
    queued = 250 * slots
    g = torch.Generator(device=device).manual_seed(seed)
    cache = PackedCache()
    positions = torch.arange(rows, dtype=torch.float32, device=device).repeat(heads)
    for _ in range(layers):
        cache.add_layer(torch.randn(heads * rows, dim, generator=g, device=device).to(torch.bfloat16),
                        torch.randn(heads * rows, dim, generator=g, device=device).to(torch.bfloat16),
                        positions.clone(), [rows] * heads, [0] * heads)
    cache.seen_tokens = rows
    queries = [(torch.randn(window, heads * groups, dim, generator=g, device=device) * 2).to(torch.bfloat16)
               for _ in range(layers)]
    gradients = [torch.randn(heads * groups, dim, generator=g, device=device) / float(np.sqrt(dim))
                 for _ in range(layers)]
    qpos = torch.arange(rows - window, rows, dtype=torch.int64, device=device)
    margin = torch.tensor([1.0], device=device)

    def run():
        saved = _snapshot(cache)
        audit_pass(cache, queries, qpos, gradients, margin, immediate, queued, 32)
        _restore(cache, saved)

    # The pass is timed bare: its launches are short enough that the host's
    # issue rate shows, so the per-call events of the roofline figure come
    # from passes of their own.
    elapsed = _timed_passes(run, steps, warmup, torch.cuda.synchronize, None)
    with ScoreTimer() as timer:
        _timed_passes(run, steps, 1, torch.cuda.synchronize, timer)
    kernel_ms = timer.total_ms()
    out = {"config": "configs[0]: llama-3.2-1b shape, 16 layers x 8 KV heads x D64, 4096 generation rows per head",
           "managed_rows": slots * rows, "candidates": slots * (rows - 32), "selected": immediate + queued,
           "evicted": immediate, "steps": steps, "warmup": warmup, "ms_per_pass": elapsed / steps,
           "tokens_per_s": slots * rows * steps / (elapsed / 1e3),
           "temporal_scores_GBps": timer.bytes / (kernel_ms / 1e3) / 1e9 if kernel_ms else None}
    if peak_gbs and kernel_ms:
        out["temporal_scores_frac"] = out["temporal_scores_GBps"] / peak_gbs
    return out


# ------------------------------------------------------------- configs[4]

# Llama-3-70B shape: 80 layers x 8 KV heads x D128, GQA group 8; a
# 32768-row cache per head, every row a generation row (no prompt rows, so
# every row but the last protect_recent is a candidate); budget 4000.
LARGE_LAYERS, LARGE_HEADS, LARGE_GROUPS, LARGE_DIM, LARGE_ROWS = 80, 8, 8, 128, 32768
LARGE_BUDGET, LARGE_WINDOW, LARGE_AUDIT_PERIOD, LARGE_EVICT_INTERVAL, LARGE_PROTECT = 4000, 250, 250, 8, 32


def large_counts(layers: int = LARGE_LAYERS, heads: int = LARGE_HEADS, rows: int = LARGE_ROWS,
                 budget: int = LARGE_BUDGET) -> dict:
    """The controller's counts for one request's first audit
    (controller.py:15-18, 148-150): slots per step = layers x heads; wall =
    budget x slots; staging = evict_interval x slots; the audit evicts down to
    wall - staging at once and queues audit_period x slots more."""
    slots = layers * heads
    wall = budget * slots
    staging = LARGE_EVICT_INTERVAL * slots
    managed = slots * rows
    immediate = managed - (wall - staging)
    queued = LARGE_AUDIT_PERIOD * slots
    return {"managed": managed, "immediate": immediate, "queued": queued, "kept": wall - staging,
            "candidates": slots * (rows - LARGE_PROTECT)}


def large_request(device, seed: int, layers=None):
    """One configs[4] request's cache and audit inputs, or only the layers in
    `layers` (a range) for a layer group: each layer is generated from its own
    seed (request seed, layer), so a group's layers equal the whole request's.
    K/V bf16 ~N(0,1); positions 0..rows-1 per head; queries (the audit's query
    history, W x 64 query heads) bf16 ~N(0,4), so the scaled logits are
    ~N(0,4) ("2 N(0,1)"); margin gradients ~N(0, 1/D)."""
    import torch

    from .kvcache import PackedCache

    layers = range(LARGE_LAYERS) if layers is None else layers
    cache = PackedCache()
    queries, gradients = [], []
    positions = torch.arange(LARGE_ROWS, dtype=torch.float32, device=device).repeat(LARGE_HEADS)
    for layer in layers:
        g = torch.Generator(device=device).manual_seed(seed * 1000 + layer)
        rows = LARGE_HEADS * LARGE_ROWS
        keys = torch.randn(rows, LARGE_DIM, generator=g, device=device).to(torch.bfloat16)
        values = torch.randn(rows, LARGE_DIM, generator=g, device=device).to(torch.bfloat16)
        cache.add_layer(keys, values, positions.clone(), [LARGE_ROWS] * LARGE_HEADS, [0] * LARGE_HEADS)
        queries.append((torch.randn(LARGE_WINDOW, LARGE_HEADS * LARGE_GROUPS, LARGE_DIM, generator=g, device=device)
                        * 2).to(torch.bfloat16))
        gradients.append(torch.randn(LARGE_HEADS * LARGE_GROUPS, LARGE_DIM, generator=g, device=device)
                         / float(np.sqrt(LARGE_DIM)))
    cache.seen_tokens = LARGE_ROWS
    return cache, queries, gradients


def _snapshot(cache):
    return [(layer.keys, layer.values, layer.positions, list(layer.head_lens), list(layer.prompt_lens),
             layer.cumulative) for layer in cache.layers]


def _restore(cache, saved):
    """Put back the layer tensors an audit replaced (its operators allocate
    fresh outputs and never write their inputs, so the originals are intact)."""
    for layer, (k, v, p, lens, prompts, cumulative) in zip(cache.layers, saved):
        layer.keys, layer.values, layer.positions, layer.cumulative = k, v, p, cumulative
        layer.head_lens, layer.prompt_lens = lens, prompts


class ScoreTimer:
    """CUDA events around every lrk_temporal_scores call an audit makes (on
    the stream it is launched on), with its algorithmic bytes: the logits read
    once, the projected values and key positions once, the scores written."""

    def __init__(self):
        self.pairs, self.bytes = [], 0

    def __enter__(self):
        import torch

        from . import audit

        self.module, self.original = audit, audit.operators
        inner = self.original()
        timer = self

        class Proxy:
            def __getattr__(self, name):
                attribute = getattr(inner, name)
                if name != "temporal_scores":
                    return attribute

                def timed(logits, projected, kpos, first, last, *rest, **kw):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    out = attribute(logits, projected, kpos, first, last, *rest, **kw)
                    b.record()
                    timer.pairs.append((a, b))
                    for lg, f, l in zip(logits, first, last):
                        w, g, length = lg.shape
                        timer.bytes += w * g * length * lg.element_size() + g * length * 4 + length * 4 + (l - f) * 4
                    return out

                return timed

        proxy = Proxy()
        audit.operators = lambda: proxy
        return self

    def __exit__(self, *exc):
        self.module.operators = self.original

    def reset(self):
        self.pairs, self.bytes = [], 0

    def total_ms(self):
        return sum(a.elapsed_time(b) for a, b in self.pairs)


def _timed_passes(run, steps: int, warmup: int, barrier, timer=None):
    for _ in range(warmup):
        run()
    barrier()
    if timer is not None:
        timer.reset()
    a, b = _events()
    barrier()
    a.record()
    for _ in range(steps):
        run()
    b.record()
    barrier()
    return a.elapsed_time(b)


def measure_large(device, requests: int = 8, steps: int = 2, warmup: int = 2, seed: int = 40, rank: int = 0,
                  barrier=None, peak_gbs=None) -> dict:
    """configs[4], request sharding: `requests` independent 70B-shaped
    requests on this GPU, each taken through one audit pass (score every
    candidate, Pool7, select immediate + queued, evict the immediate prefix:
    the first audit evicts the cache down to the budget).  Each pass starts
    from the same state (the replaced layer tensors are put back).  Timed:
    `steps` passes over all requests after `warmup`."""
    import torch

    from .audit import audit_pass

    barrier = barrier or torch.cuda.synchronize
    counts = large_counts()
    reqs = [large_request(device, seed + 100 * rank + r) for r in range(requests)]
    qpos = torch.arange(LARGE_ROWS - LARGE_WINDOW, LARGE_ROWS, dtype=torch.int64, device=device)
    margin = torch.tensor([1.0], device=device)
    evicted = []

    def run():
        evicted.clear()
        for cache, queries, gradients in reqs:
            saved = _snapshot(cache)
            result = audit_pass(cache, queries, qpos, gradients, margin, counts["immediate"], counts["queued"],
                                LARGE_PROTECT)
            evicted.append(result.evicted)
            _restore(cache, saved)

    with ScoreTimer() as timer:
        elapsed = _timed_passes(run, steps, warmup, barrier, timer)
    kernel_ms = timer.total_ms()
    out = {
        "config": (f"configs[4]: {requests} requests per GPU (request sharding, no collective), "
                   f"{LARGE_LAYERS} layers x {LARGE_HEADS} KV heads x D{LARGE_DIM}, GQA {LARGE_GROUPS}, "
                   f"{LARGE_ROWS} generation rows per head, budget {LARGE_BUDGET}, window {LARGE_WINDOW}"),
        "requests": requests, "steps": steps, "warmup": warmup,
        "managed_rows_per_request": counts["managed"], "candidates_per_request": counts["candidates"],
        "selected_per_request": counts["immediate"] + counts["queued"], "evicted_per_request": counts["immediate"],
        "evicted_check": int(evicted[0]) if evicted else None,
        "ms_per_pass": elapsed / steps,
        "tokens_per_s": requests * counts["managed"] * steps / (elapsed / 1e3),
        "temporal_scores_ms_per_pass": kernel_ms / steps,
        "temporal_scores_GBps": timer.bytes / (kernel_ms / 1e3) / 1e9 if kernel_ms else None,
    }
    if peak_gbs and kernel_ms:
        out["temporal_scores_frac"] = out["temporal_scores_GBps"] / peak_gbs
    del reqs
    return out


def measure_large_layer_groups(device, world: int, rank: int, requests: int = 8, steps: int = 2, warmup: int = 2,
                               seed: int = 40, group=None, barrier=None) -> dict:
    """configs[4], layer groups: `requests` 70B-shaped requests, each split
    into `world` contiguous groups of layers, one per rank (strong scaling:
    the total work is fixed).  One audit pass of all requests: every rank
    scores, pools, refines and compacts its own layers, and the request-wide
    bottom-k of every request comes from one select_shares call (three
    histogram all-gathers over NCCL for all requests at once)."""
    import torch

    from .distributed import layer_group_audit_requests

    barrier = barrier or torch.cuda.synchronize
    if LARGE_LAYERS % world:
        raise ValueError(f"{LARGE_LAYERS} layers do not split evenly over {world} ranks")
    per = LARGE_LAYERS // world
    counts = large_counts()
    reqs = [large_request(device, seed + r, range(rank * per, (rank + 1) * per)) for r in range(requests)]
    qpos = torch.arange(LARGE_ROWS - LARGE_WINDOW, LARGE_ROWS, dtype=torch.int64, device=device)
    margin = torch.tensor([1.0], device=device)
    gathers = []

    def run():
        saved = [_snapshot(cache) for cache, _, _ in reqs]
        gathers.clear()
        layer_group_audit_requests(reqs, qpos, margin, counts["immediate"], counts["queued"], group,
                                   protect_recent=LARGE_PROTECT, timings=gathers)
        for (cache, _, _), s in zip(reqs, saved):
            _restore(cache, s)

    with ScoreTimer() as timer:
        elapsed = _timed_passes(run, steps, warmup, barrier, timer)
    gather_us = [a.elapsed_time(b) * 1e3 for a, b in gathers]
    out = {
        "config": (f"configs[4] layer groups: {requests} requests, each split into {world} groups of {per} layers "
                   f"(strong scaling), NCCL all-gather of {requests} x 2 x 4096-bin histograms per radix round"),
        "requests": requests, "layers_per_rank": per, "steps": steps, "warmup": warmup,
        "ms_per_pass": elapsed / steps,
        "tokens_per_s": requests * counts["managed"] * steps / (elapsed / 1e3),
        "allgather_us_per_round": gather_us,
        "allgather_bytes_per_rank": requests * 2 * 4096 * 4,
    }
    del reqs
    return out
