"""Layer-group selection on the GPU.

On one GPU: the selection kernels (lrk_select_histogram, lrk_select_pick) with
the ranks emulated in one process (each rank's histograms computed on its
shard, stacked as the all-gather would, then each rank's pick) against the
torch restatement of the same rounds and against the single-table bottom-k.
Over NCCL on 2 GPUs (one process per GPU): the ranks' union equals the
single-process bottom-count, ties broken by global index; and a layer-group
audit pass equals the single-GPU one.  The NCCL tests skip with fewer than 2
GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scores(seed, n, levels):
    rng = np.random.default_rng(seed)
    if levels:
        return (rng.integers(0, levels, n) / 8).astype(np.float32)
    return rng.random(n, dtype=np.float32)


EMULATED = [
    # seed, world, per-request sizes, tie levels, ks per request (count, prefix)
    (31, 2, [50_000, 3_000, 70_001], 0, [(20_000, 500), (3_000, 3_000), (1, 1)]),
    (32, 3, [40_000, 9_999, 1], 5, [(12_345, 77), (9_000, 8_999), (1, 0)]),
    (33, 4, [120_000, 0, 2_000], 40, [(119_000, 60_000), (5, 5), (2_500, 1_000)]),
]


@pytest.mark.parametrize("seed,world,sizes,levels,ks", EMULATED)
def test_select_kernels_with_emulated_ranks(cuda, seed, world, sizes, levels, ks):
    """Every round's histograms and states equal the torch restatement's, and
    each request's shares add up to its single-table bottom-k by (key,
    index), split at the ranks' cut points."""
    import torch

    from code_for_iclr27_b200 import operators
    from code_for_iclr27_b200.distributed import (BINS, DIGITS, FIELDS, K, SHARE, TOTAL, _histogram_host,
                                                  _pick_host)
    from oracle import lrk_oracle as O

    C = operators()
    tables = [_scores(seed + i, n, levels) for i, n in enumerate(sizes)]
    tables[0][7] = np.nan  # NaN keys rank last
    cuts = [[int(x) for x in np.linspace(0, n, world + 1).round()] for n in sizes]
    requests, questions = len(sizes), 2
    start = torch.zeros(requests, questions, FIELDS, dtype=torch.int64)
    start[:, :, K] = torch.tensor(ks)
    device_states = [start.clone().to(cuda) for _ in range(world)]
    host_states = [start.clone() for _ in range(world)]
    shards = [[torch.from_numpy(t[c[r]:c[r + 1]].copy()) for t, c in zip(tables, cuts)] for r in range(world)]
    for round_index in range(len(DIGITS)):
        device_hist = [C.select_histogram([x.to(cuda) for x in shards[r]], device_states[r], round_index)
                       for r in range(world)]
        host_hist = [_histogram_host(shards[r], host_states[r], round_index) for r in range(world)]
        for d, h in zip(device_hist, host_hist):
            assert torch.equal(d.cpu(), h), f"round {round_index} histograms"
        gathered = torch.stack(device_hist)
        for r in range(world):
            C.select_pick(gathered, r, device_states[r], round_index)
            _pick_host(torch.stack(host_hist), r, host_states[r], round_index)
            assert torch.equal(device_states[r].cpu(), host_states[r]), f"round {round_index} rank {r} states"
    assert gathered.shape == (world, requests, questions, BINS)
    for i, table in enumerate(tables):
        order = np.lexsort((np.arange(table.size), O.radix_key(table)))
        owner = np.searchsorted(np.asarray(cuts[i]), order, side="right") - 1
        for q, k in enumerate(ks[i]):
            k = min(k, table.size)
            for r in range(world):
                state = device_states[r].cpu()[i, q]
                assert int(state[TOTAL]) == table.size
                assert int(state[SHARE]) == int((owner[:k] == r).sum()), f"request {i} question {q} rank {r}"


CASES = [(11, 400_000, 0, 150_000, 2048), (12, 400_000, 64, 200_000, 4096), (13, 100_000, 3, 99_000, 10)]


def _worker(rank, world, port, results):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    try:
        from code_for_iclr27_b200.distributed import prefix_split, select_smallest

        out = []
        for seed, n, levels, count, prefix in CASES:
            cuts = [int(x) for x in np.linspace(0, n, world + 1).round()]
            lo, hi = cuts[rank], cuts[rank + 1]
            local = torch.from_numpy(_scores(seed, n, levels)[lo:hi]).to(device)
            chosen = select_smallest(local, count)
            head = prefix_split(local, chosen, prefix)
            out.append(((torch.nonzero(chosen).reshape(-1) + lo).cpu().numpy(),
                        (torch.nonzero(head).reshape(-1) + lo).cpu().numpy()))
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_layer_group_selection_over_nccl():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oracle import lrk_oracle as O

    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True, start_method="spawn")
    for i, (seed, n, levels, count, prefix) in enumerate(CASES):
        keys = O.radix_key(_scores(seed, n, levels))
        order = np.lexsort((np.arange(n), keys))
        chosen = np.concatenate([results[r][i][0] for r in range(2)])
        head = np.concatenate([results[r][i][1] for r in range(2)])
        assert set(chosen.tolist()) == set(order[:count].tolist()), f"case {seed}"
        assert set(head.tolist()) == set(order[:prefix].tolist()), f"prefix of case {seed}"


def _layer_cache(device, seed, layers=4, heads=4, dim=64, window=24, groups=2):
    import torch

    from code_for_iclr27_b200.kvcache import PackedCache

    g = torch.Generator().manual_seed(seed)
    cache = PackedCache()
    for _ in range(layers):
        lens = torch.randint(300, 900, (heads,), generator=g).tolist()
        rows = sum(lens)
        keys = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(device)
        values = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(device)
        positions = torch.cat([torch.arange(n, dtype=torch.float32) for n in lens]).to(device)
        cache.add_layer(keys, values, positions, lens, [min(50, n) for n in lens])
    queries = [(torch.randn(window, heads * groups, dim, generator=g) * 2).to(torch.bfloat16).to(device)
               for _ in range(layers)]
    grads = [(torch.randn(heads * groups, dim, generator=g) / 8).to(device) for _ in range(layers)]
    top = min(min(layer.head_lens) for layer in cache.layers)
    qpos = torch.arange(top - window, top, dtype=torch.int64, device=device)
    return cache, queries, grads, qpos, torch.tensor(0.8, device=device)


def _digest(cache, offset):
    import torch

    return {offset + i: (layer.keys.view(torch.int16).cpu().numpy().copy(),
                         layer.positions.cpu().numpy().copy(), list(layer.head_lens), list(layer.prompt_lens))
            for i, layer in enumerate(cache.layers)}


def _audit_worker(rank, world, port, results):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from code_for_iclr27_b200.kvcache import PackedCache

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    try:
        from code_for_iclr27_b200.audit import audit_pass
        from code_for_iclr27_b200.distributed import layer_group_audit_pass

        cache, queries, grads, qpos, margin = _layer_cache(device, 21)
        per = len(cache.layers) // world
        mine = slice(rank * per, (rank + 1) * per)
        part = PackedCache(layers=cache.layers[mine])
        result = layer_group_audit_pass(part, queries[mine], qpos, grads[mine], margin, immediate=40, queued=150)
        out = {"part": _digest(part, rank * per), "evicted": result.evicted}
        if rank == 0:
            full, queries, grads, qpos, margin = _layer_cache(device, 21)
            expected = audit_pass(full, queries, qpos, grads, margin, immediate=40, queued=150)
            out["full"] = _digest(full, 0)
            out["full_evicted"] = expected.evicted
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_layer_group_audit_pass_equals_single_gpu():
    """A 4-layer request split into two 2-layer groups (one per GPU, NCCL
    histogram selection): the same rows are evicted from every layer as by
    the single-GPU audit pass, and the caches end bit-identical."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_audit_worker, args=(2, _free_port(), results), nprocs=2, join=True, start_method="spawn")
    full = results[0]["full"]
    assert results[0]["evicted"] + results[1]["evicted"] == results[0]["full_evicted"] == 40
    for rank in range(2):
        for layer, (keys, positions, lens, prompts) in results[rank]["part"].items():
            f_keys, f_positions, f_lens, f_prompts = full[layer]
            assert lens == f_lens and prompts == f_prompts, f"layer {layer}"
            np.testing.assert_array_equal(positions, f_positions)
            np.testing.assert_array_equal(keys, f_keys)
