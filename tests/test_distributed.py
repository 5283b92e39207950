"""Layer-group selection across ranks (gloo on CPU, world size 2 and 3).

Each rank holds a contiguous slice of one request's score table; the union of
the ranks' choices must equal the single-process bottom-`count` (the oracle's
restatement of torch.topk: smallest by (key, global index)), and queue
prefixes must split the same way."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import lrk_oracle as O


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_scores(seed, n, levels):
    rng = np.random.default_rng(seed)
    if levels:
        return (rng.integers(0, levels, n) / 8).astype(np.float32)
    return rng.random(n, dtype=np.float32)


def worker(rank, world, port, cases, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from code_for_iclr27_b200.distributed import prefix_split, queue_order, select_smallest

        out = []
        for seed, n, levels, count, prefix, cuts in cases:
            scores = torch.from_numpy(make_scores(seed, n, levels))
            lo, hi = cuts[rank], cuts[rank + 1]
            local = scores[lo:hi]
            chosen = select_smallest(local, count)
            order = queue_order(local, chosen)
            head = prefix_split(local, chosen, prefix)
            out.append(((torch.nonzero(chosen).reshape(-1) + lo).tolist(), (order + lo).tolist(),
                        (torch.nonzero(head).reshape(-1) + lo).tolist()))
        results[rank] = out
    finally:
        dist.destroy_process_group()


CASES = [
    # seed, n, tie levels (0: continuous), count, prefix, rank cut points (2 ranks)
    (1, 1000, 0, 300, 50),
    (2, 1000, 4, 300, 120),       # heavy ties at the threshold, split across ranks
    (3, 5000, 40, 2500, 1000),
    (4, 777, 2, 700, 13),
    (5, 4096, 0, 4096, 4096),     # everything
    (6, 3000, 16, 1, 1),
]


@pytest.mark.parametrize("world", [2, 3])
def test_layer_group_selection_matches_single_process(world):
    cases = []
    for seed, n, levels, count, prefix in CASES:
        cuts = [int(x) for x in np.linspace(0, n, world + 1).round()]
        cuts[1] = cuts[1] - 7 * seed  # uneven groups
        cases.append((seed, n, levels, count, prefix, cuts))
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    port = free_port()
    mp.start_processes(worker, args=(world, port, cases, results), nprocs=world, join=True, start_method="spawn")
    for case_index, (seed, n, levels, count, prefix, _) in enumerate(cases):
        scores = make_scores(seed, n, levels)
        keys = O.radix_key(scores)
        order = np.lexsort((np.arange(n), keys))
        expected = set(order[:count].tolist())
        chosen = set()
        queue = []
        head = set()
        for rank in range(world):
            picked, ordered, prefix_rows = results[rank][case_index]
            chosen |= set(picked)
            queue.append(ordered)
            head |= set(prefix_rows)
        assert chosen == expected, f"case {seed}"
        assert head == set(order[:prefix].tolist()), f"prefix of case {seed}"
        # Each rank's queue is its share of the global (key, index) order.
        position = {int(i): p for p, i in enumerate(order)}
        for ordered in queue:
            assert [position[i] for i in ordered] == sorted(position[i] for i in ordered)


def test_radix_keys_order_floats():
    from code_for_iclr27_b200.distributed import radix_keys

    x = torch.tensor([-np.inf, -3.5, -0.0, 0.0, 1e-30, 2.0, np.inf, np.nan], dtype=torch.float32)
    keys = radix_keys(x)
    assert torch.all(keys[1:] > keys[:-1])
    np.testing.assert_array_equal(keys.numpy(), O.radix_key(x.numpy()).astype(np.int64))


def lazy_worker(rank, world, port, cases, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from code_for_iclr27_b200.distributed import lazy_prefix_share, queue_order, select_smallest

        out = []
        for seed, n, levels, count, prefix, batch, cuts in cases:
            scores = torch.from_numpy(make_scores(seed, n, levels))
            local = scores[cuts[rank]:cuts[rank + 1]]
            chosen = select_smallest(local, count)
            queue = local[queue_order(local, chosen)].numpy()  # this rank's queue slots, in queue order
            shares = [lazy_prefix_share(queue, prefix)]
            queue = queue[shares[0]:]
            for _ in range(-(-count // batch) + 1):  # the same number of calls on every rank
                share = lazy_prefix_share(queue, batch)
                shares.append(share)
                queue = queue[share:]
            out.append(shares)
        results[rank] = out
    finally:
        dist.destroy_process_group()


LAZY_CASES = [
    # seed, n, tie levels, queued count, immediate prefix, lazy batch
    (11, 3000, 0, 2000, 300, 256),
    (12, 3000, 3, 2000, 150, 512),   # heavy ties inside batches and across ranks
    (13, 5000, 40, 4100, 0, 2048),
    (14, 999, 0, 999, 999, 7),       # the prefix takes everything
]


@pytest.mark.parametrize("world", [2, 3])
def test_lazy_prefix_shares_match_single_queue(world):
    """Each rank's share of every lazy batch (and of the immediate prefix)
    equals the number of its rows in the corresponding slots of the
    single-process queue (ascending (key, index)); a batch the request-wide
    queue cannot fill gives 0 on every rank."""
    cases = []
    for seed, n, levels, count, prefix, batch in LAZY_CASES:
        cuts = [int(x) for x in np.linspace(0, n, world + 1).round()]
        cuts[1] = cuts[1] - 5 * (seed % 7)  # uneven groups
        cases.append((seed, n, levels, count, prefix, batch, cuts))
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    port = free_port()
    mp.start_processes(lazy_worker, args=(world, port, cases, results), nprocs=world, join=True, start_method="spawn")
    for case_index, (seed, n, levels, count, prefix, batch, cuts) in enumerate(cases):
        scores = make_scores(seed, n, levels)
        order = np.lexsort((np.arange(n), O.radix_key(scores)))[:count]  # the single-process queue
        owner = np.searchsorted(np.asarray(cuts), order, side="right") - 1
        bounds = [(0, prefix)]
        start = prefix
        for _ in range(-(-count // batch) + 1):
            bounds.append((start, start + batch) if start + batch <= count else (start, start))
            start = min(count, start + batch) if start + batch <= count else start
        for rank in range(world):
            expected = [int((owner[a:b] == rank).sum()) for a, b in bounds]
            assert results[rank][case_index] == expected, f"case {seed}, rank {rank}"


def shares_worker(rank, world, port, cases, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from code_for_iclr27_b200.distributed import select_shares

        out = []
        for tables, ks, cuts in cases:
            local = [torch.from_numpy(t[c[rank]:c[rank + 1]].copy()) for t, c in zip(tables, cuts)]
            shares, totals = select_shares(local, ks)
            out.append((shares.tolist(), totals.tolist()))
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_select_shares_many_requests():
    """select_shares over several requests and two questions at once (the
    audit's selected count and immediate prefix), including a request with no
    scores on one rank and k beyond the request's size."""
    world = 3
    rng = np.random.default_rng(5)
    cases = []
    tables = [make_scores(41, 3000, 0), make_scores(42, 5000, 6), make_scores(43, 40, 2)]
    cuts = [[0, 1000, 2000, 3000], [0, 0, 2500, 5000], [0, 13, 40, 40]]
    ks = [[1500, 20], [4999, 4999], [100, 39]]
    cases.append((tables, ks, cuts))
    cases.append(([rng.random(7, dtype=np.float32)], [[3, 0]], [[0, 2, 5, 7]]))
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(shares_worker, args=(world, free_port(), cases, results), nprocs=world, join=True,
                       start_method="spawn")
    for c, (tables, ks, cuts) in enumerate(cases):
        for i, table in enumerate(tables):
            order = np.lexsort((np.arange(table.size), O.radix_key(table)))
            owner = np.searchsorted(np.asarray(cuts[i]), order, side="right") - 1
            for rank in range(world):
                shares, totals = results[rank][c]
                assert totals[i] == table.size
                for q, k in enumerate(ks[i]):
                    assert shares[i][q] == int((owner[:min(k, table.size)] == rank).sum()), (c, i, q, rank)
