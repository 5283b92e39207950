"""Layer-group selection over NCCL on 2 GPUs (one process per GPU): the ranks'
union equals the single-process bottom-count, ties broken by global index.
Skipped with fewer than 2 GPUs."""
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
