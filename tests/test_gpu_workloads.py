"""The side measurements bench.py reports (configs[2] batch_append, configs[3]
recall) run end to end at small sizes, and the recall path moves the right
bytes."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_recall_measurement_small(cuda):
    from code_for_iclr27_b200.workloads import measure_recall

    r = measure_recall(cuda, requests=2, pool_rows=70_000, recall_rows=64, layers=4, heads=2, cache_rows_per_head=100,
                       events=3)
    assert r["event_zero_copy_us"] > 0 and r["merge_us_per_request_event"] > 0
    assert len(r["sweep"]) == 5 and all(e["zero_copy_gather_GBps"] > 0 for e in r["sweep"])
    assert r["pinned_h2d_peak_GBps"] > 1


def test_batch_append_measurement_small(cuda):
    from code_for_iclr27_b200.workloads import measure_batch_append

    r = measure_batch_append(cuda, requests=3, layers=2, heads=2, generated=10, steps=2)
    assert r["us_per_step"] > 0 and r["GBps"] > 0


def test_host_pool_gather_matches_pool(cuda):
    """The workload's registered pool read by lrk_gather_rows returns the pool's rows."""
    import torch

    from code_for_iclr27_b200 import abi
    from code_for_iclr27_b200.workloads import _HostPool

    pool = _HostPool(5000, 128, seed=1)
    try:
        chosen = np.random.default_rng(2).choice(5000, 100, replace=False)
        idx = torch.from_numpy(chosen).to(cuda)
        out = torch.empty(100, 2, 128, dtype=torch.bfloat16, device=cuda)
        abi.check(abi.library().lrk_gather_rows(pool.device_address, 5000, pool.row_bytes, idx.data_ptr(), 100,
                                                out.data_ptr(), torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), pool.array[chosen])
    finally:
        pool.close()
