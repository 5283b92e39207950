"""The probability stash of lrk_temporal_scores against recomputing.

With room for it in the workspace, the row statistics store every candidate's
probability p and the risk step reads it (risk_stash_kernel); without, the
risk step recomputes p from the logits (risk_vec_kernel / risk_kernel).  Both must give the same scores bit for bit, NaN in the same
places, across the staging modes of the statistics (fp32 weights below 18k
keys, the lane-major packed stage above, the logits dtype for unaligned rows,
f16 and f32 logits), every group count, masked keys and queries, query
chunks, non-finite logits, padded rows and calls of more than 48 segments.
"""
import math

import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C(cuda):
    from code_for_iclr27_b200 import operators

    return operators()


def same(actual, expected):
    import torch

    actual, expected = actual.cpu(), expected.cpu()
    assert torch.equal(torch.isnan(actual), torch.isnan(expected))
    equal = torch.nan_to_num(actual, nan=0.0).view(torch.int32) == torch.nan_to_num(expected, nan=0.0).view(
        torch.int32)
    assert bool(equal.all()), f"{int((~equal).sum())} of {equal.numel()} scores differ"


CASES = [
    # dtype, window, groups, length, first, last, padded row stride, query chunk, masked queries
    ("bf16", 250, 4, 34880, 32768, 34848, 34880, 80, 0),   # configs[1] head: packed stage
    ("bf16", 250, 8, 8192, 0, 8160, 8192, 42, 3),           # configs[4]-like, every row a candidate, fp32 weights
    ("bf16", 37, 1, 20011, 100, 19000, 20011, 0, 0),        # unaligned rows: logits-dtype stage
    ("bf16", 60, 2, 25001, 5, 24990, 25008, 7, 5),          # padded aligned rows, odd length
    ("f16", 33, 4, 3001, 17, 2990, 3001, 0, 2),
    ("f32", 20, 8, 1030, 0, 1029, 1030, 6, 0),
    ("bf16", 250, 4, 4096, 0, 4064, 4096, 250, 0),          # configs[0] head
]


@pytest.mark.parametrize("dtype_name,window,groups,length,first,last,stride,chunk,masked", CASES)
def test_probability_stash_equals_recomputed_risk(C, cuda, dtype_name, window, groups, length, first, last, stride, chunk,
                                            masked):
    import torch

    dtype = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dtype_name]
    g = torch.Generator().manual_seed(length + window * 7 + groups)
    heads = 3
    logits, pvs, kpos, firsts, lasts = [], [], [], [], []
    for h in range(heads):
        n = length - 3 * h
        full = (torch.randn(window, groups, stride, generator=g) * 2 * math.sqrt(128)).to(dtype)
        if h == 1:
            full[window // 2, 0, first + 3] = float("nan")  # a non-finite candidate logit
            full[1, groups - 1, min(n - 1, first + 10)] = float("inf")
        logits.append(full.to(cuda)[:, :, :n])
        pvs.append(torch.randn(groups, n, generator=g).to(cuda))
        kpos.append(torch.arange(n, dtype=torch.float32, device=cuda))
        firsts.append(first)
        lasts.append(min(last, n - 1))
    qpos = torch.arange(length - window, length, dtype=torch.int64, device=cuda) - 50
    if masked:
        qpos[:masked] = -1  # every key masked for these queries
    margin = torch.tensor([0.8], device=cuda)
    chunks = [chunk] * heads
    stash = C.temporal_scores(logits, pvs, kpos, firsts, lasts, qpos, margin, 1 / math.sqrt(128), 1e-6, chunks,
                              probability_stash=True)
    recomputed = C.temporal_scores(logits, pvs, kpos, firsts, lasts, qpos, margin, 1 / math.sqrt(128), 1e-6, chunks,
                                   probability_stash=False)
    same(stash, recomputed)


def test_probability_stash_many_segments(C, cuda):
    """60 segments (two tables of 48), short heads of assorted lengths."""
    import torch

    g = torch.Generator().manual_seed(3)
    logits, pvs, kpos, firsts, lasts = [], [], [], [], []
    for h in range(60):
        n = 40 + 29 * h
        logits.append((torch.randn(16, 4, n, generator=g) * 20).to(torch.bfloat16).to(cuda))
        pvs.append(torch.randn(4, n, generator=g).to(cuda))
        kpos.append(torch.arange(n, dtype=torch.float32, device=cuda))
        firsts.append(n // 3)
        lasts.append(n - 2)
    qpos = torch.arange(900, 916, dtype=torch.int64, device=cuda)
    margin = torch.tensor([1.1], device=cuda)
    args = (logits, pvs, kpos, firsts, lasts, qpos, margin, 0.125, 1e-6, [5] * 60)
    same(C.temporal_scores(*args, probability_stash=True), C.temporal_scores(*args, probability_stash=False))
