"""lrk_temporal_scores_static: fused scoring without any device allocation.

Some callers cannot allocate device memory: a host whose GPU memory is all
handed out by another allocator (an inference engine that reserves the
device's memory at start-up and forbids further cudaMalloc), or a plain C host
(cgo, JNI) that has no device allocator of its own.  For them the entry point
takes its scratch from a fixed-size array compiled into liblrk instead of a
caller-provided workspace.  This test calls it through the C ABI,
three times in a row on different inputs, and checks each result against the
workspace entry point (lrk_temporal_scores) bit for bit: both run the same
kernels on the same data, so the scores must be the same floats, NaN in the
same places.  The static path compares key positions where the workspace path
uses its visible-prefix table, so one call masks keys (query positions inside
the key range), and that call has 60 segments, so the scratch rows of a second
segment table (the kernels take 48 segments per launch) are exercised too.  It
also checks that a call larger than the static scratch is refused.

It lives in its own file so that pytest collects it last.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def assert_same_scores(actual, expected):
    """Bit equality of float32 scores (NaN payloads aside: NaN where the other is NaN)."""
    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    assert actual.shape == expected.shape
    nan = np.isnan(expected)
    assert (np.isnan(actual) == nan).all()
    assert (actual[~nan].view(np.uint32) == expected[~nan].view(np.uint32)).all()


def make_call(seed, heads, window, groups, lengths, device, query_start=10 ** 6):
    """Inputs of one scoring call: bf16 logits, projected values, positions."""
    import torch

    from code_for_iclr27_b200 import abi

    g = torch.Generator().manual_seed(seed)
    tensors, outputs = [], []
    segments = (abi.ScoreSegment * heads)()
    for h in range(heads):
        length = lengths[h]
        logits = (torch.randn(window, groups, length, generator=g) * 2 * math.sqrt(128)).to(torch.bfloat16).to(device)
        pv = torch.randn(groups, length, generator=g).to(device)
        kpos = torch.arange(length, dtype=torch.float32, device=device)
        first, last = length // 4, length - 3
        out = torch.full((last - first,), -1.0, device=device)
        segments[h] = abi.ScoreSegment(logits.data_ptr(), pv.data_ptr(), length, kpos.data_ptr(), length, first, last,
                                       out.data_ptr(), length)
        tensors += [logits, pv, kpos]
        outputs.append(out)
    qpos = torch.arange(query_start, query_start + window, dtype=torch.int64, device=device)
    margin = torch.tensor([0.8], device=device)
    tensors += [qpos, margin]
    return segments, outputs, qpos, margin, tensors


def run(lib, call, window, groups, static, device):
    import torch

    from code_for_iclr27_b200 import abi

    segments, outputs, qpos, margin, _ = call
    stream = torch.cuda.current_stream(device).cuda_stream
    if static:
        status = lib.lrk_temporal_scores_static(segments, len(outputs), abi.BF16, qpos.data_ptr(), window, groups,
                                                0.125, margin.data_ptr(), 1e-6, stream)
    else:
        size = lib.lrk_temporal_scores_workspace_bytes(len(outputs), window, groups)
        workspace = torch.empty(size, dtype=torch.uint8, device=device)
        status = lib.lrk_temporal_scores(segments, len(outputs), abi.BF16, qpos.data_ptr(), window, groups, 0.125,
                                         margin.data_ptr(), 1e-6, workspace.data_ptr(), size, stream)
    abi.check(status)
    torch.cuda.synchronize(device)
    return [o.cpu().numpy().copy() for o in outputs]


def test_static_scratch_matches_workspace_entry_point():
    import torch

    from code_for_iclr27_b200 import abi

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    device = torch.device("cuda:0")
    lib = abi.library()
    # (seed, queries, groups, key counts, first query position): the third
    # call has 60 segments, two segment tables of the scoring kernels, and its
    # query positions 1000..1015 mask the later keys of its longer heads.
    calls = [(1, 60, 4, [700, 1300, 257], 10 ** 6), (2, 33, 8, [400, 2050, 90, 999, 3001], 10 ** 6),
             (3, 16, 4, [64 + 37 * i for i in range(60)], 1000)]
    inputs = [make_call(seed, len(lengths), window, groups, lengths, device, start)
              for seed, window, groups, lengths, start in calls]
    expected = [run(lib, call, window, groups, static=False, device=device)
                for call, (_, window, groups, _, _) in zip(inputs, calls)]
    for call in inputs:
        for out in call[1]:
            out.fill_(-1.0)
    # Calls in a row on the shared static scratch.
    for call, (_, window, groups, _, _), want in zip(inputs, calls, expected):
        got = run(lib, call, window, groups, static=True, device=device)
        for g, w in zip(got, want):
            assert_same_scores(g, w)


def test_static_scratch_limit_is_enforced():
    import torch

    from code_for_iclr27_b200 import abi

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    device = torch.device("cuda:0")
    lib = abi.library()
    call = make_call(3, 1, 250, 4, [300], device)
    segments, outputs, qpos, margin, _ = call
    # 1100 segments x 250 queries x 4 groups = 1.1M rows > LRK_STATIC_SCORE_ROWS.
    many = (abi.ScoreSegment * 1100)(*([segments[0]] * 1100))
    status = lib.lrk_temporal_scores_static(many, 1100, abi.BF16, qpos.data_ptr(), 250, 4, 0.125, margin.data_ptr(),
                                            1e-6, torch.cuda.current_stream(device).cuda_stream)
    assert status == abi.ERR_INVALID
    assert "LRK_STATIC_SCORE_ROWS" in lib.lrk_last_error().decode()
    assert abi.STATIC_SCORE_ROWS == 262144
