"""GPU parity of lrk_scores_from_keys (_C.scores_from_keys): the logits GEMM
and the row statistics in one tcgen05 kernel must give the scores of
score_table_fused (logits from cuBLAS / lrk_logits, then lrk_temporal_scores)
bit for bit, on heads of odd and even key counts, ragged query tiles, sorted
and unsorted key positions, and partially visible rows."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def assert_bitwise(actual, expected):
    import torch

    actual, expected = actual.cpu(), expected.cpu()
    assert actual.shape == expected.shape
    assert torch.equal(torch.isnan(actual), torch.isnan(expected)), "NaN pattern differs"
    same = torch.nan_to_num(actual) == torch.nan_to_num(expected)
    assert bool(same.all()), f"{int((~same).sum())} of {same.numel()} scores differ"


def build(seed, lens_per_layer, prompts, dim, groups, window, shuffled=(), device="cuda"):
    """A packed cache (positions 0..n-1 per head, or a permutation for the
    (layer, head) pairs in `shuffled`), queries, margin gradients and query
    positions inside the key range (rows see different prefixes)."""
    import torch

    from code_for_iclr27_b200.kvcache import PackedCache

    g = torch.Generator().manual_seed(seed)
    cache = PackedCache()
    heads = len(lens_per_layer[0])
    for layer, lens in enumerate(lens_per_layer):
        rows = sum(lens)
        keys = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(device)
        values = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(device)
        parts = []
        for head, n in enumerate(lens):
            pos = torch.arange(n, dtype=torch.float32)
            if (layer, head) in shuffled:
                pos = pos[torch.randperm(n, generator=g)]
            parts.append(pos)
        cache.add_layer(keys, values, torch.cat(parts).to(device), lens, [min(p, n) for p, n in zip(prompts, lens)])
    queries = [(torch.randn(window, heads * groups, dim, generator=g) * 2).to(torch.bfloat16).to(device)
               for _ in lens_per_layer]
    grads = [(torch.randn(heads * groups, dim, generator=g) / math.sqrt(dim)).to(device) for _ in lens_per_layer]
    top = min(min(lens) for lens in lens_per_layer)
    qpos = torch.arange(top - window - 3, top - 3, dtype=torch.int64).to(device)
    margin = torch.tensor(0.9, device=device)
    return cache, queries, grads, qpos, margin


CASES = [
    # dim, groups, window, per-layer head lengths, prompt rows per head, unsorted heads
    (128, 4, 37, [[300, 301, 1000, 1537], [129, 640, 2047, 255]], [40, 0, 100, 10], ()),
    (64, 8, 16, [[129, 256, 511, 77], [1000, 999, 130, 131]], [0, 20, 5, 0], ()),
    (128, 2, 70, [[700, 701, 702, 703]], [0, 0, 0, 0], ((0, 1), (0, 2))),
    (64, 1, 250, [[3000, 2999]], [100, 2000], ((0, 0),)),
]


@pytest.mark.parametrize("dim,groups,window,lens,prompts,shuffled", CASES)
def test_from_keys_equals_fused_table(cuda, dim, groups, window, lens, prompts, shuffled):
    from code_for_iclr27_b200.audit import score_table_from_keys, score_table_fused

    cache, queries, grads, qpos, margin = build(11 + dim + groups, lens, prompts, dim, groups, window, shuffled)
    for chunk in (250, 7):
        a = score_table_fused(cache, queries, qpos, grads, margin, protect_recent=8, query_chunk_size=chunk)
        b = score_table_from_keys(cache, queries, qpos, grads, margin, protect_recent=8, query_chunk_size=chunk)
        assert a.segments == b.segments and a.cumulative_ends == b.cumulative_ends
        assert_bitwise(b.scores, a.scores)
    assert timeouts() == 0


def timeouts():
    import ctypes

    from code_for_iclr27_b200 import abi

    count = ctypes.c_uint(0)
    abi.check(abi.library().lrk_scores_from_keys_timeouts(ctypes.byref(count)))
    return count.value


def test_from_keys_equals_fused_table_at_configs1_shape(cuda):
    """Two layers at configs[1] shape: 8 KV heads of ~34.8k rows (odd and
    even counts), D = 128, 250 queries x 4 groups, 32768 prompt rows per
    head: bit-identical scores."""
    from code_for_iclr27_b200.audit import score_table_from_keys, score_table_fused

    rng = np.random.default_rng(5)
    lens = [[32768 + int(n) for n in rng.integers(1800, 2200, 8)] for _ in range(2)]
    cache, queries, grads, qpos, margin = build(5, lens, [32768] * 8, 128, 4, 250)
    a = score_table_fused(cache, queries, qpos, grads, margin)
    b = score_table_from_keys(cache, queries, qpos, grads, margin)
    assert a.segments == b.segments
    assert_bitwise(b.scores, a.scores)
    assert timeouts() == 0


def test_from_keys_rejects_bad_calls(cuda):
    import torch

    from code_for_iclr27_b200 import operators

    C = operators()
    keys = torch.zeros(100, 128, dtype=torch.bfloat16, device=cuda)
    queries = torch.zeros(5, 8, 128, dtype=torch.bfloat16, device=cuda)
    projected = torch.zeros(4, 100, device=cuda)
    positions = torch.zeros(100, device=cuda)
    qpos = torch.arange(5, dtype=torch.int64, device=cuda)
    margin = torch.ones(1, device=cuda)
    good = [0, 0, 0, 100, 10, 90, 0]
    C.scores_from_keys([keys], [queries], [projected], [positions], [good], 4, qpos, margin, 0.1, 1e-6)
    for bad in ([0, 0, 0, 101, 10, 90, 0], [0, 2, 0, 100, 10, 90, 0], [0, 0, 0, 100, 90, 10, 0], [1, 0, 0, 100, 10, 90, 0]):
        with pytest.raises(RuntimeError):
            C.scores_from_keys([keys], [queries], [projected], [positions], [bad], 4, qpos, margin, 0.1, 1e-6)
    with pytest.raises(RuntimeError):  # head dimension 96
        k96 = torch.zeros(100, 96, dtype=torch.bfloat16, device=cuda)
        C.scores_from_keys([k96], [queries[..., :96].contiguous()], [projected], [positions], [good], 4, qpos, margin,
                           0.1, 1e-6)
