"""GPU selection: _C.topk_smallest against torch.topk on CUDA (ties
included), _C.refine / selection.refine_arrays against the oracle and against
refine_arrays' algorithm driven by torch.topk on CUDA."""
from types import SimpleNamespace

import numpy as np
import pytest

from oracle import lrk_oracle as O

pytestmark = pytest.mark.gpu

TOPK_CASES = [(1, 1), (40, 1), (40, 2), (40, 7), (40, 32), (40, 33), (40, 40), (300, 17), (300, 100), (300, 129),
              (5000, 4096), (5000, 4097), (5000, 31), (99999, 20), (99999, 5000), (100000, 20), (150000, 31),
              (150000, 70000), (600000, 300000), (200000, 2), (1000000, 32), (1000000, 33), (4000000, 5)]


@pytest.fixture(scope="module")
def C(cuda):
    from code_for_iclr27_b200 import operators

    return operators()


@pytest.mark.parametrize("n,k", TOPK_CASES)
@pytest.mark.parametrize("distinct", [3, 50, None])
def test_topk_matches_torch_cuda(C, cuda, n, k, distinct):
    import torch

    g = torch.Generator().manual_seed(n * 7 + k)
    if distinct is None:
        x = torch.rand(n, generator=g)
    else:
        x = torch.randint(0, distinct, (n,), generator=g).float() / 4
    x = x.to(cuda)
    values, indices = C.topk_smallest(x, k)
    tv, ti = torch.topk(x, k, largest=False, sorted=True)
    assert torch.equal(indices, ti), f"tie order differs from torch.topk for n={n} k={k}"
    assert torch.equal(values, tv)
    ov, oi = O.topk_smallest(x.cpu().numpy(), k)
    np.testing.assert_array_equal(oi, ti.cpu().numpy())


def torch_topk(device):
    import torch

    def topk(x, k):
        values, indices = torch.topk(torch.as_tensor(x, device=device), k, largest=False, sorted=True)
        return values.cpu().numpy(), indices.cpu().numpy()

    return topk


def make_tables(lengths, tie_levels, seed, device):
    """Raw scores and their Pool7 refinement, laid out like a score table."""
    import torch

    from code_for_iclr27_b200 import operators

    g = torch.Generator().manual_seed(seed)
    n = sum(lengths)
    if tie_levels:
        raw = torch.randint(0, tie_levels, (n,), generator=g).float() / 8
    else:
        raw = torch.rand(n, generator=g)
    raw = raw.to(device)
    ends = np.cumsum(lengths)
    bounds = torch.tensor(np.concatenate(([0], ends)), dtype=torch.int64, device=device)
    pooled = operators().pool(raw, bounds, max(lengths), 7)
    segments = [SimpleNamespace(layer=s // 8, head=s % 8, position_start=int(s % 5) * 3, count=int(c))
                for s, c in enumerate(lengths)]
    allocation = SimpleNamespace(scores=raw, segments=segments, cumulative_ends=[int(e) for e in ends])
    refinement = SimpleNamespace(scores=pooled, segments=segments, cumulative_ends=[int(e) for e in ends])
    return allocation, refinement


REFINE_CASES = [
    # (segment lengths, tie levels, count)
    ([50] * 6, 0, 120),
    ([50] * 6, 4, 120),
    ([4064] * 16, 64, 30000),      # config-0-like: many ties, large quotas
    ([2226] * 32, 200, 40000),
    ([3, 1, 40, 17, 900, 5], 3, 500),
    ([40] * 30, 10, 300),          # quotas around 10: the bitonic path
    ([120000, 10, 500], 20, 60000),  # one long segment
    ([150000, 64, 64], 40, 40),      # small quotas in a long segment
    ([7] * 3, 2, 21),
    ([1000] * 4, 5, 1),
    ([300000, 250000, 60000], 50, 450000),  # > 524k scores: the multi-CTA count scan
]


@pytest.mark.parametrize("lengths,ties,count", REFINE_CASES)
def test_refine_matches_oracle_and_torch(C, cuda, lengths, ties, count):
    import torch

    from code_for_iclr27_b200.selection import refine_arrays

    allocation, refinement = make_tables(lengths, ties, len(lengths) * 31 + count, cuda)
    references, changed, changed_heads = refine_arrays(allocation, refinement, count)
    raw, pooled = allocation.scores.cpu().numpy(), refinement.scores.cpu().numpy()
    starts = [s.position_start for s in allocation.segments]
    ends = allocation.cumulative_ends
    for topk in (None, torch_topk(cuda)):
        values, segments, positions, oc, oh = O.refine(raw, pooled, ends, starts, count, topk=topk)
        np.testing.assert_array_equal(references.scores, values)
        np.testing.assert_array_equal(references.segments, segments)
        np.testing.assert_array_equal(references.positions, positions)
        assert (changed, changed_heads) == (oc, oh)
    assert len(references) == count
    groups = references[: count // 2].groups()
    for (layer, head), positions in groups.items():
        assert np.all(np.diff(positions) > 0)


def test_refine_count_zero_and_full(C, cuda):
    from code_for_iclr27_b200.selection import refine_arrays

    allocation, refinement = make_tables([30, 40], 5, 3, cuda)
    references, changed, heads = refine_arrays(allocation, refinement, 0)
    assert len(references) == 0 and changed == 0 and heads == 0
    references, changed, heads = refine_arrays(allocation, refinement, 10 ** 9)
    assert len(references) == 70 and changed == 0


def test_refine_through_c_abi(cuda):
    import torch

    from code_for_iclr27_b200 import abi

    allocation, refinement = make_tables([500, 300, 700], 9, 11, cuda)
    n, count = 1500, 900
    ends = torch.tensor(allocation.cumulative_ends, dtype=torch.int64, device=cuda)
    starts = torch.tensor([s.position_start for s in allocation.segments], dtype=torch.int64, device=cuda)
    lib = abi.library()
    size = lib.lrk_refine_workspace_bytes(n, 3)
    workspace = torch.empty(size, dtype=torch.uint8, device=cuda)
    values = torch.empty(count, device=cuda)
    segment_ids = torch.empty(count, dtype=torch.int64, device=cuda)
    positions = torch.empty(count, dtype=torch.int64, device=cuda)
    stats = torch.empty(2, dtype=torch.int64, device=cuda)
    abi.check(lib.lrk_refine(allocation.scores.data_ptr(), refinement.scores.data_ptr(), n, ends.data_ptr(),
                             starts.data_ptr(), 3, count, workspace.data_ptr(), size, values.data_ptr(),
                             segment_ids.data_ptr(), positions.data_ptr(), stats.data_ptr(),
                             torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ev, es, ep, ec, eh = O.refine(allocation.scores.cpu().numpy(), refinement.scores.cpu().numpy(),
                                  allocation.cumulative_ends, starts.cpu().numpy(), count)
    np.testing.assert_array_equal(values.cpu().numpy(), ev)
    np.testing.assert_array_equal(segment_ids.cpu().numpy(), es)
    np.testing.assert_array_equal(positions.cpu().numpy(), ep)
    assert stats.cpu().tolist() == [ec, eh]
    # Too small a workspace is rejected before any launch.
    assert lib.lrk_refine(allocation.scores.data_ptr(), refinement.scores.data_ptr(), n, ends.data_ptr(),
                          starts.data_ptr(), 3, count, workspace.data_ptr(), size - 4096, values.data_ptr(),
                          segment_ids.data_ptr(), positions.data_ptr(), stats.data_ptr(), 0) == abi.ERR_WORKSPACE
