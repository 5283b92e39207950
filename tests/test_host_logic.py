"""Host-side queue logic (no GPU): ArrayReferences.groups and slicing follow
the reference queue's contract (selection.py, ArrayReferences)."""
import numpy as np

from code_for_iclr27_b200.selection import ArrayReferences, KVReference


def naive_groups(refs):
    out = {}
    for segment in sorted(set(refs.segments.tolist())):
        layer, head = refs.coordinates[segment]
        out[(int(layer), int(head))] = np.sort(refs.positions[refs.segments == segment])
    return out


def test_groups_matches_per_segment_sort():
    rng = np.random.default_rng(3)
    coordinates = [(layer, head) for layer in range(4) for head in range(8)]
    for n in (0, 1, 7, 512, 2048):
        segments = rng.integers(0, len(coordinates), n)
        positions = rng.integers(0, 40000, n)
        refs = ArrayReferences(rng.random(n, dtype=np.float32), segments, positions, coordinates)
        got, want = refs.groups(), naive_groups(refs)
        assert list(got) == list(want)
        for key in want:
            np.testing.assert_array_equal(got[key], want[key])


def test_slicing_and_items():
    coordinates = [(0, 0), (0, 1), (3, 2)]
    refs = ArrayReferences(np.array([0.5, 0.25, 0.125], np.float32), [2, 0, 1], [10, 20, 30], coordinates)
    assert refs[0] == KVReference(0.5, 3, 2, 10)
    tail = refs[1:]
    assert len(tail) == 2 and tail[0] == KVReference(0.25, 0, 0, 20)
    assert list(tail.groups()) == [(0, 0), (0, 1)]


def test_reference_query_view_has_the_reference_strides():
    """reference_query_view gives every head the layout of the reference's
    mapped_queries (scoring.py:260: a permuted slice of the [1, heads * G, W, D]
    history that history.py:55 concatenates, strides (D, W*D, 1)) whatever the
    input's layout -- with one group too, where a permuted view that torch
    already counts as contiguous would let torch.matmul fold it into one GEMM."""
    import torch

    from code_for_iclr27_b200.audit import reference_query_view

    for window, heads, groups, dim in ((250, 8, 4, 128), (40, 2, 1, 64), (9, 1, 1, 64), (37, 1, 8, 128)):
        layer = torch.randn(window, heads * groups, dim).to(torch.bfloat16)
        # The reference's history: one [1, heads*G, 1, D] query per step, concatenated.
        history = torch.cat([layer[w].reshape(1, heads * groups, 1, dim) for w in range(window)], dim=2)
        per_head = layer.reshape(window, heads, groups, dim).transpose(0, 1).contiguous()
        for head in range(heads):
            expected = history[0, head * groups:(head + 1) * groups].permute(1, 0, 2)
            for source in (layer[:, head * groups:(head + 1) * groups], per_head[head]):
                view = reference_query_view(source)
                assert view.stride() == expected.stride() == (dim, window * dim, 1)
                assert torch.equal(view, expected)
