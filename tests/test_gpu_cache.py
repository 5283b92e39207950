"""PackedCache bookkeeping on the GPU: remove_positions and lazy eviction
against the oracle's compaction (cache.py:92-180, controller.py:57-70)."""
import numpy as np
import pytest

from oracle import lrk_oracle as O

pytestmark = pytest.mark.gpu


def make_cache(seed, layers=3, heads=4, dim=16):
    import torch

    from code_for_iclr27_b200.kvcache import PackedCache

    g = torch.Generator().manual_seed(seed)
    cache, ident = PackedCache(), 0
    for _ in range(layers):
        lens = torch.randint(50, 400, (heads,), generator=g).tolist()
        rows = sum(lens)
        keys = torch.randn(rows, dim, generator=g).to(torch.bfloat16).cuda()
        values = torch.randn(rows, dim, generator=g).to(torch.bfloat16).cuda()
        positions = torch.arange(ident, ident + rows, dtype=torch.float32).cuda()  # unique row identities
        ident += rows
        cache.add_layer(keys, values, positions, lens, [min(30, n) for n in lens])
    return cache


def bits(tensor):
    import torch

    return tensor.cpu().view(torch.int16).numpy().copy()


def host_copy(cache):
    return [(bits(layer.keys), bits(layer.values), layer.positions.cpu().numpy().copy(), list(layer.head_lens),
             list(layer.prompt_lens)) for layer in cache.layers]


def test_remove_positions_matches_oracle():
    cache = make_cache(1)
    before = host_copy(cache)
    rng = np.random.default_rng(1)
    removals = {}
    for layer_index, layer in enumerate(cache.layers):
        for head, length in enumerate(layer.head_lens):
            if (layer_index + head) % 3 == 0:
                continue
            picks = rng.integers(0, length, 12)
            removals[(layer_index, head)] = np.concatenate([picks, picks[:3]])  # duplicates count once
    removals[(0, 3)] = []  # an empty entry is allowed
    removed = cache.remove_positions(removals)
    total = 0
    for layer_index, (keys, values, positions, lens, prompts) in enumerate(before):
        bounds = np.concatenate(([0], np.cumsum(lens)))
        rows, new_lens, new_prompts = [], list(lens), list(prompts)
        for head in range(len(lens)):
            picks = np.unique(np.asarray(removals.get((layer_index, head), []), dtype=np.int64))
            rows.append(bounds[head] + picks)
            new_lens[head] -= picks.size
            new_prompts[head] -= int(np.sum(picks < prompts[head]))
            total += picks.size
        k, v, p = O.compact(keys, values, positions, np.sort(np.concatenate(rows)))
        layer = cache.layers[layer_index]
        np.testing.assert_array_equal(bits(layer.keys), k)
        np.testing.assert_array_equal(bits(layer.values), v)
        np.testing.assert_array_equal(layer.positions.cpu().numpy(), p)
        assert layer.head_lens == new_lens and layer.prompt_lens == new_prompts
        np.testing.assert_array_equal(layer.cumulative.cpu().numpy(), np.concatenate(([0], np.cumsum(new_lens))))
    assert removed == total


def test_remove_positions_rejects_out_of_range_without_change():
    cache = make_cache(2)
    before = host_copy(cache)
    length = cache.layers[1].head_lens[2]
    with pytest.raises(IndexError):
        cache.remove_positions({(0, 0): [1, 2], (1, 2): [0, length]})
    after = host_copy(cache)
    for a, b in zip(before, after):
        for x, y in zip(a, b):
            np.testing.assert_array_equal(np.asarray(x), np.asarray(y))


def test_lazy_eviction_removes_audit_time_identities():
    """A queue of audit-time (layer, head, position) references evicted in
    three prefixes removes exactly those rows, although every prefix after the
    first sees positions shifted by earlier removals."""
    from code_for_iclr27_b200.audit import evict_prefix
    from code_for_iclr27_b200.selection import ArrayReferences

    cache = make_cache(3)
    rng = np.random.default_rng(3)
    coordinates = [(l, h) for l in range(len(cache.layers)) for h in range(len(cache.layers[0].head_lens))]
    segments, positions = [], []
    for s, (l, h) in enumerate(coordinates):
        picks = rng.choice(cache.layers[l].head_lens[h], 20, replace=False)
        segments += [s] * picks.size
        positions += picks.tolist()
    order = rng.permutation(len(segments))
    queue = ArrayReferences(rng.random(len(order), dtype=np.float32), np.asarray(segments)[order],
                            np.asarray(positions)[order], coordinates)
    identities = {}
    for s, (l, h) in enumerate(coordinates):
        layer = cache.layers[l]
        start = int(layer.bounds()[h])
        identities[s] = layer.positions.cpu().numpy().reshape(-1)[start:start + layer.head_lens[h]]
    gone = {float(identities[s][p]) for s, p in zip(queue.segments.tolist(), queue.positions.tolist())}
    expected = {l: set(cache.layers[l].positions.cpu().numpy().reshape(-1).tolist()) for l in range(len(cache.layers))}
    removed_at_audit = {}
    for count in (50, 70, len(queue) - 120):
        queue, removed_at_audit = evict_prefix(cache, queue, removed_at_audit, count)
    assert len(queue) == 0
    for l, layer in enumerate(cache.layers):
        remaining = set(layer.positions.cpu().numpy().reshape(-1).tolist())
        assert remaining == expected[l] - gone
