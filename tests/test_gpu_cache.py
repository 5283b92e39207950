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


def assert_same_cache(a, b):
    for x, y in zip(host_copy(a), host_copy(b)):
        for u, v in zip(x, y):
            np.testing.assert_array_equal(np.asarray(u), np.asarray(v))
    for x, y in zip(a.layers, b.layers):
        np.testing.assert_array_equal(x.cumulative.cpu().numpy(), y.cumulative.cpu().numpy())


def device_references(cache, seed, per_head=17, skip=3):
    """Distinct (segment, position) references in a shuffled queue order, as
    int64 CUDA tensors, over the cache's (layer, head) segments (every
    skip-th segment gets none)."""
    import torch

    rng = np.random.default_rng(seed)
    coordinates = [(l, h) for l in range(len(cache.layers)) for h in range(len(cache.layers[0].head_lens))]
    segments, positions = [], []
    for s, (l, h) in enumerate(coordinates):
        if s % skip == 1:
            continue
        picks = rng.choice(cache.layers[l].head_lens[h], per_head, replace=False)
        segments += [s] * picks.size
        positions += picks.tolist()
    order = rng.permutation(len(segments))
    seg = torch.as_tensor(np.asarray(segments)[order]).cuda()
    pos = torch.as_tensor(np.asarray(positions)[order]).cuda()
    return coordinates, seg, pos


@pytest.mark.parametrize("seed", [4, 5])
def test_remove_selected_equals_remove_positions(seed):
    """Device-planned eviction (rows formed, sorted and counted on the device,
    one multi-layer compaction call) leaves the cache bit-identical to the
    host-planned remove_positions, prompt rows included."""
    cache_a, cache_b = make_cache(seed, layers=4, heads=8), make_cache(seed, layers=4, heads=8)
    coordinates, seg, pos = device_references(cache_a, seed)
    removals = {}
    for s, p in zip(seg.cpu().numpy().tolist(), pos.cpu().numpy().tolist()):
        removals.setdefault(tuple(coordinates[s]), []).append(p)
    removed_b = cache_b.remove_positions(removals)
    removed_a = cache_a.remove_selected(coordinates, seg, pos)
    assert removed_a == removed_b == seg.numel()
    assert_same_cache(cache_a, cache_b)


def test_remove_selected_rejects_out_of_range_and_counts_duplicates_once():
    import torch

    cache = make_cache(6)
    before = host_copy(cache)
    coordinates, seg, pos = device_references(cache, 6, per_head=5)
    bad = pos.clone()
    bad[len(bad) // 2] = cache.layers[coordinates[int(seg[len(bad) // 2])][0]].head_lens[
        coordinates[int(seg[len(bad) // 2])][1]]
    with pytest.raises(IndexError):
        cache.remove_selected(coordinates, seg, bad)
    for a, b in zip(before, host_copy(cache)):
        for x, y in zip(a, b):
            np.testing.assert_array_equal(np.asarray(x), np.asarray(y))
    twin = make_cache(6)
    doubled_seg, doubled_pos = torch.cat([seg, seg[:4]]), torch.cat([pos, pos[:4]])
    assert cache.remove_selected(coordinates, doubled_seg, doubled_pos) == seg.numel()
    twin.remove_selected(coordinates, seg, pos)
    assert_same_cache(cache, twin)


def test_audit_pass_evicts_like_the_host_composition():
    """audit_pass (device-planned eviction, queue copied back while the
    compactions run) against refine_arrays + groups + remove_positions on an
    identical cache: same queue, same counters, same cache afterwards."""
    import math

    import torch

    from code_for_iclr27_b200.audit import audit_pass, pool_table, score_table_fused
    from code_for_iclr27_b200.selection import refine_arrays

    caches = [make_cache(7, layers=3, heads=4, dim=64) for _ in range(2)]
    g = torch.Generator().manual_seed(7)
    window, groups = 16, 2
    queries = [(torch.randn(window, 4 * groups, 64, generator=g) * 2).to(torch.bfloat16).cuda() for _ in range(3)]
    gradients = [(torch.randn(4 * groups, 64, generator=g) / math.sqrt(64)).cuda() for _ in range(3)]
    top = max(sum(layer.head_lens) for layer in caches[0].layers) * 3 + 10
    qpos = torch.arange(top - window, top, dtype=torch.int64).cuda()
    margin = torch.tensor([1.0]).cuda()
    result = audit_pass(caches[0], queries, qpos, gradients, margin, immediate=40, queued=100, protect_recent=8)
    table = score_table_fused(caches[1], queries, qpos, gradients, margin, 8)
    references, changed, changed_heads = refine_arrays(table, pool_table(table, 7), 140)
    removed = caches[1].remove_positions(references[:40].groups())
    assert result.evicted == removed == 40
    assert (result.changed, result.changed_heads) == (changed, changed_heads)
    np.testing.assert_array_equal(result.references.segments, references.segments)
    np.testing.assert_array_equal(result.references.positions, references.positions)
    np.testing.assert_array_equal(result.references.scores.view(np.uint32), references.scores.view(np.uint32))
    assert_same_cache(caches[0], caches[1])


def test_insert_payload_restores_evicted_rows():
    """Round trip: rows evicted from several layers and heads, reinserted with
    their K/V and positions (one multi-layer merge), leave the cache exactly
    as before the eviction -- rows back in position order, head lengths and
    cumulative lengths restored."""
    import torch

    cache = make_cache(8, layers=4, heads=4, dim=32)
    before = host_copy(cache)
    rng = np.random.default_rng(8)
    removals, metadata, payload = {}, [], []
    for layer_index, layer in enumerate(cache.layers):
        if layer_index == 2:
            continue  # an untouched layer
        bounds = layer.bounds()
        for head, length in enumerate(layer.head_lens):
            picks = np.sort(rng.choice(np.arange(30, length), 9, replace=False))  # not prompt rows
            removals[(layer_index, head)] = picks
            rows = torch.as_tensor(bounds[head] + picks, device=layer.keys.device)
            payload.append(torch.stack([layer.keys[rows], layer.values[rows]], dim=1))
            for p, position in zip(picks, layer.positions.reshape(-1)[rows].cpu().numpy()):
                metadata.append((layer_index, head, int(position)))
    cache.remove_positions(removals)
    order = rng.permutation(len(metadata))  # any payload order
    payload = torch.cat(payload)[torch.as_tensor(order, device=payload[0].device)]
    metadata = np.asarray(metadata)[order]
    assert cache.insert_payload(payload, metadata) == len(metadata)
    for layer, (keys, values, positions, lens, prompts) in zip(cache.layers, before):
        np.testing.assert_array_equal(bits(layer.keys), keys)
        np.testing.assert_array_equal(bits(layer.values), values)
        np.testing.assert_array_equal(layer.positions.cpu().numpy(), positions)
        assert layer.head_lens == lens and layer.prompt_lens == prompts
        np.testing.assert_array_equal(layer.cumulative.cpu().numpy(), np.concatenate(([0], np.cumsum(lens))))
    with pytest.raises(ValueError):  # a row that is already resident
        cache.insert_payload(payload[:1], metadata[:1])


def test_merge_layers_equals_per_layer_merge():
    import torch

    from code_for_iclr27_b200 import operators

    C = operators()
    g = torch.Generator().manual_seed(4)
    dev = "cuda"
    ins, outs = [], []
    for layer in range(5):
        rows, dim, recalled = int(torch.randint(10, 300, (1,), generator=g)), 64, int(torch.randint(0, 40, (1,), generator=g))
        keys = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(dev)
        values = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(dev)
        positions = torch.randn(rows, 1, generator=g).to(dev)
        rec = torch.randn(max(recalled, 1), 2, dim, generator=g).to(torch.bfloat16).to(dev)
        rec_pos = torch.randn(max(recalled, 1), generator=g).to(dev)
        mapping = torch.cat([torch.arange(rows), -torch.arange(recalled) - 1])[torch.randperm(rows + recalled, generator=g)]
        if layer == 3:
            mapping = mapping[:0]  # a layer with no output rows
        ins.append((keys, values, positions, rec, rec_pos, mapping.to(dev)))
        outs.append(C.merge(*ins[-1]))
    merged = C.merge_layers(*[list(t) for t in zip(*ins)])
    for i, expected in enumerate(outs):
        for got, want in zip((merged[0][i], merged[1][i], merged[2][i]), expected):
            assert torch.equal(got, want)
