"""Recall merge plans on the device (lrk_merge_plan through _C.merge_plan)
against the oracle's restatement of recall/planning.py:34-52, and the
reinsertion path that uses them (PackedCache.insert_payload, cache.py:201-253)
on the cases the reference refuses or plans on the host."""
import numpy as np
import pytest

from oracle import lrk_oracle as O

pytestmark = pytest.mark.gpu


def layer_case(rng, heads, resident_rows, recalled_rows, span):
    """Per head ascending unique resident positions, and recalled positions
    that are neither resident nor repeated, in a random order."""
    lengths = rng.integers(0, resident_rows + 1, heads)
    positions, metadata = [], []
    for head, length in enumerate(lengths.tolist()):
        pool = rng.choice(span, length + recalled_rows, replace=False)
        positions.append(np.sort(pool[:length]))
        chosen = pool[length:length + rng.integers(0, recalled_rows + 1)]
        metadata.extend((0, head, int(p)) for p in chosen)
    metadata = np.asarray(metadata, dtype=np.int64).reshape(-1, 3)
    return lengths.tolist(), np.concatenate(positions), metadata[rng.permutation(len(metadata))]


def device_plan(layers):
    """_C.merge_plan over [(lengths, positions, metadata)], the recalled rows
    of each layer sorted by (head, position) and indexed by their place in
    the layer's metadata, as the oracle indexes them."""
    import torch

    from code_for_iclr27_b200 import operators

    heads = len(layers[0][0])
    args = [[], [], [], [], []]
    for lengths, positions, metadata in layers:
        order = np.lexsort((metadata[:, 2], metadata[:, 1]))
        starts = np.searchsorted(metadata[order, 1], np.arange(heads + 1))
        args[0].append(torch.as_tensor(positions, dtype=torch.float32).cuda())
        args[1].append(torch.as_tensor(np.concatenate(([0], np.cumsum(lengths))), dtype=torch.int32).cuda())
        args[2].append(torch.as_tensor(metadata[order, 2], dtype=torch.float32).cuda())
        args[3].append(torch.as_tensor(order, dtype=torch.int64).cuda())
        args[4].append(torch.as_tensor(starts, dtype=torch.int32).cuda())
    mappings, flag = operators().merge_plan(*args)
    return [m.cpu().numpy() for m in mappings], int(flag.item())


@pytest.mark.parametrize("heads,resident,recalled,layers", [(8, 300, 40, 5), (4, 5000, 700, 3), (32, 64, 64, 70)])
def test_device_plan_equals_oracle(heads, resident, recalled, layers):
    """Every mapping entry equals the oracle's (stable argsort of resident then
    recalled positions per head), with empty heads, heads without recalled
    rows and more layers than one launch holds (64)."""
    rng = np.random.default_rng(heads * 1000 + layers)
    cases = [layer_case(rng, heads, resident, recalled, 10 * (resident + recalled) + 10) for _ in range(layers)]
    mappings, flag = device_plan(cases)
    assert flag == 0
    for (lengths, positions, metadata), mapping in zip(cases, mappings):
        expected, new_lengths = O.merge_plan(positions, lengths, metadata)
        np.testing.assert_array_equal(mapping, expected)
        assert sum(new_lengths) == mapping.size


def test_device_plan_flags():
    """Bit 1 for a recalled position that is resident or recalled twice, bit 2
    for a head whose resident positions do not ascend, bit 4 for head bounds
    that do not cover the rows; no other case sets a bit."""
    rng = np.random.default_rng(3)
    lengths, positions, metadata = layer_case(rng, 4, 100, 20, 2000)
    assert device_plan([(lengths, positions, metadata)])[1] == 0
    resident = metadata.copy()
    head = int(np.argmax(np.asarray(lengths) > 0))
    resident[0] = (0, head, positions[sum(lengths[:head])])  # the head's first resident position
    assert device_plan([(lengths, positions, resident)])[1] == 1
    repeated = np.concatenate((metadata, metadata[:1]))
    assert device_plan([(lengths, positions, repeated)])[1] == 1
    unsorted = positions.copy()
    head = int(np.argmax(np.asarray(lengths) > 2))
    first = sum(lengths[:head])
    unsorted[first], unsorted[first + 1] = unsorted[first + 1], unsorted[first]
    assert device_plan([(lengths, unsorted, metadata)])[1] & 2
    short = list(lengths)
    short[-1] -= 1  # bounds end one row before the positions do
    import torch

    from code_for_iclr27_b200 import operators

    order = np.lexsort((metadata[:, 2], metadata[:, 1]))
    starts = np.searchsorted(metadata[order, 1], np.arange(5))
    _, flag = operators().merge_plan(
        [torch.as_tensor(positions, dtype=torch.float32).cuda()],
        [torch.as_tensor(np.concatenate(([0], np.cumsum(short))), dtype=torch.int32).cuda()],
        [torch.as_tensor(metadata[order, 2], dtype=torch.float32).cuda()],
        [torch.as_tensor(order, dtype=torch.int64).cuda()],
        [torch.as_tensor(starts, dtype=torch.int32).cuda()])
    assert int(flag.item()) & 4


def test_insert_payload_unsorted_heads_and_refusals():
    """A cache whose head positions do not ascend is merged by the host plan
    (the oracle's merge); a duplicate identity raises ValueError and a head
    outside the layer raises AssertionError, each with the cache unchanged."""
    import torch

    from code_for_iclr27_b200.kvcache import PackedCache

    rng = np.random.default_rng(11)
    g = torch.Generator().manual_seed(11)
    cache, expected = PackedCache(), []
    metadata = []
    for layer_index in range(3):
        lengths, positions, meta = layer_case(rng, 4, 200, 30, 5000)
        if layer_index == 1:
            positions = positions[::-1].copy()  # every head descends
            lengths = lengths[::-1]
        rows = sum(lengths)
        keys = torch.randn(rows, 16, generator=g).to(torch.bfloat16)
        values = torch.randn(rows, 16, generator=g).to(torch.bfloat16)
        cache.add_layer(keys.cuda(), values.cuda(), torch.as_tensor(positions, dtype=torch.float32).cuda(),
                        lengths, [0] * 4)
        meta[:, 0] = layer_index
        metadata.append(meta)
        expected.append((keys, values, positions, lengths))
    metadata = np.concatenate(metadata)
    payload = torch.randn(len(metadata), 2, 16, generator=g).to(torch.bfloat16)

    def snapshot():
        return [(layer.keys.cpu(), layer.positions.cpu().numpy().copy(), list(layer.head_lens)) for layer in cache.layers]

    before = snapshot()
    bad_head = metadata.copy()
    bad_head[0, 1] = 4
    with pytest.raises(AssertionError):
        cache.insert_payload(payload.cuda(), bad_head)
    duplicate = np.concatenate((metadata, metadata[-1:]))
    with pytest.raises(ValueError, match="duplicate"):
        cache.insert_payload(torch.cat((payload, payload[-1:])).cuda(), duplicate)
    for (k0, p0, l0), (k1, p1, l1) in zip(before, snapshot()):
        assert torch.equal(k0.view(torch.int16), k1.view(torch.int16))
        np.testing.assert_array_equal(p0, p1)
        assert l0 == l1
    assert cache.insert_payload(payload.cuda(), metadata) == len(metadata)
    for layer_index, (layer, (keys, values, positions, lengths)) in enumerate(zip(cache.layers, expected)):
        rows = np.flatnonzero(metadata[:, 0] == layer_index)
        mapping, new_lengths = O.merge_plan(positions.astype(np.int64), lengths, metadata[rows])
        source = torch.cat((keys, payload[torch.as_tensor(rows), 0]))
        gather = np.where(mapping >= 0, mapping, len(positions) - mapping - 1)
        assert torch.equal(layer.keys.cpu().view(torch.int16), source[torch.as_tensor(gather)].view(torch.int16))
        merged = np.concatenate((positions, metadata[rows, 2]))[gather]
        np.testing.assert_array_equal(layer.positions.cpu().numpy().reshape(-1), merged.astype(np.float32))
        assert layer.head_lens == list(new_lengths)
        np.testing.assert_array_equal(layer.cumulative.cpu().numpy(), np.concatenate(([0], np.cumsum(new_lengths))))


def test_insert_payload_device_plan_equals_host_plan():
    """The same recall event through the device plan and the host plan leaves
    two copies of a cache bit-identical (rows, positions, lengths, bounds)."""
    import torch

    from code_for_iclr27_b200.kvcache import PackedCache

    rng = np.random.default_rng(21)
    g = torch.Generator().manual_seed(21)
    caches = [PackedCache(), PackedCache()]
    metadata = []
    for layer_index in range(6):
        lengths, positions, meta = layer_case(rng, 8, 500, 40, 20000)
        keys = torch.randn(sum(lengths), 64, generator=g).to(torch.bfloat16).cuda()
        values = torch.randn(sum(lengths), 64, generator=g).to(torch.bfloat16).cuda()
        for cache in caches:
            cache.add_layer(keys.clone(), values.clone(), torch.as_tensor(positions, dtype=torch.float32).cuda(),
                            lengths, [0] * 8)
        if layer_index != 3:  # an untouched layer
            meta[:, 0] = layer_index
            metadata.append(meta)
    metadata = np.concatenate(metadata)
    payload = torch.randn(len(metadata), 2, 64, generator=g).to(torch.bfloat16).cuda()
    assert caches[0].insert_payload(payload, metadata, plan="device") == len(metadata)
    assert caches[1].insert_payload(payload, metadata, plan="host") == len(metadata)
    for a, b in zip(caches[0].layers, caches[1].layers):
        assert torch.equal(a.keys.view(torch.int16), b.keys.view(torch.int16))
        assert torch.equal(a.values.view(torch.int16), b.values.view(torch.int16))
        assert torch.equal(a.positions, b.positions)
        assert a.head_lens == b.head_lens
        assert torch.equal(a.cumulative, b.cumulative)
    with pytest.raises(ValueError):
        caches[0].insert_payload(payload, metadata, plan="neither")
