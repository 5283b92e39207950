"""The gapped per-head KV arena (arena.py, csrc/arena.cu) against the packed cache.

Both caches start from the same rows and take the same operations -- decode
appends (one launch for all layers, and per layer), removals from the host
(remove_positions) and from a device queue (remove_selected), a whole audit
pass -- and after each, every layer of the arena read back in the packed
layout (packed_layer) equals the packed cache bit for bit: the same rows in
the same order; recall reinsertion (insert_payload, in place in the arena, a
whole-layer merge in the packed cache) keeps them equal.  FlashAttention's
cache kernel over the arena gives the
reference's decode attention (flash_attn_varlen_func over the packed layer,
attention.py:15-35) within bf16 rounding.  Malformed compaction plans set the
error flag and leave the heads unchanged.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def make_packed(device, seed=0, layers=3, heads=4, dim=128, prompt=300):
    import torch

    from code_for_iclr27_b200.kvcache import PackedCache

    g = torch.Generator().manual_seed(seed)
    cache = PackedCache()
    for _ in range(layers):
        lens = [prompt + int(x) for x in torch.randint(50, 400, (heads,), generator=g)]
        rows = sum(lens)
        keys = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(device)
        values = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(device)
        positions = torch.cat([torch.arange(n, dtype=torch.float32) for n in lens]).to(device)
        cache.add_layer(keys, values, positions, lens, [prompt] * heads)
    cache.seen_tokens = max(max(layer.head_lens) for layer in cache.layers)
    return cache


def assert_same(arena, packed):
    import torch

    for l, layer in enumerate(packed.layers):
        assert list(arena.head_lens[l]) == layer.head_lens, l
        assert list(arena.prompt_lens[l]) == layer.prompt_lens, l
        k, v, p = arena.packed_layer(l)
        assert torch.equal(k.view(torch.int16), layer.keys.view(torch.int16)), l
        assert torch.equal(v.view(torch.int16), layer.values.view(torch.int16)), l
        assert torch.equal(p, layer.positions), l
    assert arena.lengths.cpu().numpy().tolist() == arena.head_lens.reshape(-1).tolist()


def test_arena_equals_packed_through_appends_and_removals(cuda):
    import torch

    from code_for_iclr27_b200.arena import ArenaCache

    packed = make_packed(cuda, seed=1)
    arena = ArenaCache.from_packed(packed, margin=8)  # small margin: appends grow the slots
    initial_capacity = arena.capacity
    assert_same(arena, packed)
    g = torch.Generator().manual_seed(2)
    layers, heads = len(packed.layers), packed.heads
    rng = np.random.default_rng(3)
    for step in range(20):
        new_k = torch.randn(layers, 1, heads, 1, 128, generator=g).to(torch.bfloat16).to(cuda)
        new_v = torch.randn(layers, 1, heads, 1, 128, generator=g).to(torch.bfloat16).to(cuda)
        for l in range(layers):
            packed.append(l, new_k[l], new_v[l], packed.seen_tokens)
        if step % 2:
            arena.append_all(new_k, new_v, packed.seen_tokens)
        else:
            for l in range(layers):
                arena.append(l, new_k[l], new_v[l], packed.seen_tokens)
        packed.seen_tokens += 1
        if step % 5 == 4:
            removals = {}
            for l in range(layers):
                for h in rng.choice(heads, 2, replace=False).tolist():
                    n = packed.layers[l].head_lens[h]
                    removals[(l, h)] = rng.choice(n, int(rng.integers(1, 40)), replace=False)
            removals[(0, 0)] = np.concatenate([removals.get((0, 0), []), [0, 0, 5]]).astype(np.int64)  # duplicates
            assert packed.remove_positions(removals) == arena.remove_positions(removals)
        assert_same(arena, packed)
    assert arena.capacity > initial_capacity  # the slots grew and kept their rows
    # Removals from a device queue: every head, heavy (half of a head) and light.
    coordinates = [(l, h) for l in range(layers) for h in range(heads)]
    segment_ids, positions = [], []
    for s, (l, h) in enumerate(coordinates):
        n = packed.layers[l].head_lens[h]
        take = rng.choice(n, n // 2 if s == 3 else int(rng.integers(0, 6)), replace=False)
        segment_ids += [s] * take.size
        positions += take.tolist()
    seg = torch.tensor(segment_ids, dtype=torch.int64, device=cuda)
    pos = torch.tensor(positions, dtype=torch.int64, device=cuda)
    assert packed.remove_selected(coordinates, seg, pos) == arena.remove_selected(coordinates, seg, pos)
    assert_same(arena, packed)
    with pytest.raises(IndexError):
        arena.remove_positions({(1, 2): [arena.head_lens[1][2]]})
    assert_same(arena, packed)


def test_audit_pass_on_arena_equals_packed(cuda):
    """audit_pass (score, Pool7, select, evict) on both caches: the same
    scores, queue and evictions, and the same caches afterwards."""
    import torch

    from code_for_iclr27_b200.arena import ArenaCache
    from code_for_iclr27_b200.audit import audit_pass

    packed = make_packed(cuda, seed=4, layers=2, heads=4, prompt=200)
    arena = ArenaCache.from_packed(packed)
    g = torch.Generator().manual_seed(5)
    window, groups = 24, 4
    queries = [(torch.randn(window, 4 * groups, 128, generator=g) * 2).to(torch.bfloat16).to(cuda) for _ in range(2)]
    grads = [(torch.randn(4 * groups, 128, generator=g) / 11).to(cuda) for _ in range(2)]
    top = min(min(layer.head_lens) for layer in packed.layers)
    qpos = torch.arange(top - window, top, dtype=torch.int64, device=cuda)
    margin = torch.tensor([0.7], device=cuda)
    a = audit_pass(packed, queries, qpos, grads, margin, immediate=60, queued=200, protect_recent=8)
    b = audit_pass(arena, queries, qpos, grads, margin, immediate=60, queued=200, protect_recent=8)
    assert torch.equal(a.table.scores.view(torch.int32), b.table.scores.view(torch.int32))
    np.testing.assert_array_equal(a.references.segments, b.references.segments)
    np.testing.assert_array_equal(a.references.positions, b.references.positions)
    assert a.evicted == b.evicted == 60
    assert_same(arena, packed)


def test_lazy_eviction_on_the_device_equals_evict_prefix(cuda):
    """After an audit pass on both caches, lazy batches of the queue: on the
    packed cache by evict_prefix (controller.py:57-70: audit positions shifted
    by the rows already removed from their head, starting from the immediate
    prefix), on the arena by evict_logical (device only, rows found by their
    logical positions), with decode appends in between.  The caches stay
    equal bit for bit."""
    import torch

    from code_for_iclr27_b200.arena import ArenaCache
    from code_for_iclr27_b200.audit import audit_pass, evict_prefix

    packed = make_packed(cuda, seed=8, layers=2, heads=4, prompt=150)
    arena = ArenaCache.from_packed(packed)
    g = torch.Generator().manual_seed(9)
    window, groups, immediate, batch = 16, 2, 40, 37
    queries = [(torch.randn(window, 4 * groups, 128, generator=g) * 2).to(torch.bfloat16).to(cuda) for _ in range(2)]
    grads = [(torch.randn(4 * groups, 128, generator=g) / 11).to(cuda) for _ in range(2)]
    top = min(min(layer.head_lens) for layer in packed.layers)
    qpos = torch.arange(top - window, top, dtype=torch.int64, device=cuda)
    margin = torch.tensor([0.9], device=cuda)
    a = audit_pass(packed, queries, qpos, grads, margin, immediate=immediate, queued=300, protect_recent=4)
    b = audit_pass(arena, queries, qpos, grads, margin, immediate=immediate, queued=300, protect_recent=4)
    assert_same(arena, packed)
    queue, removed = a.references[immediate:], a.references[:immediate].groups()
    flat, logical = b.lazy
    start = immediate
    for step in range(5):
        new = torch.randn(2, 1, 4, 1, 128, generator=g).to(torch.bfloat16).to(cuda)
        for l in range(2):
            packed.append(l, new[l], new[l], packed.seen_tokens)
        arena.append_all(new, new, packed.seen_tokens)
        packed.seen_tokens += 1
        queue, removed = evict_prefix(packed, queue, removed, batch)
        arena.evict_logical(flat[start:start + batch], logical[start:start + batch])
        start += batch
        assert_same(arena, packed)


def test_flash_attention_reads_the_arena(cuda):
    """flash_attn_with_kvcache over the arena (k_cache [heads, capacity, 1, D],
    cache_seqlens = lengths) gives the decode attention of
    flash_attn_varlen_func over the packed layer, as attention.py:15-35 calls
    it (one query per KV head, G query heads per KV head)."""
    import torch

    flash_attn = pytest.importorskip("flash_attn")
    from code_for_iclr27_b200.arena import ArenaCache

    packed = make_packed(cuda, seed=6, layers=1, heads=8, prompt=1000)
    arena = ArenaCache.from_packed(packed, margin=100)
    heads, groups, dim = 8, 4, 128
    g = torch.Generator().manual_seed(7)
    q = torch.randn(heads, groups, dim, generator=g).to(torch.bfloat16).to(cuda)
    layer = packed.layers[0]
    cu_q = torch.arange(heads + 1, dtype=torch.int32, device=cuda)
    expected = flash_attn.flash_attn_varlen_func(
        q, layer.keys.view(-1, 1, dim), layer.values.view(-1, 1, dim), cu_q, layer.cumulative, 1,
        max(layer.head_lens), causal=True, dropout_p=0.0, softmax_scale=dim ** -0.5)
    got = flash_attn.flash_attn_with_kvcache(
        q.view(heads, 1, groups, dim), arena.keys.view(heads, arena.capacity, 1, dim),
        arena.values.view(heads, arena.capacity, 1, dim), cache_seqlens=arena.lengths, softmax_scale=dim ** -0.5,
        causal=True)
    torch.testing.assert_close(got.view(heads, groups, dim).float(), expected.float(), atol=2e-2, rtol=2e-2)


def test_arena_c_abi_and_error_flags(cuda):
    """lrk_arena_append / lrk_arena_compact through the C ABI; plans that are
    out of order or out of range set the error flag and change nothing."""
    import ctypes

    import torch

    from code_for_iclr27_b200 import abi

    lib = abi.library()
    heads, cap, dim = 3, 16, 64
    keys = torch.zeros(heads, cap, dim, dtype=torch.bfloat16, device=cuda)
    values = torch.zeros_like(keys)
    positions = torch.zeros(heads, cap, dtype=torch.float32, device=cuda)
    lengths = torch.tensor([0, 5, 16], dtype=torch.int32, device=cuda)
    arena = abi.Arena(keys.data_ptr(), values.data_ptr(), positions.data_ptr(), lengths.data_ptr(), heads, cap, dim,
                      abi.BF16)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    rows = torch.arange(heads * dim, dtype=torch.float32, device=cuda).view(heads, dim).to(torch.bfloat16)
    abi.check(lib.lrk_arena_append(ctypes.byref(arena), 0, heads, rows.data_ptr(), rows.data_ptr(), 42.0,
                                   flag.data_ptr(), stream))
    torch.cuda.synchronize()
    assert lengths.tolist() == [1, 6, 16] and int(flag) == 1  # head 2 was full
    assert torch.equal(keys[0, 0], rows[0]) and torch.equal(keys[1, 5], rows[1]) and float(positions[1, 5]) == 42.0
    before = keys.clone()
    for bad in ([2, 1], [6], [-1]):  # out of order, beyond the length, negative
        flag.zero_()
        removed = torch.tensor(bad, dtype=torch.int64, device=cuda)
        plan = torch.tensor([[1, 0, len(bad)]], dtype=torch.int64, device=cuda)
        abi.check(lib.lrk_arena_compact(ctypes.byref(arena), plan.data_ptr(), 1, removed.data_ptr(), flag.data_ptr(),
                                        stream))
        torch.cuda.synchronize()
        assert int(flag) == 1 and lengths.tolist() == [1, 6, 16] and torch.equal(keys, before)
    status = lib.lrk_arena_compact(ctypes.byref(abi.Arena(keys.data_ptr(), values.data_ptr(), positions.data_ptr(),
                                                          lengths.data_ptr(), heads, cap, 3, abi.BF16)),
                                   plan.data_ptr(), 1, removed.data_ptr(), None, stream)
    assert status == abi.ERR_INVALID  # rows of 6 bytes: not a multiple of 16


def test_arena_evict_unsorted_batch_c_abi(cuda):
    """lrk_arena_evict takes a lazy batch in queue order (unsorted, heads
    interleaved): the result equals removing the same rows with
    lrk_arena_compact; a duplicate or an absent position leaves its head
    unchanged and sets the error flag."""
    import ctypes

    import torch

    from code_for_iclr27_b200 import abi

    lib = abi.library()
    heads, cap, dim = 4, 64, 64
    g = torch.Generator().manual_seed(12)

    def fresh():
        keys = torch.randn(heads, cap, dim, generator=g).to(torch.bfloat16).to(cuda)
        positions = (torch.arange(cap, dtype=torch.float32) * 3).repeat(heads, 1).to(cuda)  # ascending, gapped
        lengths = torch.tensor([60, 10, 0, 64], dtype=torch.int32, device=cuda)
        return keys, keys.clone(), positions, lengths

    k1, v1, p1, l1 = fresh()
    k2, v2, p2, l2 = k1.clone(), v1.clone(), p1.clone(), l1.clone()
    batch_heads = torch.tensor([3, 0, 3, 1, 0, 3], dtype=torch.int64, device=cuda)
    batch_rows = torch.tensor([63, 7, 0, 9, 59, 30], dtype=torch.int64, device=cuda)
    batch_positions = (batch_rows * 3).to(torch.float32)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    a1 = abi.Arena(k1.data_ptr(), v1.data_ptr(), p1.data_ptr(), l1.data_ptr(), heads, cap, dim, abi.BF16)
    abi.check(lib.lrk_arena_evict(ctypes.byref(a1), batch_heads.data_ptr(), batch_positions.data_ptr(), 6,
                                  flag.data_ptr(), stream))
    a2 = abi.Arena(k2.data_ptr(), v2.data_ptr(), p2.data_ptr(), l2.data_ptr(), heads, cap, dim, abi.BF16)
    plan = torch.tensor([[0, 0, 2], [1, 2, 1], [3, 3, 3]], dtype=torch.int64, device=cuda)
    removed = torch.tensor([7, 59, 9, 0, 30, 63], dtype=torch.int64, device=cuda)
    abi.check(lib.lrk_arena_compact(ctypes.byref(a2), plan.data_ptr(), 3, removed.data_ptr(), None, stream))
    torch.cuda.synchronize()
    assert int(flag) == 0 and l1.tolist() == l2.tolist() == [58, 9, 0, 61]
    for h, n in enumerate(l1.tolist()):
        assert torch.equal(k1[h, :n].view(torch.int16), k2[h, :n].view(torch.int16))
        assert torch.equal(p1[h, :n], p2[h, :n])
    before = k1.clone()
    for heads_bad, positions_bad in (([0, 0], [3.0, 3.0]), ([1], [4.0])):  # duplicate; absent (not a multiple of 3)
        flag.zero_()
        hb = torch.tensor(heads_bad, dtype=torch.int64, device=cuda)
        pb = torch.tensor(positions_bad, dtype=torch.float32, device=cuda)
        abi.check(lib.lrk_arena_evict(ctypes.byref(a1), hb.data_ptr(), pb.data_ptr(), len(heads_bad),
                                      flag.data_ptr(), stream))
        torch.cuda.synchronize()
        assert int(flag) == 1 and l1.tolist() == [58, 9, 0, 61] and torch.equal(k1, before)


def test_arena_recall_insert_equals_packed_merge(cuda):
    """Rows evicted from both caches and recalled into both (the arena in
    place: lrk_arena_insert; the packed cache: the merge plan and
    merge_layers), plus rows never resident (positions above a head's last
    one): the caches stay equal.  One head receives more than one launch's
    2048 entries (two rounds), some heads none; a small margin makes the
    slots grow first.  A recalled position that is resident raises
    ValueError before either cache changes."""
    import torch

    from code_for_iclr27_b200.arena import ArenaCache

    packed = make_packed(cuda, seed=5, prompt=3000)
    arena = ArenaCache.from_packed(packed, margin=16)
    rng = np.random.default_rng(5)
    removals, payload, metadata = {}, [], []
    for l, layer in enumerate(packed.layers):
        bounds = layer.bounds()
        for h in range(packed.heads):
            if (l, h) == (1, 2):
                continue  # an untouched head
            count = 2600 if (l, h) == (0, 1) else int(rng.integers(1, 40))
            picks = np.sort(rng.choice(layer.head_lens[h], count, replace=False))
            removals[(l, h)] = picks
            rows = torch.as_tensor(bounds[h] + picks, device=cuda)
            payload.append(torch.stack([layer.keys[rows], layer.values[rows]], dim=1))
            metadata.extend((l, h, int(p)) for p in layer.positions.reshape(-1)[rows].cpu().numpy())
    for cache in (packed, arena):
        cache.remove_positions(removals)
    assert_same(arena, packed)
    # Rows never resident: positions above a head's last one.
    top = int(packed.layers[2].head_lens[3]) + int(len(removals.get((2, 3), ())))
    payload.append(torch.randn(50, 2, 128).to(torch.bfloat16).to(cuda))
    metadata.extend((2, 3, top + 10 + 7 * i) for i in range(50))
    payload = torch.cat(payload)
    metadata = np.asarray(metadata, dtype=np.int64)
    order = rng.permutation(len(metadata))  # any payload order
    payload, metadata = payload[torch.as_tensor(order, device=cuda)], metadata[order]
    bad = metadata[:3].copy()
    bad[0] = (0, 0, int(packed.layers[0].positions.reshape(-1)[0].item()))  # resident
    with pytest.raises(ValueError):
        arena.insert_payload(payload[:3], bad)
    assert_same(arena, packed)  # nothing changed
    assert arena.insert_payload(payload, metadata) == len(metadata)
    assert packed.insert_payload(payload, metadata) == len(metadata)
    assert_same(arena, packed)
