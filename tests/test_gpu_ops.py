"""GPU parity of every liblrk operator against the oracle (and, when the
reference's own CUDA modules are present under oracle/_ref, against them bit
for bit).  Byte-moving operators must be bit-exact; scoring outputs agree
with the oracle within 1e-5 relative (the oracle's numpy exp differs from
CUDA's expf by an ulp) and bit-exactly with the reference kernels."""
import ctypes
import importlib.util
import math

import numpy as np
import pytest

from oracle import lrk_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def torch_mod():
    import torch

    return torch


def bits(t):
    torch = torch_mod()
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.numpy()
    return t.numpy()


def close(actual, expected, rtol=RTOL, atol=1e-7):
    actual, expected = np.asarray(actual, np.float64), np.asarray(expected, np.float64)
    assert actual.shape == expected.shape
    assert (np.isnan(actual) == np.isnan(expected)).all(), "NaN pattern differs"
    ok = ~np.isnan(actual)
    np.testing.assert_allclose(actual[ok], expected[ok], rtol=rtol, atol=atol)


@pytest.fixture(scope="module")
def C(cuda):
    from code_for_iclr27_b200 import operators

    return operators()


@pytest.fixture(scope="module")
def L(cuda):
    from code_for_iclr27_b200 import legacy_operators

    return legacy_operators()


@pytest.fixture(scope="module")
def ref(cuda):
    """The reference's own _C / _legacy_C built from its sources (optional)."""
    from oracle import build_ref

    paths = build_ref.built_paths()
    if not {"C", "legacy_C"} <= set(paths):
        return None
    mods = {}
    for key, name in (("C", "_C"), ("legacy_C", "_legacy_C")):
        spec = importlib.util.spec_from_file_location(f"lazy_recall_reference.{name}", paths[key])
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mods[key] = mod
    return mods


def same(a, b):
    """Bit-identical values, with NaN matching NaN."""
    torch = torch_mod()
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    nan_a, nan_b = torch.isnan(a), torch.isnan(b)
    return bool(torch.equal(nan_a, nan_b) and torch.equal(a[~nan_a], b[~nan_b]))


def gen(seed):
    torch = torch_mod()
    return torch.Generator().manual_seed(seed)


def rand_kv(rows, d, dtype, g, device):
    torch = torch_mod()
    return torch.randn(rows, d, generator=g).to(dtype).to(device)


def np_kv(t):
    torch = torch_mod()
    return bits(t) if t.dtype == torch.bfloat16 else t.cpu().numpy()


# ------------------------------------------------------------- append

APPEND_CASES = [
    ("bf16", 128, [37, 0, 5, 300, 1, 2, 64, 9], 1),
    ("bf16", 64, [3, 4], 3),
    ("bf16", 128, [0, 0, 0], 1),
    ("f32", 128, [10, 20], 2),
    ("f16", 3, [7, 8, 9, 10], 1),  # 6-byte rows: narrow vector path
    ("f64", 16, [5, 1], 1),
]


@pytest.mark.parametrize("dtype_name,d,lengths,added", APPEND_CASES)
def test_append(C, ref, cuda, dtype_name, d, lengths, added):
    torch = torch_mod()
    dtype = {"bf16": torch.bfloat16, "f32": torch.float32, "f16": torch.float16, "f64": torch.float64}[dtype_name]
    g = gen(1)
    heads, rows = len(lengths), sum(lengths)
    keys, values = rand_kv(rows, d, dtype, g, cuda), rand_kv(rows, d, dtype, g, cuda)
    positions = (torch.randperm(rows + 7, generator=g)[:rows].float() * 1.5).reshape(-1, 1).to(cuda)
    nk = torch.randn(1, heads, added, d, generator=g).to(dtype).to(cuda)
    nv = torch.randn(1, heads, added, d, generator=g).to(dtype).to(cuda)
    cumulative = torch.tensor(np.concatenate(([0], np.cumsum(lengths))), dtype=torch.int32, device=cuda)
    out = C.append(keys, values, positions, nk, nv, cumulative, 40000, max(lengths))
    expect = O.append(np_kv(keys), np_kv(values), positions.cpu().numpy(), np_kv(nk), np_kv(nv),
                      cumulative.cpu().numpy(), 40000)
    for got, exp in zip(out, expect):
        np.testing.assert_array_equal(np_kv(got), exp)
    if ref is not None:
        for got, exp in zip(out, ref["C"].append(keys, values, positions, nk, nv, cumulative, 40000, max(lengths))):
            assert torch.equal(got, exp)


# ------------------------------------------------------------ compact


def removal_patterns(rows, g):
    torch = torch_mod()
    yield torch.zeros(0, dtype=torch.int64)
    yield torch.arange(rows)
    yield torch.tensor([0, rows - 1])
    yield torch.arange(rows // 4, rows // 2)
    yield torch.randperm(rows, generator=g)[: rows // 3].sort().values
    yield torch.cat([torch.arange(0, 300), torch.arange(rows - 700, rows)])


@pytest.mark.parametrize("rows,d", [(1000, 128), (4099, 64), (300007, 128)])
def test_compact(C, ref, cuda, rows, d):
    torch = torch_mod()
    g = gen(2)
    keys, values = rand_kv(rows, d, torch.bfloat16, g, cuda), rand_kv(rows, d, torch.bfloat16, g, cuda)
    positions = torch.arange(rows, dtype=torch.float32).reshape(-1, 1).to(cuda)
    k_np, v_np, p_np = bits(keys), bits(values), positions.cpu().numpy()
    for removed in removal_patterns(rows, g):
        removed = removed.to(cuda)
        out = C.compact(keys, values, positions, removed)
        expect = O.compact(k_np, v_np, p_np, removed.cpu().numpy())
        for got, exp in zip(out, expect):
            np.testing.assert_array_equal(np_kv(got), exp)
        if ref is not None and removed.numel() < rows:
            for got, exp in zip(out, ref["C"].compact(keys, values, positions, removed)):
                assert torch.equal(got, exp)


def test_compact_through_c_abi(cuda):
    """The same kernel called through the C ABI with raw pointers."""
    torch = torch_mod()
    from code_for_iclr27_b200 import abi

    g = gen(3)
    rows, d = 5000, 128
    keys, values = rand_kv(rows, d, torch.bfloat16, g, cuda), rand_kv(rows, d, torch.bfloat16, g, cuda)
    positions = torch.arange(rows, dtype=torch.float32, device=cuda)
    removed = torch.randperm(rows, generator=g)[:1234].sort().values.to(cuda)
    out_k = torch.empty(rows - 1234, d, dtype=torch.bfloat16, device=cuda)
    out_v, out_p = torch.empty_like(out_k), torch.empty(rows - 1234, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    abi.check(abi.library().lrk_compact(keys.data_ptr(), values.data_ptr(), positions.data_ptr(), rows, d, abi.BF16,
                                        removed.data_ptr(), 1234, out_k.data_ptr(), out_v.data_ptr(),
                                        out_p.data_ptr(), stream))
    torch.cuda.synchronize()
    ek, ev, ep = O.compact(bits(keys), bits(values), positions.cpu().numpy(), removed.cpu().numpy())
    np.testing.assert_array_equal(bits(out_k), ek)
    np.testing.assert_array_equal(bits(out_v), ev)
    np.testing.assert_array_equal(out_p.cpu().numpy(), ep.reshape(-1))


# --------------------------------------------------------- merge / pack


@pytest.mark.parametrize("rows,recalled_rows,d", [(500, 40, 128), (0, 5, 64), (300, 0, 128), (20000, 256, 128)])
def test_merge(C, ref, cuda, rows, recalled_rows, d):
    torch = torch_mod()
    g = gen(4)
    keys, values = rand_kv(rows, d, torch.bfloat16, g, cuda), rand_kv(rows, d, torch.bfloat16, g, cuda)
    positions = torch.arange(rows, dtype=torch.float32).reshape(-1, 1).to(cuda)
    recalled = torch.randn(recalled_rows, 2, d, generator=g).to(torch.bfloat16).to(cuda)
    recalled_pos = (torch.arange(recalled_rows, dtype=torch.float32) + 0.5).to(cuda)
    mapping = torch.cat([torch.arange(rows), -torch.arange(1, recalled_rows + 1)])
    mapping = mapping[torch.randperm(mapping.numel(), generator=g)].to(cuda)
    out = C.merge(keys, values, positions, recalled, recalled_pos, mapping)
    expect = O.merge(bits(keys), bits(values), positions.cpu().numpy(), bits(recalled), recalled_pos.cpu().numpy(),
                     mapping.cpu().numpy())
    for got, exp in zip(out, expect):
        np.testing.assert_array_equal(np_kv(got), exp)
    if ref is not None and mapping.numel():
        for got, exp in zip(out, ref["C"].merge(keys, values, positions, recalled, recalled_pos, mapping)):
            assert torch.equal(got, exp)


@pytest.mark.parametrize("count", [1, 37, 2048])
def test_pack(C, ref, cuda, count):
    torch = torch_mod()
    g = gen(5)
    rows, d = 4000, 128
    keys, values = rand_kv(rows, d, torch.bfloat16, g, cuda), rand_kv(rows, d, torch.bfloat16, g, cuda)
    positions = ((torch.rand(rows, generator=g) - 0.3) * 9000).reshape(-1, 1).to(cuda)  # fractional, some negative
    indices = torch.randperm(rows, generator=g)[:count].to(cuda)
    heads = torch.randint(0, 8, (count,), generator=g).to(cuda)
    # Write into a slice of a larger archive buffer, as recall/transport.py does.
    archive = torch.zeros(3, 2048 + 16, 2, d, dtype=torch.bfloat16, device=cuda)
    meta = torch.zeros(3, 2048 + 16, 3, dtype=torch.int64, device=cuda)
    payload, metadata = archive[1, 16:16 + count], meta[1, 16:16 + count]
    C.pack(keys, values, positions, indices, heads, 7, payload, metadata)
    ep, em = O.pack(bits(keys), bits(values), positions.cpu().numpy(), indices.cpu().numpy(), heads.cpu().numpy(), 7)
    np.testing.assert_array_equal(bits(payload), ep)
    np.testing.assert_array_equal(metadata.cpu().numpy(), em)
    assert not archive[1, :16].any() and not archive[0].any() and not archive[2].any()
    if ref is not None:
        p2 = torch.empty_like(payload)
        m2 = torch.empty_like(metadata)
        ref["C"].pack(keys, values, positions, indices, heads, 7, p2, m2)
        assert torch.equal(p2, payload) and torch.equal(m2, metadata)


# -------------------------------------------------------- batch append


@pytest.mark.parametrize("requests,heads,d", [(3, 4, 128), (9, 8, 128), (2, 8, 64)])
def test_batch_append(C, ref, cuda, requests, heads, d):
    torch = torch_mod()
    g = gen(6)
    ks, vs, ps, lens = [], [], [], []
    for r in range(requests):
        hl = torch.randint(0, 200, (heads,), generator=g).tolist()
        hl[r % heads] = 0
        n = sum(hl)
        ks.append(rand_kv(n, d, torch.bfloat16, g, cuda))
        vs.append(rand_kv(n, d, torch.bfloat16, g, cuda))
        ps.append((torch.arange(n, dtype=torch.float32) * 3).reshape(-1, 1).to(cuda))
        lens.append(hl)
    nk = torch.randn(requests, heads, 1, d, generator=g).to(torch.bfloat16).to(cuda)
    nv = torch.randn(requests, heads, 1, d, generator=g).to(torch.bfloat16).to(cuda)
    logical = [int(x) for x in torch.randint(0, 1 << 24, (requests,), generator=g)]
    out = C.batch_append(ks, vs, ps, nk, nv, lens, logical)
    expect = O.batch_append([bits(k) for k in ks], [bits(v) for v in vs], [p.cpu().numpy() for p in ps],
                            bits(nk)[:, :, 0], bits(nv)[:, :, 0], lens, logical)
    for got, exp in zip(out, expect):
        np.testing.assert_array_equal(np_kv(got), exp)
    if ref is not None:
        for got, exp in zip(out, ref["C"].batch_append(ks, vs, ps, nk, nv, lens, logical)):
            assert torch.equal(got, exp)


def test_batch_append_rejects_uncovered_rows(C, cuda):
    torch = torch_mod()
    k = torch.zeros(10, 64, dtype=torch.bfloat16, device=cuda)
    p = torch.zeros(10, 1, device=cuda)
    n = torch.zeros(1, 2, 1, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="Head lengths do not cover cache rows"):
        C.batch_append([k], [k], [p], n, n, [[4, 5]], [3])


# ------------------------------------------------------------- legacy


def test_legacy_append_and_compact(L, ref, cuda):
    torch = torch_mod()
    g = gen(7)
    head_lens = torch.tensor([10, 0, 15, 5, 12, 8], dtype=torch.int32)
    cu = torch.cat([torch.zeros(1, dtype=torch.int32), head_lens.cumsum(0).to(torch.int32)])
    for d, dtype in ((1, torch.float32), (64, torch.bfloat16), (128, torch.bfloat16)):
        cache = rand_kv(int(head_lens.sum()), d, dtype, g, cuda)
        states = torch.randn(2, 3, 2, d, generator=g).to(dtype).to(cuda)
        out = L.append_flattened_cache(cache, states, head_lens.to(cuda), cu.to(cuda))
        expect = O.append_flattened(np_kv(cache), np_kv(states), head_lens.numpy(), cu.numpy())
        np.testing.assert_array_equal(np_kv(out), expect)
        if ref is not None:
            assert torch.equal(out, ref["legacy_C"].append_flattened_cache(cache, states, head_lens.to(cuda),
                                                                            cu.to(cuda)))
    keys, values = rand_kv(700, 128, torch.bfloat16, g, cuda), rand_kv(700, 128, torch.bfloat16, g, cuda)
    keep = torch.tensor([5, 0, 699, 5, 300], dtype=torch.int64, device=cuda)
    ck, cv = L.compact_flattened_kv(keys, values, keep)
    ek, ev = O.compact_flattened(bits(keys), bits(values), keep.cpu().numpy())
    np.testing.assert_array_equal(bits(ck), ek)
    np.testing.assert_array_equal(bits(cv), ev)


@pytest.mark.parametrize("values_dtype", ["bf16", "f32"])
def test_legacy_decision_risk(L, ref, cuda, values_dtype):
    torch = torch_mod()
    g = gen(8)
    dtype = torch.bfloat16 if values_dtype == "bf16" else torch.float32
    probs = torch.rand(4, 301, generator=g).to(cuda)
    vals = torch.randn(301, 128, generator=g).to(dtype).to(cuda)
    outs, grads = torch.randn(4, 128, generator=g).to(cuda), torch.randn(4, 128, generator=g).to(cuda)
    out = L.decision_risk_scores(probs, vals, outs, grads, 0.4, 1e-6)
    expect = O.decision_risk(probs.cpu().numpy(), np_kv(vals), values_dtype, outs.cpu().numpy(), grads.cpu().numpy(),
                             0.4, 1e-6)
    close(out.cpu().numpy(), expect, atol=1e-6)
    if ref is not None:
        assert torch.equal(out, ref["legacy_C"].decision_risk_scores(probs, vals, outs, grads, 0.4, 1e-6))


# --------------------------------------------------------------- pool


@pytest.mark.parametrize("width", [1, 3, 7, 9, 63, 65])
def test_pool(C, ref, cuda, width):
    # Widths up to 65 cover the tiled kernel (half-width <= 32) and the
    # element-per-thread one beyond it.
    torch = torch_mod()
    g = gen(9)
    lengths = [1, 2, 3, 6, 7, 500, 4096, 1]
    n = sum(lengths)
    scores = (torch.randint(0, 30, (n,), generator=g).float() / 3)
    scores[10] = float("nan")
    scores[20] = float("-inf")
    scores = scores.to(cuda)
    bounds = torch.tensor(np.concatenate(([0], np.cumsum(lengths))), dtype=torch.int64, device=cuda)
    out = C.pool(scores, bounds, max(lengths), width)
    np.testing.assert_array_equal(out.cpu().numpy(), O.pool(scores.cpu().numpy(), bounds.cpu().numpy(), width))
    if ref is not None:
        assert torch.equal(out, ref["C"].pool(scores, bounds, max(lengths), width))


@pytest.mark.parametrize("offset", [0, 1])
def test_pool_tiles(C, ref, cuda, offset):
    """Segments longer than one 2048-element tile, starting at every residue
    mod 4, empty segments, NaN runs, ties; offset 1 passes a 4-byte aligned
    (not 16-byte aligned) view, which takes the element-per-thread kernel."""
    torch = torch_mod()
    g = gen(19)
    lengths = [0, 5, 2047, 2048, 2049, 0, 0, 6150, 3, 1, 4097, 9, 0, 1962 * 3 + 1]
    n = sum(lengths)
    base = (torch.randint(0, 40, (n + offset,), generator=g).float() / 4)
    base[offset + 3000:offset + 3010] = float("nan")
    base[offset + 7000] = float("inf")
    scores = base.to(cuda)[offset:]
    bounds = torch.tensor(np.concatenate(([0], np.cumsum(lengths))), dtype=torch.int64, device=cuda)
    for width in (1, 7, 15):
        out = C.pool(scores, bounds, max(lengths), width)
        np.testing.assert_array_equal(out.cpu().numpy(),
                                      O.pool(scores.cpu().numpy(), bounds.cpu().numpy(), width))
        if ref is not None:
            assert torch.equal(out, ref["C"].pool(scores, bounds, max(lengths), width))


# ------------------------------------------------------------ scoring

PROB_CASES = [
    ("bf16", 6, 4, 1), ("bf16", 3, 4, 255), ("bf16", 2, 4, 256), ("bf16", 5, 4, 4099), ("f16", 4, 2, 8192),
    ("f32", 3, 8, 1030), ("bf16", 4, 4, 35026), ("bf16", 2, 8, 60001), ("bf16", 1, 2, 120001), ("f32", 1, 2, 60001),
    ("bf16", 3, 4, 18432), ("bf16", 3, 4, 18433), ("bf16", 1, 2, 112624), ("bf16", 1, 2, 112625),
    # 16-byte aligned rows longer than the fp32-weight stage: the lane-major packed layout
    ("bf16", 3, 4, 20480), ("bf16", 2, 4, 34768), ("f16", 2, 4, 40000), ("bf16", 1, 2, 100000),
]


@pytest.mark.parametrize("dtype_name,window,groups,length", PROB_CASES)
def test_temporal_probabilities_and_risk(C, ref, cuda, dtype_name, window, groups, length):
    torch = torch_mod()
    dtype = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dtype_name]
    g = gen(10 + length)
    logits = (torch.randn(window, groups, length, generator=g) * 2 * math.sqrt(128)).to(dtype).to(cuda)
    pv = torch.randn(groups, length, generator=g).abs().to(cuda)
    qpos = torch.arange(length - window - 2, length - 2, dtype=torch.int64).to(cuda)
    kpos = torch.arange(length, dtype=torch.float32).to(cuda)
    scale = 1.0 / math.sqrt(128)
    probs, op = C.temporal_probabilities(logits, pv, qpos, kpos, scale)
    ep, eo = O.temporal_probabilities(np_kv(logits), dtype_name, pv.cpu().numpy(), qpos.cpu().numpy(),
                                      kpos.cpu().numpy(), np.float32(scale))
    close(probs.cpu().numpy(), ep, atol=1e-9)
    close(op.cpu().numpy(), eo, rtol=2e-5, atol=1e-6)
    first, last = length // 3, max(length // 3 + 1, length - 1)
    margin = torch.tensor([0.6], device=cuda)
    risk = C.temporal_risk(probs, op, pv, margin, first, last, 1e-6)
    er = O.temporal_risk(probs.cpu().numpy(), op.cpu().numpy(), pv.cpu().numpy(), np.float32(0.6), first, last, 1e-6)
    close(risk.cpu().numpy(), er, atol=1e-7)
    if ref is not None:
        rp, ro = ref["C"].temporal_probabilities(logits, pv, qpos, kpos, scale)
        assert same(rp, probs), "probabilities differ from the reference kernel"
        assert same(ro, op), "output projection differs from the reference kernel"
        assert same(ref["C"].temporal_risk(probs, op, pv, margin, first, last, 1e-6), risk)


@pytest.mark.parametrize("window,groups", [(1, 1), (7, 4), (79, 4), (250, 8), (13, 12)])
def test_temporal_risk_shapes_and_nonfinite(C, ref, cuda, window, groups):
    torch = torch_mod()
    g = gen(20 + window)
    length = 3000
    probs = torch.rand(window, groups, length, generator=g)
    probs[0, 0, 100] = float("nan")
    probs[window - 1, groups - 1, 200] = 1.0  # ratio 1/eps
    probs = probs.to(cuda)
    op = torch.randn(window, groups, generator=g).to(cuda)
    pv = torch.randn(groups, length, generator=g).to(cuda)
    margin = torch.tensor([-1.3], device=cuda)
    risk = C.temporal_risk(probs, op, pv, margin, 50, 2950, 1e-6)
    er = O.temporal_risk(probs.cpu().numpy(), op.cpu().numpy(), pv.cpu().numpy(), np.float32(-1.3), 50, 2950, 1e-6)
    close(risk.cpu().numpy(), er, atol=1e-7)
    assert math.isnan(float(risk[50]))
    if ref is not None:
        assert same(ref["C"].temporal_risk(probs, op, pv, margin, 50, 2950, 1e-6), risk)


def test_head_scores_end_to_end(C, cuda):
    """The reference's GPU scoring composition (scoring.py:174-195) run on the
    new operators equals the oracle's restatement of that composition."""
    torch = torch_mod()
    g = gen(30)
    window, groups, length, d = 20, 4, 700, 64
    q = torch.randint(-1, 2, (window, groups, d), generator=g).float()
    k = torch.randint(-1, 2, (length, d), generator=g).to(torch.bfloat16)
    v = torch.randn(length, d, generator=g).to(torch.bfloat16)
    grad = torch.randn(groups, d, generator=g)
    qpos = torch.arange(650, 650 + window, dtype=torch.int64)
    kpos = torch.arange(length, dtype=torch.float32)
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    pv = torch.matmul(grad.to(cuda), vd.float().transpose(0, 1)).contiguous()
    result = None
    for start in range(0, window, 6):
        end = min(start + 6, window)
        logits = torch.matmul(qd[start:end].to(torch.bfloat16), kd.transpose(0, 1))
        probs, op = C.temporal_probabilities(logits.contiguous(), pv, qpos[start:end].to(cuda), kpos.to(cuda),
                                             1.0 / math.sqrt(d))
        s = C.temporal_risk(probs, op, pv, torch.tensor([0.9], device=cuda), 10, 690, 1e-6)
        result = s if result is None else torch.maximum(result, s)
    expect = O.temporal_head_scores_gpu_path(q.numpy(), qpos.numpy(), O.bf16_to_f32(bits(k)), kpos.numpy(),
                                             O.bf16_to_f32(bits(v)), 10, 690, grad.numpy(), 0.9, 1e-6, 6)
    close(result.cpu().numpy(), expect, rtol=1e-4, atol=1e-6)


# ---------------------------------------------------------------- recall


def test_gather_rows_from_registered_host_pool(cuda):
    """Recall rows fetched by the GPU straight from a registered host pool
    (the archive layout [rows, 2, D] bf16, recall/cpu_worker.py:21-22)."""
    import mmap

    torch = torch_mod()
    from code_for_iclr27_b200 import abi, host_operators

    H = host_operators()
    rows, d = 20000, 128
    row_bytes = 2 * d * 2
    buffer = mmap.mmap(-1, rows * row_bytes)  # page-aligned, like the transport's SharedMemory slots
    pool = np.frombuffer(buffer, dtype=np.uint16).reshape(rows, 2, d)
    pool[:] = np.random.default_rng(0).integers(0, 65535, size=pool.shape, dtype=np.uint16)
    address = pool.__array_interface__["data"][0]
    with pytest.raises(RuntimeError):
        H.device_pointer(address)  # not registered yet: refused before any launch
    H.register_host(address, rows * row_bytes)
    try:
        device = H.device_pointer(address)
        chosen = np.random.default_rng(1).choice(rows, 256, replace=False)
        indices = torch.from_numpy(chosen).to(cuda)
        out = torch.empty(256, 2, d, dtype=torch.bfloat16, device=cuda)
        stream = torch.cuda.current_stream().cuda_stream
        abi.check(abi.library().lrk_gather_rows(device, rows, row_bytes, indices.data_ptr(), 256, out.data_ptr(),
                                                stream))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(bits(out), pool[chosen])
    finally:
        H.unregister_host(address)
        del pool
        buffer.close()


def test_row_division_is_ieee_division(cuda):
    """The scoring kernels divide each exp weight by the row denominator with a
    Markstein quotient correction; it must equal IEEE division bit for bit."""
    torch = torch_mod()
    from code_for_iclr27_b200 import abi

    lib = abi.library()
    counter = torch.zeros(1, dtype=torch.int64, device=cuda)
    for seed in (1, 2):
        abi.check(lib.lrk_check_division(1 << 28, seed, counter.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(counter.item()) == 0
