"""GPU parity of the fused scorer (lrk_temporal_scores / _C.temporal_scores).

Reference semantics: for one head, temporal_probabilities + temporal_risk over
all queries (scoring.py:179-195; per-chunk maxima equal the all-query risk).
The fused path sums in a different order, so scores must agree with the
drop-in operators -- which are bit-identical to the reference kernels -- and
with the oracle within 1e-5 relative.  The absolute floor is 1e-6 of the
largest score of the call: scores near zero (a drop close to 0) carry the
absolute, not the relative, error of the probability sums."""
import ctypes
import math

import numpy as np
import pytest

from oracle import lrk_oracle as O

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def assert_scores_close(actual, expected):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert actual.shape == expected.shape
    assert (np.isnan(actual) == np.isnan(expected)).all(), "NaN pattern differs"
    ok = ~np.isnan(expected)
    if not ok.any():
        return
    floor = 1e-6 * np.abs(expected[ok]).max()
    error = np.abs(actual[ok] - expected[ok])
    bound = RTOL * np.abs(expected[ok]) + floor
    worst = np.argmax(error - bound)
    assert (error <= bound).all(), (f"max excess at {worst}: {actual[ok][worst]} vs {expected[ok][worst]}, "
                                    f"max rel {np.max(error / np.maximum(np.abs(expected[ok]), 1e-300))}")


@pytest.fixture(scope="module")
def C(cuda):
    from code_for_iclr27_b200 import operators

    return operators()


def assert_bitwise(actual, expected):
    """Equal scores, NaN where the other has NaN."""
    import torch

    actual, expected = actual.cpu(), expected.cpu()
    assert torch.equal(torch.isnan(actual), torch.isnan(expected))
    same = torch.nan_to_num(actual) == torch.nan_to_num(expected)
    assert bool(same.all()), f"{int((~same).sum())} of {same.numel()} scores differ"


def make_head(g, device, window, groups, length, dtype, masked_queries=0):
    import torch

    logits = (torch.randn(window, groups, length, generator=g) * 2 * math.sqrt(128)).to(dtype).to(device)
    pv = torch.randn(groups, length, generator=g).to(device)
    kpos = torch.arange(length, dtype=torch.float32).to(device)
    qpos = torch.arange(length - window - 1, length - 1, dtype=torch.int64).to(device)
    if masked_queries:
        qpos[:masked_queries] = -1  # every key masked for these queries
    return logits, pv, kpos, qpos


def dropin_scores(C, logits, pv, kpos, qpos, margin, first, last, scale, chunk=79):
    import torch

    result = None
    for start in range(0, logits.shape[0], chunk):
        end = min(start + chunk, logits.shape[0])
        probs, op = C.temporal_probabilities(logits[start:end].contiguous(), pv, qpos[start:end].contiguous(), kpos,
                                             scale)
        s = C.temporal_risk(probs, op, pv, margin, first, last, 1e-6)
        result = s if result is None else torch.maximum(result, s)
    return result


CASES = [
    ("bf16", 250, 4, 4096, 0, 4064),
    ("bf16", 250, 4, 35026, 32768, 34994),
    ("bf16", 79, 8, 3000, 100, 2900),
    ("f16", 30, 4, 1027, 5, 1020),
    ("f32", 17, 2, 513, 0, 513),
    ("bf16", 6, 1, 70001, 60000, 70000),
    ("bf16", 3, 2, 120001, 100, 120000),
    ("f32", 4, 4, 60001, 59000, 60001),
    ("bf16", 8, 4, 18432, 0, 18432),
    ("bf16", 4, 4, 18433, 18000, 18433),
    # 16-byte aligned rows: lane-major packed stage, with and without a tail
    ("bf16", 9, 4, 34816, 32768, 34800),
    ("bf16", 7, 4, 20008, 100, 20000),
    ("f16", 5, 2, 40000, 0, 40000),
    ("bf16", 3, 4, 100000, 99000, 100000),
    # aligned rows just above the fp32-weight stage: the packed stage
    ("bf16", 5, 4, 36864, 100, 36000),
    ("bf16", 6, 8, 18440, 0, 18440),
    ("f16", 4, 2, 25600, 25000, 25600),
]


@pytest.mark.parametrize("dtype_name,window,groups,length,first,last", CASES)
def test_fused_matches_dropin_and_oracle(C, cuda, dtype_name, window, groups, length, first, last):
    import torch

    dtype = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dtype_name]
    g = torch.Generator().manual_seed(length + window)
    logits, pv, kpos, qpos = make_head(g, cuda, window, groups, length, dtype)
    margin = torch.tensor([0.7], device=cuda)
    scale = 1.0 / math.sqrt(128)
    fused = C.temporal_scores([logits], [pv], [kpos], [first], [last], qpos, margin, scale, 1e-6, [79])
    reference = dropin_scores(C, logits, pv, kpos, qpos, margin, first, last, scale, chunk=79)
    assert_bitwise(fused, reference)
    # One chunk of all queries equals the composition with one chunk.
    single = C.temporal_scores([logits], [pv], [kpos], [first], [last], qpos, margin, scale, 1e-6)
    assert_bitwise(single, dropin_scores(C, logits, pv, kpos, qpos, margin, first, last, scale, chunk=window))
    if length <= 5000:
        raw = logits.detach().cpu()
        raw = raw.view(torch.int16).numpy().view(np.uint16) if dtype == torch.bfloat16 else raw.numpy()
        probs, op = O.temporal_probabilities(raw, dtype_name, pv.cpu().numpy(), qpos.cpu().numpy(),
                                             kpos.cpu().numpy(), np.float32(scale))
        expect = O.temporal_risk(probs, op, pv.cpu().numpy(), np.float32(0.7), first, last, 1e-6)
        assert_scores_close(fused.cpu().numpy(), expect)


KEY_LAYOUTS = ["sorted_ties", "shuffled", "sorted_nan", "sorted_inf", "descending"]


@pytest.mark.parametrize("length", [3001, 20011, 24576, 140001])
@pytest.mark.parametrize("layout", KEY_LAYOUTS)
def test_fused_key_position_layouts(C, cuda, layout, length):
    """Masks from every kind of key-position vector: non-decreasing ones take
    the visible-prefix path (its search through sampled positions up to
    131,072 keys, a plain binary search above), the others compare positions
    per key.  Queries sit inside the key range, so each row sees a different
    prefix (some none).  The fused scores must equal the drop-in composition
    bit for bit."""
    import torch

    g = torch.Generator().manual_seed(KEY_LAYOUTS.index(layout) * 7919 + length)
    window, groups, first, last = 37, 4, 7, length - 2
    logits, pv, _, _ = make_head(g, cuda, window, groups, length, torch.bfloat16)
    if layout == "sorted_ties":
        kpos = torch.sort(torch.randint(0, length // 2, (length,), generator=g)).values.float()
    elif layout == "shuffled":
        kpos = torch.randperm(length, generator=g).float()
    elif layout == "sorted_nan":
        kpos = torch.arange(length, dtype=torch.float32)
        kpos[length // 3] = float("nan")
    elif layout == "sorted_inf":
        kpos = torch.arange(length, dtype=torch.float32)
        kpos[-5:] = float("inf")
    else:
        kpos = torch.arange(length, 0, -1, dtype=torch.float32)
    kpos = kpos.to(cuda)
    top = int(torch.nan_to_num(kpos, nan=0.0, posinf=0.0).max().item())
    qpos = torch.randint(top // 3, top + 2, (window,), generator=g, dtype=torch.int64).to(cuda)
    qpos[0] = -1  # a query that sees no key: the head's scores are NaN
    margin = torch.tensor([0.9], device=cuda)
    scale = 1.0 / math.sqrt(128)
    for queries in (qpos, qpos[1:].contiguous()):
        n = queries.shape[0]
        lg = logits[-n:].contiguous()
        fused = C.temporal_scores([lg], [pv], [kpos], [first], [last], queries, margin, scale, 1e-6).cpu()
        expected = dropin_scores(C, lg, pv, kpos, queries, margin, first, last, scale).cpu()
        assert torch.equal(torch.isnan(fused), torch.isnan(expected))
        assert torch.equal(torch.nan_to_num(fused), torch.nan_to_num(expected))


def test_fused_many_segments_strided_and_masked(C, cuda):
    """100 segments (three launches), projected values as strided views of one
    layer-wide matrix, some queries with every key masked (NaN scores)."""
    import torch

    g = torch.Generator().manual_seed(5)
    groups, window = 4, 40
    lengths = torch.randint(50, 700, (100,), generator=g).tolist()
    total = sum(lengths)
    projected = torch.randn(8 * groups, total + 3, generator=g).to(cuda)
    logits, pvs, kpos, firsts, lasts = [], [], [], [], []
    margin = torch.tensor([1.1], device=cuda)
    start = 0
    for i, length in enumerate(lengths):
        lg, _, kp, _ = make_head(g, cuda, window, groups, length, torch.bfloat16)
        head = i % 8
        logits.append(lg)
        pvs.append(projected[head * groups:(head + 1) * groups, start:start + length])
        kpos.append(kp)
        firsts.append(length // 5)
        lasts.append(length - 3)
        start += length
    # one query-position vector is shared by every segment of a call
    qpos = torch.arange(window, dtype=torch.int64, device=cuda) + 10 ** 6
    expected = [dropin_scores(C, lg, pv.contiguous(), kp, qpos, margin, f, l, 0.125)
                for lg, pv, kp, f, l in zip(logits, pvs, kpos, firsts, lasts)]
    fused = C.temporal_scores(logits, pvs, kpos, firsts, lasts, qpos, margin, 0.125, 1e-6, [79] * len(logits))
    assert_bitwise(fused, torch.cat(expected))
    # A query with every key masked makes the whole head NaN, as in the reference.
    masked_qpos = qpos.clone()
    masked_qpos[3] = -5
    fused = C.temporal_scores(logits[:2], pvs[:2], kpos[:2], firsts[:2], lasts[:2], masked_qpos, margin, 0.125, 1e-6)
    assert torch.isnan(fused).all()


def test_fused_long_aligned_segments_of_unequal_length(C, cuda):
    """Segments of 16-byte aligned rows past the fp32-weight stage: the
    persistent statistics kernel walks rows of every segment in one launch,
    with k-blocks inside and past its tensor-memory weight cache (16 blocks
    of 2048 keys), ragged tails, and segments shorter than the cache."""
    import torch

    g = torch.Generator().manual_seed(31)
    lengths = [20008, 36864, 34824, 41000, 18440]
    logits, pvs, kpos, firsts, lasts = [], [], [], [], []
    window, groups = 11, 4
    for length in lengths:
        lg, pv, kp, _ = make_head(g, cuda, window, groups, length, torch.bfloat16)
        logits.append(lg)
        pvs.append(pv)
        kpos.append(kp)
        firsts.append(length // 3)
        lasts.append(length - 32)
    qpos = torch.arange(window, dtype=torch.int64, device=cuda) + max(lengths) - window - 5000
    margin = torch.tensor([0.8], device=cuda)
    fused = C.temporal_scores(logits, pvs, kpos, firsts, lasts, qpos, margin, 0.125, 1e-6, [4] * len(lengths))
    expected = torch.cat([dropin_scores(C, lg, pv, kp, qpos, margin, f, l, 0.125, chunk=4)
                          for lg, pv, kp, f, l in zip(logits, pvs, kpos, firsts, lasts)])
    assert torch.equal(torch.isnan(fused), torch.isnan(expected))
    assert torch.equal(torch.nan_to_num(fused), torch.nan_to_num(expected))


def test_fused_through_c_abi(cuda):
    import torch

    from code_for_iclr27_b200 import abi, operators

    g = torch.Generator().manual_seed(9)
    logits, pv, kpos, qpos = make_head(g, cuda, 50, 4, 2000, torch.bfloat16)
    margin = torch.tensor([0.5], device=cuda)
    out = torch.empty(1900, device=cuda)
    segments = (abi.ScoreSegment * 1)()
    segments[0] = abi.ScoreSegment(logits.data_ptr(), pv.data_ptr(), 2000, kpos.data_ptr(), 2000, 100, 2000,
                                   out.data_ptr(), 2000)
    lib = abi.library()
    size = lib.lrk_temporal_scores_workspace_bytes(1, 50, 4)
    workspace = torch.empty(size, dtype=torch.uint8, device=cuda)
    abi.check(lib.lrk_temporal_scores(segments, 1, abi.BF16, qpos.data_ptr(), 50, 4, 0.125, margin.data_ptr(), 1e-6,
                                      workspace.data_ptr(), size, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    expected = dropin_scores(operators(), logits, pv, kpos, qpos, margin, 100, 2000, 0.125)
    assert_scores_close(out.cpu().numpy(), expected.cpu().numpy())
    assert lib.lrk_temporal_scores(segments, 1, abi.BF16, qpos.data_ptr(), 50, 4, 0.125, margin.data_ptr(), 1e-6,
                                   workspace.data_ptr(), 8, 0) == abi.ERR_WORKSPACE


def test_audit_tables_agree(cuda):
    """The audit driver's fused score table matches its drop-in score table.
    At these small head sizes cuBLAS may reduce the float32 projection g V^T in
    another order than the fused projection, so the scores agree to 1e-5
    relative; at configs[1] head size they are equal bit for bit (below)."""
    import torch

    from code_for_iclr27_b200.audit import score_table, score_table_fused
    from code_for_iclr27_b200.kvcache import PackedCache

    g = torch.Generator().manual_seed(2)
    cache = PackedCache()
    layers, heads, groups, dim, window = 2, 4, 4, 64, 30
    for layer in range(layers):
        lens = torch.randint(200, 600, (heads,), generator=g).tolist()
        rows = sum(lens)
        keys = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(cuda)
        values = torch.randn(rows, dim, generator=g).to(torch.bfloat16).to(cuda)
        positions = torch.cat([torch.arange(n, dtype=torch.float32) for n in lens]).to(cuda)
        cache.add_layer(keys, values, positions, lens, [40, 0, 100, 10])
    queries = [(torch.randn(window, heads * groups, dim, generator=g) * 2).to(torch.bfloat16).to(cuda)
               for _ in range(layers)]
    grads = [torch.randn(heads * groups, dim, generator=g).to(cuda) / 8 for _ in range(layers)]
    qpos = torch.arange(570, 570 + window, dtype=torch.int64, device=cuda)
    margin = torch.tensor(0.9, device=cuda)
    a = score_table(cache, queries, qpos, grads, margin, query_chunk_size=7)
    b = score_table_fused(cache, queries, qpos, grads, margin, query_chunk_size=7)
    assert a.segments == b.segments and a.cumulative_ends == b.cumulative_ends
    assert_scores_close(b.scores.cpu().numpy(), a.scores.cpu().numpy())


def test_configs1_layers_fused_equals_composition(cuda):
    """Two layers at configs[1] shape (8 KV heads of ~34.8k rows, D = 128,
    250 queries, 4 groups): the fused table equals the drop-in composition bit
    for bit -- same bf16 logits GEMM, projected values in the float32 GEMM's
    order, the composition's 80-query chunks."""
    import torch

    from code_for_iclr27_b200.audit import score_table, score_table_fused
    from code_for_iclr27_b200.kvcache import PackedCache

    g = torch.Generator(device=cuda).manual_seed(4)
    rng = np.random.default_rng(4)
    cache = PackedCache()
    layers, heads, groups, dim, window, prompt = 2, 8, 4, 128, 250, 32768
    for _ in range(layers):
        lens = [prompt + int(n) for n in rng.integers(1700, 2300, heads)]
        rows = sum(lens)
        keys = torch.randn(rows, dim, generator=g, device=cuda).to(torch.bfloat16)
        values = torch.randn(rows, dim, generator=g, device=cuda).to(torch.bfloat16)
        positions = torch.cat([torch.arange(n, dtype=torch.float32) for n in lens]).to(cuda)
        cache.add_layer(keys, values, positions, lens, [prompt] * heads)
    top = max(max(layer.head_lens) for layer in cache.layers)
    queries = [(torch.randn(window, heads * groups, dim, generator=g, device=cuda) * 2).to(torch.bfloat16)
               for _ in range(layers)]
    grads = [torch.randn(heads * groups, dim, generator=g, device=cuda) / math.sqrt(dim) for _ in range(layers)]
    qpos = torch.arange(top - window, top, dtype=torch.int64, device=cuda)
    margin = torch.tensor(1.0, device=cuda)
    a = score_table(cache, queries, qpos, grads, margin)
    b = score_table_fused(cache, queries, qpos, grads, margin)
    assert a.segments == b.segments
    assert_bitwise(b.scores, a.scores)


@pytest.mark.parametrize("length,gap,groups", [(3001, 11, 4), (30001, 11, 4), (30001, 0, 4), (3003, 0, 8),
                                               (30003, 0, 2)])
def test_fused_padded_logits_rows(C, cuda, length, gap, groups):
    """Logits rows with a stride larger than the row (a GEMM over a padded key
    block) score exactly like contiguous rows.  The padded rows are 16-byte
    aligned and take the vectorised kernels (the packed stage beyond 18k keys,
    vector risk loads with a ragged last vector when the candidates reach the
    row's end); the contiguous ones take the scalar kernels."""
    import torch

    g = torch.Generator().manual_seed(12 + length + groups)
    logits, pv, kpos, qpos = make_head(g, cuda, 40, groups, length, torch.bfloat16)
    padded = torch.zeros(40, groups, (length + 7) // 8 * 8, dtype=torch.bfloat16, device=cuda)
    padded[:, :, :length] = logits
    margin = torch.tensor([0.9], device=cuda)
    a = C.temporal_scores([logits], [pv], [kpos], [10], [length - gap], qpos, margin, 0.125, 1e-6)
    b = C.temporal_scores([padded[:, :, :length]], [pv], [kpos], [10], [length - gap], qpos, margin, 0.125, 1e-6)
    assert torch.equal(torch.isnan(a), torch.isnan(b))
    assert torch.equal(torch.nan_to_num(a), torch.nan_to_num(b))


PROJECT_CASES = [
    (4, "bf16", 128, 0), (8, "bf16", 128, 0), (1, "f32", 128, 0), (2, "f16", 128, 0),
    (1, "bf16", 64, 0), (8, "bf16", 64, 0), (4, "f16", 256, 0), (2, "bf16", 256, 0),
    (4, "bf16", 72, 0),    # D = 72: the thread-per-row kernel with runtime D
    (4, "bf16", 128, 1),   # values start 2 bytes past a 16-byte boundary: scalar loads
]


@pytest.mark.parametrize("groups,dtype_name,dim,offset", PROJECT_CASES)
def test_project_values(C, cuda, groups, dtype_name, dim, offset):
    """Per-head g V^T over a packed layer against a float64 reference.  Head
    lengths include empty heads and heads shorter than one warp's rows."""
    import torch

    dtype = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dtype_name]
    g = torch.Generator().manual_seed(groups * 1000 + dim + offset)
    lengths = [300, 0, 1025, 77, 4000, 12, 999, 1, 3, 5000]
    heads = len(lengths)
    rows = sum(lengths)
    storage = torch.randn(rows * dim + offset, generator=g).to(dtype).to(cuda)
    values = storage[offset:].view(rows, dim)
    grads = torch.randn(heads * groups, dim, generator=g).to(cuda)
    cumulative = torch.tensor(np.concatenate(([0], np.cumsum(lengths))), dtype=torch.int32, device=cuda)
    out = C.project_values(values, grads, cumulative, groups)
    v64, g64 = values.double().cpu(), grads.double().cpu()
    start = 0
    for h, n in enumerate(lengths):
        expect = g64[h * groups:(h + 1) * groups] @ v64[start:start + n].T
        # float32 accumulation of `dim` terms of size ~1: error ~ sqrt(dim) * 2^-24 * |sum|
        np.testing.assert_allclose(out[:, start:start + n].double().cpu().numpy(), expect.numpy(), rtol=1e-5,
                                   atol=1e-7 * dim)
        start += n


@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("groups", [1, 2, 4, 8])
def test_project_values_unrolled_equals_runtime_dim(C, cuda, groups, dim):
    """16-byte aligned rows of D = 64 / 128 take the unrolled kernel; rows
    2 bytes past a boundary take the runtime-D kernel with scalar loads.  Both
    accumulate each dot product in channel order, so the same values give the
    same bits."""
    import torch

    g = torch.Generator(device=cuda).manual_seed(groups + dim)
    lengths = [3000, 0, 513, 7, 2048]
    rows = sum(lengths)
    storage = torch.randn(rows * dim + 1, generator=g, device=cuda).to(torch.bfloat16)
    aligned = storage[:rows * dim].view(rows, dim).clone()
    shifted = storage[1:].view(rows, dim)
    shifted.copy_(aligned)
    grads = torch.randn(len(lengths) * groups, dim, generator=g, device=cuda)
    cumulative = torch.tensor(np.concatenate(([0], np.cumsum(lengths))), dtype=torch.int32, device=cuda)
    a = C.project_values(aligned, grads, cumulative, groups)
    b = C.project_values(shifted, grads, cumulative, groups)
    assert torch.equal(a, b)


def test_project_values_equal_float32_gemm_at_configs1_shape(C, cuda):
    """At configs[1] head size (~34.8k rows, D = 128, 4 groups) the projection
    equals the float32 GEMM the reference runs (scoring.py:175) bit for bit:
    both accumulate each dot product in channel order with fused multiply-adds.
    (For much smaller heads cuBLAS may pick another reduction order; there the
    projection agrees to float32 rounding, as test_project_values checks.)"""
    import torch

    g = torch.Generator(device=cuda).manual_seed(9)
    lengths = [34880, 34450, 34183, 35001]
    values = torch.randn(sum(lengths), 128, generator=g, device=cuda).to(torch.bfloat16)
    grads = torch.randn(len(lengths) * 4, 128, generator=g, device=cuda) / math.sqrt(128)
    cumulative = torch.tensor(np.concatenate(([0], np.cumsum(lengths))), dtype=torch.int32, device=cuda)
    out = C.project_values(values, grads, cumulative, 4)
    start = 0
    for h, n in enumerate(lengths):
        gemm = torch.matmul(grads[h * 4:(h + 1) * 4].float(), values[start:start + n].float().transpose(0, 1))
        assert torch.equal(out[:, start:start + n], gemm), f"head {h}"
        start += n


@pytest.mark.parametrize("rows,count,dim", [(1000, 34183, 128), (1000, 34880, 128), (320, 34191, 128),
                                            (320, 34450, 128), (8, 1, 128), (8, 2, 128), (1000, 2001, 128),
                                            (37, 513, 64), (120, 7, 64), (64, 130, 128), (129, 65, 128)])
def test_logits_equal_torch_matmul(C, cuda, rows, count, dim):
    """lrk_logits with the step torch.matmul's GEMM takes for this key count
    (8 terms for an odd count, 16 otherwise) equals torch.matmul bit for bit
    (scoring.py:184), written into padded rows."""
    import torch

    g = torch.Generator(device=cuda).manual_seed(rows + count)
    queries = (torch.randn(rows, dim, generator=g, device=cuda) * 2).to(torch.bfloat16)
    keys = torch.randn(count + 3, dim, generator=g, device=cuda).to(torch.bfloat16)[1:count + 1].contiguous()
    stride = (count + 7) // 8 * 8
    out = C.logits(queries, keys, 8 if count % 2 else 16, stride)
    assert out.shape == (rows, stride)
    assert torch.equal(out[:, :count], torch.matmul(queries, keys.transpose(0, 1)))
    from code_for_iclr27_b200 import abi

    timeouts = ctypes.c_uint(0)
    abi.check(abi.library().lrk_logits_timeouts(ctypes.byref(timeouts)))
    assert timeouts.value == 0


@pytest.mark.parametrize("rows,counts,dim", [
    (1000, [34880, 34881, 34883, 34878, 34885, 34880, 34879, 34882], 128),  # one configs[1] layer
    (2000, [300, 301, 257, 130, 7, 2, 129, 640, 1, 382, 255, 256, 3, 511, 128, 999], 128),  # ranges cross heads
    (1000, [5000 + 3 * i for i in range(20)], 128),  # more heads than one launch takes
    (37, [513, 0, 514, 1, 6000], 64),
    (129, [65, 66, 0, 4097], 128),
])
def test_logits_heads_equal_torch_matmul(C, cuda, rows, counts, dim):
    """lrk_logits_heads -- every head of a layer in one launch, each in the
    step order torch.matmul's GEMM takes for its key count -- equals
    a plain torch.matmul GEMM per head bit for bit wherever cuBLAS takes that
    order for it (plain_gemm_order_matches), and lrk_logits per head
    everywhere."""
    import torch


    g = torch.Generator(device=cuda).manual_seed(rows + sum(counts))
    heads = len(counts)
    queries = (torch.randn(heads, rows, dim, generator=g, device=cuda) * 2).to(torch.bfloat16)
    bounds = [0]
    for n in counts:
        bounds.append(bounds[-1] + n)
    keys = torch.randn(bounds[-1] + 8, dim, generator=g, device=cuda).to(torch.bfloat16)
    order = list(range(heads))[::-1]  # entries need not follow head order
    outs = C.logits_heads(queries, keys, order, [bounds[h] for h in order], [bounds[h + 1] for h in order],
                          [8 if counts[h] % 2 else 16 for h in order])
    for out, h in zip(outs, order):
        n = counts[h]
        assert out.shape == (rows, (n + 127) // 128 * 128)
        if n == 0:
            continue
        head_keys = keys[bounds[h]:bounds[h + 1]]
        if plain_gemm_order_matches(n, rows):
            assert torch.equal(out[:, :n], torch.matmul(queries[h], head_keys.transpose(0, 1))), f"head {h}"
        if h % 5 == 0 or not plain_gemm_order_matches(n, rows):
            single = C.logits(queries[h].contiguous(), head_keys.contiguous(), 8 if n % 2 else 16, out.shape[1])
            assert torch.equal(single[:, :n], out[:, :n]), f"head {h} vs lrk_logits"
    from code_for_iclr27_b200 import abi

    timeouts = ctypes.c_uint(0)
    abi.check(abi.library().lrk_logits_timeouts(ctypes.byref(timeouts)))
    assert timeouts.value == 0


def plain_gemm_order_matches(count, rows):
    """Where a plain [rows, D] x [D, count] bf16 torch.matmul GEMM takes the
    16-term (even count) or 8-term (odd count) tensor-core order (measured on
    B200 for rows 8 .. 2000: odd counts below 288 keys, and below 4098 at 8
    rows, run other kernels)."""
    return count % 2 == 0 or (count >= 1024 and rows >= 40)


def reference_chunks(head_queries, keys, chunk):
    """The reference's logits of one head (scoring.py:177-184): torch.matmul
    of the permuted query-history view, per query chunk."""
    import torch

    from code_for_iclr27_b200.audit import reference_query_view

    mapped = reference_query_view(head_queries)
    return torch.cat([torch.matmul(mapped[a:a + chunk], keys.transpose(0, 1))
                      for a in range(0, mapped.shape[0], chunk)])


@pytest.mark.parametrize("groups,window,chunk_size", [(1, 40, 250), (2, 250, 250), (4, 250, 250), (4, 37, 7),
                                                      (8, 9, 250), (8, 37, 7), (4, 100, 30)])
def test_tensor_core_order_rule_against_reference_gemm(C, cuda, groups, window, chunk_size):
    """Wherever tensor_core_order_matches says so, lrk_logits equals the
    reference's batched GEMM bit for bit; the sweep covers the small key
    counts and chunks for which cuBLAS picks other kernels."""
    import torch

    from code_for_iclr27_b200.audit import query_chunk, tensor_core_order_matches

    g = torch.Generator(device=cuda).manual_seed(groups * 1000 + window)
    queries = (torch.randn(window, groups, 128, generator=g, device=cuda) * 2).to(torch.bfloat16)
    keys = torch.randn(35000, 128, generator=g, device=cuda).to(torch.bfloat16)
    flat = queries.reshape(window * groups, 128)
    checked = 0
    for n in list(range(1, 80, 3)) + list(range(250, 330, 5)) + [1023, 1024, 1025, 2048, 2049, 4097, 16385, 34881]:
        chunk = query_chunk(chunk_size, groups, n, 2)
        if not tensor_core_order_matches(n, window, groups, chunk):
            continue
        out = C.logits(flat, keys[:n], 8 if n % 2 else 16, (n + 7) // 8 * 8)[:, :n].view(window, groups, n)
        assert torch.equal(out, reference_chunks(queries, keys[:n], chunk)), f"{n} keys"
        checked += 1
    assert checked > 0 or groups == 1


@pytest.mark.parametrize("groups", [2, 4, 8])
def test_tensor_core_order_rule_per_batch(C, cuda, groups):
    """One cuBLAS call per query chunk: at every batch size the rule lets
    through (tensor_core_order_matches with one chunk of `batch` queries),
    lrk_logits equals the reference's batched GEMM at odd key counts from
    1025 to 34,881 bit for bit."""
    import torch

    from code_for_iclr27_b200.audit import tensor_core_order_matches

    g = torch.Generator(device=cuda).manual_seed(groups)
    keys = torch.randn(34881, 128, generator=g, device=cuda).to(torch.bfloat16)
    checked = 0
    for batch in list(range(1, 31)) + [80, 81, 82, 83, 100, 170, 250]:
        queries = (torch.randn(batch, groups, 128, generator=g, device=cuda) * 2).to(torch.bfloat16)
        flat = queries.reshape(batch * groups, 128)
        for n in (1025, 4097, 16385, 24577, 34087, 34881):
            if not tensor_core_order_matches(n, batch, groups, batch):
                continue
            out = C.logits(flat, keys[:n], 8, (n + 7) // 8 * 8)[:, :n].view(batch, groups, n)
            assert torch.equal(out, reference_chunks(queries, keys[:n], batch)), f"batch {batch}, {n} keys"
            checked += 1
    assert checked > 100


@pytest.mark.parametrize("window,groups", [(250, 4), (9, 4), (100, 8), (40, 1)])
def test_layer_logits_equal_reference_chunks(C, cuda, window, groups):
    """layer_logits (the audit's logits: one lrk_logits_heads launch plus the
    reference GEMM for the heads whose order it does not reproduce) equals
    the reference's per-chunk torch.matmul (scoring.py:177-184) for every
    head of a layer."""
    import torch

    from code_for_iclr27_b200.audit import layer_logits, query_chunk

    g = torch.Generator(device=cuda).manual_seed(window * groups)
    lens = [34880, 34881, 3, 290, 1025, 2048, 35000, 511]
    bounds = [0]
    for n in lens:
        bounds.append(bounds[-1] + n)
    keys = torch.randn(bounds[-1], 128, generator=g, device=cuda).to(torch.bfloat16)
    per_head = (torch.randn(len(lens), window, groups, 128, generator=g, device=cuda) * 2).to(torch.bfloat16)
    spans = [(h, bounds[h], bounds[h + 1], query_chunk(250, groups, n, 2)) for h, n in enumerate(lens)]
    got = layer_logits(per_head.view(len(lens), window * groups, 128), keys, spans, window, groups)
    for (h, start, end, chunk), logits in zip(spans, got):
        expect = reference_chunks(per_head[h], keys[start:end], chunk)
        assert logits.shape == expect.shape
        assert torch.equal(logits, expect), f"head {h} ({end - start} keys, chunk {chunk})"


def test_layer_logits_runtime_order_check(C, cuda, monkeypatch):
    """The first head of each (groups, parity, window, chunk) class goes
    through lrk_logits and is checked against the reference GEMM; a class
    marked as failed takes the reference GEMM for all its heads (no
    lrk_logits_heads launch for them) and the logits still equal the
    reference's."""
    import torch

    from code_for_iclr27_b200 import audit

    monkeypatch.setattr(audit, "_ORDER_VERIFIED", {})
    g = torch.Generator(device=cuda).manual_seed(77)
    window, groups, lens = 250, 4, [4096, 4097, 4098]
    bounds = [0, 4096, 8193, 12291]
    keys = torch.randn(bounds[-1], 128, generator=g, device=cuda).to(torch.bfloat16)
    per_head = (torch.randn(len(lens), window, groups, 128, generator=g, device=cuda) * 2).to(torch.bfloat16)
    spans = [(h, bounds[h], bounds[h + 1], audit.query_chunk(250, groups, n, 2)) for h, n in enumerate(lens)]
    flat = per_head.view(len(lens), window * groups, 128)
    audit.layer_logits(flat, keys, spans, window, groups)
    even = audit._order_class(4096, window, groups, spans[0][3])
    odd = audit._order_class(4097, window, groups, spans[1][3])
    assert audit._ORDER_VERIFIED == {even: True, odd: True}
    audit._ORDER_VERIFIED[even] = False  # as if this cuBLAS took another order for even counts
    launched = []
    original = C.logits_heads

    def counting(per_head_arg, keys_arg, heads, *rest):
        launched.extend(heads)
        return original(per_head_arg, keys_arg, heads, *rest)

    monkeypatch.setattr(audit, "operators", lambda: type("Ops", (), {"logits_heads": staticmethod(counting)})())
    got = audit.layer_logits(flat, keys, spans, window, groups)
    assert launched == [1]  # only the odd head
    for (h, start, end, chunk), logits in zip(spans, got):
        assert torch.equal(logits, reference_chunks(per_head[h], keys[start:end], chunk))


def test_logits_heads_rejects_bad_arguments(C, cuda):
    """lrk_logits_heads checks every head like lrk_logits (step, stride,
    alignment) before anything runs."""
    import torch

    from code_for_iclr27_b200 import abi

    queries = torch.zeros(2, 16, 128, dtype=torch.bfloat16, device=cuda)
    keys = torch.zeros(64, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError):
        C.logits_heads(queries, keys, [0], [0], [64], [4])
    with pytest.raises(RuntimeError):
        C.logits_heads(queries, keys, [2], [0], [64], [16])
    out = torch.empty(16, 64, dtype=torch.bfloat16, device=cuda)
    table = (abi.LogitsHead * 1)()
    table[0].queries, table[0].keys, table[0].count = queries.data_ptr(), keys.data_ptr(), 64
    table[0].k_step, table[0].out, table[0].out_stride = 16, out.data_ptr(), 60
    lib = abi.library()
    assert lib.lrk_logits_heads(table, 1, 16, 128, None) == abi.ERR_INVALID  # stride not a multiple of 8
    table[0].out_stride, table[0].keys = 64, keys.data_ptr() + 2
    assert lib.lrk_logits_heads(table, 1, 16, 128, None) == abi.ERR_INVALID  # unaligned keys
    table[0].keys = keys.data_ptr()
    abi.check(lib.lrk_logits_heads(table, 1, 16, 128, None))
    torch.cuda.synchronize()
    assert torch.equal(out, torch.matmul(queries[0], keys.transpose(0, 1)))
