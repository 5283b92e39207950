"""Per-operator speed against the reference's own CUDA operators (built from
its sources into oracle/_ref for sm_100a), at configs[1] shapes.

Each operator is timed on the device only: the GPU is held in a sleep kernel
while the host queues REPEAT back-to-back calls behind a start event, so the
span between the events is the calls' device time and not the host's launch
overhead.  L2 is flushed (256 MiB written) before each span.  The figure is
the median over ROUNDS spans, ours and the reference's alternating.  The test
fails if an operator of ours takes more than 10 % longer than the
reference's, plus ABS_SLACK_US per call for the launch-latency-sized ones.
The table is written to pytest's tmp_path and printed (-s).

This file sorts after every parity test file except the static-scratch test,
so a speed regression cannot hide a parity result under -x.

    python -m pytest tests/test_zy_speed_vs_reference.py -m gpu -s
"""
import importlib.util
import json
import math

import pytest

pytestmark = pytest.mark.gpu
REPEAT, ROUNDS = 20, 9
ABS_SLACK_US = 0.5


@pytest.fixture(scope="module")
def modules(cuda):
    from code_for_iclr27_b200 import operators
    from oracle import build_ref

    paths = build_ref.built_paths()
    if "C" not in paths:
        pytest.skip("reference modules not built (oracle/build_ref.py)")
    spec = importlib.util.spec_from_file_location("lazy_recall_reference._C", paths["C"])
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    return operators(), ref


def span_ms(fn, flush):
    """Device time of one call: REPEAT calls queued behind a sleeping GPU."""
    import torch

    flush.zero_()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(2_000_000)  # ~1 ms at B200 clocks: the host queues every call meanwhile
    a.record()
    for _ in range(REPEAT):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / REPEAT


def paired_ms(ours, theirs, flush):
    import torch

    for _ in range(3):
        ours()
        theirs()
    torch.cuda.synchronize()
    mine, ref = [], []
    for _ in range(ROUNDS):
        mine.append(span_ms(ours, flush))
        ref.append(span_ms(theirs, flush))
    return sorted(mine)[ROUNDS // 2], sorted(ref)[ROUNDS // 2]


def test_operators_not_slower_than_reference(modules, cuda, tmp_path):
    import torch

    C, R = modules
    dev = cuda
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    rows, d = 8 * 35026, 128
    row_bytes = 4 * d + 4
    K = torch.randn(rows, d, generator=g, device=dev).to(torch.bfloat16)
    V = torch.randn(rows, d, generator=g, device=dev).to(torch.bfloat16)
    P = torch.arange(rows, dtype=torch.float32, device=dev).reshape(-1, 1)
    cases = {}
    for tag, removed_count in (("lazy64", 64), ("half", rows // 2)):
        removed = torch.randperm(rows, generator=g, device=dev)[:removed_count].sort().values
        kept = rows - removed_count
        cases[f"compact_{tag}"] = (2 * kept * row_bytes, lambda r=removed: C.compact(K, V, P, r),
                                   lambda r=removed: R.compact(K, V, P, r))
    cumulative = torch.arange(0, rows + 1, 35026, dtype=torch.int32, device=dev)
    new = torch.randn(1, 8, 1, d, generator=g, device=dev).to(torch.bfloat16)
    cases["append"] = (2 * (rows + 8) * row_bytes, lambda: C.append(K, V, P, new, new, cumulative, 40000, 35026),
                       lambda: R.append(K, V, P, new, new, cumulative, 40000, 35026))
    caches = []
    for _ in range(8):
        n = 8 * 10704
        caches.append((torch.randn(n, d, generator=g, device=dev).to(torch.bfloat16),
                       torch.randn(n, d, generator=g, device=dev).to(torch.bfloat16),
                       torch.arange(n, dtype=torch.float32, device=dev).reshape(-1, 1), [n // 8] * 8))
    bk = torch.randn(8, 8, 1, d, generator=g, device=dev).to(torch.bfloat16)
    args = ([c[0] for c in caches], [c[1] for c in caches], [c[2] for c in caches], bk, bk,
            [c[3] for c in caches], [5] * 8)
    total = sum(c[0].shape[0] for c in caches) + 64
    cases["batch_append"] = (2 * total * row_bytes, lambda: C.batch_append(*args), lambda: R.batch_append(*args))
    mk = torch.randn(16000, d, generator=g, device=dev).to(torch.bfloat16)
    mp = torch.arange(16000, dtype=torch.float32, device=dev).reshape(-1, 1)
    recalled = torch.randn(256, 2, d, generator=g, device=dev).to(torch.bfloat16)
    recalled_pos = torch.arange(256, dtype=torch.float32, device=dev)
    mapping = torch.cat([torch.arange(16000, device=dev), -torch.arange(1, 257, device=dev)])
    mapping = mapping[torch.randperm(16256, generator=g, device=dev)]
    cases["merge"] = (2 * 16256 * row_bytes, lambda: C.merge(mk, mk, mp, recalled, recalled_pos, mapping),
                      lambda: R.merge(mk, mk, mp, recalled, recalled_pos, mapping))
    indices = torch.randperm(rows, generator=g, device=dev)[:2048]
    heads = torch.randint(0, 8, (2048,), generator=g, device=dev)
    payload = torch.empty(2048, 2, d, dtype=torch.bfloat16, device=dev)
    metadata = torch.empty(2048, 3, dtype=torch.int64, device=dev)
    cases["pack"] = (2048 * (8 * d + 24), lambda: C.pack(K, V, P, indices, heads, 3, payload, metadata),
                     lambda: R.pack(K, V, P, indices, heads, 3, payload, metadata))
    for tag, window, length in (("cfg1_chunk", 79, 35026), ("cfg0_head", 250, 4096)):
        logits = (torch.randn(window, 4, length, generator=g, device=dev) * 2 * math.sqrt(128)).to(torch.bfloat16)
        pv = torch.rand(4, length, generator=g, device=dev)
        qpos = torch.arange(length - window, length, dtype=torch.int64, device=dev)
        kpos = torch.arange(length, dtype=torch.float32, device=dev)
        cases[f"probabilities_{tag}"] = (window * 4 * length * 6,
                                         lambda a=(logits, pv, qpos, kpos): C.temporal_probabilities(*a, 0.0883883),
                                         lambda a=(logits, pv, qpos, kpos): R.temporal_probabilities(*a, 0.0883883))
        probs, op = C.temporal_probabilities(logits, pv, qpos, kpos, 0.0883883)
        margin = torch.tensor([1.0], device=dev)
        first = 0 if tag == "cfg0_head" else length - 2258
        last = length - 32
        cases[f"risk_{tag}"] = (window * 4 * (last - first) * 4,
                                lambda a=(probs, op, pv, margin, first, last): C.temporal_risk(*a, 1e-6),
                                lambda a=(probs, op, pv, margin, first, last): R.temporal_risk(*a, 1e-6))
    n = 256 * 1962
    raw = torch.rand(n, generator=g, device=dev)
    bounds = torch.arange(0, n + 1, 1962, dtype=torch.int64, device=dev)
    cases["pool"] = (8 * n, lambda: C.pool(raw, bounds, 1962, 7), lambda: R.pool(raw, bounds, 1962, 7))
    report, slower = {}, []
    for name, (nbytes, ours, theirs) in cases.items():
        t_ours, t_ref = paired_ms(ours, theirs, flush)
        report[name] = {"us": t_ours * 1e3, "GBps": nbytes / t_ours / 1e6, "reference_us": t_ref * 1e3,
                        "reference_GBps": nbytes / t_ref / 1e6, "speedup": t_ref / t_ours}
        print(name, json.dumps(report[name]))
        if t_ours * 1e3 > 1.10 * t_ref * 1e3 + ABS_SLACK_US:
            slower.append(name)
    (tmp_path / "operators_vs_reference.json").write_text(json.dumps(report, indent=1))
    assert not slower, f"slower than the reference kernels: {slower}"
