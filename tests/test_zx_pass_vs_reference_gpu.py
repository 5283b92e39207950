"""A whole configs[1] audit pass through the reference's own GPU path, against
this repository's audit_pass, on one B200: the speed bar and a full-size
parity check at once.

The reference arm is the reference's unchanged Python package (oracle/_ref/py)
with its native modules bound to the reference's own CUDA operators, built
from its csrc/ for sm_100a (oracle/_ref/{C,legacy_C,host}): the controller's
audit (controller.py:140-160) -- compute_score_table (scoring.py:199-308: per
head torch.matmul logits, _C.temporal_probabilities, _C.temporal_risk),
pool_score_table, allocation_preserving_references (refine_arrays) and
LazyRecallCache.remove_positions (_C.compact per touched layer).  Our arm is
audit.audit_pass on a PackedCache holding the same rows.

Shape: 32 layers x 8 KV heads x D128, GQA 4 (Llama-3-8B), 32,768 prompt rows
and 2,000 generation rows per head, a 250-query window; 512 immediate and
64,000 queued references (the bench's configs[1] counts).  Both arms see the
same keys, values, positions, queries and gradients; the score tables must be
equal bit for bit, the queues equal, and the caches after the eviction equal
row for row.  Each arm runs once untimed, then the timed pass (CUDA events
around the whole pass; the reference's path synchronises inside it).  The
table is written to pytest's tmp_path and printed (-s).  Skipped when the
reference package or its built modules are absent.

    python -m pytest tests/test_zx_pass_vs_reference_gpu.py -m gpu -s
"""
import importlib
import importlib.util
import json
import sys
from types import SimpleNamespace

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LAYERS, HEADS, GROUPS, DIM, HIDDEN = 32, 8, 4, 128, 4096
PROMPT, GENERATED, WINDOW = 32768, 2000, 250
IMMEDIATE, QUEUED, PROTECT, POOL = 512, 64000, 32, 7


@pytest.fixture(scope="module")
def reference(cuda):
    """The reference package with its native modules bound to its own builds."""
    from oracle import build_ref
    from oracle.install_ref_py import installed

    where, paths = installed(), build_ref.built_paths()
    if where is None or not {"C", "legacy_C", "host"} <= set(paths):
        pytest.skip("reference package or its built modules absent (oracle/install_ref_py.py, build_ref.py)")
    for name in [m for m in sys.modules if m == "lazy_recall" or m.startswith("lazy_recall.")]:
        del sys.modules[name]
    sys.path.insert(0, str(where))
    try:
        package = importlib.import_module("lazy_recall")
        for key in ("C", "legacy_C", "host"):
            spec = importlib.util.spec_from_file_location(f"lazy_recall._{key}", paths[key])
            module = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(module)
            sys.modules[f"lazy_recall._{key}"] = module
            setattr(package, f"_{key}", module)
        yield SimpleNamespace(
            cache=importlib.import_module("lazy_recall.cache"),
            scoring=importlib.import_module("lazy_recall.scoring"),
            history=importlib.import_module("lazy_recall.history"),
            native=sys.modules["lazy_recall._C"],
        )
    finally:
        sys.path.remove(str(where))
        for name in [m for m in sys.modules if m == "lazy_recall" or m.startswith("lazy_recall.")]:
            del sys.modules[name]


def test_audit_pass_against_reference_gpu_path(reference, cuda, tmp_path):
    import torch

    from code_for_iclr27_b200 import operators
    from code_for_iclr27_b200.audit import audit_pass
    from code_for_iclr27_b200.kvcache import PackedCache
    from code_for_iclr27_b200.workloads import _restore, _snapshot

    assert reference.scoring.extension() is reference.native  # the reference's own _C, not ours
    assert reference.native is not operators()
    g = torch.Generator(device=cuda).manual_seed(0)
    ref_cache = reference.cache.LazyRecallCache()
    with torch.no_grad():
        for layer in range(LAYERS):
            k = torch.randn(1, HEADS, PROMPT, DIM, generator=g, device=cuda).to(torch.bfloat16)
            v = torch.randn(1, HEADS, PROMPT, DIM, generator=g, device=cuda).to(torch.bfloat16)
            ref_cache.update(k, v, layer)
        ref_cache.freeze_prompt()
        for layer in range(LAYERS):  # the generation rows: one multi-token append per layer (_C.append)
            k = torch.randn(1, HEADS, GENERATED, DIM, generator=g, device=cuda).to(torch.bfloat16)
            v = torch.randn(1, HEADS, GENERATED, DIM, generator=g, device=cuda).to(torch.bfloat16)
            ref_cache.update(k, v, layer)
    ours = PackedCache()
    for layer in range(LAYERS):
        meta = ref_cache.metadata_list[layer]
        ours.add_layer(ref_cache.key_cache[layer].clone(), ref_cache.value_cache[layer].clone(),
                       ref_cache.position_cache[layer].clone(), list(meta.head_lens_cpu), list(meta.prompt_lens_cpu))
    ours.seen_tokens = int(ref_cache._seen_tokens)

    # Queries of the last WINDOW steps, a model stub with one o_proj weight, the audit's gradients.
    seen = int(ref_cache._seen_tokens)
    history = reference.history.QueryHistory(LAYERS, WINDOW)
    steps = (torch.randn(WINDOW, LAYERS, HEADS * GROUPS, DIM, generator=g, device=cuda) * 2).to(torch.bfloat16)
    for step in range(WINDOW):
        history.append([steps[step, layer].view(1, HEADS * GROUPS, 1, DIM) for layer in range(LAYERS)],
                       seen - WINDOW + step)
    weight = torch.randn(HIDDEN, HEADS * GROUPS * DIM, generator=g, device=cuda) / 64
    config = SimpleNamespace(num_attention_heads=HEADS * GROUPS, num_key_value_heads=HEADS)
    model = SimpleNamespace(model=SimpleNamespace(layers=[SimpleNamespace(self_attn=SimpleNamespace(
        config=config, head_dim=DIM, o_proj=SimpleNamespace(weight=weight))) for _ in range(LAYERS)]))
    post = [torch.randn(1, 1, HIDDEN, generator=g, device=cuda) / 8 for _ in range(LAYERS)]
    audit = SimpleNamespace(attention_gradients=post, margin=torch.tensor(1.0, device=cuda))
    queries = [steps[:, layer].contiguous() for layer in range(LAYERS)]
    gradients = [torch.matmul(p[0, -1].float(), weight.float()).view(HEADS * GROUPS, DIM) for p in post]
    _, positions = history.layer(0)
    qpos = torch.as_tensor(positions, dtype=torch.int64, device=cuda).reshape(-1)
    margin = torch.tensor([1.0], device=cuda)

    def reference_pass(evict):
        with torch.no_grad():
            table = reference.scoring.compute_score_table(model, ref_cache, audit, history, True, PROTECT,
                                                          1e-6, 250).table
            pooled = reference.scoring.pool_score_table(table, POOL)
            references = reference.scoring.allocation_preserving_references(table, pooled,
                                                                            IMMEDIATE + QUEUED).references
            if evict:
                ref_cache.remove_positions({key: values.tolist()
                                            for key, values in references[:IMMEDIATE].groups().items()})
        return table, references

    def our_pass():
        return audit_pass(ours, queries, qpos, gradients, margin, IMMEDIATE, QUEUED, PROTECT)

    def timed(fn):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        out = fn()
        b.record()
        torch.cuda.synchronize()
        return out, a.elapsed_time(b)

    saved = _snapshot(ours)
    our_pass()  # untimed: first-use costs (streams, the step-order check's reference GEMMs)
    _restore(ours, saved)
    torch.cuda.synchronize()
    reference_pass(evict=False)  # untimed: cuBLAS and module first-use costs
    (ref_table, ref_refs), ref_ms = timed(lambda: reference_pass(evict=True))
    result, our_ms = timed(our_pass)

    # Parity at full size: scores, queue, caches after the eviction.
    assert torch.equal(result.table.scores.view(torch.int32), ref_table.scores.view(torch.int32))
    assert [(s.layer, s.head) for s in result.table.segments] == [(s.layer, s.head) for s in ref_table.segments]
    np.testing.assert_array_equal(np.asarray(result.references.scores, np.float32).view(np.uint32),
                                  np.asarray(ref_refs.scores, np.float32).view(np.uint32))
    np.testing.assert_array_equal(result.references.positions, ref_refs.positions)
    assert result.evicted == IMMEDIATE
    for layer in range(LAYERS):
        assert ours.layers[layer].head_lens == list(ref_cache.metadata_list[layer].head_lens_cpu)
        assert torch.equal(ours.layers[layer].keys.view(torch.int16), ref_cache.key_cache[layer].view(torch.int16))
        assert torch.equal(ours.layers[layer].values.view(torch.int16),
                           ref_cache.value_cache[layer].view(torch.int16))
        assert torch.equal(ours.layers[layer].positions.reshape(-1), ref_cache.position_cache[layer].reshape(-1))

    rows = LAYERS * HEADS * (PROMPT + GENERATED)
    report = {"workload": f"configs[1]: {LAYERS} layers x {HEADS} heads x ({PROMPT} + {GENERATED}) rows, D{DIM}, "
                          f"GQA {GROUPS}, window {WINDOW}, {IMMEDIATE} immediate + {QUEUED} queued",
              "reference_gpu_ms": ref_ms, "ours_ms": our_ms, "speed_up": ref_ms / our_ms,
              "reference_tokens_per_s": rows / (ref_ms / 1e3), "ours_tokens_per_s": rows / (our_ms / 1e3)}
    (tmp_path / "audit_pass_vs_reference_gpu.json").write_text(json.dumps(report, indent=1))
    print(json.dumps(report, indent=1))
    assert our_ms < ref_ms
