"""The reference's own Python, unchanged, running on this repository's operators.

The reference package (installed unchanged into oracle/_ref/py by
oracle/install_ref_py.py, CPU math path) imports its native modules as
``lazy_recall._C``, ``lazy_recall._legacy_C`` and ``lazy_recall._host``
(cuda_ops.py:4-13, _core/cuda_ops.py:11-14, recall/transport.py:18).  Here
those names are bound to code_for_iclr27_b200's modules before the package is
imported -- the drop-in -- and the reference's own classes and functions run:

* LazyRecallCache (cache.py:29-253): prefill, decode appends (_C.append),
  remove_positions (_C.compact), insert_payload (_C.merge);
* compute_score_table (scoring.py:198-308) with temporal_head_scores' GPU
  branch (_C.temporal_probabilities + _C.temporal_risk), pool_score_table
  (_C.pool) and refine_arrays (selection.py:52-88).

Each is compared with the same calls on CPU tensors, which take the
reference's own CPU branches: the cache byte for byte, the scores within
1e-5 relative (the query and key entries are small integers, so both paths
see the same logits), Pool7 exactly.  The reference's refine_arrays (torch.topk
on CUDA) on the GPU tables is compared with this repository's refine_arrays
exactly (CPU and CUDA topk may break ties differently, so the CPU branch is
not the yardstick there).  Skipped when oracle/_ref/py is absent.
"""
import importlib
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
RTOL = 1e-5


@pytest.fixture(scope="module")
def reference(cuda):
    """The reference package with its native modules bound to ours."""
    from oracle.install_ref_py import installed

    where = installed()
    if where is None:
        pytest.skip("reference package not installed (oracle/install_ref_py.py)")
    import code_for_iclr27_b200 as ours

    for name in [m for m in sys.modules if m == "lazy_recall" or m.startswith("lazy_recall.")]:
        del sys.modules[name]
    sys.path.insert(0, str(where))
    try:
        package = importlib.import_module("lazy_recall")
        for name, module in (("_C", ours.operators()), ("_legacy_C", ours.legacy_operators()),
                             ("_host", ours.host_operators())):
            sys.modules[f"lazy_recall.{name}"] = module
            setattr(package, name, module)
        modules = SimpleNamespace(
            cache=importlib.import_module("lazy_recall.cache"),
            scoring=importlib.import_module("lazy_recall.scoring"),
            history=importlib.import_module("lazy_recall.history"),
            selection=importlib.import_module("lazy_recall.selection"),
            cuda_ops=importlib.import_module("lazy_recall.cuda_ops"),
            core_ops=importlib.import_module("lazy_recall._core.cuda_ops"),
        )
        assert modules.cuda_ops.extension() is ours.operators()
        assert modules.core_ops.extension_available()
        yield modules
    finally:
        sys.path.remove(str(where))
        for name in [m for m in sys.modules if m == "lazy_recall" or m.startswith("lazy_recall.")]:
            del sys.modules[name]


def u16(t):
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy()


def same_cache(gpu, cpu):
    for layer in range(len(cpu.key_cache)):
        assert gpu.metadata_list[layer].head_lens_cpu == cpu.metadata_list[layer].head_lens_cpu, layer
        np.testing.assert_array_equal(u16(gpu.key_cache[layer]), u16(cpu.key_cache[layer]))
        np.testing.assert_array_equal(u16(gpu.value_cache[layer]), u16(cpu.value_cache[layer]))
        np.testing.assert_array_equal(gpu.position_cache[layer].cpu().numpy(), cpu.position_cache[layer].numpy())
        np.testing.assert_array_equal(gpu.metadata_list[layer].cu_seqlens_k.cpu().numpy(),
                                      cpu.metadata_list[layer].cu_seqlens_k.numpy())


def build_caches(reference, cuda, layers=2, heads=4, dim=64, prompt=40, steps=6, seed=0):
    """The same LazyRecallCache built on the GPU (through our operators) and on
    the CPU (the reference's CPU branch): prefill, freeze, decode appends."""
    import torch

    g = torch.Generator().manual_seed(seed)
    caches = {"gpu": reference.cache.LazyRecallCache(), "cpu": reference.cache.LazyRecallCache()}
    states = []
    for layer in range(layers):
        states.append((torch.randint(-2, 3, (1, heads, prompt, dim), generator=g).to(torch.bfloat16),
                       torch.randn(1, heads, prompt, dim, generator=g).to(torch.bfloat16)))
    with torch.no_grad():
        for where, cache in caches.items():
            device = cuda if where == "gpu" else torch.device("cpu")
            for layer, (k, v) in enumerate(states):
                cache.update(k.to(device), v.to(device), layer)
            cache.freeze_prompt()
        for _ in range(steps):
            new = [(torch.randint(-2, 3, (1, heads, 1, dim), generator=g).to(torch.bfloat16),
                    torch.randn(1, heads, 1, dim, generator=g).to(torch.bfloat16)) for _ in range(layers)]
            for where, cache in caches.items():
                device = cuda if where == "gpu" else torch.device("cpu")
                for layer, (k, v) in enumerate(new):
                    cache.update(k.to(device), v.to(device), layer)
    return caches["gpu"], caches["cpu"]


def test_reference_cache_lifecycle_on_our_operators(reference, cuda):
    """LazyRecallCache.update / remove_positions / insert_payload, the
    reference's code, on our _C: the cache equals the CPU branch's byte for
    byte after every phase."""
    import torch

    gpu, cpu = build_caches(reference, cuda)
    same_cache(gpu, cpu)
    removals = {(0, 1): [2, 5, 6, 41], (1, 3): [0, 19, 44], (1, 0): [7]}
    for cache in (gpu, cpu):
        cache.remove_positions(removals)
    same_cache(gpu, cpu)
    g = torch.Generator().manual_seed(5)
    payload = torch.randn(4, 2, 64, generator=g).to(torch.bfloat16)
    metadata = np.asarray([[0, 1, 5], [1, 3, 19], [0, 1, 41], [1, 3, 0]], np.int64)
    gpu.insert_payload(payload.to(cuda), metadata)
    cpu.insert_payload(payload, metadata)
    same_cache(gpu, cpu)
    # A decode step after the recall: appends on the merged layout.
    new = [(torch.randn(1, 4, 1, 64, generator=g).to(torch.bfloat16),) * 2 for _ in range(2)]
    with torch.no_grad():
        for layer, (k, v) in enumerate(new):
            gpu.update(k.to(cuda), v.to(cuda), layer)
            cpu.update(k, v, layer)
    same_cache(gpu, cpu)


def model_stub(layers, heads, groups, dim, hidden, seed):
    """What compute_score_table reads of a model: per layer the attention's
    head counts, head_dim and o_proj weight (scoring.py:218-237)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    config = SimpleNamespace(num_attention_heads=heads * groups, num_key_value_heads=heads)
    blocks = [SimpleNamespace(self_attn=SimpleNamespace(
        config=config, head_dim=dim,
        o_proj=SimpleNamespace(weight=torch.randn(hidden, heads * groups * dim, generator=g) / 16)))
        for _ in range(layers)]
    return SimpleNamespace(model=SimpleNamespace(layers=blocks))


def test_reference_score_table_and_selection_on_our_operators(reference, cuda):
    """compute_score_table + pool_score_table, the reference's code: on GPU
    tensors through our _C, on CPU tensors through its CPU branches (scores
    within 1e-5, Pool7 exact on the same scores); then the reference's
    refine_arrays on the GPU tables against ours, exactly."""
    import torch

    layers, heads, groups, dim, hidden, window = 2, 4, 2, 64, 48, 12
    gpu, cpu = build_caches(reference, cuda, layers=layers, heads=heads, dim=dim, steps=window + 30)
    model_cpu = model_stub(layers, heads, groups, dim, hidden, 1)
    model_gpu = SimpleNamespace(model=SimpleNamespace(layers=[SimpleNamespace(self_attn=SimpleNamespace(
        config=b.self_attn.config, head_dim=dim, o_proj=SimpleNamespace(weight=b.self_attn.o_proj.weight.to(cuda))))
        for b in model_cpu.model.layers]))
    g = torch.Generator().manual_seed(2)
    grads = [torch.randn(1, 1, hidden, generator=g) for _ in range(layers)]
    history = {"gpu": reference.history.QueryHistory(layers, window),
               "cpu": reference.history.QueryHistory(layers, window)}
    seen = cpu._seen_tokens
    for step in range(window):
        queries = [torch.randint(-2, 3, (1, heads * groups, 1, dim), generator=g).to(torch.bfloat16)
                   for _ in range(layers)]
        history["gpu"].append([q.to(cuda) for q in queries], seen - window + step)
        history["cpu"].append(queries, seen - window + step)
    audit = {"gpu": SimpleNamespace(attention_gradients=[x.to(cuda) for x in grads],
                                    margin=torch.tensor(0.9, device=cuda)),
             "cpu": SimpleNamespace(attention_gradients=grads, margin=torch.tensor(0.9))}
    results = {}
    for where, cache, model in (("gpu", gpu, model_gpu), ("cpu", cpu, model_cpu)):
        with torch.no_grad():
            table = reference.scoring.compute_score_table(model, cache, audit[where], history[where],
                                                          protect_prompt=True, protect_recent=4,
                                                          query_chunk_size=5).table
        pooled = reference.scoring.pool_score_table(table, 7)
        results[where] = (table, pooled)
    (tg, pg), (tc, pc) = results["gpu"], results["cpu"]
    assert tg.segments == tc.segments and tg.cumulative_ends == tc.cumulative_ends
    a, b = tg.scores.cpu().numpy().astype(np.float64), tc.scores.numpy().astype(np.float64)
    floor = 1e-6 * np.abs(b).max()
    assert (np.abs(a - b) <= RTOL * np.abs(b) + floor).all()
    # Pool7 on our _C equals the reference's CPU max_pool1d on the same scores.
    same_input = reference.scoring.pool_score_table(
        type(tc)(tg.scores.cpu(), list(tc.segments), list(tc.cumulative_ends), 0.0), 7)
    np.testing.assert_array_equal(pg.scores.cpu().numpy(), same_input.scores.numpy())
    # refine_arrays, the reference's own code (torch.topk on CUDA), on the
    # GPU tables equals this repository's refine_arrays (lrk_refine) exactly:
    # queue order, raw scores, positions and change counts.
    from code_for_iclr27_b200.selection import refine_arrays as ours

    count = tg.scores.numel() // 3
    refs_ref, changed_ref, heads_ref = reference.selection.refine_arrays(tg, pg, count)
    refs_ours, changed_ours, heads_ours = ours(tg, pg, count)
    assert len(refs_ref) == len(refs_ours) == count
    np.testing.assert_array_equal(np.asarray(refs_ours.scores, np.float32).view(np.uint32),
                                  np.asarray(refs_ref.scores, np.float32).view(np.uint32))
    np.testing.assert_array_equal(refs_ours.segments, refs_ref.segments)
    np.testing.assert_array_equal(refs_ours.positions, refs_ref.positions)
    assert (changed_ours, heads_ours) == (changed_ref, heads_ref)
