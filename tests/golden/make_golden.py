"""Generate the golden fixtures that pin oracle/lrk_oracle.py to the reference.

The reference (LazyRecall v0.3.1) ships no tests and no known-answer vectors,
so these fixtures are made by running the reference itself on seeded inputs:

  cpu  imports the reference's Python package (its CPU math path: the
       PyTorch fallbacks that run when the CUDA extension is not built) and
       records inputs and outputs -> tests/golden/reference_cpu.npz
       python tests/golden/make_golden.py cpu --reference <reference>/src

  gpu  loads the reference's own CUDA operator modules, built from its
       sources by oracle/build_ref.py into oracle/_ref/, and records their
       outputs; also records torch.topk on CUDA for tie-heavy inputs (the
       selection step calls torch.topk) -> tests/golden/reference_gpu.npz
       python tests/golden/make_golden.py gpu   (on a machine with a GPU)

Both write float arrays as-is and bf16 data as uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import importlib.util
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def bits(tensor):
    import torch

    t = tensor.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


# ------------------------------------------------------------------ cpu


def make_cpu(reference_src: str, out: Path):
    sys.path.insert(0, reference_src)
    import torch
    import torch.nn.functional as F  # noqa: F401

    from lazy_recall import scoring, selection
    from lazy_recall._core import cuda_ops
    from lazy_recall._core.scoring import ScoreSegment, ScoreTable
    from lazy_recall.cache import LazyRecallCache
    from lazy_recall.recall import planning

    assert not cuda_ops.extension_available(), "the reference's CPU path needs the extension absent"
    fixtures = {}
    g = torch.Generator().manual_seed(20261201)

    # Scoring, CPU math path (scoring.py:75-149).  Integer-valued Q and K with
    # D=64 make Q K^T / sqrt(D) exact in bf16, so the fixture does not depend
    # on the BLAS summation order; V and the margin gradient are random.
    cases = [
        dict(window=7, groups=4, length=300, dim=64, start=5, end=280, chunk=3, qlo=250),
        dict(window=5, groups=2, length=513, dim=64, start=0, end=513, chunk=250, qlo=600),
        dict(window=9, groups=8, length=130, dim=16, start=17, end=98, chunk=4, qlo=100),
    ]
    for i, c in enumerate(cases):
        q = torch.randint(-1, 2, (c["window"], c["groups"], c["dim"]), generator=g).to(torch.float32)
        k = torch.randint(-1, 2, (c["length"], c["dim"]), generator=g).to(torch.bfloat16)
        v = torch.randn(c["length"], c["dim"], generator=g).to(torch.bfloat16)
        kpos = torch.arange(c["length"], dtype=torch.float32)
        qpos = torch.arange(c["qlo"], c["qlo"] + c["window"], dtype=torch.int64)
        grad = torch.randn(c["groups"], c["dim"], generator=g)
        margin = torch.tensor(0.75)
        scores = scoring.temporal_head_scores_reference(q, qpos, k, kpos, v, c["start"], c["end"], grad, margin,
                                                        1e-6, c["chunk"])
        p = f"scores{i}_"
        fixtures.update({p + "queries": q.numpy(), p + "qpos": qpos.numpy(), p + "keys": bits(k),
                         p + "kpos": kpos.numpy(), p + "values": bits(v), p + "grad": grad.numpy(),
                         p + "margin": margin.numpy(), p + "meta": np.asarray([c["start"], c["end"], c["chunk"]]),
                         p + "out": scores.numpy()})

    # Pool7, CPU path (scoring.py:336-353), with ties and uneven segments.
    raw = torch.randint(0, 40, (1000,), generator=g).to(torch.float32) / 8
    counts = [1, 2, 7, 13, 300, 677]
    ends = list(np.cumsum(counts))
    segments = [ScoreSegment(layer=i // 4, head=i % 4, position_start=3 * i, count=n) for i, n in enumerate(counts)]
    table = ScoreTable(raw, segments, ends, 0.0)
    pooled = scoring.pool_score_table(table, 7)
    fixtures.update({"pool_scores": raw.numpy(), "pool_ends": np.asarray(ends), "pool_out": pooled.scores.numpy()})

    # Selection (selection.py:52-88) on tie-free tables (CPU topk tie order is
    # not the CUDA one; CUDA tie cases come from the gpu fixtures).
    for i, (n_segments, length, count) in enumerate([(6, 50, 120), (12, 37, 1), (5, 400, 1999), (3, 9, 27)]):
        n = n_segments * length
        raw = torch.randperm(n, generator=g).to(torch.float32) / n + 0.5
        refined = torch.randperm(n, generator=g).to(torch.float32) / n
        segs = [ScoreSegment(layer=s // 2, head=s % 2, position_start=int(s % 3) * 5, count=length)
                for s in range(n_segments)]
        ends = [length * (s + 1) for s in range(n_segments)]
        a = ScoreTable(raw, segs, ends, 0.0)
        b = ScoreTable(refined, segs, ends, 0.0)
        references, changed, changed_heads = selection.refine_arrays(a, b, count)
        p = f"refine{i}_"
        fixtures.update({p + "raw": raw.numpy(), p + "pooled": refined.numpy(), p + "ends": np.asarray(ends),
                         p + "starts": np.asarray([s.position_start for s in segs]), p + "count": np.asarray(count),
                         p + "values": references.scores, p + "segments": references.segments,
                         p + "positions": references.positions, p + "coordinates": references.coordinates,
                         p + "changed": np.asarray([changed, changed_heads])})

    # Flat cache lifecycle on CPU: prefill, appends, removals (index_select
    # compaction, cache.py:162-167), a recall insert (torch.cat + index_select
    # merge, cache.py:240-245) -- LazyRecallCache's own CPU branch.
    cache = LazyRecallCache()
    heads, dim = 4, 16
    for layer in range(2):
        ks = torch.randn(1, heads, 20, dim, generator=g).to(torch.bfloat16)
        vs = torch.randn(1, heads, 20, dim, generator=g).to(torch.bfloat16)
        cache.update(ks, vs, layer)
    cache.freeze_prompt()
    history = []

    def snap(tag):
        for layer in range(2):
            history.append((f"cache_{tag}_L{layer}_", cache.key_cache[layer], cache.value_cache[layer],
                            cache.position_cache[layer], list(cache.metadata_list[layer].head_lens_cpu)))

    snap("prefill")
    new_states = []
    for step in range(3):
        for layer in range(2):
            ks = torch.randn(1, heads, 1, dim, generator=g).to(torch.bfloat16)
            vs = torch.randn(1, heads, 1, dim, generator=g).to(torch.bfloat16)
            new_states.append((f"cache_step{step}_L{layer}_", ks, vs))
            cache.update(ks, vs, layer)
    snap("appended")
    removals = {(0, 1): [2, 5, 6, 21], (1, 3): [0, 19, 22], (1, 0): [7]}
    cache.remove_positions(removals)
    snap("removed")
    payload = torch.randn(4, 2, dim, generator=g).to(torch.bfloat16)
    metadata = np.asarray([[0, 1, 5], [1, 3, 19], [0, 1, 21], [1, 3, 0]], np.int64)
    cache.insert_payload(payload, metadata)
    snap("merged")
    for prefix, k, v, pos, lengths in history:
        fixtures.update({prefix + "keys": bits(k), prefix + "values": bits(v), prefix + "positions": pos.numpy(),
                         prefix + "lengths": np.asarray(lengths)})
    for prefix, k, v in new_states:
        fixtures.update({prefix + "new_keys": bits(k), prefix + "new_values": bits(v)})
    fixtures["cache_removals"] = np.asarray([[l, h, p] for (l, h), ps in removals.items() for p in ps])
    fixtures.update({"cache_payload": bits(payload), "cache_metadata": metadata})

    # merge_plan (recall/planning.py:34-52).
    old = np.asarray([3, 7, 9, 1, 2, 8, 11, 4], np.int64)
    plan_meta = np.asarray([[0, 0, 5], [0, 1, 0], [0, 0, 10], [0, 2, 6], [0, 1, 3]], np.int64)
    mapping, lengths = planning.merge_plan(old, [3, 4, 1], plan_meta)
    fixtures.update({"plan_old": old, "plan_meta": plan_meta, "plan_mapping": mapping,
                     "plan_lengths": np.asarray(lengths)})

    # Legacy decision risk, PyTorch twin (_core/cuda_ops.py:228-273).
    probs = torch.rand(4, 37, generator=g)
    probs[0, 3] = 0.9999999
    vals = torch.randn(37, 24, generator=g).to(torch.bfloat16)
    outs = torch.randn(4, 24, generator=g)
    grads = torch.randn(4, 24, generator=g)
    risk = cuda_ops.decision_risk_scores_pytorch(probs, vals, outs, grads, 1.25, 1e-6)
    fixtures.update({"drisk_probs": probs.numpy(), "drisk_values": bits(vals), "drisk_outputs": outs.numpy(),
                     "drisk_grads": grads.numpy(), "drisk_out": risk.numpy()})
    np.savez_compressed(out, **fixtures)
    print(f"wrote {out} ({len(fixtures)} arrays)")


# ------------------------------------------------------------------ gpu


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(f"lazy_recall_reference.{name}", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def make_gpu(out: Path):
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import build_ref

    paths = build_ref.built_paths()
    if not {"C", "legacy_C"} <= set(paths):
        raise SystemExit("reference modules missing under oracle/_ref; run oracle/build_ref.py first")
    ref = _load("_C", paths["C"])
    legacy = _load("_legacy_C", paths["legacy_C"])
    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(7)
    fx = {}

    def rn(*shape, dtype=torch.float32):
        return torch.randn(*shape, generator=g).to(dtype).to(dev)

    # temporal_probabilities / temporal_risk for three logit dtypes.
    for i, (dtype, tag, window, groups, length, start, end) in enumerate([
            (torch.bfloat16, "bf16", 6, 4, 300, 3, 290), (torch.float16, "f16", 3, 2, 4113, 0, 4113),
            (torch.float32, "f32", 2, 8, 1030, 500, 1029), (torch.bfloat16, "bf16", 2, 4, 70001, 69000, 69990)]):
        logits = (rn(window, groups, length) * 2 * math.sqrt(64)).to(dtype)
        pv = rn(groups, length).abs()
        qpos = torch.arange(length - window - 5, length - 5, device=dev, dtype=torch.int64)
        kpos = torch.arange(length, device=dev, dtype=torch.float32)
        probs, op = ref.temporal_probabilities(logits, pv, qpos, kpos, 0.125)
        margin = torch.tensor([0.8], device=dev)
        risk = ref.temporal_risk(probs, op, pv, margin, start, end, 1e-6)
        p = f"tp{i}_"
        fx.update({p + "logits": bits(logits), p + "dtype": np.asarray(tag), p + "pv": bits(pv),
                   p + "qpos": bits(qpos), p + "kpos": bits(kpos), p + "op": bits(op), p + "risk": bits(risk),
                   p + "interval": np.asarray([start, end]), p + "margin": bits(margin)})
        if length <= 5000:
            fx[p + "probs"] = bits(probs)
        else:
            fx[p + "probs_rows"] = bits(probs[:, :, start:end])

    # Risk with a non-finite probability and window < 8.
    probs = torch.rand(3, 2, 50, generator=g).to(dev)
    probs[1, 0, 10] = float("nan")
    probs[2, 1, 20] = 1.0
    op = rn(3, 2)
    pv = rn(2, 50)
    risk = ref.temporal_risk(probs, op, pv, torch.tensor([-0.3], device=dev), 2, 48, 1e-6)
    fx.update({"risk_nan_probs": bits(probs), "risk_nan_op": bits(op), "risk_nan_pv": bits(pv), "risk_nan_out": bits(risk)})

    # Data movement, bf16 D=128 and D=64.
    for d in (128, 64):
        heads = 8
        lengths = torch.randint(0, 300, (heads,), generator=g)
        lengths[3] = 0
        rows = int(lengths.sum())
        cumulative = torch.cat([torch.zeros(1, dtype=torch.int64), lengths.cumsum(0)]).to(torch.int32).to(dev)
        keys, values = rn(rows, d, dtype=torch.bfloat16), rn(rows, d, dtype=torch.bfloat16)
        positions = torch.randperm(rows + 50, generator=g)[:rows].to(torch.float32).reshape(-1, 1).to(dev)
        new_keys, new_values = rn(1, heads, 2, d, dtype=torch.bfloat16), rn(1, heads, 2, d, dtype=torch.bfloat16)
        appended = ref.append(keys, values, positions, new_keys, new_values, cumulative, 12345, int(lengths.max()))
        removed = torch.randperm(rows, generator=g)[: rows // 3].sort().values.to(dev)
        compacted = ref.compact(keys, values, positions, removed)
        recalled = rn(9, 2, d, dtype=torch.bfloat16)
        recalled_pos = torch.arange(9, dtype=torch.float32, device=dev) + 0.5
        mapping = torch.cat([torch.arange(rows), -torch.arange(1, 10)])[torch.randperm(rows + 9, generator=g)].to(dev)
        merged = ref.merge(keys, values, positions, recalled, recalled_pos, mapping)
        indices = torch.randperm(rows, generator=g)[:40].to(dev)
        head_ids = torch.randint(0, heads, (40,), generator=g).to(dev)
        payload = torch.empty(40, 2, d, dtype=torch.bfloat16, device=dev)
        metadata = torch.empty(40, 3, dtype=torch.int64, device=dev)
        ref.pack(keys, values, positions, indices, head_ids, 5, payload, metadata)
        p = f"move{d}_"
        fx.update({p + "keys": bits(keys), p + "values": bits(values), p + "positions": bits(positions),
                   p + "cumulative": bits(cumulative), p + "new_keys": bits(new_keys),
                   p + "new_values": bits(new_values), p + "removed": bits(removed), p + "recalled": bits(recalled),
                   p + "recalled_pos": bits(recalled_pos), p + "mapping": bits(mapping), p + "indices": bits(indices),
                   p + "heads": bits(head_ids), p + "payload": bits(payload), p + "metadata": bits(metadata)})
        for j, name in enumerate(["keys", "values", "positions", "cumulative", "lengths"]):
            fx[p + "append_" + name] = bits(appended[j])
        for j, name in enumerate(["keys", "values", "positions"]):
            fx[p + "compact_" + name] = bits(compacted[j])
            fx[p + "merge_" + name] = bits(merged[j])

    # batch_append: three requests, one with an empty head.
    d, heads = 128, 4
    ks, vs, ps, lens = [], [], [], []
    for r in range(3):
        hl = torch.randint(0, 40, (heads,), generator=g).tolist()
        if r == 1:
            hl[2] = 0
        n = sum(hl)
        ks.append(rn(n, d, dtype=torch.bfloat16))
        vs.append(rn(n, d, dtype=torch.bfloat16))
        ps.append(torch.arange(n, dtype=torch.float32, device=dev).reshape(-1, 1))
        lens.append(hl)
    nk, nv = rn(3, heads, 1, d, dtype=torch.bfloat16), rn(3, heads, 1, d, dtype=torch.bfloat16)
    logical = [101, 7, 99999]
    bk, bv, bp = ref.batch_append(ks, vs, ps, nk, nv, lens, logical)
    for r in range(3):
        fx.update({f"batch_keys{r}": bits(ks[r]), f"batch_values{r}": bits(vs[r]), f"batch_positions{r}": bits(ps[r]),
                   f"batch_lengths{r}": np.asarray(lens[r])})
    fx.update({"batch_new_keys": bits(nk), "batch_new_values": bits(nv), "batch_logical": np.asarray(logical),
               "batch_out_keys": bits(bk), "batch_out_values": bits(bv), "batch_out_positions": bits(bp)})

    # Pool on device.
    scores = (torch.randint(0, 50, (2000,), generator=g).to(torch.float32) / 4).to(dev)
    bounds = torch.tensor([0, 1, 3, 10, 700, 2000], dtype=torch.int64, device=dev)
    pooled = ref.pool(scores, bounds, 1300, 7)
    fx.update({"gpool_scores": bits(scores), "gpool_bounds": bits(bounds), "gpool_out": bits(pooled)})

    # Legacy ops.
    cache = rn(50, 1)
    states = rn(2, 3, 2, 1)
    head_lens = torch.tensor([10, 0, 15, 5, 12, 8], dtype=torch.int32, device=dev)
    cu = torch.cat([torch.zeros(1, dtype=torch.int32, device=dev), head_lens.cumsum(0).to(torch.int32)])
    appended = legacy.append_flattened_cache(cache, states, head_lens, cu)
    lk, lv = rn(60, 64, dtype=torch.bfloat16), rn(60, 64, dtype=torch.bfloat16)
    keep = torch.tensor([0, 3, 4, 59, 10, 10], dtype=torch.int64, device=dev)
    ck, cv = legacy.compact_flattened_kv(lk, lv, keep)
    probs = torch.rand(4, 33, generator=g).to(dev)
    dvals, douts, dgrads = rn(33, 40, dtype=torch.bfloat16), rn(4, 40), rn(4, 40)
    drisk = legacy.decision_risk_scores(probs, dvals, douts, dgrads, -0.7, 1e-6)
    fx.update({"legacy_cache": bits(cache), "legacy_states": bits(states), "legacy_head_lens": bits(head_lens),
               "legacy_cu": bits(cu), "legacy_appended": bits(appended), "legacy_keys": bits(lk),
               "legacy_values": bits(lv), "legacy_keep": bits(keep), "legacy_ck": bits(ck), "legacy_cv": bits(cv),
               "legacy_probs": bits(probs), "legacy_dvals": bits(dvals), "legacy_douts": bits(douts),
               "legacy_dgrads": bits(dgrads), "legacy_drisk": bits(drisk)})

    # torch.topk(largest=False, sorted=True) on CUDA with heavy ties.
    # Inputs are stored as uint16 codes (x = code / 4) and indices as int32 to
    # keep the fixture small; slices over 10^6 are checked live by the GPU tests.
    cases = [(40, 1), (40, 2), (40, 7), (40, 32), (40, 33), (300, 17), (300, 100), (300, 129), (5000, 4096),
             (5000, 31), (99999, 20), (99999, 5000), (100000, 20), (150000, 31), (150000, 70000)]
    for i, (n, k) in enumerate(cases):
        codes = torch.randint(0, max(3, n // 50), (n,), generator=g)
        x = (codes.to(torch.float32) / 4).to(dev)
        _, indices_k = torch.topk(x, k, largest=False, sorted=True)
        fx.update({f"topk{i}_codes": codes.numpy().astype(np.uint16), f"topk{i}_k": np.asarray(k),
                   f"topk{i}_indices": indices_k.cpu().numpy().astype(np.int32)})
    np.savez_compressed(out, **fx)
    print(f"wrote {out} ({len(fx)} arrays)")


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("which", choices=["cpu", "gpu"])
    parser.add_argument("--reference", default=None,
                        help="the reference's src/ directory (default: oracle/reference_root.py's tree + /src)")
    parser.add_argument("--out", default=None)
    args = parser.parse_args()
    if args.which == "cpu":
        if args.reference is None:
            sys.path.insert(0, str(ROOT))
            from oracle.reference_root import reference_root

            root = reference_root()
            if root is None:
                raise SystemExit("reference sources not found: pass --reference or set LAZY_RECALL_REFERENCE")
            args.reference = str(root / "src")
        make_cpu(args.reference, Path(args.out or HERE / "reference_cpu.npz"))
    else:
        make_gpu(Path(args.out or HERE / "reference_gpu.npz"))


if __name__ == "__main__":
    main()
