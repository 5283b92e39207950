"""The oracle against golden fixtures produced by the reference itself.

reference_cpu.npz: the reference's Python CPU math path (make_golden.py cpu).
reference_gpu.npz: the reference's own CUDA operators built from its sources,
and torch.topk on CUDA (make_golden.py gpu).
"""
import numpy as np
import pytest

from oracle import lrk_oracle as O

RTOL = 1e-5


def close(actual, expected, rtol=RTOL, atol=1e-7):
    actual, expected = np.asarray(actual, np.float64), np.asarray(expected, np.float64)
    assert actual.shape == expected.shape
    same_nan = np.isnan(actual) == np.isnan(expected)
    assert same_nan.all(), "NaN pattern differs"
    a, e = actual[~np.isnan(actual)], expected[~np.isnan(expected)]
    np.testing.assert_allclose(a, e, rtol=rtol, atol=atol)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_scores_cpu_path(golden_cpu, case):
    g = golden_cpu
    p = f"scores{case}_"
    start, end, chunk = (int(v) for v in g[p + "meta"])
    keys, values = O.bf16_to_f32(g[p + "keys"]), O.bf16_to_f32(g[p + "values"])
    args = (g[p + "queries"], g[p + "qpos"], keys, g[p + "kpos"], values, start, end, g[p + "grad"],
            g[p + "margin"], 1e-6, chunk)
    close(O.temporal_head_scores_cpu_path(*args), g[p + "out"])
    # The GPU decomposition (probabilities + risk kernels) agrees on exact logits.
    close(O.temporal_head_scores_gpu_path(*args), g[p + "out"], rtol=2e-5)


def test_pool_cpu_path(golden_cpu):
    g = golden_cpu
    bounds = np.concatenate(([0], g["pool_ends"]))
    np.testing.assert_array_equal(O.pool(g["pool_scores"], bounds, 7), g["pool_out"])


@pytest.mark.parametrize("case", [0, 1, 2, 3])
def test_refine_cpu_path(golden_cpu, case):
    g = golden_cpu
    p = f"refine{case}_"
    values, segments, positions, changed, heads = O.refine(g[p + "raw"], g[p + "pooled"], g[p + "ends"],
                                                           g[p + "starts"], int(g[p + "count"]))
    np.testing.assert_array_equal(values, g[p + "values"])
    np.testing.assert_array_equal(segments, g[p + "segments"])
    np.testing.assert_array_equal(positions, g[p + "positions"])
    assert [changed, heads] == list(g[p + "changed"])


def test_cache_lifecycle_cpu_path(golden_cpu):
    """Append, compaction and recall merge replayed on the oracle reproduce the
    reference LazyRecallCache's CPU branch byte for byte."""
    g = golden_cpu
    state = {}
    for layer in range(2):
        p = f"cache_prefill_L{layer}_"
        state[layer] = [g[p + "keys"], g[p + "values"], g[p + "positions"].reshape(-1), list(g[p + "lengths"])]
    seen = 20
    for step in range(3):
        for layer in range(2):
            p = f"cache_step{step}_L{layer}_"
            keys, values, positions, lengths = state[layer]
            cumulative = np.concatenate(([0], np.cumsum(lengths)))
            k, v, pos, _, new_lengths = O.append(keys, values, positions, g[p + "new_keys"], g[p + "new_values"],
                                                 cumulative, seen)
            state[layer] = [k, v, pos.reshape(-1), list(new_lengths)]
        seen += 1
    for layer in range(2):
        p = f"cache_appended_L{layer}_"
        np.testing.assert_array_equal(state[layer][0], g[p + "keys"])
        np.testing.assert_array_equal(state[layer][1], g[p + "values"])
        np.testing.assert_array_equal(state[layer][2], g[p + "positions"].reshape(-1))
    removals = g["cache_removals"]
    for layer in range(2):
        keys, values, positions, lengths = state[layer]
        bounds = np.concatenate(([0], np.cumsum(lengths)))
        rows = sorted(int(bounds[h] + pos) for l, h, pos in removals if l == layer)
        k, v, pos = O.compact(keys, values, positions, np.asarray(rows, np.int64))
        for l, h, _ in removals:
            if l == layer:
                lengths[h] -= 1
        state[layer] = [k, v, pos.reshape(-1), lengths]
        p = f"cache_removed_L{layer}_"
        np.testing.assert_array_equal(k, g[p + "keys"])
        np.testing.assert_array_equal(pos.reshape(-1), g[p + "positions"].reshape(-1))
        assert lengths == list(g[p + "lengths"])
    payload, metadata = g["cache_payload"], g["cache_metadata"]
    for layer in range(2):
        rows = np.flatnonzero(metadata[:, 0] == layer)
        keys, values, positions, lengths = state[layer]
        mapping, new_lengths = O.merge_plan(positions.astype(np.int64), lengths, metadata[rows])
        k, v, pos = O.merge(keys, values, positions, payload[rows], metadata[rows, 2].astype(np.float32), mapping)
        p = f"cache_merged_L{layer}_"
        np.testing.assert_array_equal(k, g[p + "keys"])
        np.testing.assert_array_equal(v, g[p + "values"])
        np.testing.assert_array_equal(pos.reshape(-1), g[p + "positions"].reshape(-1))
        assert list(new_lengths) == list(g[p + "lengths"])


def test_merge_plan_cpu_path(golden_cpu):
    g = golden_cpu
    mapping, lengths = O.merge_plan(g["plan_old"], [3, 4, 1], g["plan_meta"])
    np.testing.assert_array_equal(mapping, g["plan_mapping"])
    assert list(lengths) == list(g["plan_lengths"])


def test_decision_risk_cpu_path(golden_cpu):
    g = golden_cpu
    out = O.decision_risk(g["drisk_probs"], g["drisk_values"], "bf16", g["drisk_outputs"], g["drisk_grads"], 1.25, 1e-6)
    close(out, g["drisk_out"])


def test_bf16_rounding_is_nearest_even():
    x = np.asarray([1.0, 1.00390625, 1.01171875, -2.5e-3, np.inf, -np.inf, 3.0e38], np.float32)
    back = O.bf16_to_f32(O.f32_to_bf16(x))
    assert back[1] == 1.0 and back[2] == np.float32(1.015625)
    assert np.isinf(back[4]) and np.isinf(back[5])
    assert np.isnan(O.bf16_to_f32(O.f32_to_bf16(np.asarray([np.nan], np.float32))))[0]


# ------------------------------------------------ reference CUDA fixtures


@pytest.mark.parametrize("case", [0, 1, 2, 3])
def test_probabilities_and_risk_vs_reference_cuda(golden_gpu, case):
    g = golden_gpu
    p = f"tp{case}_"
    dtype = str(g[p + "dtype"])
    logits = g[p + "logits"]
    probs, op = O.temporal_probabilities(logits, dtype, g[p + "pv"], g[p + "qpos"], g[p + "kpos"], 0.125)
    start, end = (int(v) for v in g[p + "interval"])
    close(op, g[p + "op"], rtol=1e-5, atol=1e-7)
    if p + "probs" in g:
        close(probs, g[p + "probs"], atol=1e-9)
    else:
        close(probs[:, :, start:end], g[p + "probs_rows"], atol=1e-9)
    risk = O.temporal_risk(probs, op, g[p + "pv"], g[p + "margin"], start, end, 1e-6)
    close(risk, g[p + "risk"], rtol=1e-5, atol=1e-9)


def test_risk_nonfinite_vs_reference_cuda(golden_gpu):
    g = golden_gpu
    out = O.temporal_risk(g["risk_nan_probs"], g["risk_nan_op"], g["risk_nan_pv"], np.float32(-0.3), 2, 48, 1e-6)
    close(out, g["risk_nan_out"])


@pytest.mark.parametrize("d", [128, 64])
def test_movement_vs_reference_cuda(golden_gpu, d):
    g = golden_gpu
    p = f"move{d}_"
    keys, values, positions = g[p + "keys"], g[p + "values"], g[p + "positions"]
    out = O.append(keys, values, positions, g[p + "new_keys"], g[p + "new_values"], g[p + "cumulative"], 12345)
    for got, name in zip(out, ["keys", "values", "positions", "cumulative", "lengths"]):
        np.testing.assert_array_equal(got, g[p + "append_" + name])
    out = O.compact(keys, values, positions, g[p + "removed"])
    for got, name in zip(out, ["keys", "values", "positions"]):
        np.testing.assert_array_equal(got, g[p + "compact_" + name])
    out = O.merge(keys, values, positions, g[p + "recalled"], g[p + "recalled_pos"], g[p + "mapping"])
    for got, name in zip(out, ["keys", "values", "positions"]):
        np.testing.assert_array_equal(got, g[p + "merge_" + name])
    payload, metadata = O.pack(keys, values, positions, g[p + "indices"], g[p + "heads"], 5)
    np.testing.assert_array_equal(payload, g[p + "payload"])
    np.testing.assert_array_equal(metadata, g[p + "metadata"])


def test_batch_append_vs_reference_cuda(golden_gpu):
    g = golden_gpu
    out = O.batch_append([g[f"batch_keys{r}"] for r in range(3)], [g[f"batch_values{r}"] for r in range(3)],
                         [g[f"batch_positions{r}"] for r in range(3)], g["batch_new_keys"][:, :, 0],
                         g["batch_new_values"][:, :, 0], [list(g[f"batch_lengths{r}"]) for r in range(3)],
                         list(g["batch_logical"]))
    for got, name in zip(out, ["keys", "values", "positions"]):
        np.testing.assert_array_equal(got, g["batch_out_" + name])


def test_pool_vs_reference_cuda(golden_gpu):
    g = golden_gpu
    np.testing.assert_array_equal(O.pool(g["gpool_scores"], g["gpool_bounds"], 7), g["gpool_out"])


def test_legacy_vs_reference_cuda(golden_gpu):
    g = golden_gpu
    np.testing.assert_array_equal(O.append_flattened(g["legacy_cache"], g["legacy_states"], g["legacy_head_lens"],
                                                     g["legacy_cu"]), g["legacy_appended"])
    k, v = O.compact_flattened(g["legacy_keys"], g["legacy_values"], g["legacy_keep"])
    np.testing.assert_array_equal(k, g["legacy_ck"])
    np.testing.assert_array_equal(v, g["legacy_cv"])
    out = O.decision_risk(g["legacy_probs"], g["legacy_dvals"], "bf16", g["legacy_douts"], g["legacy_dgrads"], -0.7,
                          1e-6)
    close(out, g["legacy_drisk"])


def test_topk_ties_vs_torch_cuda(golden_gpu):
    """The oracle's restatement of torch.topk(largest=False, sorted=True) on
    CUDA picks and orders tied elements exactly like PyTorch 2.11 did."""
    g = golden_gpu
    i = 0
    while f"topk{i}_codes" in g:
        x = g[f"topk{i}_codes"].astype(np.float32) / 4
        values, indices = O.topk_smallest(x, int(g[f"topk{i}_k"]))
        np.testing.assert_array_equal(indices, g[f"topk{i}_indices"], err_msg=f"case {i}")
        np.testing.assert_array_equal(values, x[g[f"topk{i}_indices"]])
        i += 1
    assert i > 0
