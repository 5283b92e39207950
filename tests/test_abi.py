"""The C-ABI library and the operator modules, without a GPU: symbols,
signatures, host-side validation (which returns before any CUDA call)."""
import ctypes
import re
from pathlib import Path

import pytest

from code_for_iclr27_b200 import abi, host_operators, legacy_operators, operators

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "lrk.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(lrk_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(abi.LIBRARY_PATH))
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(abi.SIGNATURES), "abi.py must bind exactly the header's entry points"


def test_host_queries():
    lib = abi.library()
    assert lib.lrk_version() >= 100
    assert [lib.lrk_dtype_size(c) for c in (abi.F32, abi.F64, abi.F16, abi.BF16, 99)] == [4, 8, 2, 2, 0]
    assert lib.lrk_refine_workspace_bytes(1000, 8) > 24 * 1000
    assert lib.lrk_topk_workspace_bytes(1 << 20) >= 24 * (1 << 20)


def test_invalid_arguments_rejected_before_launch():
    lib = abi.library()
    status = lib.lrk_compact(None, None, None, 10, 128, abi.BF16, None, 11, None, None, None, None)
    assert status == abi.ERR_INVALID
    assert "compaction" in lib.lrk_last_error().decode()
    assert lib.lrk_pool(None, 10, None, 1, 5, 4, None, None) == abi.ERR_INVALID  # even width
    assert lib.lrk_temporal_risk(None, None, None, None, None, 4, 2, 10, 5, 5, 1e-6, None) == abi.ERR_INVALID
    assert lib.lrk_append(None, None, None, 0, None, None, None, 4, 1, 64, 77, 0, None, None, None, None, None,
                          None) == abi.ERR_INVALID  # unknown dtype
    segments = (abi.Segment * 2)()
    segments[0].destination_row, segments[0].length = 0, 3
    segments[1].destination_row, segments[1].length = 5, 1  # gap: should be 4
    assert lib.lrk_batch_append(segments, 2, 1, 1, 64, abi.BF16, 1, 1, 1, 6, None) == abi.ERR_INVALID
    with pytest.raises(abi.LrkError):
        abi.check(lib.lrk_refine(None, None, 10, None, None, 0, 3, None, 0, None, None, None, None, None))
    keyed = (abi.KeySegment * 1)()
    keyed[0].first, keyed[0].last = 5, 5  # empty candidate interval
    assert lib.lrk_scores_from_keys_workspace_bytes(keyed, 1, 10, 4) == 0
    assert lib.lrk_scores_from_keys(keyed, 1, None, 0, None, 10, 4, 96, 0.1, None, 1e-6, None, 0,
                                    None) == abi.ERR_INVALID  # head dimension 96
    assert lib.lrk_scores_from_keys(keyed, 1, None, 0, None, 10, 4, 128, 0.1, None, 1e-6, None, 0,
                                    None) == abi.ERR_INVALID  # no layers


def test_logits_heads_checks_every_head_first():
    """lrk_logits_heads rejects a table with any bad head before launching
    anything (include/lrk.h), so these calls need no GPU."""
    lib = abi.library()
    table = (abi.LogitsHead * 2)()
    for h in table:
        h.queries, h.keys, h.out, h.count, h.k_step, h.out_stride = 256, 512, 1024, 100, 16, 104
    table[1].k_step = 4
    assert lib.lrk_logits_heads(table, 2, 8, 128, None) == abi.ERR_INVALID  # step 4
    table[1].k_step, table[1].out_stride = 8, 100
    assert lib.lrk_logits_heads(table, 2, 8, 128, None) == abi.ERR_INVALID  # stride not a multiple of 8
    table[1].out_stride = 104
    assert lib.lrk_logits_heads(table, 2, 8, 96, None) == abi.ERR_INVALID  # head dimension 96
    table[0].keys = 520
    assert lib.lrk_logits_heads(table, 2, 8, 128, None) == abi.ERR_INVALID  # unaligned keys
    assert lib.lrk_logits_heads(None, 2, 8, 128, None) == abi.ERR_INVALID
    assert lib.lrk_logits_heads(None, 0, 8, 128, None) == abi.OK
    assert lib.lrk_logits_heads(table, 2, 0, 128, None) == abi.OK  # no rows: nothing to do, like lrk_logits
    table[0].keys, table[0].count, table[1].count = 512, 0, 0
    assert lib.lrk_logits_heads(table, 2, 8, 128, None) == abi.OK  # no keys


def test_zero_sized_calls_are_noops():
    lib = abi.library()
    assert lib.lrk_compact(None, None, None, 5, 64, abi.BF16, None, 5, None, None, None, None) == abi.OK
    assert lib.lrk_merge(None, None, None, 0, None, None, 0, None, 0, 64, abi.BF16, None, None, None, None) == abi.OK
    assert lib.lrk_pack(None, None, None, 0, 64, abi.BF16, None, None, 0, 0, None, None, None) == abi.OK


def test_modules_expose_reference_operator_names():
    # csrc/bindings.cpp:21-28, csrc/cache_legacy.cu:305-307, csrc/host.cpp:16-17
    C = operators()
    for name in ["temporal_probabilities", "temporal_risk", "append", "compact", "pool", "merge", "pack",
                 "batch_append", "refine", "topk_smallest"]:
        assert callable(getattr(C, name)), name
    for name in ["append_flattened_cache", "compact_flattened_kv", "decision_risk_scores"]:
        assert callable(getattr(legacy_operators(), name))
    for name in ["register_host", "unregister_host"]:
        assert callable(getattr(host_operators(), name))


def test_shim_rejects_cpu_tensors_like_the_reference():
    import torch

    C = operators()
    k = torch.zeros(4, 8, dtype=torch.bfloat16)
    pos = torch.zeros(4, 1)
    with pytest.raises(RuntimeError, match="Expected contiguous CUDA tensor"):
        C.compact(k, k, pos, torch.zeros(0, dtype=torch.long))
    with pytest.raises(RuntimeError, match="Contiguous CUDA states required"):
        C.batch_append([k], [k], [pos], torch.zeros(1, 2, 1, 8), torch.zeros(1, 2, 1, 8), [[2, 2]], [4])
    with pytest.raises(RuntimeError, match="cache must be CUDA"):
        legacy_operators().append_flattened_cache(k, torch.zeros(1, 1, 1, 8, dtype=torch.bfloat16),
                                                  torch.zeros(1, dtype=torch.int32), torch.zeros(2, dtype=torch.int32))


def test_no_cpu_fallback_in_selection():
    import torch
    from types import SimpleNamespace

    from code_for_iclr27_b200.selection import refine_arrays

    seg = [SimpleNamespace(layer=0, head=0, position_start=0, count=4)]
    table = SimpleNamespace(scores=torch.rand(4), segments=seg, cumulative_ends=[4])
    with pytest.raises(RuntimeError, match="CUDA"):
        refine_arrays(table, table, 2)
