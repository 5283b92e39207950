"""ctypes binding of liblrk's C ABI (include/lrk.h).

This is the same surface a non-Python host (cgo, JNI, N-API) would bind.
Pointers are passed as integers (e.g. ``tensor.data_ptr()``), streams as the
integer value of a ``cudaStream_t`` (``torch.cuda.current_stream().cuda_stream``).
Every entry point returns an lrk_status; :func:`check` raises on failure.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from . import LIBRARY_PATH

OK, ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_WORKSPACE = 0, 1, 2, 3, 4
F32, F64, F16, BF16 = 0, 1, 2, 3
STATIC_SCORE_ROWS = 262144  # LRK_STATIC_SCORE_ROWS in include/lrk.h
# Layer-group selection state (LRK_SELECT_* in include/lrk.h).
SELECT_BINS, SELECT_ROUNDS, SELECT_STATE_FIELDS = 4096, 3, 8
SELECT_K, SELECT_PREFIX, SELECT_NEED, SELECT_BELOW, SELECT_LOCAL_BELOW, SELECT_TOTAL, SELECT_SHARE = range(7)

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F = ctypes.c_float
D = ctypes.c_double
SIZE = ctypes.c_size_t


class Segment(ctypes.Structure):
    """lrk_segment (include/lrk.h)."""
    _fields_ = [("keys", P), ("values", P), ("positions", P), ("source_row", I64), ("length", I64),
                ("destination_row", I64), ("logical_position", I64)]


class ScoreSegment(ctypes.Structure):
    """lrk_score_segment (include/lrk.h)."""
    _fields_ = [("logits", P), ("projected_values", P), ("projected_stride", I64), ("key_positions", P),
                ("length", I64), ("first", I64), ("last", I64), ("scores", P), ("logits_stride", I64),
                ("query_chunk", I64)]


class MergeLayer(ctypes.Structure):
    """lrk_merge_layer (include/lrk.h)."""
    _fields_ = [("keys", P), ("values", P), ("positions", P), ("rows", I64), ("recalled", P),
                ("recalled_positions", P), ("recalled_rows", I64), ("mapping", P), ("out_rows", I64)]


class LogitsHead(ctypes.Structure):
    """lrk_logits_head (include/lrk.h)."""
    _fields_ = [("queries", P), ("keys", P), ("count", I64), ("k_step", I64), ("out", P), ("out_stride", I64)]


class KeyLayer(ctypes.Structure):
    """lrk_key_layer (include/lrk.h)."""
    _fields_ = [("keys", P), ("rows", I64)]


class KeySegment(ctypes.Structure):
    """lrk_key_segment (include/lrk.h)."""
    _fields_ = [("layer", I64), ("queries", P), ("query_stride", I64), ("projected_values", P),
                ("projected_stride", I64), ("key_positions", P), ("key_row", I64), ("length", I64), ("first", I64),
                ("last", I64), ("scores", P), ("query_chunk", I64)]


class PlanLayer(ctypes.Structure):
    """lrk_plan_layer (include/lrk.h)."""
    _fields_ = [("positions", P), ("head_starts", P), ("recalled_positions", P), ("recalled_index", P),
                ("recalled_starts", P), ("rows", I64), ("recalled", I64), ("mapping", P)]


class Arena(ctypes.Structure):
    """lrk_arena (include/lrk.h)."""
    _fields_ = [("keys", P), ("values", P), ("positions", P), ("lengths", P), ("heads_total", I64),
                ("capacity", I64), ("dimension", I64), ("dtype", I32)]


SIGNATURES = {
    "lrk_last_error": (ctypes.c_char_p, []),
    "lrk_version": (I32, []),
    "lrk_dtype_size": (I32, [I32]),
    "lrk_temporal_probabilities": (I32, [P, I32, P, P, P, P, P, I64, I64, I64, F, P]),
    "lrk_temporal_risk": (I32, [P, P, P, P, P, I64, I64, I64, I64, I64, F, P]),
    "lrk_pool": (I32, [P, I64, P, I64, I64, I64, P, P]),
    "lrk_temporal_scores_workspace_bytes": (SIZE, [I64, I64, I64]),
    "lrk_temporal_scores_stash_bytes": (SIZE, [ctypes.POINTER(ScoreSegment), I64, I64, I64]),
    "lrk_temporal_scores": (I32, [ctypes.POINTER(ScoreSegment), I64, I32, P, I64, I64, F, P, F, P, SIZE, P]),
    "lrk_temporal_scores_static": (I32, [ctypes.POINTER(ScoreSegment), I64, I32, P, I64, I64, F, P, F, P]),
    "lrk_decision_risk": (I32, [P, P, I32, P, P, I64, I64, I64, D, F, P, P]),
    "lrk_append": (I32, [P, P, P, I64, P, P, P, I64, I64, I64, I32, I64, P, P, P, P, P, P]),
    "lrk_compact": (I32, [P, P, P, I64, I64, I32, P, I64, P, P, P, P]),
    "lrk_merge": (I32, [P, P, P, I64, P, P, I64, P, I64, I64, I32, P, P, P, P]),
    "lrk_merge_layers": (I32, [ctypes.POINTER(MergeLayer), I64, I64, I32, P, P, P, P]),
    "lrk_pack": (I32, [P, P, P, I64, I64, I32, P, P, I64, I64, P, P, P]),
    "lrk_batch_append": (I32, [ctypes.POINTER(Segment), I64, P, P, I64, I32, P, P, P, I64, P]),
    "lrk_append_flattened": (I32, [P, I64, P, I64, I64, I64, I32, P, P, P, I64, P]),
    "lrk_compact_flattened": (I32, [P, P, I64, I64, I32, P, I64, P, P, P]),
    "lrk_refine_workspace_bytes": (SIZE, [I64, I64]),
    "lrk_refine": (I32, [P, P, I64, P, P, I64, I64, P, SIZE, P, P, P, P, P]),
    "lrk_topk_workspace_bytes": (SIZE, [I64]),
    "lrk_topk_smallest": (I32, [P, I64, I64, P, SIZE, P, P, P]),
    "lrk_gather_rows": (I32, [P, I64, I64, P, I64, P, P]),
    "lrk_project_values": (I32, [P, I32, I64, I64, P, P, I64, I64, P, P]),
    "lrk_check_division": (I32, [ctypes.c_uint64, ctypes.c_uint64, P, P]),
    "lrk_logits": (I32, [P, I64, P, I64, I64, I64, P, I64, P]),
    "lrk_logits_heads": (I32, [P, I64, I64, I64, P]),
    "lrk_logits_timeouts": (I32, [P]),
    "lrk_scores_from_keys_workspace_bytes": (SIZE, [ctypes.POINTER(KeySegment), I64, I64, I64]),
    "lrk_scores_from_keys": (I32, [ctypes.POINTER(KeySegment), I64, ctypes.POINTER(KeyLayer), I64, P, I64, I64, I64,
                                   F, P, F, P, SIZE, P]),
    "lrk_scores_from_keys_timeouts": (I32, [P]),
    "lrk_host_device_pointer": (I32, [P, ctypes.POINTER(P)]),
    "lrk_register_host": (I32, [P, SIZE]),
    "lrk_unregister_host": (I32, [P]),
    "lrk_select_histogram": (I32, [ctypes.POINTER(P), ctypes.POINTER(I64), I64, I64, I32, P, P, P]),
    "lrk_select_pick": (I32, [P, I64, I64, I64, I64, I32, P, P]),
    "lrk_arena_append": (I32, [ctypes.POINTER(Arena), I64, I64, P, P, F, P, P]),
    "lrk_arena_compact": (I32, [ctypes.POINTER(Arena), P, I64, P, P, P]),
    "lrk_arena_compact_positions": (I32, [ctypes.POINTER(Arena), P, I64, P, P, P]),
    "lrk_arena_evict": (I32, [ctypes.POINTER(Arena), P, P, I64, P, P]),
    "lrk_merge_plan": (I32, [ctypes.POINTER(PlanLayer), I64, I64, P, P]),
    "lrk_arena_insert": (I32, [ctypes.POINTER(Arena), P, I64, P, P, I32, P, P]),
}

_library = None


def library(path: str | Path | None = None) -> ctypes.CDLL:
    """Load liblrk.so once and declare every entry point's types."""
    global _library
    if _library is None or path is not None:
        lib = ctypes.CDLL(str(path or LIBRARY_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            function = getattr(lib, name)
            function.restype = restype
            function.argtypes = argtypes
        if path is not None:
            return lib
        _library = lib
    return _library


class LrkError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"liblrk status {status}: {message}")
        self.status = status


def check(status: int) -> None:
    if status != OK:
        raise LrkError(status, library().lrk_last_error().decode(errors="replace"))


def dtype_code(torch_dtype) -> int:
    import torch

    return {torch.float32: F32, torch.float64: F64, torch.float16: F16, torch.bfloat16: BF16}[torch_dtype]
