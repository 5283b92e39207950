"""B200-native (sm_100a) KV-cache management hot path for LazyRecall.

The package holds liblrk.so (hand-written CUDA kernels behind the C ABI in
include/lrk.h) and three extension modules with the reference's operator
names and signatures:

  _C         temporal_probabilities, temporal_risk, append, compact, pool,
             merge, pack, batch_append (+ refine, topk_smallest,
             temporal_scores, project_values, logits, compact_layers)
  _legacy_C  append_flattened_cache, compact_flattened_kv, decision_risk_scores
  _host      register_host, unregister_host

Build them in place with ``python -m code_for_iclr27_b200.build``.  There is
no CPU fallback: importing an operator module that was not built raises.
"""
from __future__ import annotations

import importlib
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "liblrk.so"

__all__ = ["operators", "legacy_operators", "host_operators", "upload", "LIBRARY_PATH"]


def _module(name: str):
    try:
        return importlib.import_module(f"{__name__}.{name}")
    except ImportError as error:
        raise RuntimeError(
            f"{__name__}.{name} is not built (liblrk CUDA extension missing). "
            f"Run: python -m {__name__}.build") from error


def upload(array, device, dtype=None):
    """A host array as a CUDA tensor, copied through pinned staging memory so
    that the copy is only queued on the current stream.  (A copy from
    pageable memory makes the host wait for the work queued before it, which
    stops the host from running ahead of the device.)"""
    import torch

    return torch.as_tensor(array, dtype=dtype).pin_memory().to(device, non_blocking=True)


def operators():
    """The lazy_recall._C replacement module."""
    return _module("_C")


def legacy_operators():
    """The lazy_recall._legacy_C replacement module."""
    return _module("_legacy_C")


def host_operators():
    """The lazy_recall._host replacement module."""
    return _module("_host")
