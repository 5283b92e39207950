"""Build the reference's own CUDA operator modules from its sources into oracle/_ref/.

Test infrastructure only.  The reference (LazyRecall) ships three torch
extension modules built by its setup.py (setup.py:19-27):
``lazy_recall._C`` from csrc/bindings.cpp, csrc/scoring.cu, csrc/recall.cu,
csrc/batch_append.cu; ``lazy_recall._legacy_C`` from csrc/cache_legacy.cu and
``lazy_recall._host`` from csrc/host.cpp.  This recipe compiles those source
files where they lie (it never copies them) with the reference's own nvcc
flags (setup.py:15-18) for sm_100a, so that GPU parity tests can compare the
new kernels with the reference kernels on identical inputs.  The reference's
setup.py is not run.

Usage: python oracle/build_ref.py [REFERENCE_ROOT]  (default: oracle/reference_root.py)
Outputs: oracle/_ref/{C,legacy_C,host}/<module>.so (git-ignored, travels with
the repository snapshot to the GPU box).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"

MODULES = {
    "C": ("_C", ["csrc/bindings.cpp", "csrc/scoring.cu", "csrc/recall.cu", "csrc/batch_append.cu"]),
    "legacy_C": ("_legacy_C", ["csrc/cache_legacy.cu"]),
    "host": ("_host", ["csrc/host.cpp"]),
}


def built_paths():
    """Return {key: path-to-.so} for modules already built (any missing key is absent)."""
    found = {}
    for key, (name, _) in MODULES.items():
        for candidate in (OUT / key).glob(f"{name}*.so"):
            found[key] = candidate
    return found


def build(reference_root: str, verbose: bool = False) -> dict:
    root = Path(reference_root)
    if not (root / "csrc" / "scoring.cu").exists():
        raise FileNotFoundError(f"reference sources not found under {root}")
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils.cpp_extension import CUDA_HOME, load

    cuda_home = Path(CUDA_HOME or "/usr/local/cuda")

    nvcc = ["-O3", "-std=c++17", "--fmad=false", "-U__CUDA_NO_HALF_OPERATORS__",
            "-U__CUDA_NO_HALF_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-lineinfo"]
    done = built_paths()
    for key, (name, sources) in MODULES.items():
        if key in done:
            continue
        directory = OUT / key
        directory.mkdir(parents=True, exist_ok=True)
        # setup.py:10-14 adds CUDA_HOME/include for every module; _host has no
        # .cu source, so it also needs the CUDA runtime on its link line.
        ldflags = [f"-L{cuda_home / 'lib64'}", "-lcudart"] if key == "host" else []
        load(name=name, sources=[str(root / s) for s in sources], build_directory=str(directory),
             extra_cflags=["-O3", "-std=c++17"], extra_cuda_cflags=nvcc, extra_ldflags=ldflags,
             extra_include_paths=[str(cuda_home / "include")], verbose=verbose, is_python_module=True)
    return built_paths()


if __name__ == "__main__":
    sys.path.insert(0, str(HERE.parent))
    from oracle.reference_root import reference_root

    root = sys.argv[1] if len(sys.argv) > 1 else reference_root()
    if root is None:
        raise SystemExit("reference sources not found: pass REFERENCE_ROOT or set LAZY_RECALL_REFERENCE")
    paths = build(str(root), verbose=True)
    for key, path in sorted(paths.items()):
        print(key, path)
