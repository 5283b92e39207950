"""Install the reference's own Python package, unchanged, into oracle/_ref/py.

Test and baseline infrastructure only.  The reference (LazyRecall) builds its
CUDA extensions only when LAZY_RECALL_BUILD_CUDA is not "0" (setup.py:8); with
it set to "0" the package is pure Python and its operators take the CPU math
path (scoring.py:75-149, selection.py:52-88, cache.py:162-167 ...).  This
recipe installs that configuration with pip (no index, no build isolation, no
dependencies: torch and numpy are already in the image) from a temporary copy
of the reference tree (its build writes into the source tree, which may be
read-only), into oracle/_ref/py.  oracle/_ref is git-ignored and travels with
the repository snapshot to the GPU box, where bench.py --impl reference times
the reference's CPU path and the drop-in tests run the reference's own Python
on this repository's operator modules.

Usage: python oracle/install_ref_py.py [REFERENCE_ROOT]  (default: oracle/reference_root.py)
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref" / "py"


def installed() -> Path | None:
    """oracle/_ref/py when it holds the reference package, else None."""
    return TARGET if (TARGET / "lazy_recall" / "scoring.py").exists() else None


def install(reference_root: str, force: bool = False) -> Path:
    root = Path(reference_root)
    if not (root / "src" / "lazy_recall" / "scoring.py").exists():
        raise FileNotFoundError(f"reference package not found under {root}")
    if installed() and not force:
        return TARGET
    with tempfile.TemporaryDirectory() as scratch:
        source = Path(scratch) / "reference"
        shutil.copytree(root, source, ignore=shutil.ignore_patterns(".git", "build", "*.egg-info", "__pycache__"))
        if TARGET.exists():
            shutil.rmtree(TARGET)
        env = dict(os.environ, LAZY_RECALL_BUILD_CUDA="0")
        subprocess.run([sys.executable, "-m", "pip", "install", "--quiet", "--no-index", "--no-build-isolation",
                        "--no-deps", "--target", str(TARGET), str(source)], check=True, env=env, cwd=scratch)
    return TARGET


if __name__ == "__main__":
    sys.path.insert(0, str(HERE.parent))
    from oracle.reference_root import reference_root

    root = sys.argv[1] if len(sys.argv) > 1 else reference_root()
    if root is None:
        raise SystemExit("reference sources not found: pass REFERENCE_ROOT or set LAZY_RECALL_REFERENCE")
    print(install(str(root), force=True))
