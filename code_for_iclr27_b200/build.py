"""In-tree build of liblrk.so and the three operator modules.

liblrk.so   <- csrc/host.cu, move.cu, score.cu, select.cu, fused.cu, project.cu, logits.cu,
               logits_tc.cu, scores_tc.cu, groups.cu,
               arena.cu, plan.cu (nvcc, sm_100a)
_C          <- csrc/shim_C.cpp        (torch extension, links liblrk)
_legacy_C   <- csrc/shim_legacy_C.cpp (torch extension, links liblrk)
_host       <- csrc/shim_host.cpp     (pybind11 only, links liblrk)

Every artefact lands next to this file, so the built tree travels as a
whole; the modules find liblrk.so through an $ORIGIN rpath.  Targets are
rebuilt only when a source or header is newer than the artefact.

    python -m code_for_iclr27_b200.build [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
OBJ = ROOT / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")

CUDA_SOURCES = {
    "host.cu": [],
    "move.cu": [],
    # Same no-contraction rule as the reference scoring build (setup.py:15-16).
    "score.cu": ["--fmad=false"],
    "select.cu": [],
    "fused.cu": ["--fmad=false"],
    "project.cu": [],
    "logits.cu": [],
    "logits_tc.cu": [],
    "scores_tc.cu": ["--fmad=false"],
    "groups.cu": [],
    "arena.cu": [],
    "plan.cu": [],
}
MODULES = {"_C": "shim_C.cpp", "_legacy_C": "shim_legacy_C.cpp", "_host": "shim_host.cpp"}
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
LIBRARY = PACKAGE / "liblrk.so"


def module_path(name: str) -> Path:
    return PACKAGE / f"{name}{EXT_SUFFIX}"


def _headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(target: Path, sources) -> bool:
    if not target.exists():
        return True
    newest = max(Path(s).stat().st_mtime for s in sources)
    return newest > target.stat().st_mtime


def _run(command, label):
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"{label} failed ({result.returncode}):\n{' '.join(command)}\n{result.stdout}\n{result.stderr}")
    return result.stderr


def _nvcc_object(source: str, extra, force: bool) -> Path:
    src = CSRC / source
    obj = OBJ / (source + ".o")
    if force or _stale(obj, [src, *_headers()]):
        command = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
                   f"-I{INCLUDE}", f"-I{CSRC}", *extra, "-c", str(src), "-o", str(obj)]
        log = _run(command, f"nvcc {source}")
        (OBJ / (source + ".ptxas.txt")).write_text(log)
    return obj


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce

    includes = [*ce.include_paths(device_type="cuda")]
    library_dirs = [*ce.library_paths(device_type="cuda")]
    abi = int(bool(torch._C._GLIBCXX_USE_CXX11_ABI))
    defines = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    pybind_abi = getattr(ce, "_get_pybind11_abi_build_flags", None)
    if pybind_abi is not None:
        defines += list(pybind_abi())
    libraries = ["c10", "torch", "torch_cpu", "torch_python", "c10_cuda", "torch_cuda"]
    return includes, library_dirs, defines, libraries


def _module(name: str, source: str, force: bool) -> Path:
    target = module_path(name)
    src = CSRC / source
    if not (force or _stale(target, [src, LIBRARY, *_headers()])):
        return target
    python_include = sysconfig.get_paths()["include"]
    import pybind11

    common = ["g++", "-O3", "-std=c++17", "-fPIC", "-shared", f"-DTORCH_EXTENSION_NAME={name}",
              f"-I{INCLUDE}", f"-I{CSRC}", f"-I{python_include}", f"-I{pybind11.get_include()}",
              f"-I{CUDA_HOME / 'include'}"]
    link = [f"-L{PACKAGE}", "-llrk", "-Wl,-rpath,$ORIGIN"]
    if name == "_host":
        command = [*common, str(src), "-o", str(target), *link]
    else:
        includes, library_dirs, defines, libraries = _torch_flags()
        command = [*common, *defines, *[f"-I{i}" for i in includes], str(src), "-o", str(target), *link,
                   *[f"-L{d}" for d in library_dirs], *[f"-Wl,-rpath,{d}" for d in library_dirs],
                   *[f"-l{lib}" for lib in libraries]]
    _run(command, f"g++ {source}")
    return target


def build(force: bool = False, jobs: int | None = None) -> dict:
    """Compile everything that is stale; return {name: path}."""
    if not Path(NVCC).exists():
        raise RuntimeError(f"nvcc not found at {NVCC}")
    OBJ.mkdir(parents=True, exist_ok=True)
    jobs = jobs or min(8, os.cpu_count() or 4)
    with futures.ThreadPoolExecutor(jobs) as pool:
        objects = list(pool.map(lambda item: _nvcc_object(item[0], item[1], force), CUDA_SOURCES.items()))
    if force or _stale(LIBRARY, objects):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), "-cudart", "static"], "link liblrk")
    with futures.ThreadPoolExecutor(jobs) as pool:
        paths = dict(zip(MODULES, pool.map(lambda item: _module(item[0], item[1], force), MODULES.items())))
    paths["liblrk"] = LIBRARY
    return paths


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    args = parser.parse_args(argv)
    for name, path in build(args.force, args.jobs).items():
        print(f"{name}: {path}")


if __name__ == "__main__":
    sys.exit(main())
