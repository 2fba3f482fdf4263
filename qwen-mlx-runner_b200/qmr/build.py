"""Build recipe for libqmr.so (sm_100a) in-tree, next to the package.

The library is built with nvcc directly: no JIT cache, so the shared object
travels with the source tree.  IEEE subnormals must stay enabled (no -ftz,
no --use_fast_math): the streaming kernels extract quantised values as exact
subnormal floats.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

PKG_ROOT = pathlib.Path(__file__).resolve().parents[1]  # qwen-mlx-runner_b200/
CSRC = PKG_ROOT / "csrc"
LIB_PATH = PKG_ROOT / "libqmr.so"
REPO_ROOT = PKG_ROOT.parent

SOURCES = ["matrix.cu", "abi.cpp"]
HEADERS = ["matrix_kernels.cuh", "qmr_internal.h", "tile.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-ftz=false",
    "-prec-div=true",
    "-prec-sqrt=true",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wall",
    "-shared",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libqmr")
    return path


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [REPO_ROOT / "include" / "qmr.h"]
    return any(d.stat().st_mtime > built for d in deps)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compile libqmr.so if any source is newer than it (or force)."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-I", str(REPO_ROOT / "include"), "-o", str(tmp)]
    cmd += [str(CSRC / s) for s in SOURCES]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"nvcc failed building libqmr ({proc.returncode})")
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
