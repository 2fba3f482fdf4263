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

# (source, extra flags, object name): translation units compile in parallel.
UNITS = [
    ("matrix.cu", [], "matrix.o"),
    ("abi.cpp", [], "abi.o"),
    ("kernels_reg.cu", [], "kernels_reg.o"),
    ("kernels_tile.cu", [], "kernels_tile.o"),
    ("kernels_mma.cu", ["-DQMR_MMA_BITS=4"], "kernels_mma4.o"),
    ("kernels_mma.cu", ["-DQMR_MMA_BITS=8"], "kernels_mma8.o"),
    ("static_scratch.cu", [], "static_scratch.o"),
    ("decode.cu", [], "decode.o"),
    ("engine.cpp", [], "engine.o"),
    ("checkpoint.cpp", [], "checkpoint.o"),
]
SOURCES = sorted({u[0] for u in UNITS})
HEADERS = ["matrix_kernels.cuh", "qmr_internal.h", "tile.cuh", "mma_stream.cuh", "launch.h", "pipe.cuh", "decode.h",
           "checkpoint.h"]
OBJ_DIR = PKG_ROOT / "_build"

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
    from concurrent.futures import ThreadPoolExecutor
    OBJ_DIR.mkdir(exist_ok=True)
    tool = nvcc()

    def compile_unit(unit):
        src, extra, obj = unit
        cmd = [tool, *NVCC_FLAGS, *extra, "-c"]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        cmd += ["-I", str(REPO_ROOT / "include"), "-o", str(OBJ_DIR / obj), str(CSRC / src)]
        return subprocess.run(cmd, capture_output=True, text=True)

    with ThreadPoolExecutor(max_workers=min(len(UNITS), os.cpu_count() or 1)) as pool:
        results = list(pool.map(compile_unit, UNITS))
    for unit, proc in zip(UNITS, results):
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            raise RuntimeError(f"nvcc failed on {unit[0]} ({proc.returncode})")
        if verbose:
            sys.stderr.write(proc.stderr)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [tool, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp)]
    link += [str(OBJ_DIR / u[2]) for u in UNITS]
    proc = subprocess.run(link, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"nvcc failed linking libqmr ({proc.returncode})")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
