"""Builds the CUDA library ``libdsai.so`` in-tree for sm_100a.

The library is plain nvcc output (no torch headers): the kernels, the C ABI
declared in ``include/dsai.h`` and a statically linked CUDA runtime, so it
loads on a machine without a GPU driver (symbols can be inspected there) and
runs on a B200.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libdsai.so"
SOURCES = ["score.cu", "score_mq.cu", "fused.cu", "select.cu", "api.cu", "graph.cu", "noalloc.cu", "writer.cu", "attn.cu"]
HEADERS = ["common.cuh", "sm100.cuh", "launch.h", "tiles.cuh", "radix.cuh", "graph.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared", "-cudart", "static",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build libdsai.so")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [REPO / "include" / "dsai.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles libdsai.so next to this file if it is missing or stale."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(REPO / "include"), "-o", str(tmp),
           *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
