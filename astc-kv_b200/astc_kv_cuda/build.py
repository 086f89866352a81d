"""Build recipe for libakv_cuda.so (sm_100a), in-tree.

``python -m astc_kv_cuda.build`` (with ``astc-kv_b200`` on ``sys.path``) or
``build()`` compiles ``csrc/`` with nvcc for ``-gencode
arch=compute_100a,code=sm_100a`` into ``astc_kv_cuda/libakv_cuda.so``. No GPU
is needed to build.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB = PKG / "libakv_cuda.so"

SOURCES = ["akv_cuda.cu", "akv_tables.cpp", "akv_encode.cpp"]
HEADERS = ["akv_astc_device.cuh", "akv_common.cuh", "akv_decode_kernels.cuh", "akv_attention_kernels.cuh", "akv_tables.h",
           "akv_attn_fp16.cuh",
           "akv_attn_fast.cuh", "akv_decode_fast.cuh"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libakv_cuda.so")


def _stale() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "akv_cuda.h", INCLUDE / "akv_host.h", Path(__file__)]
    return any(d.stat().st_mtime > mtime for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
           "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-shared", "-I", str(INCLUDE),
           "-o", str(LIB)] + [str(CSRC / s) for s in SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    tmp = LIB.with_suffix(".so.tmp")
    cmd[cmd.index(str(LIB))] = str(tmp)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
