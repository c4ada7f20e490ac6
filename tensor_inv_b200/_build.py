"""Build ``libtensor_inv_crt.so`` in-tree with nvcc for sm_100a.

``python -m tensor_inv_b200._build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` to an object with ``-gencode arch=compute_100a,code=sm_100a`` and links them
into ``tensor_inv_b200/libtensor_inv_crt.so`` (static CUDA runtime, no libtorch).  Objects
go to ``tensor_inv_b200/_build/``; a source is recompiled only when it, or a header, is newer
than its object.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libtensor_inv_crt.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; set NVCC or put CUDA 12.8+ on PATH")
    return cand


def build(verbose: bool = False, force: bool = False, extra_flags=()) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    objects = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        stale = (force or not obj.exists() or obj.stat().st_mtime < src.stat().st_mtime
                 or obj.stat().st_mtime < newest_header)
        if stale:
            cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *extra_flags, "-I", str(INCLUDE),
                   "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objects):
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(LIB), *map(str, objects)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
