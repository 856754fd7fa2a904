"""Build the in-tree CUDA library (sm_100a only).

    python -m thunderllamax_b200.build

compiles csrc/*.cu with nvcc for sm_100a and links libtlx_b200.so next to this
file (in-tree, so it travels with the repository snapshot).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libtlx_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]
SOURCES = ["gemv.cu", "capi.cu", "moe.cu", "prefill.cu", "noalloc.cu", "lookup.cu", "attention.cu", "peer.cu", "w4a8.cu"]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found")
    return exe


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        if not os.path.exists(path):
            continue
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, *FLAGS, *(extra or []), "-c", path, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None)
