"""Compile reference kernels into oracle/_ref/ (test infrastructure only).

    python oracle/build_ref.py            # TLX_REFERENCE overrides /root/reference

Each listed kernel is one self-contained .cu file of the reference tree
(engine/<name>.cu, extern "C"); nvcc compiles it as written, from where it
lies, into oracle/_ref/<name>.cubin for sm_100a.  The GPU parity tests load these
cubins and run the reference's own kernels next to the library's on the same
device inputs.  Nothing in the product loads them; the directory is git-ignored
and travels to the GPU box with the working tree.  Without the reference tree the
script does nothing and the tests that need a cubin are skipped.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF = os.environ.get("TLX_REFERENCE", "/root/reference")

# (engine-relative source, kernel name): kernels whose every access was checked by
# reading against the shapes the tests launch them with (integer / index / copy work
# of the verify cycle).  Fixed shapes compiled into them: amx3 / h_argmax read
# 248320 fp16 logits per row, accept11k copies 5120-float rows, acceptsel11k
# copies [48][5] x (786432 + 30720) floats and indexes its slot by m in 0..10.
KERNELS = [(f"lookup{n}_nw32.cu", f"lookup{n}_nw32") for n in range(5, 12)] + [
    ("accept11k.cu", "accept11k"),
    ("acceptsel11k.cu", "acceptsel11k"),
    ("h_argmax.cu", "h_argmax"),
    ("amx3.cu", "amx3"),
    ("mm/MM_P7_acc36.cu", "acc36"),
]


def build(verbose: bool = False) -> list[str]:
    src_dir = os.path.join(REF, "engine")
    if not os.path.isdir(src_dir):
        return []
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    os.makedirs(OUT, exist_ok=True)
    built = []
    for rel, name in KERNELS:
        src = os.path.join(src_dir, rel)
        if not os.path.exists(src):
            continue
        out = os.path.join(OUT, name + ".cubin")
        cmd = [nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-o", out, src]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        built.append(out)
    return built


if __name__ == "__main__":
    print("\n".join(build(verbose="-v" in sys.argv)))
