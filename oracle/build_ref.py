"""Compile reference kernels into oracle/_ref/ (test infrastructure only).

    python oracle/build_ref.py   # reference tree: TLX_REFERENCE, else ../reference beside the repository

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
REPO_ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")
# the reference checkout: TLX_REFERENCE, else a "reference" directory beside this repository
REF = os.environ.get("TLX_REFERENCE") or os.path.normpath(os.path.join(REPO_ROOT, "..", "reference"))

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
# the ROWS = 11 split-KV attention set, with the compile-time shapes the reference
# builds it with (engine/build_k11.py: CTXK = 100352, S = 256 chunks of 392 keys,
# TILE 32, 32 warps); the kernels read and write only inside [8][CTXK] caches and
# [4][S][66] partials, which the tests allocate at exactly these sizes
ATTN_CTX, ATTN_S = 100352, 256
ATTN_KERNELS = [
    ("spk_preqh.cu", "spk_pre11", ["-DKPRE=spk_pre11", f"-DCTXK={ATTN_CTX}", "-DROWS=11"]),
    ("spk_g4hm.cu", "spk_a11", ["-DKNAME=spk_a11", f"-DCTXK={ATTN_CTX}", "-DROWS=11", f"-DS={ATTN_S}",
                                f"-DCH={ATTN_CTX // ATTN_S}", "-DTILE=32", "-DNW=32"]),
    ("skv_split.cu:K2S", "spk_c11", ["-DK2S=spk_c11", f"-DCTXK={ATTN_CTX}", "-DROWS=11", f"-DS={ATTN_S}",
                                 f"-DCH={ATTN_CTX // ATTN_S}", "-DUNROLL=4"]),
]

# the W4A8 prefill pair with the compile-time shapes the reference builds it with
# (engine/build_p8w4.py:33-38): p8q8x reads [M][5120] fp16 rows and writes [M][5120]
# int8 plus [M][40] scales and sums, M = its grid; p8w4ffn7 reads two weight planes
# of [17408 / 8][40][32] 16-byte units, [M][5120] int8 and [M][40] scales, a
# 1024-byte codebook, and writes [M][17408] fp16 for M = 64 * (grid / 272)
W4A8_KERNELS = [
    ("pfk_q8.cu", "p8q8x", ["-DKNAME=p8q8x", "-DKDIM=5120"]),
    ("p8_w4ffn7.cu", "p8w4ffn7", ["-DKNAME=p8w4ffn7", "-DKDIM=5120", "-DNDIM=17408", "-DNTHR=256", "-DNTILE=64",
                                  "-DKCH=128", "-DMTILE=64"]),
]


def _one_kernel(src: str, macro: str, out: str) -> str:
    """The file's preamble plus the one kernel whose name is `macro` (what the
    reference's own build does for its multi-kernel files, engine/build_k11.py
    split_skv), written as a build input under oracle/_ref."""
    text = open(src).read()
    head = 'extern "C" __global__'
    first = text.find(head)
    bodies = text[first:].split(head)[1:]
    body = [b for b in bodies if f") {macro}(" in b.split("\n", 1)[0]]
    assert len(body) == 1, (src, macro)
    with open(out, "w") as f:
        f.write(text[:first] + head + body[0].rstrip() + "\n")
    return out


def build(verbose: bool = False) -> list[str]:
    src_dir = os.path.join(REF, "engine")
    if not os.path.isdir(src_dir):
        return []
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    os.makedirs(OUT, exist_ok=True)
    built = []
    for rel, name, defs in [(r, n, []) for r, n in KERNELS] + ATTN_KERNELS + W4A8_KERNELS:
        src = os.path.join(src_dir, rel.split(":")[0])
        if not os.path.exists(src):
            continue
        if ":" in rel:
            src = _one_kernel(src, rel.split(":")[1], os.path.join(OUT, name + ".cu"))
        out = os.path.join(OUT, name + ".cubin")
        cmd = [nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", *defs, "-o", out, src]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        if ":" in rel:
            os.remove(src)   # the extracted input is not kept
        built.append(out)
    return built


if __name__ == "__main__":
    print("\n".join(build(verbose="-v" in sys.argv)))
