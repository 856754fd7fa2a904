"""Generate the golden fixture that pins the W4A8 oracle (oracle/w4a8.py) to the
reference.

Run where the reference tree is available (TLX_REFERENCE, else a "reference"
directory beside this repository):

    python tests/golden/gen_golden_w4a8.py

It runs the reference's OWN code on seeded inputs and writes
tests/golden/golden_w4a8.npz:
- the token quantiser loop of engine/p8_w4_test.py:59-70 (the reference's numpy
  check of its p8q8x kernel), compiled alone from that file as written;
- the linearised codebook and ``dq_lin`` of engine/p8_w4ffn7_test.py:43-46,62-88
  (the reference's numpy model of its p8w4ffn7 weights), compiled alone as written,
  on rows in the reference's row-region layout;
- ``pack_tensor`` of engine/pack_w7.py:40-73, the packed7 layout p8w4ffn7 reads.
Those test scripts drive the reference's GPU engine at import, so only the listed
statements are taken out of them.  Nothing at test time reads the reference tree.
"""
from __future__ import annotations

import ast
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from gen_golden import REF, load_reference, region_repack_iq3  # noqa: E402
from thunderllamax_b200 import synth  # noqa: E402

K = 512
NCH = K // 128


def _module(path):
    return ast.parse(open(path).read(), path)


def reference_quantiser(x16: np.ndarray):
    """The module-level ``for c in range(NCH)`` loop of engine/p8_w4_test.py that
    builds xq, sx, rs from xf."""
    path = os.path.join(REF, "engine", "p8_w4_test.py")
    tree = _module(path)
    loops = [n for n in tree.body if isinstance(n, ast.For) and isinstance(n.target, ast.Name)
             and n.target.id == "c" and "rs[" in ast.unparse(n)]
    assert len(loops) == 1
    m = x16.shape[0]
    ns = {"np": np, "NCH": NCH, "xf": x16, "xq": np.zeros((m, K), dtype=np.int8),
          "sx": np.zeros((m, NCH), dtype=np.float32), "rs": np.zeros((m, NCH), dtype=np.int32)}
    exec(compile(ast.Module(body=loops, type_ignores=[]), path, "exec"), ns)
    return ns["xq"], ns["sx"], ns["rs"]


def reference_linearised(pack_w4):
    """lut8 (DELTA, G, lut8 assignments) and dq_lin (nested in lin_ref) of
    engine/p8_w4ffn7_test.py."""
    path = os.path.join(REF, "engine", "p8_w4ffn7_test.py")
    tree = _module(path)
    assigns = [n for n in tree.body if isinstance(n, ast.Assign) and len(n.targets) == 1
               and isinstance(n.targets[0], ast.Name) and n.targets[0].id in ("DELTA", "G", "lut8")]
    assert [a.targets[0].id for a in assigns] == ["DELTA", "G", "lut8"]
    ns = {"np": np, "grid_f32": pack_w4.grid_f32, "KD": K}
    exec(compile(ast.Module(body=assigns, type_ignores=[]), path, "exec"), ns)
    lin_ref = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "lin_ref"]
    dq = [n for n in lin_ref[0].body if isinstance(n, ast.FunctionDef) and n.name == "dq_lin"]
    assert len(dq) == 1
    exec(compile(ast.Module(body=dq, type_ignores=[]), path, "exec"), ns)
    return ns["lut8"], ns["dq_lin"]


def main():
    _, _, pack_w4, _ = load_reference()
    sys.path.insert(0, os.path.join(REF, "engine"))
    import pack_w7

    rng = np.random.default_rng(20261202)
    g = {}
    x = (rng.standard_normal((8, K)) * 0.7).astype(np.float16)
    x[1, 128:256] = 0                                                # an all-zero chunk: s = 1e-6 / 127
    x[2, 256:384] = (rng.standard_normal(128) * 1e-7).astype(np.float16)   # max below 1e-6
    x[3] = np.clip(rng.standard_normal(K) * 1.5e4, -6e4, 6e4).astype(np.float16)   # near the fp16 range
    ties = np.arange(128, dtype=np.float32) - 63.5                   # .5 steps: s = 1, ties to even
    ties[0] = 127.0
    x[4, 0:128] = ties.astype(np.float16)
    x[5, 384:512] = -x[5, 384:512]
    g["q8_x"] = x
    g["q8_xq"], g["q8_sx"], g["q8_rs"] = reference_quantiser(x)

    lut8, dq_lin = reference_linearised(pack_w4)
    raw = synth.iq3xxs_blocks(rng, 16, K)
    region = region_repack_iq3(raw, K)
    g["lut8"] = lut8
    g["lin_raw"] = raw
    g["lin_w"] = dq_lin(region)
    g["packed7"] = np.frombuffer(pack_w7.pack_tensor(np.ascontiguousarray(region), K)[0], dtype=np.uint8)

    out = os.path.join(HERE, "golden_w4a8.npz")
    np.savez_compressed(out, **g)
    print(out, {k: v.shape for k, v in g.items()})


if __name__ == "__main__":
    main()
