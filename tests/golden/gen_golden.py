"""Generate the golden fixtures that pin the oracle to the reference.

Run where the reference tree is available (TLX_REFERENCE, else a "reference"
directory beside this repository):

    python tests/golden/gen_golden.py

It imports the reference's OWN numpy ports -- engine/mm/MM_P2_ports.py
(dq_q6_k, gxup4_ref, gxdn4_ref, gxdn6_ref, rt_prod_ref, cmb_ref),
engine/mm/MM_P0_d2_repack.py (dq_iq4_xs), engine/pack_w4.py
(dequant_iq3xxs), engine/mm/mm_mtp_anchor.py (dq_q4_k_np) and
engine/chain_sim.py (dequant_q5k_rows) -- with the ggml tables they would take from tinygrad injected
from gguf-py, runs them on seeded synthetic blocks, and writes the inputs and
outputs to tests/golden/golden_v1.npz.  Nothing at test time reads the
reference tree; the tests only read the .npz.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from thunderllamax_b200 import synth  # noqa: E402
from inputs import cmb_inputs, router_inputs  # noqa: E402

# the reference checkout: TLX_REFERENCE, else a "reference" directory beside this repository
REF = os.environ.get("TLX_REFERENCE") or os.path.normpath(os.path.join(REPO_ROOT, "..", "reference"))


def load_reference():
    sys.path[:0] = [os.path.join(REF, "engine", "mm"), os.path.join(REF, "engine")]
    from gguf import quants

    if quants.IQ3_XXS.grid is None:
        quants.IQ3_XXS.init_grid()
    import MM_P0_d2_repack as P0
    import MM_P2_ports as P2
    import pack_w4

    tables = {"iq4nl": np.asarray(quants.IQ4_NL.kvalues, dtype=np.float32)}
    P0.get_tables = lambda: tables
    P2.get_tables = lambda: tables
    pack_w4._GRID = np.asarray(quants.IQ3_XXS.grid, dtype=np.float32).reshape(256, 4)
    return P0, P2, pack_w4, quants


def reference_q4k_port(P0):
    """dq_q4_k_np and its helper from engine/mm/mm_mtp_anchor.py, taken from that
    file as written (the module's own imports need the reference's model tree, so
    only these two definitions are compiled and run)."""
    import ast

    path = os.path.join(REF, "engine", "mm", "mm_mtp_anchor.py")
    tree = ast.parse(open(path).read(), path)
    defs = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in ("_get_scale_min_k4", "dq_q4_k_np")]
    ns = {"np": np, "_f16": P0._f16}
    exec(compile(ast.Module(body=defs, type_ignores=[]), path, "exec"), ns)
    return ns["dq_q4_k_np"]


def reference_q5k_port():
    """dequant_q5k_rows from engine/chain_sim.py (the reference's numpy restatement of
    its Q5_K row dequant), compiled alone as written: the module's own imports need
    the reference's model tree.  It reads whole 5120-weight rows (20 blocks)."""
    import ast

    path = os.path.join(REF, "engine", "chain_sim.py")
    tree = ast.parse(open(path).read(), path)
    defs = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "dequant_q5k_rows"]
    ns = {"np": np, "DIM": 5120, "F32": np.float32, "F16": np.float16}
    exec(compile(ast.Module(body=defs, type_ignores=[]), path, "exec"), ns)
    return ns["dequant_q5k_rows"]


def region_repack_iq3(raw: np.ndarray, k: int) -> np.ndarray:
    """GGUF IQ3_XXS rows -> the reference's row-region layout
    [qs 64*NB][scales 32*NB][d 2*NB] (engine/pack_w1c.py:18-31), the input
    format of pack_w4.dequant_iq3xxs."""
    n = raw.shape[0]
    nb = k // 256
    x = raw.reshape(n, nb, 98)
    out = np.empty((n, 98 * nb), dtype=np.uint8)
    out[:, :64 * nb] = x[:, :, 2:66].reshape(n, 64 * nb)
    out[:, 64 * nb:96 * nb] = x[:, :, 66:98].reshape(n, 32 * nb)
    out[:, 96 * nb:] = x[:, :, 0:2].reshape(n, 2 * nb)
    return out


def main():
    P0, P2, pack_w4, quants = load_reference()
    rng = np.random.default_rng(20261201)
    g = {}

    # Q6_K: config distribution plus full-range int8 sub-scales (real checkpoints)
    q6 = synth.q6k_blocks(rng, 8, 512)
    q6w = q6.copy().reshape(8, 2, 210)
    q6w[4:, :, 192:208] = rng.integers(-128, 128, (4, 2, 16)).astype(np.int8).view(np.uint8)
    q6 = q6w.reshape(8, 420)
    g["q6k_raw"] = q6
    g["q6k_ref"] = P2.dq_q6_k(q6, 512)

    iq4 = synth.iq4xs_blocks(rng, 8, 512)
    g["iq4xs_raw"] = iq4
    g["iq4xs_ref"] = P0.dq_iq4_xs(iq4, 512)

    iq3 = synth.iq3xxs_blocks(rng, 8, 512)
    g["iq3xxs_raw"] = iq3
    g["iq3xxs_ref_f16"] = pack_w4.dequant_iq3xxs(region_repack_iq3(iq3, 512), 512)
    g["iq3xxs_gguf_f32"] = quants.dequantize(iq3, quants.GGMLQuantizationType.IQ3_XXS).reshape(8, 512)

    # MoE expert lanes: gate/up k=2048 IQ4_XS (+silu*u), down k=512 IQ4_XS / Q6_K
    rows_g = synth.iq4xs_blocks(rng, 16, 2048)
    rows_u = synth.iq4xs_blocks(rng, 16, 2048)
    x2048 = rng.standard_normal(2048, dtype=np.float32)
    g["gxup4_rows_g"], g["gxup4_rows_u"], g["gxup4_x"] = rows_g, rows_u, x2048
    g["gxup4_ref"] = P2.gxup4_ref(rows_g, rows_u, x2048)
    rows_d4 = synth.iq4xs_blocks(rng, 32, 512)
    rows_d6 = synth.q6k_blocks(rng, 32, 512)
    act = rng.standard_normal(512, dtype=np.float32)
    g["gxdn_rows4"], g["gxdn_rows6"], g["gxdn_act"] = rows_d4, rows_d6, act
    g["gxdn4_ref"] = P2.gxdn4_ref(rows_d4, act)
    g["gxdn6_ref"] = P2.gxdn6_ref(rows_d6, act)

    # router (inputs regenerated from the seed in tests/golden/inputs.py)
    Wr, wsh, h = router_inputs()
    rt = P2.rt_prod_ref(Wr, wsh, h, range(h.shape[0]))
    g["router_ids"] = np.stack([rt[p][0] for p in range(h.shape[0])]).astype(np.int32)
    g["router_gates"] = np.stack([rt[p][1] for p in range(h.shape[0])]).astype(np.float32)
    g["router_sg"] = np.array([rt[p][2] for p in range(h.shape[0])], dtype=np.float32)
    g["router_logits"] = np.stack([P2.logits_ref(Wr, h, p) for p in range(h.shape[0])])

    gates, sg, part, shared = cmb_inputs()
    g["cmb_ref"] = P2.cmb_ref(gates, sg, part, shared)

    # Q4_K (the v rows of aq3k8v11): the reference's numpy port dq_q4_k_np
    # (engine/mm/mm_mtp_anchor.py:47-80), run as defined there, and gguf-py
    rng4 = np.random.default_rng(20261202)
    q4 = synth.q4k_blocks(rng4, 8, 512)
    g["q4k_raw"] = q4
    g["q4k_ref"] = reference_q4k_port(P0)(q4, 512)
    g["q4k_gguf_f32"] = quants.dequantize(q4, quants.GGMLQuantizationType.Q4_K).reshape(8, 512)

    # Q5_K (the GDN qkv rows of q5g8v11): the reference's dequant_q5k_rows
    # (engine/chain_sim.py:111-150) on whole 5120-weight rows, and gguf-py;
    # Q8_0 (the o-projection rows of k3aonw32_11): dq_q8_0 (engine/mm/MM_P2_ports.py:48-54)
    rng5 = np.random.default_rng(20261203)
    q5 = synth.q5k_blocks(rng5, 3, 5120)
    g["q5k_raw"] = q5
    g["q5k_ref"] = reference_q5k_port()(q5, np.arange(3))
    g["q5k_gguf_f32"] = quants.dequantize(q5, quants.GGMLQuantizationType.Q5_K).reshape(3, 5120)
    q8 = synth.q8_0_blocks(rng5, 8, 512)
    g["q8_0_raw"] = q8
    g["q8_0_ref"] = P2.dq_q8_0(q8, 512)
    g["q8_0_gguf_f32"] = quants.dequantize(q8, quants.GGMLQuantizationType.Q8_0).reshape(8, 512)

    out = os.path.join(HERE, "golden_v1.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out} ({os.path.getsize(out)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
