"""The W4A8 prefill tier, restated in numpy (oracle; test infrastructure).

The reference's int8-activation FFN replaces the fp16 gate/up GEMM of a prefill
chunk with two launches (engine/pf_prefill.py:1155-1158):

  p8q8x     fp16 tokens -> int8 per (token, 128-k chunk) with an fp32 absmax
            scale and the chunk's integer sum (engine/pfk_q8.cu:24-59);
  p8w4ffn7  gate and up on the IQ3_XXS weights read through a LINEARISED
            codebook: each grid magnitude g becomes the 4-bit level
            clip(rint(g / 4.0507), 0, 15), the 32-weight group scale gains the
            factor 4.0507, and the GEMM multiplies int8 tokens by signed levels
            (engine/p8_w4ffn7.cu:4-12, 83-116, 118-160); epilogue silu(g) * u.

The functions below restate that arithmetic: the quantiser bit for bit, the
weights exactly as the reference's own numpy model builds them
(engine/p8_w4ffn7_test.py:62-88 ``dq_lin``: float32 scale products), and the
GEMM in float64 on the dequantised int8 tokens (p8_w4ffn7_test.py:89-91).
"""
from __future__ import annotations

import numpy as np

from .dequant import QK, _f16
from .path import matvec_f64, silu_f64
from .tables import iq3xxs_grid_bytes, ksigns_iq2xs

LDELTA = 4.0507   # the codebook step (engine/p8_w4ffn7.cu:42 LDELTA, engine/pf_prefill.py:994)
KCH = 128         # tokens are quantised per 128-k chunk (engine/pfk_q8.cu:15 NCH = KDIM / 128)


def lut8_levels() -> np.ndarray:
    """int8[1024]: level of grid entry i, magnitude j at [4 i + j]
    (engine/pf_prefill.py:994; the kernel's lut8 argument, p8_w4ffn7.cu:11)."""
    g = iq3xxs_grid_bytes().astype(np.float32).reshape(-1)
    return np.clip(np.rint(g / LDELTA), 0, 15).astype(np.int8)


def act_quant_q8(x: np.ndarray):
    """fp16 x[m, k] (k % 128 == 0) -> (xq int8[m, k], sx f32[m, k/128], rs int32[m, k/128]).

    Per chunk: am = max|x|, s = max(am, 1e-6) * (1/127) in fp32,
    q = clamp(rint(x / s), -127, 127) (IEEE division, ties to even), rs = sum of
    the stored q (engine/pfk_q8.cu:40-58; the reference's numpy check of the
    kernel, engine/p8_w4_test.py:59-70)."""
    x = np.asarray(x, dtype=np.float16)
    m, k = x.shape
    assert k % KCH == 0, k
    seg = x.astype(np.float32).reshape(m, k // KCH, KCH)
    am = np.maximum(np.abs(seg).max(axis=2), np.float32(1e-6))
    s = (am * np.float32(1.0 / 127.0)).astype(np.float32)
    with np.errstate(invalid="ignore"):
        q = np.clip(np.rint(seg / s[..., None]), -127, 127).astype(np.int8)
    rs = q.astype(np.int32).sum(axis=2).astype(np.int32)
    return q.reshape(m, k), s, rs


def dequant_iq3xxs_lin(raw: np.ndarray, k: int, lut8: np.ndarray = None) -> np.ndarray:
    """IQ3_XXS rows (GGUF block order d | qs[64] | scales[32]) on the linearised
    codebook -> f32 [n, k].

    Group ib of a block: sdb = ((d * ((sw >> 28) + 0.5)) * 0.5) * 4.0507 in fp32;
    weight = sdb * (level * sign), the sign field and its parity bit as in
    IQ3_XXS (engine/p8_w4ffn7_test.py:69-86 ``dq_lin``; the kernel's
    engine/p8_w4ffn7.cu:86-88 ``dbd`` and :94-113)."""
    lut = lut8_levels() if lut8 is None else np.asarray(lut8, dtype=np.int8)
    n = raw.shape[0]
    nb = k // QK
    blk = np.ascontiguousarray(raw).reshape(n, nb, 98)
    d = _f16(blk[..., 0:2])                                            # [n, nb]
    qs = blk[..., 2:66]                                                # [n, nb, 64]
    sw = np.ascontiguousarray(blk[..., 66:98]).view(np.uint32)         # [n, nb, 8]
    sdb = ((d[..., None] * ((sw >> 28).astype(np.float32) + np.float32(0.5))) * np.float32(0.5)) \
        * np.float32(LDELTA)                                           # [n, nb, 8]
    fields = (sw[..., None] >> (np.arange(4, dtype=np.uint32) * 7)) & 0x7F   # [n, nb, 8, 4]
    s8 = ksigns_iq2xs()[fields]
    bits = (s8[..., None] >> np.arange(8, dtype=np.uint8)) & 1          # [n, nb, 8, 4, 8]
    sign = np.where(bits != 0, np.float32(-1.0), np.float32(1.0))
    lv = lut.reshape(256, 4)[qs].astype(np.float32).reshape(n, nb, 8, 4, 8)
    w = sdb[..., None, None] * (lv * sign)
    return w.reshape(n, k).astype(np.float32)


def dequant_tokens(xq: np.ndarray, sx: np.ndarray) -> np.ndarray:
    """xdeq[t, k] = xq[t, k] * sx[t, k // 128] in float64 (p8_w4ffn7_test.py:89)."""
    k = xq.shape[1]
    return xq.astype(np.float64) * np.asarray(sx, dtype=np.float64)[:, np.arange(k) // KCH]


def w4a8_gate_up_f64(xq, sx, gate_raw, up_raw, lut8=None, rows=None, chunk_rows=4096):
    """act[t, r] = silu(g) * u with g = xdeq Wg^T, u = xdeq Wu^T in float64 on the
    linearised weights (p8_w4ffn7_test.py:89-91; the kernel's silu(g) * u epilogue,
    p8_w4ffn7.cu:229-255).  rows: optional weight-row indices (a sample)."""
    k = xq.shape[1]
    X = dequant_tokens(xq, sx)
    if rows is not None:
        gate_raw, up_raw = gate_raw[rows], up_raw[rows]
    n = gate_raw.shape[0]
    act = np.empty((X.shape[0], n), dtype=np.float64)
    for r0 in range(0, n, chunk_rows):
        g = matvec_f64(dequant_iq3xxs_lin(gate_raw[r0:r0 + chunk_rows], k, lut8), X)
        u = matvec_f64(dequant_iq3xxs_lin(up_raw[r0:r0 + chunk_rows], k, lut8), X)
        act[:, r0:r0 + g.shape[1]] = silu_f64(g) * u
    return act
