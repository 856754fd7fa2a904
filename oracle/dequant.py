"""ggml block dequantisation, restated in numpy (oracle; test infrastructure).

All six formats dequantise EXACTLY in fp32: every weight is a product of an
fp16 scale with small integers whose significands fit in 24 bits, so the fp32
values below equal the real-number values.  The reference's dense GEMVs round
each weight to fp16 before use (engine/ffn8v11.cu:115-117 ``__float2half``);
that rounding is an artefact of its fp16-product kernels, not of the format, and
is not part of this oracle (the golden fixtures keep the reference's
fp16-rounded port too, and the tests relate the two).
"""
from __future__ import annotations

import numpy as np

from .tables import iq3xxs_grid_bytes, iq4nl_kvalues, ksigns_iq2xs

QK = 256


def _f16(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b).view(np.float16)[..., 0].astype(np.float32)


def dequant_iq3xxs(raw: np.ndarray, k: int) -> np.ndarray:
    """IQ3_XXS rows (GGUF block order d | qs[64] | scales[32]) -> f32 [n, k].

    Per 32-weight group ib: sw = scales word ib, db = d*(0.5 + (sw>>28))*0.5;
    unit l (8 weights) takes sign field (sw >> 7l) & 127 expanded to 8 bits
    with even parity, and two grid entries qs[8ib+2l], qs[8ib+2l+1].
    Follows reference engine/pack_w4.py:39-69 (``dequant_iq3xxs``) and the
    lane math of engine/ffn8v11.cu:103-116, without the final fp16 round.
    """
    n = raw.shape[0]
    nb = k // QK
    blk = np.ascontiguousarray(raw).reshape(n, nb, 98)
    d = _f16(blk[..., 0:2])                                            # [n, nb]
    qs = blk[..., 2:66]                                                # [n, nb, 64]
    sw = np.ascontiguousarray(blk[..., 66:98]).view(np.uint32)         # [n, nb, 8]
    db = d[..., None] * ((sw >> 28).astype(np.float32) + np.float32(0.5)) * np.float32(0.5)
    fields = (sw[..., None] >> (np.arange(4, dtype=np.uint32) * 7)) & 0x7F   # [n, nb, 8, 4]
    s8 = ksigns_iq2xs()[fields]                                        # [n, nb, 8, 4]
    bits = (s8[..., None] >> np.arange(8, dtype=np.uint8)) & 1          # [n, nb, 8, 4, 8]
    sign = np.where(bits != 0, np.float32(-1.0), np.float32(1.0))
    g = iq3xxs_grid_bytes()[qs].astype(np.float32).reshape(n, nb, 8, 4, 8)
    w = (db[..., None, None] * g) * sign
    return w.reshape(n, k).astype(np.float32)


def dequant_q6k(raw: np.ndarray, k: int) -> np.ndarray:
    """Q6_K rows (ql[128] | qh[64] | sc[16] int8 | d f16) -> f32 [n, k].

    Weight i = 128h + 32j + l (h half, j quarter, l 0..31):
    q = ((ql[64h + 32(j&1) + l] >> 4(j>>1)) & 15) | (((qh[32h + l] >> 2j) & 3) << 4),
    w = (d * sc[i >> 4]) * (q - 32).  Reference engine/mm/MM_P2_ports.py:21-45
    (``dq_q6_k``) and engine/mm/MM_P6_h6kam.cu:45-56.  The index arithmetic is
    done by reshapes: ql viewed as [h][j & 1][l] shifted by 4(j >> 1) gives the low
    nibbles in weight order [h][j >> 1][j & 1][l] = [h][j][l]; qh viewed as [h][l]
    shifted by 2j gives the high bits in [h][j][l].
    """
    n = raw.shape[0]
    nb = k // QK
    blk = np.ascontiguousarray(raw).reshape(n, nb, 210)
    ql = blk[..., 0:128].reshape(n, nb, 2, 1, 2, 32)
    qh = blk[..., 128:192].reshape(n, nb, 2, 1, 32)
    lo = (ql >> np.array([0, 4], np.uint8).reshape(2, 1, 1)) & 15                # [n, nb, h, j>>1, j&1, l]
    hi = (qh >> np.array([0, 2, 4, 6], np.uint8).reshape(4, 1)) & 3              # [n, nb, h, j, l]
    q = (lo.reshape(n, nb, QK) | (hi.reshape(n, nb, QK) << 4)).view(np.int8) - np.int8(32)
    sc = blk[..., 192:208].view(np.int8).astype(np.float32)
    d = _f16(blk[..., 208:210])
    t = d[..., None] * sc                                              # [n, nb, 16] (d*sc first)
    w = t[..., None] * q.reshape(n, nb, 16, 16).astype(np.float32)
    return w.reshape(n, k)


def dequant_iq4xs(raw: np.ndarray, k: int) -> np.ndarray:
    """IQ4_XS rows (d f16 | scales_h u16 | scales_l[4] | qs[128]) -> f32 [n, k].

    Group ib (32 weights): ls = ((scales_l[ib>>1] >> 4(ib&1)) & 15) | (((scales_h >> 2ib) & 3) << 4),
    dl = d * (ls - 32); element e < 16 is the low nibble of qs[16ib + e], e >= 16
    the high nibble of qs[16ib + e - 16]; w = dl * kvalues[nibble].
    Reference engine/mm/MM_P0_d2_repack.py:78-93 (``dq_iq4_xs``).
    """
    n = raw.shape[0]
    nb = k // QK
    blk = np.ascontiguousarray(raw).reshape(n, nb, 136)
    d = _f16(blk[..., 0:2])
    sh = np.ascontiguousarray(blk[..., 2:4]).view(np.uint16)[..., 0].astype(np.int32)
    sl = blk[..., 4:8].astype(np.int32)
    qs = blk[..., 8:136].reshape(n, nb, 8, 16).astype(np.int32)
    ib = np.arange(8)
    ls = ((sl[..., ib >> 1] >> (4 * (ib & 1))) & 15) | (((sh[..., None] >> (2 * ib)) & 3) << 4)
    dl = d[..., None] * (ls - 32).astype(np.float32)                   # [n, nb, 8]
    nib = np.concatenate([qs & 15, qs >> 4], axis=-1)                  # [n, nb, 8, 32]
    w = dl[..., None] * iq4nl_kvalues()[nib]
    return w.reshape(n, k).astype(np.float32)


def _scale_min_k4(sc: np.ndarray):
    """The 12 packed scale bytes of a K-quant block -> (scale, min) uint8 [..., 8]:
    sub-blocks 0..3 take the low 6 bits of bytes j / j+4; 4..7 join a nibble of
    byte j+4 with the top 2 bits of byte j-4 / j (ggml get_scale_min_k4)."""
    s = np.empty(sc.shape[:-1] + (8,), dtype=np.uint8)
    m = np.empty_like(s)
    s[..., :4] = sc[..., 0:4] & 63
    m[..., :4] = sc[..., 4:8] & 63
    s[..., 4:] = (sc[..., 8:12] & 0xF) | ((sc[..., 0:4] >> 6) << 4)
    m[..., 4:] = (sc[..., 8:12] >> 4) | ((sc[..., 4:8] >> 6) << 4)
    return s, m


def dequant_q4k(raw: np.ndarray, k: int) -> np.ndarray:
    """Q4_K rows (d f16 | dmin f16 | scales[12] | qs[128]) -> f32 [n, k].

    Sub-block s (32 weights): w = (d * sc_s) * q - dmin * mn_s, q the low nibbles of
    qs[32j .. 32j+32) for s = 2j and the high nibbles for s = 2j+1.  Follows the
    v-row branch of engine/aq3k8v11.cu:156-172 and the reference's numpy port
    engine/mm/mm_mtp_anchor.py:47-80 (dq_q4_k_np), including its fp32 evaluation
    order (one rounding, in the subtraction)."""
    n = raw.shape[0]
    nb = k // QK
    blk = np.ascontiguousarray(raw).reshape(n, nb, 144)
    d = _f16(blk[..., 0:2])                                      # [n, nb]
    dmin = _f16(blk[..., 2:4])
    sc, mn = _scale_min_k4(blk[..., 4:16])                        # [n, nb, 8]
    qs = blk[..., 16:144].reshape(n, nb, 4, 32)
    q = np.stack([qs & 0xF, qs >> 4], axis=3).reshape(n, nb, 8, 32).astype(np.float32)
    d1 = d[..., None] * sc.astype(np.float32)                     # exact in fp32
    m1 = dmin[..., None] * mn.astype(np.float32)                  # exact in fp32
    w = d1[..., None] * q - m1[..., None]
    return w.reshape(n, k).astype(np.float32)


def dequant_q5k(raw: np.ndarray, k: int) -> np.ndarray:
    """Q5_K rows (d f16 | dmin f16 | scales[12] | qh[32] | qs[128]) -> f32 [n, k].

    Sub-block s (32 weights, element e): q = nibble + 16 * bit s of qh[e], the nibble
    being the low one of qs[32j + e] for s = 2j and the high one for s = 2j+1;
    w = (d * sc_s) * q - dmin * mn_s.  Follows the qkv branch of
    engine/q5g8v11.cu:76-93 and the reference's numpy restatement
    engine/chain_sim.py:111-150 (dequant_q5k_rows), in its fp32 evaluation order."""
    n = raw.shape[0]
    nb = k // QK
    blk = np.ascontiguousarray(raw).reshape(n, nb, 176)
    d = _f16(blk[..., 0:2])
    dmin = _f16(blk[..., 2:4])
    sc, mn = _scale_min_k4(blk[..., 4:16])                        # [n, nb, 8]
    qh = blk[..., 16:48]                                          # [n, nb, 32]
    qs = blk[..., 48:176].reshape(n, nb, 4, 32)
    nib = np.stack([qs & 0xF, qs >> 4], axis=3).reshape(n, nb, 8, 32).astype(np.int32)
    hbit = (qh[:, :, None, :] >> np.arange(8, dtype=np.uint8)[None, None, :, None]) & 1   # [n, nb, 8, 32]
    q = (nib + 16 * hbit.astype(np.int32)).astype(np.float32)
    d1 = d[..., None] * sc.astype(np.float32)
    m1 = dmin[..., None] * mn.astype(np.float32)
    w = d1[..., None] * q - m1[..., None]
    return w.reshape(n, k).astype(np.float32)


def dequant_q8_0(raw: np.ndarray, k: int) -> np.ndarray:
    """Q8_0 rows (blocks of 32: d f16 | qs[32] int8) -> f32 [n, k]: w = d * q (exact
    in fp32).  Follows engine/mm/MM_P2_ports.py:48-54 (dq_q8_0).  The reference's
    GPU o-projection then rounds each weight to fp16 (engine/k3aonw32_11.cu:100-101);
    that rounding belongs to the kernel's numerics, not to the format."""
    n = raw.shape[0]
    nb = k // 32
    blk = np.ascontiguousarray(raw).reshape(n, nb, 34)
    d = _f16(blk[..., 0:2])
    q = blk[..., 2:34].view(np.int8).astype(np.float32)
    return (d[..., None] * q).reshape(n, k).astype(np.float32)


_DQ = {"iq3_xxs": dequant_iq3xxs, "q6_k": dequant_q6k, "iq4_xs": dequant_iq4xs, "q4_k": dequant_q4k,
       "q5_k": dequant_q5k, "q8_0": dequant_q8_0}


def dequant(qtype: str, raw: np.ndarray, k: int, chunk_rows: int = 8192) -> np.ndarray:
    """Dequantise in row chunks (bounded temporary memory)."""
    n = raw.shape[0]
    out = np.empty((n, k), dtype=np.float32)
    for r0 in range(0, n, chunk_rows):
        out[r0:r0 + chunk_rows] = _DQ[qtype](raw[r0:r0 + chunk_rows], k)
    return out
