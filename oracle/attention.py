"""Split-KV int8 attention of the verify step, restated in numpy (oracle; test
infrastructure only).

Shapes of the reference model's full-attention layers: 24 query heads, 4 KV heads
(6 query heads per KV head), head dim 256, rotary on the first 64 dims (32 pairs
(d, d + 32)), KV cache int8 with one fp16 scale per 32 dims.

* ``attn_pre`` follows engine/spk_preqh.cu:13-90: per token t and head, RMS norm
  over 256 dims (eps 1e-6) rounded to fp16, times the norm weight, rotary at
  position pos + t, q scaled by 1/16 and rounded to fp16 (qw16); k the same with
  the k norm weight, rounded to fp16; k and the raw v quantised per 32 dims to int8
  (scale = max|x| / 127 as fp16, or 1e-8 for an all-zero group; stored as q + 128)
  into the cache at position pos + t.
* ``attn_decode`` follows engine/spk_g4hm.cu (scores, causal mask, online softmax
  over split chunks) and engine/skv_split.cu:176-199 (the combine and the sigmoid
  output gate from the second half of each head's q projection row): for token t
  of head h, keys 0 .. pos + t of KV head h / 6, dequantised as fp16(q * scale),
  softmax(qw16 . k) . v times sigmoid(gate), in float64.
"""
from __future__ import annotations

import numpy as np

NQ, NKV, HD, GQ = 24, 4, 256, 6
QROW = 2 * HD * NQ          # 12288: per head 256 q then 256 gate values
KROW = HD * NKV             # 1024
EPS = 1e-6


def rope_freqs() -> np.ndarray:
    """The 32 rotary frequencies the reference uploads (theta 1e7 over 64 dims)."""
    return (1.0 / (1e7 ** (np.arange(0, 64, 2, dtype=np.float64) / 64.0))).astype(np.float32)


def _f16(x):
    return np.asarray(x, dtype=np.float64).astype(np.float16).astype(np.float64)


def _norm_rope(v, w, ang):
    """fp16(v * rsqrt(mean(v^2) + eps)) * w, then rotary on dims 0..63."""
    r = 1.0 / np.sqrt(np.sum(v * v) / HD + EPS)
    x = _f16(v * r) * w.astype(np.float64)
    cs, sn = np.cos(ang), np.sin(ang)
    out = x.copy()
    out[:32] = x[:32] * cs - x[32:64] * sn
    out[32:64] = x[32:64] * cs + x[:32] * sn
    return out


def _quant8(x):
    """Per 32-dim group: scale = fp16(max|x| / 127), or fp16(1e-8) for an all-zero
    group; byte = rint(clamp(x / scale, -127, 127)) + 128 (engine/spk_preqh.cu:77-83).

    fp16(1e-8) is 0 (below the smallest fp16 subnormal), so an all-zero group divides
    0 by 0.  The reference clamps with fmaxf / fminf, which return the non-NaN
    operand: NaN -> fmaxf(NaN, -127) = -127 -> byte 1.  Likewise a non-zero group
    whose scale underflows to 0 gives +-inf -> +-127 for its non-zero entries.
    np.fmax / np.fmin have the same NaN rule."""
    q = np.empty(HD, dtype=np.uint8)
    s = np.empty(HD // 32, dtype=np.float16)
    for gi in range(HD // 32):
        seg = x[gi * 32:(gi + 1) * 32]
        m = np.abs(seg).max()
        sc = np.float16(m / 127.0 if m > 0 else 1e-8)
        s[gi] = sc
        with np.errstate(divide="ignore", invalid="ignore"):
            r = seg / np.float64(sc)
        qi = np.rint(np.fmin(np.fmax(r, -127.0), 127.0)).astype(np.int64)
        q[gi * 32:(gi + 1) * 32] = (qi + 128).astype(np.uint8)
    return q, s


def attn_pre(qrow, krow, vrow, qnw, knw, freqs, pos, kv, sc):
    """qrow [T][12288], krow / vrow [T][1024] fp16; kv uint8 [8][ctx][256] and sc
    fp16 [8][ctx][8] updated in place at positions pos .. pos + T - 1.  Returns qw16
    [T][24][256] fp16."""
    T = qrow.shape[0]
    qw16 = np.empty((T, NQ, HD), dtype=np.float16)
    for t in range(T):
        ang = (np.float32(pos + t) * freqs.astype(np.float32)).astype(np.float64)   # fp32 angle
        for h in range(NQ):
            q = qrow[t, h * 2 * HD:h * 2 * HD + HD].astype(np.float64)
            qw16[t, h] = (_norm_rope(q, qnw, ang) * 0.0625).astype(np.float16)
        for g in range(NKV):
            k = krow[t, g * HD:(g + 1) * HD].astype(np.float64)
            kf = _f16(_norm_rope(k, knw, ang))
            v = vrow[t, g * HD:(g + 1) * HD].astype(np.float64)
            kv[g, pos + t], sc[g, pos + t] = _quant8(kf)
            kv[NKV + g, pos + t], sc[NKV + g, pos + t] = _quant8(v)
    return qw16


def dequant_cache(kv, sc, head, n):
    """Rows 0 .. n-1 of cache head `head` as float64 values fp16((b - 128) * scale)."""
    b = kv[head, :n].astype(np.float64) - 128.0
    s = np.repeat(sc[head, :n].astype(np.float64), 32, axis=1)
    return _f16(b * s)


def attn_decode(qw16, kv, sc, qrow, pos):
    """ao [T][6144] float64: gated causal attention of the T verify rows."""
    T = qw16.shape[0]
    ao = np.zeros((T, NQ * HD), dtype=np.float64)
    n = pos + T
    keys = np.arange(n)
    for g in range(NKV):
        K = dequant_cache(kv, sc, g, n)
        V = dequant_cache(kv, sc, NKV + g, n)
        Q = qw16[:, g * GQ:(g + 1) * GQ].astype(np.float64).reshape(T * GQ, HD)     # row t * GQ + hl
        S = K @ Q.T                                                                   # [n][T * GQ]
        lim = np.repeat(pos + np.arange(T), GQ)                                       # row sees keys <= lim
        S = np.where(keys[:, None] <= lim[None, :], S, -np.inf)
        P = np.exp(S - S.max(axis=0, keepdims=True))
        out = (P.T @ V) / P.sum(axis=0)[:, None]                                      # [T * GQ][HD]
        for t in range(T):
            for hl in range(GQ):
                h = g * GQ + hl
                gate = qrow[t, h * 2 * HD + HD:(h + 1) * 2 * HD].astype(np.float64)
                ao[t, h * HD:(h + 1) * HD] = out[t * GQ + hl] / (1.0 + np.exp(-gate))
    return ao
