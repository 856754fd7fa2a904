"""The verify path above the dequantiser, restated in numpy (oracle).

float64 arithmetic on the exact fp32 dequantised weights and the exact
(bf16/fp32) activations: this is the "true" value that the GPU's fp32
accumulation is compared against (tolerance max|err| <= 2e-3 * ||row||_2 for
outputs, bit-exact for argmax ids and accept results).
"""
from __future__ import annotations

import numpy as np

from .dequant import dequant, dequant_iq4xs


def matvec_f64(W: np.ndarray, X: np.ndarray) -> np.ndarray:
    """Y[t, r] = sum_k W[r, k] X[t, k] in float64.  The K-row matvec of the
    reference's dense GEMVs (engine/ffn8v11.cu:88-133: one weight read for all
    rows) and its numpy check ``W.astype(f32) @ x`` (lineage/a3a/a3a_bench.py:176)."""
    return np.asarray(X, dtype=np.float64) @ np.asarray(W, dtype=np.float64).T


def silu_f64(g: np.ndarray) -> np.ndarray:
    """silu(g) = g / (1 + exp(-g)) (engine/ffn8v11.cu:22-24; MM_P2_ports.py:187-188)."""
    g = np.asarray(g, dtype=np.float64)
    with np.errstate(over="ignore"):
        return g / (1.0 + np.exp(-g))


def ffn_f64(X, gate_raw, up_raw, down_raw, gate_q="iq3_xxs", up_q="iq3_xxs", down_q="q6_k",
            residual=None):
    """gact = silu(X Wg^T) * (X Wu^T); y = residual + gact Wd^T.
    Reference call chain engine/mtp.py:1127-1128 (ffn8v11r7 -> down8nw32v11r7),
    semantics engine/ffn8v11.cu:127-132 and engine/down8nw32_11.cu:120-125."""
    X = np.asarray(X, dtype=np.float64)
    k = X.shape[1]
    n = gate_raw.shape[0]
    g = matvec_f64(dequant(gate_q, gate_raw, k), X)
    u = matvec_f64(dequant(up_q, up_raw, k), X)
    gact = silu_f64(g) * u
    y = matvec_f64(dequant(down_q, down_raw, n), gact)
    if residual is not None:
        y = y + np.asarray(residual, dtype=np.float64)
    return gact, y


def head_logits_f64(X, w_raw, qtype="q6_k", chunk_rows=16384):
    """logits[t, v] for the full vocabulary, dequantising in row chunks."""
    X = np.asarray(X, dtype=np.float64)
    k = X.shape[1]
    V = w_raw.shape[0]
    out = np.empty((X.shape[0], V), dtype=np.float64)
    for r0 in range(0, V, chunk_rows):
        W = dequant(qtype, w_raw[r0:r0 + chunk_rows], k)
        out[:, r0:r0 + W.shape[0]] = matvec_f64(W, X)
    return out


def argmax_rows(logits: np.ndarray):
    """Per-row (max, index) of the reference scan: best starts at -1e30 and only a
    strictly greater value (or an equal one at a lower index) replaces it, so the
    LOWEST index wins ties and NaN, -inf and values <= -1e30 never win; a row with
    no candidate yields index 0 (engine/amx3.cu:124-139, engine/h_argmax.cu:20-33;
    the fused head's packed key gives the same lowest-row tie-break,
    engine/mm/MM_P6_h6kam.cu:76-80)."""
    L = np.asarray(logits, dtype=np.float64)
    with np.errstate(invalid="ignore"):
        cand = L > -1e30
    clean = np.where(cand, L, -np.inf)
    idx = np.argmax(clean, axis=1).astype(np.int32)
    mx = L[np.arange(L.shape[0]), idx]
    return mx, idx


def lookup_ngram(tok_hist, pos: int, n_drafts: int, scan_end: int):
    """n-gram draft proposal of engine/lookup11_nw32.cu:17-58 (and its K = 4..9
    siblings, which differ only in K and scan_end).

    Suffix s = hist[pos-8 .. pos-1]; every start i in [0, pos - scan_end] scores
    l = the length of the common prefix of hist[i .. i+7] and s (the nested ifs of
    lines 28-35); the winner is the largest (l, i) (the key (l << 20) | i, line 36,
    maximised over the CTA, lines 38-41).  Returns (l_hist value, drafts): l_hist =
    1000000 + pos when pos < scan_end, else l + 1 (line 45); drafts = hist[i+8 ..
    i+8+K-1] when l >= 8 (lines 46-57), else None (the ring is left unchanged)."""
    h = np.asarray(tok_hist, dtype=np.int64)
    if pos < scan_end:
        return 1000000 + pos, None
    s = h[pos - 8:pos]
    iend = pos - scan_end
    starts = np.arange(iend + 1)
    # l = number of leading positions j with hist[i+j] == s[j]
    eq = np.stack([h[starts + j] == s[j] for j in range(8)], axis=1)      # [n, 8]
    l = np.where(eq.all(axis=1), 8, np.argmin(eq, axis=1))
    best_l = int(l.max())
    if best_l == 0:
        return 1, None
    i = int(starts[l == best_l].max())
    drafts = h[i + 8:i + 8 + n_drafts].astype(np.int32) if best_l >= 8 else None
    return best_l + 1, drafts


def acceptsel11k(rec4, conv4, m, conv_x, rec_x):
    """acceptsel11k (engine/acceptsel11k.cu:8-40): slot m of the GDN state becomes the
    live slot 4.  rec4 [B][5][R], conv4 [B][5][C]; rec from rec4[:, m] for m <= 4,
    else rec_x[m - 5] (rec6x .. rec11x); conv from conv4[:, m] for m <= 3, else
    conv_x[m - 4] (conv5x .. conv11x).  Returns the new (rec4, conv4)."""
    rec4 = np.array(rec4, copy=True)
    conv4 = np.array(conv4, copy=True)
    if not 0 <= m <= 10:
        return rec4, conv4
    rec4[:, 4] = rec4[:, m] if m <= 4 else np.asarray(rec_x[m - 5])
    conv4[:, 4] = conv4[:, m] if m <= 3 else np.asarray(conv_x[m - 4])
    return rec4, conv4


def h_argmax(logits_row, tok_hist, pos):
    """h_argmax (T = 1) with its side effects (engine/h_argmax.cu:13-42): the
    argmax of one row of logits (argmax_rows rules), then tok_slot = idx,
    tok_hist[pos] = idx, pos + 1.  Returns (idx, tok_hist', pos')."""
    idx = int(argmax_rows(np.asarray(logits_row)[None, :])[1][0])
    hist = np.array(tok_hist, dtype=np.int32, copy=True)
    hist[pos] = idx
    return idx, hist, pos + 1


def head_argmax(X, w_raw, qtype="q6_k", row_offset=0):
    lg = head_logits_f64(X, w_raw, qtype)
    mx, idx = argmax_rows(lg)
    return mx, idx + np.int32(row_offset), lg


def min_top2_gap(logits: np.ndarray) -> np.ndarray:
    """Per row: top-1 minus top-2 logit (the margin an fp32 GPU sum must not
    cross for the argmax to stay bit-exact)."""
    part = np.partition(np.asarray(logits, dtype=np.float64), -2, axis=1)
    return part[:, -1] - part[:, -2]


def accept(amds, drafts, k=None):
    """Greedy acceptance: m = length of the longest prefix with
    amds[s] == drafts[s] (s < K), bonus = amds[m].
    Reference engine/mm/MM_P7_acc36.cu:18-24 (acc36) and the unrolled ladder of
    engine/accept11k.cu:25-36."""
    amds = np.asarray(amds).astype(np.int64)
    drafts = np.asarray(drafts).astype(np.int64)
    K = len(drafts) if k is None else int(k)
    m = 0
    while m < K and amds[m] == drafts[m]:
        m += 1
    return m, int(amds[m])


def accept11k(amds, drafts, state, xA=None, hd_d0=None, hd_d1=None, dim=5120):
    """accept11k with its commit side effects (engine/accept11k.cu:11-58).

    ``state`` is a dict with int scalars ``pos``, ``cyc``, ``cur``, ``m_slot`` and
    arrays ``tok_hist``, ``m_hist``, ``l_hist``; returns (new_state, emit[22],
    h_seed, dhd_seed)."""
    m, bonus = accept(amds, drafts, 10)
    st = {kk: (v.copy() if isinstance(v, np.ndarray) else v) for kk, v in state.items()}
    pos = st["pos"]
    st["tok_hist"][pos:pos + m + 1] = np.asarray(amds[:m + 1], dtype=np.int32)
    st["cur"] = bonus
    st["pos"] = pos + m + 1
    st["m_slot"] = m
    cyc = st["cyc"]
    st["m_hist"][cyc] = m
    emit = np.zeros(22, dtype=np.int32)
    emit[0] = pos + m + 1
    emit[1] = m
    emit[2:13] = np.asarray(amds[:11], dtype=np.int32)
    emit[13] = 0
    emit[14] = cyc
    emit[15] = st["l_hist"][cyc]
    st["cyc"] = cyc + 1
    h_seed = None if xA is None else np.asarray(xA, np.float32).reshape(-1)[m * dim:(m + 1) * dim].copy()
    dhd_seed = None
    if hd_d0 is not None:
        dhd_seed = np.asarray(hd_d0 if m == 0 else hd_d1, np.float32).copy()
    return st, emit, h_seed, dhd_seed


def router_top8(Wr, wsh, h):
    """MoE router per position: logits = Wr h (f64), top-8 by 8 masked-argmax
    passes (strict '>', ties to the lower expert id), gates = softmax over the
    selected 8 (exp(l - max)/sum), sg = sigmoid(wsh . h).
    Reference engine/mm/MM_P1_rt8e256.cu:38-61 and its numpy twin
    engine/mm/MM_P2_ports.py:273-292 (``rt_prod_ref``).
    Returns (ids int32[P,8], gates f64[P,8], sg f64[P], logits f64[P,E])."""
    h = np.asarray(h, dtype=np.float64)
    lg = h @ np.asarray(Wr, dtype=np.float64).T
    P, E = lg.shape
    ids = np.empty((P, 8), dtype=np.int32)
    gates = np.empty((P, 8), dtype=np.float64)
    for p in range(P):
        l = lg[p].copy()
        mx = l.max()
        ex = []
        for r in range(8):
            be = int(np.argmax(l))
            ids[p, r] = be
            ex.append(np.exp(l[be] - mx))
            l[be] = -np.inf
        ex = np.asarray(ex)
        gates[p] = ex / ex.sum()
    sg = 1.0 / (1.0 + np.exp(-(h @ np.asarray(wsh, dtype=np.float64))))
    return ids, gates, sg, lg


def moe_verify_f64(h, Wr, wsh, experts_gate, experts_up, experts_down,
                   shared_gate, shared_up, shared_down, hres=None):
    """One MoE layer of the verify step for P positions.

    experts_*: uint8 IQ4_XS rows, [E][rows][row_bytes]; gate/up are 512 x 2048,
    down 2048 x 512.  y = hres + sum_r gates[r] * down_e(silu(g_e) u_e) + sg * shared.
    Reference chain engine/mm/MM_P7_lib.py:505-511 (rt8e256 -> shexp8 ->
    gx8e256up4 -> gx8e256dn -> cmbz2048); combine order r ascending then the
    shared expert then the residual (engine/mm/MM_P34_cmbz2048.cu:20-27)."""
    h = np.asarray(h, dtype=np.float64)
    P, H = h.shape
    ids, gates, sg, lg = router_top8(Wr, wsh, h)
    inner = experts_gate.shape[1]
    cache = {}

    def expert(key, gr, ur, dr):
        # dequantised once per expert; keyed by expert id ("shared" for the shared one)
        if key not in cache:
            cache[key] = (dequant_iq4xs(gr, H), dequant_iq4xs(ur, H), dequant_iq4xs(dr, inner))
        return cache[key]

    y = np.zeros((P, H), dtype=np.float64)
    parts = np.zeros((P, 8, H), dtype=np.float64)
    for p in range(P):
        for r in range(8):
            e = int(ids[p, r])
            Wg, Wu, Wd = expert(e, experts_gate[e], experts_up[e], experts_down[e])
            act = silu_f64(Wg.astype(np.float64) @ h[p]) * (Wu.astype(np.float64) @ h[p])
            parts[p, r] = Wd.astype(np.float64) @ act
    Sg, Su, Sd = expert("shared", shared_gate, shared_up, shared_down)
    shared = np.zeros((P, H), dtype=np.float64)
    for p in range(P):
        act = silu_f64(Sg.astype(np.float64) @ h[p]) * (Su.astype(np.float64) @ h[p])
        shared[p] = Sd.astype(np.float64) @ act
    for p in range(P):
        acc = np.zeros(H, dtype=np.float64)
        for r in range(8):
            acc += gates[p, r] * parts[p, r]
        acc += sg[p] * shared[p]
        y[p] = acc if hres is None else np.asarray(hres[p], np.float64) + acc
    return {"ids": ids, "gates": gates, "sg": sg, "logits": lg, "parts": parts,
            "shared": shared, "y": y}
