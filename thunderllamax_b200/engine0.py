"""Reference-shaped host surface: ``Bufs`` + ``load_progs`` over the CUDA library.

Mirrors the reference's engine0 call surface (engine/engine0.py:65-106): the
host preallocates every buffer once, uploads with ``up``/``win_up``, reads back
with ``down``/``down_at``, and launches named programs with buffer arguments
only, ``prog(*bufs)`` in the reference's argument order.  Shapes are fixed when
the programs are loaded (the reference bakes them into each cubin as
``#define``s); launch geometry is chosen by the library, not by the caller.

Buffers are torch CUDA tensors used purely as device memory.  Weight buffers
hold the B200 tile layout (``pack``) instead of the reference's row-region /
packed7 planes.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops
from ._lib import TLXError


class Bufs:
    """Named device buffers (engine/engine0.py:65-95)."""

    def __init__(self, device="cuda"):
        self.d: dict[str, torch.Tensor] = {}
        self.device = device

    def alloc(self, name, nbytes, dtype=torch.uint8):
        el = torch.empty((), dtype=dtype).element_size()
        self.d[name] = torch.empty(int(nbytes) // el, dtype=dtype, device=self.device)
        return self.d[name]

    def up(self, name, arr):
        t = torch.from_numpy(np.ascontiguousarray(arr)).to(self.device)
        self.d[name] = t
        return t

    def poison(self, name, nbytes, dtype, val):
        """Poison-filled scratch (engine/engine0.py:76-79)."""
        t = self.alloc(name, nbytes, dtype)
        t.fill_(val)
        return t

    def pack(self, name, qtype, gguf_rows, k):
        """Upload GGUF rows and repack them into the tile layout on the device."""
        self.d[name] = ops.pack_tiles(qtype, gguf_rows, k)
        return self.d[name]

    def down(self, name, shape=None, dtype=None):
        t = self.d[name]
        torch.cuda.current_stream().synchronize()
        a = t.cpu().numpy()
        if dtype is not None:
            a = a.view(dtype)
        return a.reshape(shape) if shape is not None else a

    def win_up(self, name, off, arr):
        """Windowed upload into an EXISTING buffer (no reallocation)."""
        a = np.ascontiguousarray(arr)
        dst = self.d[name].view(torch.uint8)[off:off + a.nbytes]
        dst.copy_(torch.from_numpy(a.view(np.uint8).reshape(-1)), non_blocking=False)

    def down_at(self, name, off, n, dtype=np.int32):
        nb = n * np.dtype(dtype).itemsize
        src = self.d[name].view(torch.uint8)[off:off + nb]
        return src.cpu().numpy().view(dtype).copy()


class Prog:
    def __init__(self, name, fn):
        self.name = name
        self.fn = fn

    def __call__(self, *bufs, **_launch):
        # global_size/local_size/wait from the reference call sites are accepted and
        # ignored: the library sizes its own persistent grids.
        return self.fn(*bufs)

    def __repr__(self):
        return f"Prog({self.name})"


def _contig_drafts(drings):
    base = drings[0]
    for i, d in enumerate(drings):
        if d.data_ptr() != base.data_ptr() + 4 * i:
            raise TLXError("dring0..N must be consecutive int32 views of one buffer (Bufs.dring_views)")
    return base.as_strided((len(drings),), (1,))


def dring_views(P: Bufs, k: int = 10):
    """Allocate dring0..dring{k-1} as consecutive 1-int views of one buffer."""
    ring = P.alloc("dring", 4 * k, torch.int32)
    ring.zero_()
    for i in range(k):
        P.d[f"dring{i}"] = ring[i:i + 1]
    return ring


def load_progs(dim=5120, ffn=17408, vocab=151936, rows=11, ffn_q="iq3_xxs", down_q="q6_k", head_q="q6_k"):
    """Programs with the reference kernel names, shapes fixed at load time."""
    ops.require_device()
    ws = {
        "ffn": ops.Workspace.for_shape(ops.MODE_GATE_UP, ffn_q, ffn, dim, rows),
        "down": ops.Workspace.for_shape(ops.MODE_STORE, down_q, dim, ffn, rows, torch.float16),
        "head": ops.Workspace.for_shape(ops.MODE_STORE, head_q, vocab, dim, rows),
        "head_am": ops.Workspace.for_shape(ops.MODE_ARGMAX, head_q, vocab, dim, rows),
    }

    def ffn8v11(wg, wu, gridf, hhx, gact):
        # engine/ffn8v11.cu:88-133: gact = silu(Wg hhx) * (Wu hhx), fp16 out
        del gridf  # the library keeps its own copy of the grid (same table)
        ops.ffn_gate_up(ffn_q, wg, wu, hhx.view(rows, dim), ffn, ws["ffn"], gact=gact.view(rows, ffn))

    def down8nw32_11(wd, gridf, gact, hh, y):
        # engine/down8nw32_11.cu:88-126: y = hh + W gact
        del gridf
        ops.gemv(down_q, wd, gact.view(rows, ffn), dim, ws["down"], y=y.view(rows, dim), residual=hh.view(rows, dim))

    def head8v11(w, xh, logits):
        # engine/head8v11.cu:88-121: logits [rows][vocab] (fp16 or fp32)
        ops.gemv(head_q, w, xh.view(rows, dim), vocab, ws["head"], y=logits.view(rows, vocab))

    def amx3(logits, amds):
        ops.argmax_rows(logits.view(rows, vocab), amds=amds)

    def head_argmax(w, xh, amds):
        # fused head8v11 + amx3 (no logits round trip)
        ops.head_argmax(head_q, w, xh.view(rows, dim), vocab, ws["head_am"], out_idx=amds)

    accept11k = load_progs_small_accept(dim).fn

    def acc36(amds, drafts, mb, eb, K):
        ops.accept(amds, drafts, int(K), mb=mb, eb=eb)

    attn = {}

    def aq3k8v11(wq, wk, wv4, gridf, xh4, qrow4, krow4, vrow4):
        # engine/aq3k8v11.cu:88-179: q 12288 / k 1024 (IQ3_XXS) and v 1024 (Q4_K) rows,
        # fp16 xh4 [rows][dim] -> fp16 [rows][n]
        del gridf
        nq, nk, nv = qrow4.numel() // rows, krow4.numel() // rows, vrow4.numel() // rows
        key = (nq, nk, nv)
        if key not in attn:
            attn[key] = ops.AttnProjections(rows, dim, nq, nk, nv, torch.float16)
        attn[key](wq, wk, wv4, xh4.view(rows, dim), q=qrow4.view(rows, nq), k=krow4.view(rows, nk),
                  v=vrow4.view(rows, nv))

    gdn = {}

    def q5g8v11(wq5, wq3g, gridf, xh4, qkv4, gate4):
        # engine/q5g8v11.cu:68-150: qkv 10240 (Q5_K) and gate 6144 (IQ3_XXS) rows,
        # fp16 xh4 [rows][dim] -> fp16 [rows][n]
        del gridf
        nqkv, ngate = qkv4.numel() // rows, gate4.numel() // rows
        if (nqkv, ngate) not in gdn:
            gdn[(nqkv, ngate)] = ops.GdnProjections(rows, dim, nqkv, ngate, torch.float16)
        gdn[(nqkv, ngate)](wq5, wq3g, xh4.view(rows, dim), qkv=qkv4.view(rows, nqkv), gate=gate4.view(rows, ngate))

    oproj_ws = {}

    def _oproj(qtype, w, z4, attn_out4):
        kz = z4.numel() // rows
        if (qtype, kz) not in oproj_ws:
            oproj_ws[(qtype, kz)] = ops.Workspace.for_shape(ops.MODE_STORE, qtype, dim, kz, rows, torch.float16)
        ops.gemv(qtype, w, z4.view(rows, kz), dim, oproj_ws[(qtype, kz)], y=attn_out4.view(rows, dim))

    def op38nw32_11(wo, gridf, z4, attn_out4):
        # engine/op38nw32_11.cu:88-120: GDN o-projection, IQ3_XXS 5120 x 6144, fp16 in/out
        del gridf
        _oproj("iq3_xxs", wo, z4, attn_out4)

    def k3aonw32_11(wq8, z4, attn_out4):
        # engine/k3aonw32_11.cu:88-116: GDN o-projection, Q8_0 5120 x 6144, fp16 in/out
        _oproj("q8_0", wq8, z4, attn_out4)

    lookups = {}

    def make_lookup(n):
        # engine/lookup{n}_nw32.cu: (tok_hist, pos_slot, cur_slot, dring0..dring{n-2}, l_hist, cyc_slot)
        k = n - 1

        def lookup(tok_hist, pos_slot, cur_slot, *rest):
            del cur_slot  # read but unused by the reference kernels too
            drings, l_hist, cyc_slot = rest[:k], rest[k], rest[k + 1]
            if k not in lookups:
                lookups[k] = ops.Lookup(k)
            lookups[k](tok_hist, pos_slot, cyc_slot, _contig_drafts(list(drings)), l_hist)
        return lookup

    attn = {}   # rows -> the Attention whose workspace spk_a11 filled last

    def _attn(rows, kv):
        ctx = kv.numel() // (8 * 256)
        key = (rows, ctx)
        if attn.get("obj", {}).get(key) is None:
            attn.setdefault("obj", {})[key] = ops.Attention(rows, ctx)
        attn[rows] = attn["obj"][key]
        return attn[rows]

    def spk_pre11(qrow, krow, vrow, qnw, knw, freqs, kv, sc, pos_slot, qw, qw16):
        # engine/spk_preqh.cu:13-90 (the fp32 qw output is not produced; spk_a11 reads qw16)
        del qw
        n = qrow.numel() // 12288
        _attn(n, kv).pre(qrow, krow, vrow, qnw, knw, freqs, pos_slot, kv, sc, qw16)

    def spk_a11(kv, sc, qw16, pos_slot, pm, ps, pA):
        # engine/spk_g4hm.cu: partials go to the library's workspace, not pm / ps / pA
        del pm, ps, pA
        n = qw16.numel() // (24 * 256)
        _attn(n, kv).split(kv, sc, qw16, pos_slot)

    def spk_c11(pm, ps, pA, qrow, ao):
        # engine/skv_split.cu:176-199: combine + sigmoid gate -> ao [rows][6144] fp16
        del pm, ps, pA
        n = qrow.numel() // 12288
        attn[n].combine(qrow, ao.view(n, 6144))

    def acceptsel11k(rec4, conv4, m_slot, *scratch):
        # engine/acceptsel11k.cu:8-40: conv5x..conv11x then rec6x..rec11x, as the reference
        ops.acceptsel11k(rec4, conv4, m_slot, scratch[:7], scratch[7:13])

    def h_argmax(logits, tok_slot, pos_slot, tok_hist):
        # engine/h_argmax.cu:13-42 (T = 1 decode tail)
        ops.h_argmax(logits, tok_slot, pos_slot, tok_hist)

    progs = {"ffn8v11": ffn8v11, "down8nw32_11": down8nw32_11, "head8v11": head8v11, "amx3": amx3,
             "head_argmax": head_argmax, "accept11k": accept11k, "acc36": acc36, "acceptsel11k": acceptsel11k,
             "h_argmax": h_argmax, "aq3k8v11": aq3k8v11, "q5g8v11": q5g8v11, "op38nw32_11": op38nw32_11,
             "k3aonw32_11": k3aonw32_11, "spk_pre11": spk_pre11, "spk_a11": spk_a11, "spk_c11": spk_c11}
    for n in range(5, 12):
        progs[f"lookup{n}_nw32"] = make_lookup(n)
    return {k: Prog(k, v) for k, v in progs.items()}


def run_accept11k(amds, drafts, state, xA, hd_d0, hd_d1, dim):
    """Run accept11k once on host-provided state; returns the new state (test helper)."""
    ops.require_device()
    P = Bufs()
    ring = dring_views(P, 10)
    ring.copy_(torch.from_numpy(np.asarray(drafts, np.int32)))
    P.up("amds", np.asarray(amds, np.int32))
    P.up("xA", np.asarray(xA, np.float32))
    for nm in ("m_slot", "cyc_slot", "pos_slot", "cur_slot"):
        P.up(nm, np.zeros(1, np.int32))
    P.d["pos_slot"].fill_(state["pos"])
    P.d["cyc_slot"].fill_(state["cyc"])
    P.up("m_hist", state["m_hist"].astype(np.int32))
    P.up("l_hist", state["l_hist"].astype(np.int32))
    P.up("tok_hist", state["tok_hist"].astype(np.int32))
    P.alloc("h_seed", 4 * dim, torch.float32)
    P.alloc("dhd_seed", 4 * dim, torch.float32)
    P.up("hd_d0", np.asarray(hd_d0, np.float32))
    P.up("hd_d1", np.asarray(hd_d1, np.float32))
    P.alloc("emit", 4 * 26, torch.int32).zero_()
    d = P.d
    accept11k_prog = load_progs_small_accept(dim)
    accept11k_prog(d["amds"], *[d[f"dring{i}"] for i in range(10)], d["xA"], d["m_slot"], d["m_hist"],
                   d["cyc_slot"], d["pos_slot"], d["cur_slot"], d["tok_hist"], d["h_seed"], d["hd_d0"],
                   d["hd_d1"], d["dhd_seed"], d["emit"], d["l_hist"])
    torch.cuda.synchronize()
    return {"pos": int(d["pos_slot"].item()), "cur": int(d["cur_slot"].item()), "cyc": int(d["cyc_slot"].item()),
            "m_slot": int(d["m_slot"].item()), "tok_hist": d["tok_hist"].cpu().numpy(),
            "m_hist": d["m_hist"].cpu().numpy(), "emit": d["emit"].cpu().numpy(),
            "h_seed": d["h_seed"].cpu().numpy(), "dhd_seed": d["dhd_seed"].cpu().numpy()}


def load_progs_small_accept(dim):
    """Only the accept11k program (no weight-shaped workspaces)."""
    from ._lib import check, lib
    from .ops import _ptr, _stream

    def accept11k(amds, *args):
        drings, rest = args[:10], args[10:]
        (xA, m_slot, m_hist, cyc_slot, pos_slot, cur_slot, tok_hist, h_seed, hd_d0, hd_d1, dhd_seed, emit,
         l_hist) = rest
        drafts = _contig_drafts(drings)
        check(lib().tlx_accept11k(_ptr(amds), _ptr(drafts), _ptr(xA), _ptr(m_slot), _ptr(m_hist), _ptr(cyc_slot),
                                  _ptr(pos_slot), _ptr(cur_slot), _ptr(tok_hist), _ptr(h_seed), _ptr(hd_d0),
                                  _ptr(hd_d1), _ptr(dhd_seed), _ptr(emit), _ptr(l_hist), dim, _stream(amds)),
              "accept11k")

    return Prog("accept11k", accept11k)
