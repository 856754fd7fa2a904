"""Torch-buffer front end of the CUDA library.

Torch tensors are used only as device buffers: every call passes raw pointers
to the C ABI (``_lib``) on the tensor's current stream.  Nothing here computes
on the CPU or falls back to torch kernels.
"""
from __future__ import annotations

import contextlib
import ctypes
import functools

import numpy as np
import torch

from . import _lib
from ._lib import (MODE_ARGMAX, MODE_GATE_UP, MODE_STORE, QTYPES, TLX_DT_BF16, TLX_DT_F16, TLX_DT_F32,
                   TLX_DT_IMAGE, TLXError, check)

_DT = {torch.float32: TLX_DT_F32, torch.float16: TLX_DT_F16, torch.bfloat16: TLX_DT_BF16}


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t=None):
    dev = t.device if t is not None else torch.device("cuda")
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def require_device():
    if not torch.cuda.is_available():
        raise TLXError("no CUDA device: the verify path has no CPU implementation")
    check(_lib.lib().tlx_device_check(), "device check (needs an sm_100 B200)")


def qtype_id(q) -> int:
    return QTYPES[q] if isinstance(q, str) else int(q)


@functools.lru_cache(maxsize=None)
def _grid_numpy():
    from .tables import iq3xxs_grid_u32

    return iq3xxs_grid_u32()


@functools.lru_cache(maxsize=None)
def grid(device: str = "cuda") -> torch.Tensor:
    """The IQ3_XXS grid (256 u32, from gguf-py) resident on the device
    (the reference's ``gridf`` buffer, engine/engine0.py:108-112)."""
    return torch.from_numpy(_grid_numpy().view(np.int32).copy()).to(device)


def tiled_bytes(qtype, n_rows: int, k: int) -> int:
    return int(_lib.lib().tlx_tiled_bytes(qtype_id(qtype), n_rows, k))


def pack_tiles_host(qtype, rows: np.ndarray, k: int) -> np.ndarray:
    """GGUF rows (uint8 [n, row_bytes]) -> tile layout (uint8, host)."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    n = rows.shape[0]
    out = np.empty(tiled_bytes(qtype, n, k), dtype=np.uint8)
    check(_lib.lib().tlx_pack_tiles(qtype_id(qtype), rows.ctypes.data, n, k, rows.shape[1], out.ctypes.data),
          "pack_tiles")
    return out


def unpack_tiles_host(qtype, tiled: np.ndarray, n_rows: int, k: int, row_bytes: int) -> np.ndarray:
    out = np.zeros((n_rows, row_bytes), dtype=np.uint8)
    tiled = np.ascontiguousarray(tiled, dtype=np.uint8)
    check(_lib.lib().tlx_unpack_tiles(qtype_id(qtype), tiled.ctypes.data, n_rows, k, out.ctypes.data), "unpack")
    return out


def pack_tiles(qtype, rows, k: int) -> torch.Tensor:
    """GGUF rows (numpy or CUDA uint8 [n, row_bytes]) -> tiled device buffer."""
    require_device()
    if isinstance(rows, np.ndarray):
        rows = torch.from_numpy(np.ascontiguousarray(rows, dtype=np.uint8)).cuda()
    rows = rows.contiguous()
    n = rows.shape[0]
    out = torch.empty(tiled_bytes(qtype, n, k), dtype=torch.uint8, device=rows.device)
    check(_lib.lib().tlx_pack_tiles_device(qtype_id(qtype), _ptr(rows), n, k, rows.stride(0), _ptr(out),
                                           _stream(rows)), "pack_tiles_device")
    return out


class Workspace:
    """Caller-owned scratch (split-tile partials, counters, argmax partials).
    Zeroed once; kernels leave it zeroed after each launch."""

    def __init__(self, nbytes: int, device="cuda"):
        self.nbytes = max(int(nbytes), 256)
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        check(_lib.lib().tlx_workspace_init(_ptr(self.buf), self.nbytes, _stream(self.buf)), "workspace_init")

    @classmethod
    def for_shape(cls, mode: int, qtype, n_rows: int, k: int, m: int, x_dtype=torch.bfloat16, device="cuda"):
        dt = TLX_DT_IMAGE if x_dtype == "image" else _DT[x_dtype]
        nb = _lib.lib().tlx_gemv_workspace_bytes(mode, qtype_id(qtype), n_rows, k, m, dt)
        if nb == 0:
            raise TLXError(f"unsupported shape for workspace: mode={mode} {qtype} n={n_rows} k={k} m={m}")
        return cls(nb, device)

    def error(self) -> int:
        v = ctypes.c_uint32(0)
        check(_lib.lib().tlx_workspace_error(_ptr(self.buf), ctypes.byref(v)), "workspace_error")
        return int(v.value)

    def reset(self):
        check(_lib.lib().tlx_workspace_init(_ptr(self.buf), self.nbytes, _stream(self.buf)), "workspace_init")


def plan(mode: int, qtype, n_rows: int, k: int, m: int, x_dtype=torch.bfloat16) -> dict:
    info = (ctypes.c_int32 * 12)()
    dt = TLX_DT_IMAGE if x_dtype == "image" else _DT[x_dtype]
    check(_lib.lib().tlx_gemv_plan(mode, qtype_id(qtype), n_rows, k, m, dt, info, 12), "plan")
    keys = ["tiles", "blocks", "segments", "blocks_per_segment", "ctas", "ctas_per_segment", "max_pieces",
            "columns", "ntiles", "warps_per_cta", "stages", "smem"]
    return dict(zip(keys, list(info)))


def set_max_ctas(n: int) -> None:
    _lib.lib().tlx_set_max_ctas(int(n))


@contextlib.contextmanager
def cta_budget(n: int):
    """GEMV launches and workspace sizes inside the block use at most n CTAs (0: one
    per SM); the setting returns to one per SM afterwards."""
    set_max_ctas(n)
    try:
        yield
    finally:
        set_max_ctas(0)


class Image:
    """Activations staged as the fp16 mma-fragment image the GEMV kernels bulk-copy
    (``tlx_stage_activations``, or gate/up writing gact for the down projection)."""

    def __init__(self, m: int, k: int, device="cuda", buf: torch.Tensor = None):
        self.m, self.k = int(m), int(k)
        nb = int(_lib.lib().tlx_activation_image_bytes(self.m, self.k, TLX_DT_F16))
        if nb == 0:
            raise TLXError(f"unsupported activation image shape m={m} k={k}")
        self.buf = buf if buf is not None else torch.empty(nb, dtype=torch.uint8, device=device)
        self.shape = (self.m, self.k)

    def data_ptr(self):
        return self.buf.data_ptr()

    @property
    def device(self):
        return self.buf.device


def stage(x: torch.Tensor, image: "Image" = None) -> "Image":
    dt, ldx = _x_args(x)
    if dt == TLX_DT_F32:
        raise TLXError("fp32 activations are staged inside each call (3 columns per token)")
    m, k = x.shape
    image = image if image is not None else Image(m, k, x.device)
    check(_lib.lib().tlx_stage_activations(_ptr(x), dt, ldx, m, k, _ptr(image.buf), _stream(x)), "stage")
    return image


def _x_args(x):
    if isinstance(x, Image):
        return TLX_DT_IMAGE, 0
    if x.dim() != 2 or x.stride(1) != 1:
        raise TLXError("x must be a row-major [m, k] tensor")
    if x.dtype not in _DT:
        raise TLXError(f"unsupported activation dtype {x.dtype}")
    return _DT[x.dtype], x.stride(0)


def _y_dtype(y):
    if isinstance(y, Image):
        return TLX_DT_IMAGE
    if y.dtype not in (torch.float32, torch.float16):
        raise TLXError("outputs are fp32 or fp16")
    return _DT[y.dtype]


def gemv(qtype, w: torch.Tensor, x: torch.Tensor, n_rows: int, ws: Workspace, y: torch.Tensor = None,
         residual: torch.Tensor = None, out_dtype=torch.float32) -> torch.Tensor:
    """y[t][r] = (W x_t)[r] (+ residual[t][r]); W tiled."""
    q = qtype_id(qtype)
    dt, ldx = _x_args(x)
    m, k = x.shape
    if y is None:
        y = torch.empty((m, n_rows), dtype=out_dtype, device=x.device)
    g = grid(str(x.device)) if q == _lib.TLX_IQ3_XXS else None
    rc = _lib.lib().tlx_gemv(q, _ptr(w), _ptr(g), _ptr(x), dt, ldx, m, n_rows, k, _ptr(residual),
                             residual.stride(0) if residual is not None else 0, _ptr(y), _y_dtype(y), y.stride(0),
                             _ptr(ws.buf), ws.nbytes, _stream(x))
    check(rc, "gemv")
    return y


def ffn_gate_up(qtype, w_gate: torch.Tensor, w_up: torch.Tensor, x: torch.Tensor, n_rows: int, ws: Workspace,
                gact: torch.Tensor = None, out_dtype=torch.float32) -> torch.Tensor:
    q = qtype_id(qtype)
    dt, ldx = _x_args(x)
    m, k = x.shape
    if gact is None:
        gact = torch.empty((m, n_rows), dtype=out_dtype, device=x.device)
    g = grid(str(x.device)) if q == _lib.TLX_IQ3_XXS else None
    rc = _lib.lib().tlx_ffn_gate_up(q, _ptr(w_gate), _ptr(w_up), _ptr(g), _ptr(x), dt, ldx, m, n_rows, k,
                                    _ptr(gact), _y_dtype(gact), 0 if isinstance(gact, Image) else gact.stride(0),
                                    _ptr(ws.buf), ws.nbytes,
                                    _stream(x))
    check(rc, "ffn_gate_up")
    return gact


def head_argmax(qtype, w: torch.Tensor, x: torch.Tensor, n_rows: int, ws: Workspace, row_offset: int = 0,
                out_max=None, out_idx=None, out_keys=None, drafts=None, accept_out=None):
    q = qtype_id(qtype)
    dt, ldx = _x_args(x)
    m, k = x.shape
    dev = x.device
    if out_max is None:
        out_max = torch.empty(m, dtype=torch.float32, device=dev)
    if out_idx is None:
        out_idx = torch.empty(m, dtype=torch.int32, device=dev)
    g = grid(str(dev)) if q == _lib.TLX_IQ3_XXS else None
    nd = 0 if drafts is None else int(drafts.numel())
    rc = _lib.lib().tlx_head_argmax(q, _ptr(w), _ptr(g), _ptr(x), dt, ldx, m, n_rows, k, row_offset,
                                    _ptr(out_max), _ptr(out_idx), _ptr(out_keys), _ptr(drafts), nd,
                                    _ptr(accept_out), _ptr(ws.buf), ws.nbytes, _stream(x))
    check(rc, "head_argmax")
    return out_max, out_idx


def argmax_rows(logits: torch.Tensor, amds: torch.Tensor = None) -> torch.Tensor:
    m, n = logits.shape
    if amds is None:
        amds = torch.empty(m, dtype=torch.int32, device=logits.device)
    dt = {torch.float32: TLX_DT_F32, torch.float16: TLX_DT_F16}.get(logits.dtype)
    if dt is None:
        raise TLXError("logits must be fp32 or fp16")
    check(_lib.lib().tlx_argmax_rows(_ptr(logits), dt, m, n, logits.stride(0), _ptr(amds), _stream(logits)),
          "argmax_rows")
    return amds


def h_argmax(logits: torch.Tensor, tok_slot: torch.Tensor, pos_slot: torch.Tensor, tok_hist: torch.Tensor) -> None:
    """h_argmax(logits, tok_slot, pos_slot, tok_hist): argmax of one row of logits,
    then tok_slot[0] = idx, tok_hist[pos_slot[0]] = idx, pos_slot[0] += 1 (all on the
    device, stream-ordered; engine/h_argmax.cu argument order)."""
    if logits.dim() != 1 or not logits.is_contiguous():
        raise TLXError("h_argmax takes one contiguous row of logits")
    dt = {torch.float32: TLX_DT_F32, torch.float16: TLX_DT_F16}.get(logits.dtype)
    if dt is None:
        raise TLXError("logits must be fp32 or fp16")
    for t in (tok_slot, pos_slot, tok_hist):
        if t.dtype != torch.int32 or t.device != logits.device:
            raise TLXError("tok_slot / pos_slot / tok_hist are int32 tensors on the logits' device")
    check(_lib.lib().tlx_h_argmax(_ptr(logits), dt, logits.numel(), _ptr(tok_slot), _ptr(pos_slot), _ptr(tok_hist),
                                  _stream(logits)), "h_argmax")


class AttnProjections:
    """aq3k8v11: q / k (IQ3_XXS) and v (Q4_K) projections of m rows of x, one staging
    of x shared by the three GEMVs (tlx_aq3k8v11).  Outputs fp16 [m][n]."""

    def __init__(self, m: int, k: int, nq: int, nk: int, nv: int, x_dtype=torch.float16, device="cuda"):
        self.m, self.k, self.nq, self.nk, self.nv = int(m), int(k), int(nq), int(nk), int(nv)
        self.dt = _DT[x_dtype]
        nb = int(_lib.lib().tlx_aq3k8v11_workspace_bytes(self.m, self.k, self.nq, self.nk, self.nv, self.dt))
        if nb == 0:
            raise TLXError(f"unsupported aq3k8v11 shape m={m} k={k} nq={nq} nk={nk} nv={nv} {x_dtype}")
        self.ws = Workspace(nb, device)

    def __call__(self, wq, wk, wv, x: torch.Tensor, q=None, k=None, v=None):
        require_device()
        if x.dim() != 2 or x.stride(1) != 1 or tuple(x.shape) != (self.m, self.k) or _DT.get(x.dtype) != self.dt:
            raise TLXError("x must be a row-major [m][k] tensor of the workspace's dtype")
        q = q if q is not None else torch.empty((self.m, self.nq), dtype=torch.float16, device=x.device)
        k = k if k is not None else torch.empty((self.m, self.nk), dtype=torch.float16, device=x.device)
        v = v if v is not None else torch.empty((self.m, self.nv), dtype=torch.float16, device=x.device)
        check(_lib.lib().tlx_aq3k8v11(_ptr(wq), _ptr(wk), _ptr(wv), _ptr(grid(str(x.device))), _ptr(x), self.dt,
                                      x.stride(0), self.m, self.k, self.nq, self.nk, self.nv, _ptr(q), _ptr(k),
                                      _ptr(v), _ptr(self.ws.buf), self.ws.nbytes, _stream(x)), "aq3k8v11")
        return q, k, v

    def error(self) -> int:
        e = ctypes.c_uint32(0)
        check(_lib.lib().tlx_aq3k8v11_error(_ptr(self.ws.buf), self.m, self.k, self.nq, self.nk, self.nv, self.dt,
                                            ctypes.byref(e)), "aq3k8v11_error")
        return int(e.value)


class GdnProjections:
    """q5g8v11: the GDN block's qkv (Q5_K) and gate (IQ3_XXS) projections of m rows of
    x, one staging of x shared by the two GEMVs (tlx_q5g8v11).  Outputs fp16 [m][n]."""

    def __init__(self, m: int, k: int, nqkv: int, ngate: int, x_dtype=torch.float16, device="cuda"):
        self.m, self.k, self.nqkv, self.ngate = int(m), int(k), int(nqkv), int(ngate)
        self.dt = _DT[x_dtype]
        nb = int(_lib.lib().tlx_q5g8v11_workspace_bytes(self.m, self.k, self.nqkv, self.ngate, self.dt))
        if nb == 0:
            raise TLXError(f"unsupported q5g8v11 shape m={m} k={k} nqkv={nqkv} ngate={ngate} {x_dtype}")
        self.ws = Workspace(nb, device)

    def __call__(self, wqkv, wgate, x: torch.Tensor, qkv=None, gate=None):
        require_device()
        if x.dim() != 2 or x.stride(1) != 1 or tuple(x.shape) != (self.m, self.k) or _DT.get(x.dtype) != self.dt:
            raise TLXError("x must be a row-major [m][k] tensor of the workspace's dtype")
        qkv = qkv if qkv is not None else torch.empty((self.m, self.nqkv), dtype=torch.float16, device=x.device)
        gate = gate if gate is not None else torch.empty((self.m, self.ngate), dtype=torch.float16, device=x.device)
        check(_lib.lib().tlx_q5g8v11(_ptr(wqkv), _ptr(wgate), _ptr(grid(str(x.device))), _ptr(x), self.dt,
                                     x.stride(0), self.m, self.k, self.nqkv, self.ngate, _ptr(qkv), _ptr(gate),
                                     _ptr(self.ws.buf), self.ws.nbytes, _stream(x)), "q5g8v11")
        return qkv, gate

    def error(self) -> int:
        e = ctypes.c_uint32(0)
        check(_lib.lib().tlx_q5g8v11_error(_ptr(self.ws.buf), self.m, self.k, self.nqkv, self.ngate, self.dt,
                                           ctypes.byref(e)), "q5g8v11_error")
        return int(e.value)


# lookup{K+1}_nw32: K drafts and the scan end (starts i <= pos - scan_end), per the
# reference kernels engine/lookup5_nw32.cu .. engine/lookup11_nw32.cu
LOOKUP_SCAN_END = {4: 12, 5: 13, 6: 14, 7: 15, 8: 17, 9: 18, 10: 19}


class Lookup:
    """n-gram draft proposal over the device token history (tlx_lookup): on an
    8-token suffix match the next K history tokens become the drafts; l_hist[cyc]
    records the match length + 1.  One launch, stream-ordered, workspace reused."""

    def __init__(self, n_drafts: int = 10, scan_end: int = None, device="cuda"):
        self.k = int(n_drafts)
        self.scan_end = int(scan_end if scan_end is not None else LOOKUP_SCAN_END[self.k])
        self.ws = Workspace(int(_lib.lib().tlx_lookup_workspace_bytes()), device)

    def __call__(self, tok_hist: torch.Tensor, pos_slot: torch.Tensor, cyc_slot: torch.Tensor,
                 drafts: torch.Tensor, l_hist: torch.Tensor) -> None:
        require_device()
        for t in (tok_hist, pos_slot, cyc_slot, drafts, l_hist):
            if t.dtype != torch.int32 or not t.is_contiguous():
                raise TLXError("lookup buffers are contiguous int32")
        if drafts.numel() < self.k:
            raise TLXError(f"drafts holds {drafts.numel()} < {self.k} entries")
        check(_lib.lib().tlx_lookup(_ptr(tok_hist), tok_hist.numel(), _ptr(pos_slot), _ptr(cyc_slot), _ptr(drafts),
                                    self.k, self.scan_end, _ptr(l_hist), _ptr(self.ws.buf), self.ws.nbytes,
                                    _stream(tok_hist)), "lookup")


class Attention:
    """Split-KV int8 attention of the full-attention layers for `rows` verify rows
    (tlx_attn_pre / tlx_attn_split / tlx_attn_combine): the int8 KV cache
    kv [8][ctx][256] uint8 with scales sc [8][ctx][8] fp16, pos on the device."""

    HEADS, KV_HEADS, HEAD_DIM = 24, 4, 256

    def __init__(self, rows: int, ctx: int, device="cuda"):
        self.rows, self.ctx = int(rows), int(ctx)
        nb = int(_lib.lib().tlx_attn_workspace_bytes(self.rows))
        if nb == 0:
            raise TLXError(f"unsupported attention rows={rows}")
        self.ws = Workspace(nb, device)

    def new_cache(self, device="cuda"):
        kv = torch.full((8, self.ctx, 256), 128, dtype=torch.uint8, device=device)
        sc = torch.zeros((8, self.ctx, 8), dtype=torch.float16, device=device)
        return kv, sc

    def pre(self, qrow, krow, vrow, qnw, knw, freqs, pos_slot, kv, sc, qw16=None):
        require_device()
        if qw16 is None:
            qw16 = torch.empty((self.rows, self.HEADS, 256), dtype=torch.float16, device=qrow.device)
        check(_lib.lib().tlx_attn_pre(_ptr(qrow), _ptr(krow), _ptr(vrow), _ptr(qnw), _ptr(knw), _ptr(freqs),
                                      _ptr(pos_slot), self.rows, self.ctx, _ptr(kv), _ptr(sc), _ptr(qw16),
                                      _stream(qrow)), "attn_pre")
        return qw16

    def split(self, kv, sc, qw16, pos_slot):
        check(_lib.lib().tlx_attn_split(_ptr(kv), _ptr(sc), _ptr(qw16), _ptr(pos_slot), self.rows, self.ctx,
                                        _ptr(self.ws.buf), self.ws.nbytes, _stream(kv)), "attn_split")

    def combine(self, qrow, ao=None):
        if ao is None:
            ao = torch.empty((self.rows, self.HEADS * 256), dtype=torch.float16, device=qrow.device)
        check(_lib.lib().tlx_attn_combine(_ptr(self.ws.buf), self.ws.nbytes, _ptr(qrow), self.rows, _ptr(ao),
                                          _stream(qrow)), "attn_combine")
        return ao

    def error(self) -> int:
        """The split kernel's error bits (a bounded wait that gave up); synchronous."""
        return self.ws.error()

    def decode(self, kv, sc, qw16, qrow, pos_slot, ao=None):
        require_device()
        if ao is None:
            ao = torch.empty((self.rows, self.HEADS * 256), dtype=torch.float16, device=qrow.device)
        check(_lib.lib().tlx_attn_decode(_ptr(kv), _ptr(sc), _ptr(qw16), _ptr(qrow), _ptr(pos_slot), self.rows,
                                         self.ctx, _ptr(ao), _ptr(self.ws.buf), self.ws.nbytes, _stream(kv)),
              "attn_decode")
        return ao


GDN_BLOCKS, GDN_REC, GDN_CONV = 48, 786432, 30720  # engine/acceptsel11k.cu:22-38


def acceptsel11k(rec4: torch.Tensor, conv4: torch.Tensor, m_slot: torch.Tensor, conv_x, rec_x,
                 n_blocks: int = GDN_BLOCKS, rec_elems: int = GDN_REC, conv_elems: int = GDN_CONV) -> None:
    """acceptsel11k(rec4, conv4, m_slot, conv5x..conv11x, rec6x..rec11x): the accepted
    GDN state slot m_slot[0] becomes the live slot 4 (device-side, stream-ordered)."""
    conv_x, rec_x = list(conv_x), list(rec_x)
    if len(conv_x) != 7 or len(rec_x) != 6:
        raise TLXError("acceptsel11k takes 7 conv scratch buffers (conv5x..11x) and 6 rec (rec6x..11x)")
    for t, n in [(rec4, n_blocks * 5 * rec_elems), (conv4, n_blocks * 5 * conv_elems)] + \
                [(t, n_blocks * conv_elems) for t in conv_x] + [(t, n_blocks * rec_elems) for t in rec_x]:
        if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < n:
            raise TLXError("acceptsel11k buffers are contiguous fp32 of the stated sizes")
    if m_slot.dtype != torch.int32:
        raise TLXError("m_slot is int32")
    cx = (ctypes.c_void_p * 7)(*[t.data_ptr() for t in conv_x])
    rx = (ctypes.c_void_p * 6)(*[t.data_ptr() for t in rec_x])
    check(_lib.lib().tlx_acceptsel11k(_ptr(rec4), _ptr(conv4), _ptr(m_slot), cx, rx, n_blocks, rec_elems, conv_elems,
                                      _stream(rec4)), "acceptsel11k")


class GdnSlots:
    """GDN state commit as a slot index: a device table of the rec / conv buffer
    addresses of the eleven draft positions and the live state per GDN block
    (tlx_gdn_slots_init over the same buffers acceptsel11k takes).  flip(m_slot)
    makes the live entry name draft m's buffer instead of copying it
    (tlx_acceptsel11k_flip)."""

    LIVE = 11

    def __init__(self, rec4: torch.Tensor, conv4: torch.Tensor, conv_x, rec_x, n_blocks: int = GDN_BLOCKS,
                 rec_elems: int = GDN_REC, conv_elems: int = GDN_CONV):
        conv_x, rec_x = list(conv_x), list(rec_x)
        if len(conv_x) != 7 or len(rec_x) != 6:
            raise TLXError("the slot table takes 7 conv scratch buffers (conv5x..11x) and 6 rec (rec6x..11x)")
        for t, n in [(rec4, n_blocks * 5 * rec_elems), (conv4, n_blocks * 5 * conv_elems)] + \
                    [(t, n_blocks * conv_elems) for t in conv_x] + [(t, n_blocks * rec_elems) for t in rec_x]:
            if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < n:
                raise TLXError("slot-table buffers are contiguous fp32 of the stated sizes")
        self.n_blocks = n_blocks
        nb = int(_lib.lib().tlx_gdn_slots_bytes(n_blocks))
        self.table = torch.empty(nb // 8, dtype=torch.int64, device=rec4.device)
        cx = (ctypes.c_void_p * 7)(*[t.data_ptr() for t in conv_x])
        rx = (ctypes.c_void_p * 6)(*[t.data_ptr() for t in rec_x])
        check(_lib.lib().tlx_gdn_slots_init(_ptr(self.table), _ptr(rec4), _ptr(conv4), cx, rx, n_blocks, rec_elems,
                                            conv_elems, _stream(rec4)), "gdn_slots_init")

    def flip(self, m_slot: torch.Tensor) -> None:
        if m_slot.dtype != torch.int32:
            raise TLXError("m_slot is int32")
        check(_lib.lib().tlx_acceptsel11k_flip(_ptr(self.table), _ptr(m_slot), self.n_blocks, _stream(self.table)),
              "acceptsel11k_flip")

    def entries(self) -> torch.Tensor:
        """[n_blocks][2 (rec, conv)][12] device addresses (host copy)."""
        return self.table.view(self.n_blocks, 2, 12).cpu()


def argmax_merge(keys: torch.Tensor, out_max=None, out_idx=None, drafts=None, accept_out=None):
    n_shards, m = keys.shape
    dev = keys.device
    if out_max is None:
        out_max = torch.empty(m, dtype=torch.float32, device=dev)
    if out_idx is None:
        out_idx = torch.empty(m, dtype=torch.int32, device=dev)
    nd = 0 if drafts is None else int(drafts.numel())
    check(_lib.lib().tlx_argmax_merge(_ptr(keys), n_shards, m, _ptr(out_max), _ptr(out_idx), _ptr(drafts), nd,
                                      _ptr(accept_out), _stream(keys)), "argmax_merge")
    return out_max, out_idx


def accept(amds: torch.Tensor, drafts: torch.Tensor, k: int = None, mb=None, eb=None):
    dev = amds.device
    k = int(drafts.numel()) if k is None else int(k)
    if mb is None:
        mb = torch.empty(1, dtype=torch.int32, device=dev)
    if eb is None:
        eb = torch.empty(2, dtype=torch.int32, device=dev)
    check(_lib.lib().tlx_accept(_ptr(amds), _ptr(drafts), k, _ptr(mb), _ptr(eb), _stream(amds)), "accept")
    return mb, eb


__all__ = ["Workspace", "Image", "stage", "pack_tiles", "pack_tiles_host", "unpack_tiles_host", "tiled_bytes", "gemv", "ffn_gate_up",
           "head_argmax", "argmax_rows", "h_argmax", "acceptsel11k", "GdnSlots", "AttnProjections", "GdnProjections", "Lookup", "Attention", "argmax_merge", "accept", "grid", "plan", "set_max_ctas", "require_device",
           "MODE_STORE", "MODE_GATE_UP", "MODE_ARGMAX"]
