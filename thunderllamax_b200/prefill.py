"""Prefill-sized FFN contraction on the tcgen05 tensor cores.

    act = silu(X Wg^T) * (X Wu^T)     IQ3_XXS 5120 -> 17408, fp32 act
    Y   = act Wd^T                    Q6_K 17408 -> 5120, fp32

for 2048 tokens: the reference's prefill GEMM pool (engine/pf_gemm3.cu,
engine/pf_gemm3m.cu: IQ3 dequant -> fp16 shared memory -> mma.sync) as two
launches of libtlx_b200 (``tlx_prefill_ffn_gate_up``, ``tlx_prefill_gemm``)
that dequantise each weight tile once per 256 tokens into shared memory and run
tcgen05.mma with fp32 accumulators in tensor memory.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib, ops
from ._lib import TLX_DT_BF16, TLX_DT_F16, TLXError, check


@dataclass(frozen=True)
class PrefillShape:
    tokens: int = 2048
    dim: int = 5120
    ffn: int = 17408
    ffn_q: str = "iq3_xxs"
    down_q: str = "q6_k"

    def flops(self) -> int:
        """Multiply-adds x 2 of gate + up + down."""
        return 2 * self.tokens * self.dim * self.ffn * 3


class PrefillWorkspace:
    """Device error word + fp16 staging of bf16 tokens and their per-row scales (zeroed once)."""

    def __init__(self, m: int, k: int, device="cuda"):
        nb = int(_lib.lib().tlx_prefill_workspace_bytes(m, k))
        if nb == 0:
            raise TLXError(f"unsupported prefill shape m={m} k={k}")
        self.nbytes = nb
        self.buf = torch.zeros(nb, dtype=torch.uint8, device=device)

    def error(self) -> int:
        torch.cuda.synchronize()
        return int(self.buf[:4].view(torch.int32).item())


def _x_args(x: torch.Tensor):
    if x.dim() != 2 or x.stride(1) != 1:
        raise TLXError("x must be a row-major [tokens, k] tensor")
    if x.dtype == torch.bfloat16:
        return TLX_DT_BF16
    if x.dtype == torch.float16:
        return TLX_DT_F16
    if x.dtype == torch.float32:
        return _lib.TLX_DT_F32
    raise TLXError(f"prefill tokens are bf16, fp16 or fp32, not {x.dtype}")


def gate_up(qtype, w_gate: torch.Tensor, w_up: torch.Tensor, x: torch.Tensor, n_rows: int, ws: PrefillWorkspace,
            act: torch.Tensor = None) -> torch.Tensor:
    """act[t][r] = silu((Wg x_t)[r]) * (Wu x_t)[r] in fp32; weights tiled (ops.pack_tiles).  fp32 because the
    product of two large projections can leave the fp16 range; gemm() stages it back to fp16 with a
    power-of-two scale per row."""
    ops.require_device()
    q = ops.qtype_id(qtype)
    dt = _x_args(x)
    m, k = x.shape
    if act is None:
        act = torch.empty((m, n_rows), dtype=torch.float32, device=x.device)
    g = ops.grid(str(x.device)) if q == _lib.TLX_IQ3_XXS else None
    rc = _lib.lib().tlx_prefill_ffn_gate_up(q, ops._ptr(w_gate), ops._ptr(w_up), ops._ptr(g), ops._ptr(x), dt,
                                            x.stride(0), m, n_rows, k, ops._ptr(act), act.stride(0),
                                            ops._ptr(ws.buf), ws.nbytes, ops._stream(x))
    check(rc, "prefill_ffn_gate_up")
    return act


def gemm(qtype, w: torch.Tensor, x: torch.Tensor, n_rows: int, ws: PrefillWorkspace,
         y: torch.Tensor = None) -> torch.Tensor:
    """y[t][r] = (W x_t)[r] in fp32; W tiled."""
    ops.require_device()
    q = ops.qtype_id(qtype)
    dt = _x_args(x)
    m, k = x.shape
    if y is None:
        y = torch.empty((m, n_rows), dtype=torch.float32, device=x.device)
    g = ops.grid(str(x.device)) if q == _lib.TLX_IQ3_XXS else None
    rc = _lib.lib().tlx_prefill_gemm(q, ops._ptr(w), ops._ptr(g), ops._ptr(x), dt, x.stride(0), m, n_rows, k,
                                     ops._ptr(y), y.stride(0), ops._ptr(ws.buf), ws.nbytes, ops._stream(x))
    check(rc, "prefill_gemm")
    return y


def lut8(device: str = "cuda") -> torch.Tensor:
    """The W4A8 tier's linearised codebook (int8[1024]) resident on the device."""
    from .tables import iq3xxs_levels_lut8

    return torch.from_numpy(iq3xxs_levels_lut8().copy()).to(device)


def _check_chunk_table(t: torch.Tensor, dtype, m: int, k: int, name: str):
    """One value per (token, 128-k chunk), contiguous: the layout the kernels index."""
    if t.dtype != dtype or tuple(t.shape) != (m, k // 128) or not t.is_contiguous():
        raise TLXError(f"{name} must be a contiguous {dtype} [tokens, k / 128] tensor")


def act_quant_q8(x: torch.Tensor, xq: torch.Tensor = None, sx: torch.Tensor = None, rs: torch.Tensor = None):
    """fp16 x[m, k] -> (xq int8 [m, k], sx fp32 [m, k/128], rs int32 [m, k/128]): per (token, 128-k
    chunk) s = max(max|x|, 1e-6) / 127, xq = clamp(rint(x / s)), rs = sum of xq (reference p8q8x,
    engine/pfk_q8.cu:24-59)."""
    ops.require_device()
    if x.dim() != 2 or x.stride(1) != 1 or x.dtype != torch.float16:
        raise TLXError("x must be a row-major fp16 [tokens, k] tensor")
    m, k = x.shape
    if xq is None:
        xq = torch.empty((m, k), dtype=torch.int8, device=x.device)
    if sx is None:
        sx = torch.empty((m, k // 128), dtype=torch.float32, device=x.device)
    if rs is None:
        rs = torch.empty((m, k // 128), dtype=torch.int32, device=x.device)
    if xq.dtype != torch.int8 or tuple(xq.shape) != (m, k) or xq.stride(1) != 1:
        raise TLXError("xq must be a row-major int8 [tokens, k] tensor")
    _check_chunk_table(sx, torch.float32, m, k, "sx")
    _check_chunk_table(rs, torch.int32, m, k, "rs")
    rc = _lib.lib().tlx_act_quant_q8(ops._ptr(x), x.stride(0), m, k, ops._ptr(xq), xq.stride(0), ops._ptr(sx),
                                     ops._ptr(rs), ops._stream(x))
    check(rc, "act_quant_q8")
    return xq, sx, rs


def w4a8_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, xq: torch.Tensor, sx: torch.Tensor, n_rows: int,
                 ws: PrefillWorkspace, act: torch.Tensor = None, lut: torch.Tensor = None) -> torch.Tensor:
    """act[t][r] = silu(g) * u in fp32 on int8 tokens (xq, sx from act_quant_q8) and the tiled IQ3_XXS
    weights read through the linearised codebook (reference p8w4ffn7, engine/p8_w4ffn7.cu:118-255)."""
    ops.require_device()
    if xq.dim() != 2 or xq.stride(1) != 1 or xq.dtype != torch.int8:
        raise TLXError("xq must be a row-major int8 [tokens, k] tensor")
    m, k = xq.shape
    _check_chunk_table(sx, torch.float32, m, k, "sx")
    if act is None:
        act = torch.empty((m, n_rows), dtype=torch.float32, device=xq.device)
    if lut is None:
        lut = lut8(str(xq.device))
    if lut.dtype != torch.int8 or lut.numel() != 1024 or not lut.is_contiguous():
        raise TLXError("lut must be the 1024-entry int8 codebook (prefill.lut8())")
    if act.dtype != torch.float32 or act.shape[0] != m or act.shape[1] < n_rows or act.stride(1) != 1:
        raise TLXError("act must be a row-major fp32 [tokens, >= n_rows] tensor")
    rc = _lib.lib().tlx_prefill_w4a8_gate_up(ops._ptr(w_gate), ops._ptr(w_up), ops._ptr(lut), ops._ptr(xq),
                                             xq.stride(0), ops._ptr(sx), m, n_rows, k, ops._ptr(act), act.stride(0),
                                             ops._ptr(ws.buf), ws.nbytes, ops._stream(xq))
    check(rc, "prefill_w4a8_gate_up")
    return act


class PrefillFFN:
    """The config-5 FFN on one GPU: gate/up (+SiLU) then down, two launches (+ the
    bf16 -> fp16 token staging)."""

    def __init__(self, shape: PrefillShape = PrefillShape(), seed: int = 0, weights: dict = None):
        from .verify import synth_tiled

        ops.require_device()
        self.shape = s = shape
        self.w = weights if weights is not None else {
            "gate": synth_tiled(s.ffn_q, s.ffn, s.dim, seed + 1),
            "up": synth_tiled(s.ffn_q, s.ffn, s.dim, seed + 2),
            "down": synth_tiled(s.down_q, s.dim, s.ffn, seed + 3),
        }
        self.x = torch.zeros((s.tokens, s.dim), dtype=torch.bfloat16, device="cuda")
        self.act = torch.empty((s.tokens, s.ffn), dtype=torch.float32, device="cuda")
        self.y = torch.empty((s.tokens, s.dim), dtype=torch.float32, device="cuda")
        self.ws = PrefillWorkspace(s.tokens, s.dim)
        self.ws_down = PrefillWorkspace(s.tokens, s.ffn)

    def launch(self):
        s = self.shape
        gate_up(s.ffn_q, self.w["gate"], self.w["up"], self.x, s.ffn, self.ws, act=self.act)
        gemm(s.down_q, self.w["down"], self.act, s.dim, self.ws_down, y=self.y)
