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
