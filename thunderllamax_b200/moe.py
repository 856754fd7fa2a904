"""The MoE verify layer on B200.

P positions (MTP K=4 + 1 = 5) of hidden 2048 go through an fp32 router over 256
experts (top-8, softmax gates over the 8, sigmoid shared-expert gate), the 8
routed SiLU-gated IQ4_XS experts (2048 -> 512 -> 2048) plus the shared expert,
and the gated combine with the residual.  This is the reference's MoE layer
sequence rt8e256 -> shexp8 -> gx8e256up4 -> gx8e256dn -> cmbz2048
(engine/mm/MM_P7_lib.py:505-511), run as four launches of libtlx_b200
(``tlx_moe_verify``): router, expert gate/up, act image, expert down + combine.

Expert parallelism: a rank passes its expert range [e0, e1); only those experts
are read and combined (the shared expert and the residual on rank 0), and the
per-rank partial outputs are summed with one NCCL all-reduce.  The positions are
replicated on every rank (they are the verify step's rows), so token dispatch
needs no data movement: each rank reads the replicated h for its experts, and the
combine is the all-reduce.
"""
from __future__ import annotations

import ctypes
import functools
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, ops, synth
from ._lib import TLXError, check


@dataclass(frozen=True)
class MoeShape:
    positions: int = 5
    experts: int = 256
    hidden: int = 2048
    inner: int = 512
    top_k: int = 8

    def expert_bytes(self) -> int:
        """GGUF bytes of one expert (gate + up + down, IQ4_XS)."""
        return 3 * self.inner * synth.row_bytes("iq4_xs", self.hidden)

    def router_bytes(self) -> int:
        return (self.experts + 1) * self.hidden * 4


@functools.lru_cache(maxsize=None)
def kvalues(device: str = "cuda") -> torch.Tensor:
    """The 16 IQ4_NL levels (from gguf-py at run time) on the device."""
    from .tables import iq4nl_kvalues

    return torch.from_numpy(iq4nl_kvalues().copy()).to(device)


def synth_host(shape: MoeShape, seed: int = 0) -> dict:
    """Seeded config-4 weights as GGUF-layout host arrays: router fp32 N(0, 0.02),
    the shared-expert gate row N(0, 0.02) (not given by the config; drawn from the
    same seed), IQ4_XS experts [E][rows][row_bytes] and the shared expert."""
    rng = np.random.default_rng(seed)
    E, H, I = shape.experts, shape.hidden, shape.inner
    wr = rng.normal(0.0, 0.02, (E, H)).astype(np.float32)
    wsh = rng.normal(0.0, 0.02, H).astype(np.float32)
    gate = synth.iq4xs_blocks(rng, E * I, H).reshape(E, I, -1)
    up = synth.iq4xs_blocks(rng, E * I, H).reshape(E, I, -1)
    down = synth.iq4xs_blocks(rng, E * H, I).reshape(E, H, -1)
    sgate = synth.iq4xs_blocks(rng, I, H)
    sup = synth.iq4xs_blocks(rng, I, H)
    sdown = synth.iq4xs_blocks(rng, H, I)
    return {"wr": wr, "wsh": wsh, "gate": gate, "up": up, "down": down, "sgate": sgate, "sup": sup, "sdown": sdown}


def to_device(shape: MoeShape, host: dict, e0: int = 0, e1: int = None, shared: bool = True) -> dict:
    """Router (replicated), experts [e0, e1) and optionally the shared expert, tiled
    on the device.  Expert tensors stay indexed by global expert id (the kernels
    address expert e at e * bytes_per_expert), so a rank holds [0, e1) of the
    buffer but only [e0, e1) is filled and read."""
    E, H, I = shape.experts, shape.hidden, shape.inner
    e1 = E if e1 is None else e1
    dev = {"wr": torch.from_numpy(host["wr"]).cuda(), "wsh": torch.from_numpy(host["wsh"]).cuda()}
    gu = ops.tiled_bytes("iq4_xs", I, H)
    dn = ops.tiled_bytes("iq4_xs", H, I)
    for name, rows, k, per in (("gate", I, H, gu), ("up", I, H, gu), ("down", H, I, dn)):
        buf = torch.zeros(max(e1, 1) * per, dtype=torch.uint8, device="cuda")
        if e1 > e0:
            raw = host[name][e0:e1].reshape((e1 - e0) * rows, -1)
            buf[e0 * per:e1 * per].copy_(ops.pack_tiles("iq4_xs", raw, k))
        dev[name] = buf
    if shared:
        dev["sgate"] = ops.pack_tiles("iq4_xs", host["sgate"], H)
        dev["sup"] = ops.pack_tiles("iq4_xs", host["sup"], H)
        dev["sdown"] = ops.pack_tiles("iq4_xs", host["sdown"], I)
    else:
        dev["sgate"] = dev["sup"] = dev["sdown"] = None
    return dev


class MoeWorkspace:
    """Caller-owned scratch of the MoE layer: zero-filled once, self re-arming."""

    def __init__(self, shape: MoeShape, device="cuda"):
        nb = int(_lib.lib().tlx_moe_workspace_bytes(shape.positions, shape.experts, shape.hidden, shape.inner))
        if nb == 0:
            raise TLXError(f"unsupported MoE shape {shape}")
        self.shape = shape
        self.nbytes = nb
        self.buf = torch.zeros(nb, dtype=torch.uint8, device=device)

    def error(self) -> int:
        v = ctypes.c_uint32(0)
        s = self.shape
        check(_lib.lib().tlx_moe_workspace_error(ops._ptr(self.buf), s.positions, s.experts, s.hidden, s.inner,
                                                 ctypes.byref(v), ops._stream(self.buf)), "moe_workspace_error")
        return int(v.value)


def moe_verify(shape: MoeShape, w: dict, h: torch.Tensor, ws: MoeWorkspace, y: torch.Tensor,
               hres: torch.Tensor = None, ids: torch.Tensor = None, gates: torch.Tensor = None,
               sg: torch.Tensor = None, e0: int = 0, e1: int = None):
    """y = hres + MoE(h) over the experts in [e0, e1) (+ the shared one if w has it)."""
    ops.require_device()
    s = shape
    e1 = s.experts if e1 is None else e1
    if h.dtype != torch.bfloat16 or h.dim() != 2 or tuple(h.shape) != (s.positions, s.hidden) or h.stride(1) != 1:
        raise TLXError("h must be a row-major bf16 [positions, hidden] tensor")
    if y.dtype != torch.float32 or y.stride(1) != 1:
        raise TLXError("y must be a row-major fp32 tensor")
    P = ops._ptr
    rc = _lib.lib().tlx_moe_verify(P(w["wr"]), P(w["wsh"]), P(w["gate"]), P(w["up"]), P(w["down"]),
                                   P(w["sgate"]), P(w["sup"]), P(w["sdown"]), P(kvalues(str(h.device))), P(h),
                                   h.stride(0), P(hres), hres.stride(0) if hres is not None else 0, P(y), y.stride(0),
                                   P(ids), P(gates), P(sg), s.positions, s.experts, s.hidden, s.inner, e0, e1,
                                   P(ws.buf), ws.nbytes, ops._stream(h))
    check(rc, "moe_verify")
    return y


class MoeVerifyStep:
    """One MoE verify layer on one GPU (or one rank's expert range), graph-captured."""

    LAUNCHES_PER_STEP = 4

    def __init__(self, shape: MoeShape = MoeShape(), seed: int = 0, host: dict = None, e0: int = 0, e1: int = None,
                 shared: bool = True):
        ops.require_device()
        self.shape = s = shape
        self.e0, self.e1 = e0, (s.experts if e1 is None else e1)
        self.host = host if host is not None else synth_host(s, seed)
        self.w = to_device(s, self.host, self.e0, self.e1, shared)
        dev = "cuda"
        self.h = torch.zeros((s.positions, s.hidden), dtype=torch.bfloat16, device=dev)
        self.hres = torch.zeros((s.positions, s.hidden), dtype=torch.float32, device=dev) if shared else None
        self.y = torch.zeros((s.positions, s.hidden), dtype=torch.float32, device=dev)
        self.ids = torch.zeros((s.positions, s.top_k), dtype=torch.int32, device=dev)
        self.gates = torch.zeros((s.positions, s.top_k), dtype=torch.float32, device=dev)
        self.sg = torch.zeros(s.positions, dtype=torch.float32, device=dev)
        self.ws = MoeWorkspace(s, dev)
        self.graph = None

    def launch(self):
        moe_verify(self.shape, self.w, self.h, self.ws, self.y, hres=self.hres, ids=self.ids, gates=self.gates,
                   sg=self.sg, e0=self.e0, e1=self.e1)

    def capture(self):
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            self.launch()
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.launch()
        self.graph = g
        return g

    def replay(self):
        if self.graph is None:
            self.capture()
        self.graph.replay()

    def set_inputs(self, h, hres=None):
        self.h.copy_(h, non_blocking=True)
        if hres is not None and self.hres is not None:
            self.hres.copy_(hres, non_blocking=True)

    def touched_bytes(self) -> int:
        """Algorithmic bytes of the last step: router + shared expert + each distinct
        routed expert of this rank's range once (read back from ids)."""
        s = self.shape
        ids = self.ids.cpu().numpy().reshape(-1)
        u = len({int(e) for e in ids if self.e0 <= e < self.e1})
        shared = 1 if self.w["sgate"] is not None else 0
        return s.router_bytes() + (u + shared) * s.expert_bytes()
