"""The K-row speculative verify step on one GPU.

One step = the dense FFN of the probe trunk followed by the LM head:

    gact = silu(Wg X) * (Wu X)        IQ3_XXS, 11 x 5120 -> 11 x 17408 (fp16)
    Y    = R + Wd gact                Q6_K,   11 x 17408 -> 11 x 5120  (fp32)
    (max, idx)[t] = argmax_v (Wh H)   Q6_K,   11 x 5120 -> 151936 vocab, no logits
    m, bonus = accept(idx, drafts)    greedy draft acceptance

which is the reference's per-layer ffn8v11r7 -> down8nw32v11r7 pair
(engine/mtp.py:1127-1128) and its head8v11 -> amx3 -> accept11k tail
(engine/mtp.py:1159-1161, :749-753).  Five launches per step (two tiny
activation-staging kernels and the three GEMVs; gate/up writes gact directly in
the image format down reads), captured in a CUDA graph (the reference's
pre-recorded ParityGraph, engine/gcycle.py:22-73).

The FFN chain and the head read different inputs, so the step runs them side by
side: the stream forks, the head runs on a side stream over `head_ctas` SMs while
gate/up -> down run on the caller's stream over the other `ffn_ctas` SMs, and the
streams join (event record / wait, which a graph capture turns into two parallel
branches).  Each GEMV is bound by per-SM instruction throughput, so splitting the
SMs costs nothing in total work, while each chain's launch ramp, first-copy
latency and split-tile tail are hidden behind the other chain's streaming.
`ffn_ctas=0` runs the three GEMVs one after another on all SMs.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import ops, synth


@dataclass
class VerifyShape:
    dim: int = 5120
    ffn: int = 17408
    vocab: int = 151936
    rows: int = 11           # K + 1 probe rows
    ffn_q: str = "iq3_xxs"
    down_q: str = "q6_k"
    head_q: str = "q6_k"

    @property
    def n_drafts(self) -> int:
        return self.rows - 1

    def weight_bytes(self) -> dict:
        return {"gate": self.ffn * synth.row_bytes(self.ffn_q, self.dim),
                "up": self.ffn * synth.row_bytes(self.ffn_q, self.dim),
                "down": self.dim * synth.row_bytes(self.down_q, self.ffn),
                "head": self.vocab * synth.row_bytes(self.head_q, self.dim)}

    def algorithmic_bytes(self) -> dict:
        """Bytes a roofline-optimal step must move: weights once, activations in, results out."""
        wb = self.weight_bytes()
        r, d, f = self.rows, self.dim, self.ffn
        return {"ffn_gate_up": wb["gate"] + wb["up"] + r * d * 2 + r * f * 2,
                "ffn_down": wb["down"] + r * f * 2 + r * d * 4 * 2,
                "head_argmax": wb["head"] + r * d * 2 + r * 8}


def synth_tiled(qtype: str, n_rows: int, k: int, seed: int, rows: tuple[int, int] | None = None,
                cols: tuple[int, int] | None = None) -> torch.Tensor:
    """The seeded synthetic (n_rows x k) GGUF matrix (synth.matrix_rows), or its row
    range `rows` / column range `cols` (multiples of 256: a k shard), repacked on
    the device into one tiled buffer, one 8192-row chunk at a time."""
    r0, r1 = rows if rows is not None else (0, n_rows)
    k0, k1 = cols if cols is not None else (0, k)
    if k0 % synth.QK or k1 % synth.QK or not 0 <= k0 < k1 <= k:
        raise ValueError(f"column range [{k0}, {k1}) is not a 256-aligned part of [0, {k})")
    kk = k1 - k0
    bb = synth.BLOCK_BYTES[qtype]           # bytes per 256 weights of a row
    out = torch.empty(ops.tiled_bytes(qtype, r1 - r0, kk), dtype=torch.uint8, device="cuda")
    per_tile = ops.tiled_bytes(qtype, 16, kk)
    step = synth.CHUNK_ROWS
    a = r0
    while a < r1:
        b = min(a - (a % step) + step, r1)          # to the next chunk boundary
        raw = synth.matrix_rows(qtype, n_rows, k, seed, a, b)
        if cols is not None:
            raw = np.ascontiguousarray(raw[:, (k0 // synth.QK) * bb:(k1 // synth.QK) * bb])
        t = ops.pack_tiles(qtype, raw, kk)
        off = ((a - r0) // 16) * per_tile
        out[off:off + t.numel()].copy_(t)
        a = b
    return out


def default_split_ctas(sms: int) -> int:
    """CTAs of the FFN chain when it runs beside the head on one GPU (the head gets
    the rest); 0 (serial) on parts too small to split."""
    return 45 if sms >= 128 else 0


class StepIO:
    """The step's host-facing buffers, packed so that a step moves its inputs with ONE
    host-to-device copy and its record with ONE device-to-host copy: the device input
    buffer holds x | h (bf16 [rows][dim] each) | drafts (int32), the output buffer the
    accept record (m, bonus) then the rows' argmax ids (int32), and the kernels read and
    write views of them.  host_buffers() gives pinned host buffers of the same layouts."""

    def _alloc_io(self, rows: int, dim: int, n_drafts: int, dev="cuda"):
        xb = rows * dim * 2
        self._in_bytes = 2 * xb + n_drafts * 4
        self.inbuf = torch.zeros(self._in_bytes, dtype=torch.uint8, device=dev)
        self.x = self.inbuf[:xb].view(torch.bfloat16).view(rows, dim)
        self.h = self.inbuf[xb:2 * xb].view(torch.bfloat16).view(rows, dim)
        self.drafts = self.inbuf[2 * xb:].view(torch.int32)
        self.outbuf = torch.zeros(2 + rows, dtype=torch.int32, device=dev)
        self.accept_out = self.outbuf[:2]
        self.out_idx = self.outbuf[2:]

    def host_buffers(self):
        """(in_pinned uint8, out_pinned int32, the in buffer's x / h / drafts views)."""
        xb = self.x.numel() * 2
        inp = torch.zeros(self._in_bytes, dtype=torch.uint8).pin_memory()
        outp = torch.zeros(self.outbuf.numel(), dtype=torch.int32).pin_memory()
        views = {"x": inp[:xb].view(torch.bfloat16).view(self.x.shape),
                 "h": inp[xb:2 * xb].view(torch.bfloat16).view(self.h.shape),
                 "drafts": inp[2 * xb:].view(torch.int32)}
        return inp, outp, views

    def step_host_packed(self, in_pinned, out_pinned):
        """End-to-end step through host buffers: ONE H2D copy of x | h | drafts, the
        graph replay, ONE D2H copy of (m, bonus, argmax ids)."""
        self.inbuf.copy_(in_pinned, non_blocking=True)
        self.replay()
        out_pinned.copy_(self.outbuf, non_blocking=True)


class VerifyStep(StepIO):
    def __init__(self, shape: VerifyShape = VerifyShape(), seed: int = 0, weights: dict | None = None,
                 ffn_ctas: int | None = None):
        ops.require_device()
        self.shape = s = shape
        self.w = weights if weights is not None else {
            "gate": synth_tiled(s.ffn_q, s.ffn, s.dim, seed + 1),
            "up": synth_tiled(s.ffn_q, s.ffn, s.dim, seed + 2),
            "down": synth_tiled(s.down_q, s.dim, s.ffn, seed + 3),
            "head": synth_tiled(s.head_q, s.vocab, s.dim, seed + 4),
        }
        dev = "cuda"
        self._alloc_io(s.rows, s.dim, s.n_drafts, dev)      # x, h, drafts, accept_out, out_idx
        self.res = torch.zeros((s.rows, s.dim), dtype=torch.float32, device=dev)
        # gate/up writes gact straight into the fp16 activation image down reads
        self.gact = ops.Image(s.rows, s.ffn, dev)
        self.y = torch.empty((s.rows, s.dim), dtype=torch.float32, device=dev)
        self.out_max = torch.empty(s.rows, dtype=torch.float32, device=dev)
        # workspaces of the kernels alone on every SM (launch_<kernel>) ...
        self.ws = {
            "ffn_gate_up": ops.Workspace.for_shape(ops.MODE_GATE_UP, s.ffn_q, s.ffn, s.dim, s.rows),
            "ffn_down": ops.Workspace.for_shape(ops.MODE_STORE, s.down_q, s.dim, s.ffn, s.rows, "image"),
            "head_argmax": ops.Workspace.for_shape(ops.MODE_ARGMAX, s.head_q, s.vocab, s.dim, s.rows),
        }
        # ... and of the step's two chains side by side, each sized by its CTA budget
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        self.ffn_ctas = default_split_ctas(sms) if ffn_ctas is None else int(ffn_ctas)
        if not 0 <= self.ffn_ctas < sms:
            raise ValueError(f"ffn_ctas must be in [0, {sms}), not {self.ffn_ctas}")
        self.head_ctas = sms - self.ffn_ctas if self.ffn_ctas else 0
        self.side = None
        self.ws_step = self.ws
        if self.ffn_ctas:
            with ops.cta_budget(self.ffn_ctas):
                self.ws_step = {
                    "ffn_gate_up": ops.Workspace.for_shape(ops.MODE_GATE_UP, s.ffn_q, s.ffn, s.dim, s.rows),
                    "ffn_down": ops.Workspace.for_shape(ops.MODE_STORE, s.down_q, s.dim, s.ffn, s.rows, "image"),
                }
            with ops.cta_budget(self.head_ctas):
                self.ws_step["head_argmax"] = ops.Workspace.for_shape(ops.MODE_ARGMAX, s.head_q, s.vocab, s.dim,
                                                                      s.rows)
            self.side = torch.cuda.Stream()
        self.graph = None

    # ---- the three launches (ws: which workspace set; the CTA budget is the caller's) ----
    def launch_ffn_gate_up(self, ws=None):
        s = self.shape
        ws = self.ws if ws is None else ws
        ops.ffn_gate_up(s.ffn_q, self.w["gate"], self.w["up"], self.x, s.ffn, ws["ffn_gate_up"], gact=self.gact)

    def launch_ffn_down(self, ws=None):
        s = self.shape
        ws = self.ws if ws is None else ws
        ops.gemv(s.down_q, self.w["down"], self.gact, s.dim, ws["ffn_down"], y=self.y, residual=self.res)

    def launch_head_argmax(self, ws=None):
        s = self.shape
        ws = self.ws if ws is None else ws
        ops.head_argmax(s.head_q, self.w["head"], self.h, s.vocab, ws["head_argmax"], out_max=self.out_max,
                        out_idx=self.out_idx, drafts=self.drafts, accept_out=self.accept_out)

    KERNELS = ("ffn_gate_up", "ffn_down", "head_argmax")
    # stage(X) + gate/up, down, stage(H) + head
    LAUNCHES_PER_STEP = 5

    def workspace_errors(self) -> dict:
        """Error words of every workspace the step and the kernels alone use."""
        out = {f"{k}": w.error() for k, w in self.ws.items()}
        if self.ws_step is not self.ws:
            out.update({f"{k}_step": w.error() for k, w in self.ws_step.items()})
        return out

    def launch(self):
        if not self.ffn_ctas:
            self.launch_ffn_gate_up()
            self.launch_ffn_down()
            self.launch_head_argmax()
            return
        cur = torch.cuda.current_stream()
        self.side.wait_stream(cur)
        with torch.cuda.stream(self.side):
            with ops.cta_budget(self.head_ctas):
                self.launch_head_argmax(self.ws_step)
        with ops.cta_budget(self.ffn_ctas):
            self.launch_ffn_gate_up(self.ws_step)
            self.launch_ffn_down(self.ws_step)
        cur.wait_stream(self.side)

    def capture(self):
        """Record the step once as a CUDA graph (after a warm-up launch)."""
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

    def set_inputs(self, x, h, res=None, drafts=None):
        self.x.copy_(x, non_blocking=True)
        self.h.copy_(h, non_blocking=True)
        if res is not None:
            self.res.copy_(res, non_blocking=True)
        if drafts is not None:
            self.drafts.copy_(drafts, non_blocking=True)

    def step_host(self, x_pinned, h_pinned, drafts_pinned, out_pinned):
        """End-to-end step through host buffers: H2D inputs, graph replay, D2H of
        the accept record (m, bonus) and the 11 argmax ids."""
        self.set_inputs(x_pinned, h_pinned, drafts=drafts_pinned)
        self.replay()
        out_pinned[:2].copy_(self.accept_out, non_blocking=True)
        out_pinned[2:].copy_(self.out_idx, non_blocking=True)
