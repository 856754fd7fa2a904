"""The verify step sharded across the GPUs of one node (one process per GPU).

The reference is single-GPU (README.md:412-413); this is the B200 node layout:

* FFN gate/up: output rows split by whole 256-row blocks (the gact image a
  rank produces is exactly the k range of down it consumes).
* FFN down: split by k (columns) to match; every rank produces a partial
  11 x 5120 fp32 sum, and every rank adds all ranks' partials in rank order
  (the residual first).
* LM head: split by vocabulary; each rank's fused head emits 11 packed
  (max, index) keys with global row ids; every rank merges all ranks' keys and
  runs greedy accept (deterministic, identical on all ranks).

The MoE verify layer (config 4) and the prefill FFN (config 5) shard the same way:

* MoE: expert parallel.  The router is replicated (every rank computes the same
  top-8); rank r runs only the routed experts of its contiguous range
  [e0, e1) and rank 0 also the shared expert and the residual; ONE all-reduce of
  the [positions][hidden] fp32 partials gives the layer.  Token dispatch moves no
  data: the verify step's positions are replicated on every rank.
* Prefill FFN: tensor parallel.  gate/up split by whole 256-row blocks, down by
  the matching k range; each rank's tcgen05 down GEMM writes a partial
  [tokens][dim] fp32 sum, added by ONE all-reduce.

The summation order of an all-reduce differs from the single-GPU combine, so
sharded results agree with the one-GPU path to fp32 rounding, not bit for bit.

The verify step's default exchange (comm="peer") uses no collective library: every
rank maps every other rank's communication buffer (CUDA IPC), the down and head
kernels write their results into their own buffer and raise release flags in every
rank's buffer, and the finish kernel / the head's last CTA read the peers' results
over NVLink.  comm="nccl" keeps the all-reduce + all-gather form.  The MoE and
prefill steps use one NCCL all-reduce each.  Collectives go through
``torch.distributed`` (NCCL on GPUs; gloo in the CPU tests of the host-side
plumbing) and are captured in the step's CUDA graph.  No load of peer memory uses
TMA or multicast.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import ops
from .verify import StepIO, VerifyShape, synth_tiled


def block_ranges(n_blocks: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, near-equal split of n_blocks 256-row blocks over ranks."""
    return [((n_blocks * r) // world, (n_blocks * (r + 1)) // world) for r in range(world)]


def row_ranges(n_rows: int, world: int, quantum: int = 16) -> list[tuple[int, int]]:
    """Contiguous split of n_rows in multiples of `quantum` rows (the last rank
    takes the remainder)."""
    units = (n_rows + quantum - 1) // quantum
    out = []
    for r in range(world):
        u0, u1 = (units * r) // world, (units * (r + 1)) // world
        out.append((min(u0 * quantum, n_rows), min(u1 * quantum, n_rows)))
    return out


class PeerComm:
    """The communication buffers of the sharded verify step over peer memory: one per
    rank on its own GPU (tlx_peer_buffer_alloc), every peer's mapped into this process
    through a CUDA IPC handle exchanged over the process group.  `ptrs` is the array of
    the `world` buffers as seen from this process (the kernels write their results into
    their own buffer, raise a release flag in every rank's buffer and read the peers'
    results over NVLink once the flags are up)."""

    def __init__(self, rank: int, world: int, m: int, ny: int, group=None):
        import ctypes

        from . import _lib

        self._lib = L = _lib.lib()
        nb = int(L.tlx_peer_buffer_bytes(world, m, ny))
        if nb == 0:
            raise ValueError(f"no peer buffer for world={world} m={m} ny={ny}")
        buf = ctypes.c_void_p()
        _lib.check(L.tlx_peer_buffer_alloc(nb, ctypes.byref(buf)), "peer_buffer_alloc")
        self.local, self.nbytes = buf.value, nb
        hsize = int(L.tlx_ipc_handle_bytes())
        handle = (ctypes.c_uint8 * hsize)()
        off = ctypes.c_uint64()
        _lib.check(L.tlx_ipc_handle(self.local, handle, ctypes.byref(off)), "ipc_handle")
        infos = [None] * world
        dist.all_gather_object(infos, (bytes(handle), int(off.value)), group=group)
        self.opened, ptrs = [], []
        for r, (h, o) in enumerate(infos):
            if r == rank:
                ptrs.append(self.local)
                continue
            hb = (ctypes.c_uint8 * hsize).from_buffer_copy(h)
            base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.check(L.tlx_ipc_open(hb, o, ctypes.byref(base), ctypes.byref(ptr)), "ipc_open")
            self.opened.append(base.value)
            ptrs.append(ptr.value)
        self.ptrs = (ctypes.c_void_p * world)(*ptrs)
        # every buffer is zeroed and mapped everywhere before any step writes into it
        dist.barrier(group=group)

    def close(self, group=None):
        """Collective: every rank's GPU idle, every mapping of every buffer closed,
        then each rank frees its own buffer."""
        if self.local is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=group)          # no kernel of any rank still writes into a peer buffer
        for b in self.opened:
            self._lib.tlx_ipc_close(b)
        self.opened = []
        dist.barrier(group=group)          # every mapping of this rank's buffer is closed
        self._lib.tlx_peer_buffer_free(self.local)
        self.local = None


def default_ffn_ctas(world: int, sms: int) -> int:
    """CTAs for the FFN stream of the peer step (the head gets the rest)."""
    return {2: 48, 4: 64, 8: 64}.get(world, 64) if sms >= 128 else 0


def allreduce_partial(y: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the per-rank partial down-projection outputs in place."""
    dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y


def gather_keys(local_keys: torch.Tensor, all_keys: torch.Tensor, group=None) -> torch.Tensor:
    """[m] int64 keys of this rank -> [world, m] keys of every rank."""
    dist.all_gather_into_tensor(all_keys.view(-1), local_keys, group=group)  # concatenated form (NCCL and gloo)
    return all_keys


class ShardedVerifyStep(StepIO):
    """VerifyStep over `world` GPUs; this object is rank `rank`'s share.

    comm = "peer" (default): the down projection's partials and the head's argmax keys
    travel through peer memory inside the two kernels (PeerComm, tlx_gemv_peer,
    tlx_head_argmax_peer): no NCCL call and no merge kernel in the step.
    comm = "nccl": one NCCL all-reduce of the partials and one all-gather of the keys,
    then a merge kernel (the collective-library baseline of the same split)."""

    KERNELS = ("ffn_gate_up", "ffn_down", "head_argmax")

    def __init__(self, shape: VerifyShape, rank: int, world: int, seed: int = 0, weights: dict | None = None,
                 group=None, comm: str = "peer", ffn_ctas: int | None = None):
        ops.require_device()
        if comm not in ("peer", "nccl"):
            raise ValueError(f"comm must be 'peer' or 'nccl', not {comm!r}")
        self.comm = comm
        # stage/gate-up, down, stage/head, then the finish kernel (peer) or the merge (nccl)
        self.LAUNCHES_PER_STEP = 6
        self.COLLECTIVES = ("down partials and head keys over peer memory inside the kernels" if comm == "peer"
                            else "NCCL all-reduce of the down partials + NCCL all-gather of the head keys")
        self.shape = s = shape
        self.rank, self.world, self.group = rank, world, group
        nb_ffn = s.ffn // 256
        b0, b1 = block_ranges(nb_ffn, world)[rank]
        self.f0, self.f1 = 256 * b0, 256 * b1          # this rank's FFN rows / down k range
        self.v0, self.v1 = row_ranges(s.vocab, world)[rank]
        self.n_ffn = self.f1 - self.f0
        self.n_voc = self.v1 - self.v0
        if self.n_ffn <= 0 or self.n_voc <= 0:
            raise ValueError(f"rank {rank} of {world} has an empty shard")
        if weights is None:
            # this rank's slices of the ONE seeded model VerifyStep(seed) uses: gate/up
            # rows [f0, f1), down columns [f0, f1), head rows [v0, v1)
            weights = {"gate": synth_tiled(s.ffn_q, s.ffn, s.dim, seed + 1, rows=(self.f0, self.f1)),
                       "up": synth_tiled(s.ffn_q, s.ffn, s.dim, seed + 2, rows=(self.f0, self.f1)),
                       "down": synth_tiled(s.down_q, s.dim, s.ffn, seed + 3, cols=(self.f0, self.f1)),
                       "head": synth_tiled(s.head_q, s.vocab, s.dim, seed + 4, rows=(self.v0, self.v1))}
        self.w = weights
        dev = "cuda"
        self._alloc_io(s.rows, s.dim, s.n_drafts, dev)      # x, h, drafts, accept_out, out_idx
        self.res = torch.zeros((s.rows, s.dim), dtype=torch.float32, device=dev)
        self.gact = ops.Image(s.rows, self.n_ffn, dev)
        self.y = torch.empty((s.rows, s.dim), dtype=torch.float32, device=dev)
        self.local_keys = torch.zeros(s.rows, dtype=torch.int64, device=dev)
        self.all_keys = torch.zeros((world, s.rows), dtype=torch.int64, device=dev)
        self.out_max = torch.empty(s.rows, dtype=torch.float32, device=dev)
        # peer mode: the FFN (gate/up -> down) and the head run on two streams at once,
        # each on its own share of the SMs; both are latency-bound at these shard sizes,
        # so running them side by side hides one's fixed costs behind the other
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        if comm == "peer":
            self.ffn_ctas = ffn_ctas if ffn_ctas is not None else default_ffn_ctas(world, sms)
            self.head_ctas = sms - self.ffn_ctas if self.ffn_ctas else 0
        else:
            self.ffn_ctas = self.head_ctas = 0
        with ops.cta_budget(self.ffn_ctas):
            self.ws = {
                "ffn_gate_up": ops.Workspace.for_shape(ops.MODE_GATE_UP, s.ffn_q, self.n_ffn, s.dim, s.rows),
                "ffn_down": ops.Workspace.for_shape(ops.MODE_STORE, s.down_q, s.dim, self.n_ffn, s.rows, "image"),
            }
        with ops.cta_budget(self.head_ctas):
            self.ws["head_argmax"] = ops.Workspace.for_shape(ops.MODE_ARGMAX, s.head_q, self.n_voc, s.dim, s.rows)
        self.peer = PeerComm(rank, world, s.rows, s.dim, group) if comm == "peer" else None
        self.side = torch.cuda.Stream() if comm == "peer" else None
        self.finish_err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.graph = None

    def algorithmic_bytes_per_rank(self) -> dict:
        s = self.shape
        from .synth import row_bytes

        r, d = s.rows, s.dim
        return {"ffn_gate_up": 2 * self.n_ffn * row_bytes(s.ffn_q, d) + r * d * 2 + r * self.n_ffn * 2,
                "ffn_down": d * row_bytes(s.down_q, self.n_ffn) + r * self.n_ffn * 2 + r * d * 4 * 2,
                "head_argmax": self.n_voc * row_bytes(s.head_q, d) + r * d * 2 + r * 8}

    def launch_ffn_gate_up(self):
        s = self.shape
        with ops.cta_budget(self.ffn_ctas):
            ops.ffn_gate_up(s.ffn_q, self.w["gate"], self.w["up"], self.x, self.n_ffn, self.ws["ffn_gate_up"],
                            gact=self.gact)

    def launch_ffn_down(self):
        s = self.shape
        res = self.res if self.rank == 0 else None
        with ops.cta_budget(self.ffn_ctas):
            ops.gemv(s.down_q, self.w["down"], self.gact, s.dim, self.ws["ffn_down"], y=self.y, residual=res)

    def launch_head_argmax(self):
        s = self.shape
        with ops.cta_budget(self.head_ctas):
            ops.head_argmax(s.head_q, self.w["head"], self.h, self.n_voc, self.ws["head_argmax"],
                            row_offset=self.v0, out_keys=self.local_keys)

    def launch_ffn_down_peer(self):
        """This rank's down partial into its own peer buffer, flagged to every rank
        (tlx_gemv_peer)."""
        from . import _lib

        s = self.shape
        w = self.ws["ffn_down"]
        _lib.check(_lib.lib().tlx_gemv_peer(ops.qtype_id(s.down_q), ops._ptr(self.w["down"]), None,
                                            ops._ptr(self.gact), _lib.TLX_DT_IMAGE, 0, s.rows, s.dim, self.n_ffn,
                                            self.world, self.rank, self.peer.ptrs, self.ffn_ctas, ops._ptr(w.buf),
                                            w.nbytes, ops._stream(self.x)), "gemv_peer")

    def launch_head_argmax_peer(self):
        """This rank's vocabulary shard of the head, then the merge of the ranks' keys +
        greedy accept in its last CTA (tlx_head_argmax_peer)."""
        from . import _lib

        s = self.shape
        w = self.ws["head_argmax"]
        dt, ldx = ops._x_args(self.h)
        g = ops.grid("cuda") if s.head_q == "iq3_xxs" else None
        with ops.cta_budget(self.head_ctas):     # the staging of h is sized by the same plan
            _lib.check(_lib.lib().tlx_head_argmax_peer(
                ops.qtype_id(s.head_q), ops._ptr(self.w["head"]), ops._ptr(g), ops._ptr(self.h), dt, ldx, s.rows,
                self.n_voc, s.dim, self.v0, ops._ptr(self.out_max), ops._ptr(self.out_idx), ops._ptr(self.drafts),
                s.n_drafts, ops._ptr(self.accept_out), self.world, self.rank, self.peer.ptrs, self.head_ctas,
                ops._ptr(w.buf), w.nbytes, ops._stream(self.h)), "head_argmax_peer")

    def launch_finish(self):
        """y = residual + the ranks' down partials, and the step counter advances."""
        from . import _lib

        s = self.shape
        _lib.check(_lib.lib().tlx_peer_finish(self.world, self.rank, self.peer.ptrs, s.rows, s.dim,
                                              ops._ptr(self.res), s.dim, ops._ptr(self.y), s.dim,
                                              ops._ptr(self.finish_err), ops._stream(self.y)), "peer_finish")

    def launch(self):
        if self.comm == "peer":
            cur = torch.cuda.current_stream()
            self.side.wait_stream(cur)
            with torch.cuda.stream(self.side):
                self.launch_head_argmax_peer()
            self.launch_ffn_gate_up()
            self.launch_ffn_down_peer()
            cur.wait_stream(self.side)
            self.launch_finish()
            return
        self.launch_ffn_gate_up()
        self.launch_ffn_down()
        allreduce_partial(self.y, self.group)
        self.launch_head_argmax()
        gather_keys(self.local_keys, self.all_keys, self.group)
        ops.argmax_merge(self.all_keys, out_max=self.out_max, out_idx=self.out_idx, drafts=self.drafts,
                         accept_out=self.accept_out)

    COLLECTIVES = "NCCL all-reduce of the down partials + NCCL all-gather of the head keys"

    def launch_allreduce(self):
        allreduce_partial(self.y, self.group)

    def launch_gather_merge(self):
        gather_keys(self.local_keys, self.all_keys, self.group)
        ops.argmax_merge(self.all_keys, out_max=self.out_max, out_idx=self.out_idx, drafts=self.drafts,
                         accept_out=self.accept_out)

    def phase_times(self, time_graph, graph_of, max_over_ranks, torch_mod, reps: int = 20, replays: int = 5):
        """Device time (us, max over ranks) of each piece of the step alone, each
        captured `reps` times back to back in its own graph, and of the whole step; `gap`
        is the step minus the sum of the pieces.  The GEMVs are timed as their local
        (exchange-free) launches; with comm = "nccl" the collectives are timed alone too,
        with comm = "peer" the exchange lives inside the step's kernels, so the gap is
        the exchange plus the launch ramps."""
        out = {}
        pieces = [("ffn_gate_up", self.launch_ffn_gate_up), ("ffn_down", self.launch_ffn_down),
                  ("head_argmax", self.launch_head_argmax)]
        if self.comm == "nccl":
            pieces += [("allreduce_y", self.launch_allreduce), ("gather_merge_keys", self.launch_gather_merge)]
        # the same three kernels chained as in the step but without any exchange: the
        # step minus this is what the exchange costs
        chain = ("kernels_chained_no_exchange",
                 lambda: (self.launch_ffn_gate_up(), self.launch_ffn_down(), self.launch_head_argmax()))
        for name, fn in pieces:
            g = graph_of(lambda fn=fn: [fn() for _ in range(reps)], torch_mod)
            g.replay()
            out[name] = round(max_over_ranks(time_graph(g.replay, replays, torch_mod) / reps) * 1000, 2)
            del g
        out["step"] = round(max_over_ranks(time_graph(self.replay, replays * reps, torch_mod)) * 1000, 2)
        out["gap"] = round(out["step"] - sum(v for k, v in out.items() if k != "step"), 2)
        parts = {k: v for k, v in out.items() if k not in ("step",)}
        out["limiter"] = max(parts, key=parts.get)
        g = graph_of(lambda: [chain[1]() for _ in range(reps)], torch_mod)
        g.replay()
        out[chain[0]] = round(max_over_ranks(time_graph(g.replay, replays, torch_mod) / reps) * 1000, 2)
        del g
        return out

    def capture(self):
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(2):
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

    def release(self):
        """Drop the captured graph (it may hold NCCL work) before the process group goes,
        and unmap / free the peer buffers."""
        self.graph = None
        torch.cuda.synchronize()
        if self.peer is not None:
            self.peer.close(self.group)
            self.peer = None

    def set_inputs(self, x, h, res=None, drafts=None):
        self.x.copy_(x, non_blocking=True)
        self.h.copy_(h, non_blocking=True)
        if res is not None:
            self.res.copy_(res, non_blocking=True)
        if drafts is not None:
            self.drafts.copy_(drafts, non_blocking=True)

    def step_host(self, x_pinned, h_pinned, drafts_pinned, out_pinned):
        self.set_inputs(x_pinned, h_pinned, drafts=drafts_pinned)
        self.replay()
        out_pinned[:2].copy_(self.accept_out, non_blocking=True)
        out_pinned[2:].copy_(self.out_idx, non_blocking=True)


def shard_gguf_rows(raw: np.ndarray, r0: int, r1: int) -> np.ndarray:
    """Rows [r0, r1) of a GGUF matrix (row split: gate/up/head)."""
    return np.ascontiguousarray(raw[r0:r1])


def shard_gguf_cols(raw: np.ndarray, k0: int, k1: int, block_bytes: int) -> np.ndarray:
    """Columns [k0, k1) (multiples of 256) of a GGUF matrix (k split: down)."""
    return np.ascontiguousarray(raw[:, (k0 // 256) * block_bytes:(k1 // 256) * block_bytes])


class _GraphStep:
    """Capture / replay / release of one rank's step as a CUDA graph (the graph holds
    NCCL work, so release it before the process group is destroyed)."""

    graph = None

    def capture(self):
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(2):
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

    def release(self):
        self.graph = None
        torch.cuda.synchronize()


def expert_ranges(n_experts: int, world: int) -> list[tuple[int, int]]:
    """Contiguous expert ranges per rank (32 of 256 per rank at 8 ranks)."""
    return block_ranges(n_experts, world)


class ShardedMoeVerifyStep(_GraphStep):
    """The MoE verify layer, expert parallel: this rank's experts, then the sum of the
    ranks' partial layer outputs.

    comm = "peer" (default at world > 1): the partial goes into this rank's peer
    buffer with its flag raised in every rank's buffer (tlx_peer_publish), and
    tlx_peer_finish adds all ranks' partials read over NVLink, in rank order (the
    same bits on every rank); no collective library in the layer.
    comm = "nccl": one NCCL all-reduce of the partials."""

    def __init__(self, shape=None, rank: int = 0, world: int = 1, seed: int = 0, host: dict | None = None,
                 group=None, comm: str = "peer"):
        from .moe import MoeShape, MoeVerifyStep, synth_host

        if comm not in ("peer", "nccl"):
            raise ValueError(f"comm must be 'peer' or 'nccl', not {comm!r}")
        shape = shape if shape is not None else MoeShape()
        self.shape, self.rank, self.world, self.group = shape, rank, world, group
        self.comm = comm if world > 1 else "nccl"
        self.e0, self.e1 = expert_ranges(shape.experts, world)[rank]
        host = host if host is not None else synth_host(shape, seed)
        self.local = MoeVerifyStep(shape, host=host, e0=self.e0, e1=self.e1, shared=(rank == 0))
        self.peer = None
        if self.comm == "peer":
            self.peer = PeerComm(rank, world, shape.positions, shape.hidden, group)
            self.y = torch.empty_like(self.local.y)
            self.finish_err = torch.zeros(1, dtype=torch.int32, device=self.y.device)
        else:
            self.y = self.local.y

    def launch(self):
        self.local.launch()
        if self.peer is None:
            allreduce_partial(self.y, self.group)
            return
        from . import _lib

        s, part = self.shape, self.local.y
        L = _lib.lib()
        _lib.check(L.tlx_peer_publish(self.world, self.rank, self.peer.ptrs, s.positions, s.hidden, ops._ptr(part),
                                      s.hidden, ops._stream(part)), "peer_publish")
        _lib.check(L.tlx_peer_finish(self.world, self.rank, self.peer.ptrs, s.positions, s.hidden, None, 0,
                                     ops._ptr(self.y), s.hidden, ops._ptr(self.finish_err), ops._stream(part)),
                   "peer_finish")

    def release(self):
        """Drop the graph, then unmap / free the peer buffers (collective)."""
        self.graph = None
        torch.cuda.synchronize()
        if self.peer is not None:
            self.peer.close(self.group)
            self.peer = None

    def set_inputs(self, h, hres=None):
        self.local.set_inputs(h, hres if self.rank == 0 else None)

    def touched_bytes(self) -> int:
        return self.local.touched_bytes()


class ShardedPrefillFFN(_GraphStep):
    """The prefill FFN, tensor parallel: this rank's gate/up rows and down k range,
    then one all-reduce of the partial [tokens][dim] output."""

    def __init__(self, shape=None, rank: int = 0, world: int = 1, seed: int = 0, weights: dict | None = None,
                 group=None):
        from .prefill import PrefillShape, PrefillWorkspace

        ops.require_device()
        s = self.shape = shape if shape is not None else PrefillShape()
        self.rank, self.world, self.group = rank, world, group
        b0, b1 = block_ranges(s.ffn // 256, world)[rank]
        self.f0, self.f1 = 256 * b0, 256 * b1
        self.n_ffn = self.f1 - self.f0
        if self.n_ffn <= 0:
            raise ValueError(f"rank {rank} of {world} has an empty FFN shard")
        if weights is None:
            # this rank's slices of the seeded model PrefillFFN(seed) uses
            weights = {"gate": synth_tiled(s.ffn_q, s.ffn, s.dim, seed + 1, rows=(self.f0, self.f1)),
                       "up": synth_tiled(s.ffn_q, s.ffn, s.dim, seed + 2, rows=(self.f0, self.f1)),
                       "down": synth_tiled(s.down_q, s.dim, s.ffn, seed + 3, cols=(self.f0, self.f1))}
        self.w = weights
        self.x = torch.zeros((s.tokens, s.dim), dtype=torch.bfloat16, device="cuda")
        self.act = torch.empty((s.tokens, self.n_ffn), dtype=torch.float32, device="cuda")
        self.y = torch.empty((s.tokens, s.dim), dtype=torch.float32, device="cuda")
        self.ws = PrefillWorkspace(s.tokens, s.dim)
        self.ws_down = PrefillWorkspace(s.tokens, self.n_ffn)

    def flops_per_rank(self) -> int:
        s = self.shape
        return 2 * s.tokens * s.dim * self.n_ffn * 3

    def launch(self):
        from .prefill import gate_up, gemm

        s = self.shape
        gate_up(s.ffn_q, self.w["gate"], self.w["up"], self.x, self.n_ffn, self.ws, act=self.act)
        gemm(s.down_q, self.w["down"], self.act, s.dim, self.ws_down, y=self.y)
        allreduce_partial(self.y, self.group)

    def set_inputs(self, x):
        self.x.copy_(x, non_blocking=True)
