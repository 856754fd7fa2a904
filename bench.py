"""Benchmark: the K=11 speculative verify step (BASELINE configs 2 + 3) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = IQ3_XXS gate/up (+SiLU) -> Q6_K down over 11 rows, then the Q6_K
151936-vocab LM head fused with per-row argmax and greedy accept.  value =
weight bytes streamed per step / step time (GB/s, whole job); us_per_step is
reported beside it.  At N > 1 (torchrun) the step is sharded: FFN rows (gate/up)
and the matching k range of down per rank with one NCCL all-reduce of the
11 x 5120 fp32 partial outputs; the head by vocabulary with one NCCL all-gather
of 11 packed (max, index) keys per rank.

--impl reference times the reference algorithm's CPU implementation (the numpy
oracle port, all host cores) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "µs per K=11 verify step + weight GB/s (% HBM roofline) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 2 ** 20
# DRAM bytes (read + write) per head row of the fused head/argmax launch, from one
# ncu --set full capture of that kernel alone at the full vocabulary 151936
# (profiles/tile_gemv_head_argmax_full.txt: 640.37 MB read + 5.62 MB written),
# scaled to a launch by its row count (a vocabulary shard at N > 1)
HEAD_TRAFFIC_BYTES_PER_ROW = (640_373_248 + 5_624_320) / 151936


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------------ clocks ----
class ClockSampler:
    """SM clock, power and clock-event reasons of this rank's GPU, sampled from a
    background thread while the timed legs run.  NVML (nvidia_ml_py) is polled every
    2 ms, so even a few-millisecond timed region gets samples; without NVML,
    ``nvidia-smi -lms 50`` is read instead.  Read-only: no GPU setting is touched."""

    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_s: float = 0.002):
        self.gpu, self.period = gpu_index, period_s
        self.proc, self.samples, self.stop = None, [], threading.Event()
        self.source = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.gpu)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def _poll_nvml(self, nv, hd):
        mx = float(nv.nvmlDeviceGetMaxClockInfo(hd, nv.NVML_CLOCK_SM))
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(hd, nv.NVML_CLOCK_SM)), mx,
                                     nv.nvmlDeviceGetPowerUsage(hd) / 1000.0, int(get_reasons(hd))))
            except Exception:
                pass
            time.sleep(self.period)

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            try:
                bits = sum(self.REASONS[nm] for nm, v in zip(("hw_slowdown", "hw_thermal_slowdown",
                                                              "sw_thermal_slowdown", "sw_power_cap"), parts[5:9])
                           if v.lower() == "active")
                self.samples.append((float(parts[1]), float(parts[2]), float(parts[3]), bits))
            except (ValueError, IndexError):
                continue

    def __enter__(self):
        try:
            nv, hd = self._nvml_handle()
            self.t = threading.Thread(target=self._poll_nvml, args=(nv, hd), daemon=True)
            self.source = "nvml, 2 ms"
        except Exception:
            try:
                self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                              "--format=csv,noheader,nounits", "-lms", "50"],
                                             stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.t = threading.Thread(target=self._read_smi, daemon=True)
                self.source = "nvidia-smi, 50 ms"
            except Exception:
                return self
        self.t.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.source is not None:
            self.t.join(timeout=5)

    def summary(self):
        if not self.samples:
            return None
        reasons = sorted(nm for nm, bit in self.REASONS.items() if any(s[3] & bit for s in self.samples))
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": max(s[1] for s in self.samples),
                "power_w_max": round(max(s[2] for s in self.samples), 1), "reasons": reasons,
                "samples": len(self.samples), "source": self.source,
                "window": "the timed step replays, the per-kernel graphs and the end-to-end steps"}


# ------------------------------------------------------------- CPU port ------
# The verify step on host cores: the reference's numpy path, restated by the oracle
# package (GGUF blocks dequantised to fp32 as engine/pack_w4.py:39-69 and
# engine/mm/MM_P2_ports.py:21-45 do, then an fp32 matmul, ``W.astype(f32) @ xh`` of
# lineage/a3a/a3a_bench.py:176).  Every matrix is split by rows over worker
# processes; each worker generates its own rows of the seeded model once
# (synth.matrix_rows, the rows the GPU arm packs) and keeps them.  One step is the
# whole workload, nothing scaled or extrapolated:
#   phase 1  gate/up rows -> act = silu(g) * u;  head rows -> per-token (max, row)
#   phase 2  down rows over the full act, + residual
# then the host merges the head's (max, row) pairs (strict >, lowest row on ties,
# as engine/amx3.cu:124-128) and runs greedy accept (engine/accept11k.cu:25-36).

DEQUANT_ROWS = 2048          # rows dequantised at a time (bounded fp32 temporaries)


def _matrices(dims, seed):
    """name -> (qtype, n_rows, k, seed) of VerifyStep(seed)'s model."""
    dim, ffn, vocab, ffn_q, down_q, head_q = dims
    return {"gate": (ffn_q, ffn, dim, seed + 1), "up": (ffn_q, ffn, dim, seed + 2),
            "down": (down_q, dim, ffn, seed + 3), "head": (head_q, vocab, dim, seed + 4)}


def _cpu_worker(conn, dims, seed, mine):
    """One host process of CpuVerifyStep: owns rows mine[name] = (r0, r1) of each matrix."""
    from threadpoolctl import threadpool_limits

    import oracle
    from thunderllamax_b200 import synth

    mats = _matrices(dims, seed)
    raw = {nm: synth.matrix_rows(q, n, k, sd, *mine[nm]) for nm, (q, n, k, sd) in mats.items()}

    def matmul_rows(nm, x):
        """[rows of mine][tokens] = W[rows] @ x^T in fp32, dequantising DEQUANT_ROWS at a time."""
        q, _, k, _ = mats[nm]
        r = raw[nm]
        out = np.empty((r.shape[0], x.shape[0]), dtype=np.float32)
        for a in range(0, r.shape[0], DEQUANT_ROWS):
            W = oracle.dequant(q, r[a:a + DEQUANT_ROWS], k)
            out[a:a + W.shape[0]] = W @ x.T
        return out

    conn.send("ready")
    with threadpool_limits(1):
        while True:
            msg = conn.recv()
            if msg[0] == "stop":
                break
            if msg[0] == "phase1":
                x, h = msg[1], msg[2]
                g, u = matmul_rows("gate", x), matmul_rows("up", x)
                with np.errstate(over="ignore"):                                  # exp(-g) -> inf: act -> -0
                    act = (g / (np.float32(1) + np.exp(-g))) * u               # [rows][tokens]
                lg = matmul_rows("head", h)                                       # [rows][tokens]
                best = np.argmax(lg, axis=0)                                      # first (lowest) row of the max
                conn.send((act, lg[best, np.arange(lg.shape[1])], best + mine["head"][0]))
            elif msg[0] == "phase2":
                conn.send(matmul_rows("down", msg[1]))


class CpuVerifyStep:
    """The K=11 verify step on `procs` host processes (one thread each)."""

    def __init__(self, shape, seed: int, procs: int):
        import multiprocessing as mp

        self.shape, self.procs = shape, max(1, int(procs))
        dims = (shape.dim, shape.ffn, shape.vocab, shape.ffn_q, shape.down_q, shape.head_q)
        mats = _matrices(dims, seed)
        split = {nm: [((n * i) // self.procs, (n * (i + 1)) // self.procs) for i in range(self.procs)]
                 for nm, (_, n, _, _) in mats.items()}
        ctx = mp.get_context("spawn")
        self.conns, self.workers = [], []
        for i in range(self.procs):
            a, b = ctx.Pipe()
            w = ctx.Process(target=_cpu_worker, args=(b, dims, seed, {nm: split[nm][i] for nm in split}), daemon=True)
            w.start()
            self.conns.append(a)
            self.workers.append(w)
        for c in self.conns:
            if c.recv() != "ready":
                raise RuntimeError("CPU worker failed to start")

    def step(self, x, h, res, drafts):
        """x, h [tokens][dim] fp32 (the bf16 rows), res [tokens][dim] fp32, drafts int32.
        Returns (y [tokens][dim], ids [tokens], (m, bonus))."""
        for c in self.conns:
            c.send(("phase1", x, h))
        parts = [c.recv() for c in self.conns]
        act = np.concatenate([p[0] for p in parts], axis=0).T.copy()            # [tokens][ffn]
        for c in self.conns:
            c.send(("phase2", act))
        y = np.concatenate([c.recv() for c in self.conns], axis=0).T + res
        best_v = np.full(x.shape[0], -np.inf, dtype=np.float32)
        best_i = np.zeros(x.shape[0], dtype=np.int64)
        for _, v, i in parts:                                                      # workers in row order
            take = v > best_v
            best_v = np.where(take, v, best_v)
            best_i = np.where(take, i, best_i)
        m = 0
        while m < len(drafts) and best_i[m] == drafts[m]:
            m += 1
        return y, best_i, (m, int(best_i[m]))

    def close(self):
        for c in self.conns:
            try:
                c.send(("stop",))
            except Exception:
                pass
        for w in self.workers:
            w.join(timeout=10)


def _cpu_inputs(shape, seed=1234):
    """The GPU arm's step inputs (same seeds), as fp32 host arrays."""
    from thunderllamax_b200 import synth

    rng = np.random.default_rng(seed)
    x = synth.bf16_bits_to_f32(synth.bf16_normal(rng, (shape.rows, shape.dim)))
    h = synth.bf16_bits_to_f32(synth.bf16_normal(rng, (shape.rows, shape.dim)))
    return x, h, np.zeros((shape.rows, shape.dim), np.float32)


def time_cpu_steps(cpu, shape, warmup, steps, drafts=None):
    """Mean wall time (s) of `steps` whole CPU verify steps after `warmup` ones."""
    x, h, res = _cpu_inputs(shape)
    drafts = np.zeros(shape.n_drafts, np.int32) if drafts is None else drafts
    for _ in range(warmup):
        cpu.step(x, h, res, drafts)
    t0 = time.perf_counter()
    for _ in range(steps):
        out = cpu.step(x, h, res, drafts)
    return (time.perf_counter() - t0) / max(1, steps), out


# ------------------------------------------------------------- helpers -------
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def emit(obj):
    print(json.dumps(obj), flush=True)


WORKLOAD = ("K=11 verify step: IQ3_XXS gate/up 17408x5120 (+SiLU) -> Q6_K down 5120x17408 -> Q6_K head "
            "151936x5120 fused argmax + greedy accept")


def bench_config(shape, ws):
    """The `config` both arms print (identical keys and values for the same run)."""
    return {"workload": WORKLOAD, "rows": shape.rows, "ffn": shape.ffn, "vocab": shape.vocab,
            "weight_bytes_per_step": sum(shape.weight_bytes().values()),
            "parallelism": f"tp{ws}" if ws > 1 else "single"}


def run_reference(args):
    ws, rank, _ = dist_env()
    from thunderllamax_b200.verify import VerifyShape

    shape = VerifyShape()
    if rank != 0:
        return 0
    procs = os.cpu_count() or 1
    cpu = CpuVerifyStep(shape, 0, procs)
    try:
        sec, _ = time_cpu_steps(cpu, shape, args.warmup, args.steps)
    finally:
        cpu.close()
    total = sum(shape.weight_bytes().values())
    gbs = total / sec / 1e9
    sample = (f"{args.steps} whole verify steps (all four matrices, {total / 1e6:.0f} MB of GGUF blocks each) after "
              f"{args.warmup} warm-up steps; numpy fp32 dequant + fp32 matmul (the reference's numpy path, restated "
              f"by the oracle package) in {procs} worker processes of one thread each (os.cpu_count() = "
              f"{os.cpu_count()}); wall clock per step")
    emit({"metric": METRIC, "impl": "reference", "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1000, 3),
          "us_per_step": round(sec * 1e6, 1), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
          "dtype": "f32", "data": "synthetic (seeded GGUF-layout IQ3_XXS/Q6_K blocks and bf16 N(0,1) rows per "
                                  "BASELINE configs 2+3)",
          "config": bench_config(shape, ws),
          "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": procs, "kind": "port", "sample": sample},
          "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    return 0


def time_graph(fn_replay, steps, torch):
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(steps):
        fn_replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps  # ms


def measure_moe(args, torch, peak):
    """BASELINE config 4 (MoE verify layer, 5 positions) on this GPU: graph replays
    timed with CUDA events; bytes = router + shared + distinct routed experts."""
    from thunderllamax_b200 import moe, synth

    shape = moe.MoeShape()
    step = moe.MoeVerifyStep(shape, seed=0)
    rng = np.random.default_rng(4321)
    bits = synth.bf16_normal(rng, (shape.positions, shape.hidden))
    h = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
    hres = torch.from_numpy(rng.standard_normal((shape.positions, shape.hidden)).astype(np.float32))
    step.set_inputs(h.cuda(), hres.cuda())
    step.capture()
    for _ in range(5):
        step.replay()
    n = max(20, min(2000, args.steps))
    ms = time_graph(step.replay, n, torch)
    touched = step.touched_bytes()
    out = {"workload": "MoE verify layer: fp32 router 2048->256 top-8 + shared, IQ4_XS experts 2048->512->2048, "
                       "5 positions",
           "us_per_step": round(ms * 1000, 2), "bytes_per_step": touched,
           "gbs": round(touched / (ms * 1e-3) / 1e9, 1),
           "frac_of_peak": round(touched / (ms * 1e-3) / 1e9 / peak, 4),
           "launches_per_step": step.LAUNCHES_PER_STEP, "err_word": step.ws.error()}
    if not args.no_cpu:
        import oracle

        t0 = time.perf_counter()
        oracle.moe_verify_f64(synth.bf16_bits_to_f32(bits).astype(np.float64), step.host["wr"], step.host["wsh"],
                              step.host["gate"], step.host["up"], step.host["down"], step.host["sgate"],
                              step.host["sup"], step.host["sdown"], hres=hres.numpy())
        cpu_s = time.perf_counter() - t0
        out["cpu_baseline"] = {"us_per_step": round(cpu_s * 1e6, 1), "cores": 1, "kind": "port",
                               "sample": "one full MoE step of the numpy f64 oracle"}
    return out


def measure_prefill(args, torch, weights):
    """BASELINE config 5 (2048-token FFN, tcgen05): CUDA events around the two GEMM
    launches (+ bf16 -> fp16 token staging); FLOPs = 2 * tokens * dim * ffn * 3."""
    from thunderllamax_b200 import prefill, synth

    shape = prefill.PrefillShape()
    step = prefill.PrefillFFN(shape, weights=weights)
    rng = np.random.default_rng(777)
    step.x.copy_(torch.from_numpy(synth.bf16_normal(rng, (shape.tokens, shape.dim)).view(np.int16))
                 .view(torch.bfloat16))
    for _ in range(3):
        step.launch()
    n = 20
    ms = time_graph(step.launch, n, torch)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
        peak, kind = float(peaks["bf16_tflops"]), "measured cuBLAS bf16 burst"
    except Exception:
        peak, kind = 1590.0, "fallback"
    tflops = shape.flops() / (ms * 1e-3) / 1e12
    out = {"workload": "prefill FFN: 2048 tokens, IQ3_XXS gate/up 5120->17408 (+SiLU) -> Q6_K down 17408->5120, "
                       "fp16 tcgen05 with fp32 TMEM accumulators",
           "ms_per_step": round(ms, 4), "flops_per_step": shape.flops(), "tflops": round(tflops, 1),
           "peak_tflops": peak, "peak_kind": kind, "frac_of_peak": round(tflops / peak, 4),
           "launches_per_step": 3, "err_word": [step.ws.error(), step.ws_down.error()]}

    # the W4A8 tier in place of the fp16 gate/up: fp16 tokens -> int8 (quantiser), then
    # the gate/up on the linearised codebook (token staging + the tcgen05 contraction)
    gu_flops = 2 * shape.tokens * shape.dim * shape.ffn * 2
    x16 = step.x.to(torch.float16)
    xq = torch.empty((shape.tokens, shape.dim), dtype=torch.int8, device="cuda")
    sx = torch.empty((shape.tokens, shape.dim // 128), dtype=torch.float32, device="cuda")
    rs = torch.empty_like(sx, dtype=torch.int32)
    lut = prefill.lut8()

    def fp16_gate_up():
        prefill.gate_up(shape.ffn_q, step.w["gate"], step.w["up"], step.x, shape.ffn, step.ws, act=step.act)

    def w4a8_gate_up():
        prefill.act_quant_q8(x16, xq=xq, sx=sx, rs=rs)
        prefill.w4a8_gate_up(step.w["gate"], step.w["up"], xq, sx, shape.ffn, step.ws, act=step.act, lut=lut)

    for fn in (fp16_gate_up, w4a8_gate_up):
        for _ in range(3):
            fn()
    ms16 = time_graph(fp16_gate_up, n, torch)
    ms8 = time_graph(w4a8_gate_up, n, torch)
    out["w4a8_gate_up"] = {
        "workload": "gate/up only (5120 -> 17408 x2 + SiLU, 2048 tokens): W4A8 tier (int8 tokens, linearised "
                    "IQ3_XXS levels; quantiser + token staging + tcgen05 contraction) against the fp16 tier "
                    "(bf16 -> fp16 staging + the same contraction)",
        "ms": round(ms8, 4), "tflops": round(gu_flops / (ms8 * 1e-3) / 1e12, 1),
        "fp16_tier_ms": round(ms16, 4), "fp16_tier_tflops": round(gu_flops / (ms16 * 1e-3) / 1e12, 1),
        "launches": 3, "err_word": step.ws.error()}
    return out


def measure_moe_exchange(torch, dist, shape, ws, max_over_ranks, reps: int = 20):
    """The MoE layer's cross-GPU exchange alone, two ways, each captured `reps` times
    in one CUDA graph and timed with CUDA events (max over ranks):
    - replicated positions (what ShardedMoeVerifyStep does): every rank holds all P
      positions, computes its experts' share of the layer output, and one NCCL
      all-reduce sums the [P][hidden] fp32 partials;
    - token dispatch: positions owned round-robin by ranks, an NCCL all-to-all sends
      each owner's bf16 rows to every rank (the experts of a position can sit on any
      rank), and a second all-to-all returns each rank's fp32 partial rows to the
      owners (which then add them).
    Every rank takes the same collective steps in the same order."""
    P, H = shape.positions, shape.hidden
    per = -(-P // ws)                                # positions per owner, padded
    y = torch.zeros((P, H), dtype=torch.float32, device="cuda")
    send_h = torch.zeros((ws * per, H), dtype=torch.bfloat16, device="cuda")
    recv_h = torch.empty_like(send_h)
    send_y = torch.zeros((ws * per, H), dtype=torch.float32, device="cuda")
    recv_y = torch.empty_like(send_y)

    def allreduce():
        for _ in range(reps):
            dist.all_reduce(y)

    def a2a():
        for _ in range(reps):
            dist.all_to_all_single(recv_h, send_h)
            dist.all_to_all_single(recv_y, send_y)

    res = {}
    for name, fn in (("allreduce_replicated_us", allreduce), ("all_to_all_dispatch_combine_us", a2a)):
        g = _graph_of(fn, torch)
        g.replay()
        dist.barrier()
        res[name] = round(max_over_ranks(time_graph(g.replay, 5, torch) / reps) * 1000, 2)
        del g
    torch.cuda.synchronize()
    res["bytes"] = {"allreduce": P * H * 4, "dispatch": ws * per * H * 2, "combine": ws * per * H * 4}
    res["chosen"] = ("replicated positions + one all-reduce" if res["allreduce_replicated_us"]
                     <= res["all_to_all_dispatch_combine_us"] else "token dispatch (all-to-all) would be faster")
    return res


def measure_sharded_extras(args, torch, ws, rank, peak):
    """At N > 1: the MoE verify layer expert parallel and the prefill FFN tensor
    parallel over all ranks (ShardedMoeVerifyStep / ShardedPrefillFFN, one NCCL
    all-reduce each), CUDA-graph replays timed with CUDA events on every rank, the
    max over ranks reported.  Every rank runs this, in the same order."""
    import torch.distributed as dist
    from thunderllamax_b200 import synth
    from thunderllamax_b200.dist import ShardedMoeVerifyStep, ShardedPrefillFFN
    from thunderllamax_b200.moe import MoeShape
    from thunderllamax_b200.prefill import PrefillShape

    def max_over_ranks(v):
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    out = {}
    if not args.no_moe:
        from thunderllamax_b200.moe import synth_host

        shape = MoeShape()
        host = synth_host(shape, 0)
        rng = np.random.default_rng(4321)
        bits = synth.bf16_normal(rng, (shape.positions, shape.hidden))
        hres = rng.standard_normal((shape.positions, shape.hidden)).astype(np.float32)
        res, ys, err = {}, {}, 0
        for comm in ("peer", "nccl"):
            step = ShardedMoeVerifyStep(shape, rank, ws, host=host, comm=comm)
            step.set_inputs(torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda(),
                            torch.from_numpy(hres).cuda())
            step.capture()
            for _ in range(5):
                step.replay()
            dist.barrier()
            torch.cuda.synchronize()
            res[comm] = max_over_ranks(time_graph(step.replay, max(20, min(2000, args.steps)), torch))
            ys[comm] = step.y.clone()
            touched = sum_over_ranks(step.touched_bytes())
            err |= step.local.ws.error() | (int(step.finish_err.item()) if comm == "peer" else 0)
            step.release()
            del step
        ms = res["peer"]
        y_err = float(((ys["peer"] - ys["nccl"]).abs().amax(dim=1) / ys["nccl"].norm(dim=1)).max())
        out["moe_verify"] = {"workload": f"MoE verify layer, expert parallel over {ws} GPUs "
                                         f"({shape.experts // ws} experts per rank), router replicated, the "
                                         "ranks' fp32 partials summed over peer memory (tlx_peer_publish + "
                                         "tlx_peer_finish)",
                             "us_per_step": round(ms * 1000, 2), "bytes_per_step": int(touched),
                             "gbs": round(touched / (ms * 1e-3) / 1e9, 1),
                             "frac_of_peak": round(touched / (ms * 1e-3) / 1e9 / (peak * ws), 4),
                             "us_per_step_nccl_allreduce": round(res["nccl"] * 1000, 2),
                             "peer_vs_nccl_y_max_err_over_row_norm": y_err,
                             "timing": "CUDA graph replay, max over ranks", "err_word": err}
        out["moe_exchange"] = measure_moe_exchange(torch, dist, shape, ws, max_over_ranks)
    if not args.no_prefill:
        shape = PrefillShape()
        step = ShardedPrefillFFN(shape, rank, ws, seed=0)
        rng = np.random.default_rng(777)
        step.set_inputs(torch.from_numpy(synth.bf16_normal(rng, (shape.tokens, shape.dim)).view(np.int16))
                        .view(torch.bfloat16).cuda())
        step.capture()
        for _ in range(3):
            step.replay()
        dist.barrier()
        torch.cuda.synchronize()
        ms = max_over_ranks(time_graph(step.replay, 20, torch))
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                bf16_peak, kind = float(json.load(f)["bf16_tflops"]), "measured cuBLAS bf16 burst"
        except Exception:
            bf16_peak, kind = 1590.0, "fallback"
        tflops = shape.flops() / (ms * 1e-3) / 1e12
        out["prefill_ffn"] = {"workload": f"prefill FFN 2048 tokens, tensor parallel over {ws} GPUs (gate/up rows, "
                                          "down k), one NCCL all-reduce of the 2048 x 5120 fp32 partials",
                              "ms_per_step": round(ms, 4), "flops_per_step": shape.flops(),
                              "tflops": round(tflops, 1), "peak_tflops": bf16_peak * ws, "peak_kind": kind + " x N",
                              "frac_of_peak": round(tflops / (bf16_peak * ws), 4),
                              "timing": "CUDA graph replay, max over ranks",
                              "err_word": [step.ws.error(), step.ws_down.error()]}
        step.release()
        del step
    return out


def _timed_cold(launch, n, torch):
    """Mean device time (ms) of `launch` with L2 flushed before each call (a 256 MB
    read outside the timed events, leaving clean lines): for working sets that would
    otherwise stay in the 126 MB L2 between iterations."""
    flush = torch.ones(256 << 18, dtype=torch.int32, device="cuda")
    total = 0.0
    for _ in range(n):
        flush.sum()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        launch()
        e1.record()
        torch.cuda.synchronize()
        total += e0.elapsed_time(e1)
    return total / n


def measure_attn_qkv(args, torch, peak):
    """aq3k8v11 at the reference shape (q 12288 / k 1024 IQ3_XXS, v 1024 Q4_K, k 5120,
    11 rows, fp16 x): staging + three GEMVs, cold L2; bytes = weights + x + outputs."""
    from thunderllamax_b200 import ops, synth
    from thunderllamax_b200.verify import synth_tiled

    m, k, nq, nk, nv = 11, 5120, 12288, 1024, 1024
    wq, wk, wv = synth_tiled("iq3_xxs", nq, k, 31), synth_tiled("iq3_xxs", nk, k, 32), synth_tiled("q4_k", nv, k, 33)
    rng = np.random.default_rng(34)
    x = torch.from_numpy(synth.bf16_bits_to_f32(synth.bf16_normal(rng, (m, k))).astype(np.float16)).cuda()
    proj = ops.AttnProjections(m, k, nq, nk, nv, torch.float16)
    outs = [torch.empty((m, n), dtype=torch.float16, device="cuda") for n in (nq, nk, nv)]
    for _ in range(3):
        proj(wq, wk, wv, x, *outs)
    # one CUDA graph for the five launches, so the timed region is device time
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        proj(wq, wk, wv, x, *outs)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        proj(wq, wk, wv, x, *outs)
    ms = _timed_cold(graph.replay, 20, torch)
    nbytes = (nq + nk) * synth.row_bytes("iq3_xxs", k) + nv * synth.row_bytes("q4_k", k) + m * k * 2 + m * (nq + nk + nv) * 2
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": "aq3k8v11: q 12288 + k 1024 rows IQ3_XXS, v 1024 rows Q4_K, k 5120, 11 fp16 rows",
            "us_per_call": round(ms * 1000, 2), "bytes_per_call": int(nbytes), "gbs": round(gbs, 1),
            "frac_of_peak": round(gbs / peak, 4), "launches_per_call": 5, "graph": "CUDA graph replay",
            "l2": "flushed before each call",
            "err_word": proj.error()}


RAMP_S = 0.3


def ramp_replays(replay, torch, dist=None) -> int:
    """Untimed replays for about RAMP_S seconds (the count is rank 0's, broadcast so
    that every rank replays, and so exchanges, the same number of steps)."""
    import time

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    replay()
    torch.cuda.synchronize()
    one = max(time.perf_counter() - t0, 1e-5)
    n = torch.tensor([min(20000, max(10, int(RAMP_S / one)))], device="cuda")
    if dist is not None:
        dist.broadcast(n, 0)
    n = int(n.item())
    for _ in range(n):
        replay()
    torch.cuda.synchronize()
    return n


def _graph_of(fn, torch):
    """Capture fn (after one eager call on a side stream) as a CUDA graph."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        fn()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph


def measure_gdn_qkv(args, torch, peak):
    """q5g8v11 at the reference shape (qkv 10240 rows Q5_K, gate 6144 rows IQ3_XXS,
    k 5120, 11 fp16 rows): staging + two GEMVs, cold L2; bytes = weights + x + outputs."""
    from thunderllamax_b200 import ops, synth
    from thunderllamax_b200.verify import synth_tiled

    m, k, nqkv, ngate = 11, 5120, 10240, 6144
    wqkv, wg = synth_tiled("q5_k", nqkv, k, 41), synth_tiled("iq3_xxs", ngate, k, 42)
    rng = np.random.default_rng(43)
    x = torch.from_numpy(synth.bf16_bits_to_f32(synth.bf16_normal(rng, (m, k))).astype(np.float16)).cuda()
    proj = ops.GdnProjections(m, k, nqkv, ngate, torch.float16)
    outs = [torch.empty((m, n), dtype=torch.float16, device="cuda") for n in (nqkv, ngate)]
    for _ in range(3):
        proj(wqkv, wg, x, *outs)
    graph = _graph_of(lambda: proj(wqkv, wg, x, *outs), torch)
    ms = _timed_cold(graph.replay, 20, torch)
    wbytes = nqkv * synth.row_bytes("q5_k", k) + ngate * synth.row_bytes("iq3_xxs", k)
    nbytes = wbytes + m * k * 2 + m * (nqkv + ngate) * 2
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": "q5g8v11: qkv 10240 rows Q5_K + gate 6144 rows IQ3_XXS, k 5120, 11 fp16 rows",
            "us_per_call": round(ms * 1000, 2), "bytes_per_call": int(nbytes), "gbs": round(gbs, 1),
            "frac_of_peak": round(gbs / peak, 4), "launches_per_call": 4, "graph": "CUDA graph replay",
            "l2": "flushed before each call", "err_word": proj.error()}


def measure_o_proj(args, torch, peak):
    """op38nw32_11 (IQ3_XXS) and k3aonw32_11 (Q8_0): attn_out [11][5120] = W z with
    z [11][6144] fp16, fp16 out, one GEMV each (its staging included), cold L2."""
    from thunderllamax_b200 import ops, synth
    from thunderllamax_b200.verify import synth_tiled

    m, n, k = 11, 5120, 6144
    rng = np.random.default_rng(44)
    z = torch.from_numpy(synth.bf16_bits_to_f32(synth.bf16_normal(rng, (m, k))).astype(np.float16)).cuda()
    out = {}
    for qt, seed in (("iq3_xxs", 45), ("q8_0", 46)):
        w = synth_tiled(qt, n, k, seed)
        ws = ops.Workspace.for_shape(ops.MODE_STORE, qt, n, k, m, torch.float16)
        y = torch.empty((m, n), dtype=torch.float16, device="cuda")
        fn = lambda: ops.gemv(qt, w, z, n, ws, y=y)  # noqa: E731
        for _ in range(3):
            fn()
        graph = _graph_of(fn, torch)
        ms = _timed_cold(graph.replay, 20, torch)
        nbytes = n * synth.row_bytes(qt, k) + m * k * 2 + m * n * 2
        gbs = nbytes / (ms * 1e-3) / 1e9
        out["op38nw32_11" if qt == "iq3_xxs" else "k3aonw32_11"] = {
            "qtype": qt, "us_per_call": round(ms * 1000, 2), "bytes_per_call": int(nbytes), "gbs": round(gbs, 1),
            "frac_of_peak": round(gbs / peak, 4), "err_word": ws.error()}
        del graph
    out["workload"] = "GDN o-projection 5120 x 6144, 11 fp16 rows, CUDA graph replay, L2 flushed before each call"
    return out


def measure_lookup(args, torch, peak):
    """lookup11_nw32 (the K = 10 n-gram drafter) over a 100K-token history with the
    suffix planted near the start (the whole range is scanned); CUDA graph replay.
    Bytes = the history scanned (4 B per start)."""
    import time
    from thunderllamax_b200 import ops
    import oracle

    n = 100_000
    rng = np.random.default_rng(47)
    h = rng.integers(0, 50_000, n).astype(np.int32)
    h[n - 8:n] = h[1000:1008]
    hist = torch.from_numpy(h).cuda()
    pos = torch.tensor([n], dtype=torch.int32, device="cuda")
    cyc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ring = torch.zeros(10, dtype=torch.int32, device="cuda")
    l_hist = torch.zeros(4, dtype=torch.int32, device="cuda")
    lk = ops.Lookup(10)
    fn = lambda: lk(hist, pos, cyc, ring, l_hist)  # noqa: E731
    for _ in range(3):
        fn()

    def twenty():
        for _ in range(20):
            fn()
    graph = _graph_of(twenty, torch)          # 20 back-to-back launches per replay
    ms = time_graph(graph.replay, 10, torch) / 20
    t0 = time.perf_counter()
    ref = oracle.lookup_ngram(h, n, 10, 19)
    cpu_ms = (time.perf_counter() - t0) * 1000
    ok = int(l_hist[0]) == ref[0] and np.array_equal(ring.cpu().numpy(), ref[1])
    return {"workload": "lookup11_nw32: K = 10 drafts from a 100000-token history (8-token suffix, full scan)",
            "us_per_call": round(ms * 1000, 2), "bytes_per_call": 4 * n,
            "gbs": round(4 * n / (ms * 1e-3) / 1e9, 1), "launches_per_call": 1, "graph": "CUDA graph replay",
            "matches_oracle": bool(ok),
            "cpu_baseline": {"us_per_call": round(cpu_ms * 1000, 1), "cores": 1, "kind": "port",
                             "sample": "the numpy oracle on the same history"}}


def measure_attention(args, torch, peak):
    """Split-KV int8 attention of one full-attention layer for the 11 verify rows at
    32K and 100K tokens of context (spk_pre11 + spk_a11 + spk_c11 as tlx_attn_pre +
    tlx_attn_split + tlx_attn_combine), 10 layers per CUDA graph replay.  Bytes =
    the K / V cache rows and scales read."""
    from thunderllamax_b200 import ops
    import oracle

    rows, ctx = 11, 100352
    rng = np.random.default_rng(48)
    q = torch.from_numpy(rng.standard_normal((rows, 12288)).astype(np.float16)).cuda()
    k = torch.from_numpy(rng.standard_normal((rows, 1024)).astype(np.float16)).cuda()
    v = torch.from_numpy(rng.standard_normal((rows, 1024)).astype(np.float16)).cuda()
    qn, kn = torch.ones(256, device="cuda"), torch.ones(256, device="cuda")
    fr = torch.from_numpy(oracle.rope_freqs()).cuda()
    kv = torch.randint(1, 256, (8, ctx, 256), dtype=torch.uint8, device="cuda")
    sc = (torch.rand((8, ctx, 8), device="cuda") * 0.02 + 0.01).half()
    at = ops.Attention(rows, ctx)
    out = {"workload": "full-attention layer, 11 verify rows, 24 q / 4 KV heads x 256, int8 KV cache",
           "graph": "CUDA graph replay, 10 layers per replay"}
    for pos in (32000, 100000):
        pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
        qw16 = torch.empty((rows, 24, 256), dtype=torch.float16, device="cuda")
        ao = torch.empty((rows, 6144), dtype=torch.float16, device="cuda")

        def layer():
            at.pre(q, k, v, qn, kn, fr, pos_t, kv, sc, qw16)
            at.decode(kv, sc, qw16, q, pos_t, ao)
        layer()

        def ten():
            for _ in range(10):
                layer()
        graph = _graph_of(ten, torch)
        ms = time_graph(graph.replay, 5, torch) / 10
        nbytes = 8 * (pos + rows) * (256 + 16)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[f"ctx_{pos}"] = {"us_per_layer": round(ms * 1000, 2), "kv_bytes": nbytes, "gbs": round(gbs, 1),
                             "frac_of_peak": round(gbs / peak, 4), "launches_per_layer": 3}
        del graph
    return out


def measure_acceptsel(args, torch, peak):
    """acceptsel11k at the reference size (48 GDN blocks x (786432 + 30720) fp32, m = 7):
    bytes = the slot read + the live slot written."""
    from thunderllamax_b200 import ops

    B, R, C = ops.GDN_BLOCKS, ops.GDN_REC, ops.GDN_CONV
    rec4 = torch.zeros((B, 5, R), device="cuda")
    conv4 = torch.zeros((B, 5, C), device="cuda")
    rec_x = [torch.zeros((B, R), device="cuda") for _ in range(6)]
    conv_x = [torch.zeros((B, C), device="cuda") for _ in range(7)]
    m_slot = torch.tensor([7], dtype=torch.int32, device="cuda")
    launch = lambda: ops.acceptsel11k(rec4, conv4, m_slot, conv_x, rec_x)  # noqa: E731
    for _ in range(3):
        launch()
    ms = time_graph(launch, 20, torch)       # 314 MB per call: larger than L2
    nbytes = 2 * B * (R + C) * 4
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": "acceptsel11k: 48 GDN blocks, rec 786432 + conv 30720 fp32 each, slot 7 -> live",
            "us_per_call": round(ms * 1000, 2), "bytes_per_call": int(nbytes), "gbs": round(gbs, 1),
            "frac_of_peak": round(gbs / peak, 4), "launches_per_call": 1}


def run_ours(args):
    import torch

    ws, rank, local = dist_env()
    if args.gpus != ws and ws > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ws}")
    torch.cuda.set_device(local)
    from thunderllamax_b200 import synth
    from thunderllamax_b200.verify import VerifyShape, VerifyStep

    shape = VerifyShape(vocab=args.vocab, ffn=args.ffn)
    dist = None
    if ws > 1:
        import datetime

        import torch.distributed as dist
        from thunderllamax_b200.dist import ShardedVerifyStep

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    step = ShardedVerifyStep(shape, rank, ws, seed=0) if ws > 1 else VerifyStep(shape, seed=0)

    rng = np.random.default_rng(1234)
    x_bits = synth.bf16_normal(rng, (shape.rows, shape.dim))
    h_bits = synth.bf16_normal(rng, (shape.rows, shape.dim))
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16)
    h = torch.from_numpy(h_bits.view(np.int16)).view(torch.bfloat16)
    # drafts per the head + accept configuration: j ~ U{0..10}; drafts before j are the
    # head's argmax of their row (from one untimed pass), later ones uniform ids
    step.set_inputs(x.cuda(), h.cuda(), drafts=torch.zeros(shape.n_drafts, dtype=torch.int32).cuda())
    step.launch()
    torch.cuda.synchronize()
    amds = step.out_idx.cpu().numpy()
    d_np, draft_j = synth.drafts_for(amds, shape.n_drafts, shape.vocab, np.random.default_rng(4321))
    drafts = torch.from_numpy(d_np)
    step.set_inputs(x.cuda(), h.cuda(), drafts=drafts.cuda())
    step.capture()

    check = None
    if ws > 1:
        check = check_unsharded(step, shape, x, h, drafts, rank, torch, dist)

    clk = ClockSampler(local).__enter__()     # runs across every timed leg below (step, kernels, e2e)
    # the GPU sat idle while the model was generated on the host: untimed replays for
    # RAMP_S seconds bring its clocks and power state to steady load, then the W
    # warm-up steps, then the K timed steps (same count on every rank)
    ramp = ramp_replays(step.replay, torch, dist)
    for _ in range(max(3, args.warmup)):
        step.replay()
    barrier()
    ms = time_graph(step.replay, args.steps, torch)
    barrier()
    ms_max = max_over_ranks(ms)
    accepted = step.accept_out.cpu().tolist()

    # per-kernel durations: each kernel captured R times back to back in its own
    # graph, replayed with CUDA events on the launching stream
    per_kernel = {}
    R = 20
    for name in step.KERNELS:
        g = _graph_of(lambda fn=getattr(step, f"launch_{name}"): [fn() for _ in range(R)], torch)
        g.replay()
        per_kernel[name] = max_over_ranks(time_graph(g.replay, max(3, args.steps // R), torch) / R)
        del g
    phases = None
    if ws > 1:
        phases = step.phase_times(time_graph, _graph_of, max_over_ranks, torch)
        step.replay()
        torch.cuda.synchronize()

    # end to end through host buffers (pinned), one host wait per step
    # one pinned buffer for the step's inputs (x | h | drafts) and one for its record:
    # one H2D and one D2H copy per step
    inp, outp, views = step.host_buffers()
    views["x"].copy_(x)
    views["h"].copy_(h)
    views["drafts"].copy_(drafts)
    for _ in range(3):
        step.step_host_packed(inp, outp)
        torch.cuda.current_stream().synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step.step_host_packed(inp, outp)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    h2d = x.numel() * 2 + h.numel() * 2 + drafts.numel() * 4
    d2h = outp.numel() * 4
    clk.__exit__(None, None, None)

    total_w = sum(shape.weight_bytes().values())
    value = total_w / (ms_max * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    alg = step.algorithmic_bytes_per_rank() if hasattr(step, "algorithmic_bytes_per_rank") else shape.algorithmic_bytes()
    head_ms = per_kernel["head_argmax"]
    head_rows = getattr(step, "n_voc", shape.vocab)
    achieved = alg["head_argmax"] / (head_ms * 1e-3) / 1e9
    kernels = {k: {"us": round(v * 1000, 2), "gbs": round(alg[k] / (v * 1e-3) / 1e9, 1),
                   "frac_of_peak": round(alg[k] / (v * 1e-3) / 1e9 / peak, 4)} for k, v in per_kernel.items()}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        port = CpuVerifyStep(shape, 0, 1)
        try:
            sec, out = time_cpu_steps(port, shape, 0, 1, drafts=d_np)
        finally:
            port.close()
        cpu = {"value": round(total_w / sec / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": "one whole verify step (all four matrices) on one host core: numpy fp32 dequant + fp32 "
                         "matmul, the reference's numpy path restated by the oracle package; wall clock, "
                         "nothing extrapolated",
               "us_per_step": round(sec * 1e6, 1), "argmax_ids_match_gpu": bool(np.array_equal(out[1], amds))}
    extras = {"drafts": {"recipe": "j ~ U{0..10}; drafts before j = the head's argmax, later uniform ids",
                         "j": draft_j, "accepted": accepted[0], "bonus": accepted[1]}}
    if check is not None:
        extras["matches_unsharded"] = check
    if phases is not None:
        extras["phases"] = phases
    if rank == 0 and ws == 1 and not args.no_moe:
        extras["moe_verify"] = measure_moe(args, torch, peak)
    if rank == 0 and ws == 1 and not args.no_prefill and shape.ffn == 17408 and shape.dim == 5120:
        extras["prefill_ffn"] = measure_prefill(args, torch, {k: step.w[k] for k in ("gate", "up", "down")})
    if rank == 0 and ws == 1 and not args.no_extras:
        extras["attn_qkv"] = measure_attn_qkv(args, torch, peak)
        extras["acceptsel11k"] = measure_acceptsel(args, torch, peak)
        extras["gdn_qkv"] = measure_gdn_qkv(args, torch, peak)
        extras["o_proj"] = measure_o_proj(args, torch, peak)
        extras["lookup11"] = measure_lookup(args, torch, peak)
        extras["attention"] = measure_attention(args, torch, peak)
    if ws > 1:
        step.release()
        extras.update(measure_sharded_extras(args, torch, ws, rank, peak))
    clocks = clk.summary()
    if rank == 0:
        emit({"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "us_per_step": round(ms_max * 1000, 2),
              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16xf16->f32 (u8 blocks)",
              "data": "synthetic (seeded GGUF-layout IQ3_XXS/Q6_K blocks and bf16 N(0,1) rows per BASELINE configs 2+3)",
              "config": bench_config(shape, ws),
              "timing": {"graph": f"CUDA graph replay, {step.LAUNCHES_PER_STEP} launches/step"
                                  + (f" ({step.COLLECTIVES})" if ws > 1 else ""),
                         "schedule": (f"FFN chain (gate/up -> down) on {step.ffn_ctas} SMs beside the head on "
                                      f"{step.head_ctas} SMs, two graph branches" if step.ffn_ctas
                                      else "the three GEMVs in sequence on every SM"),
                         "kernels": "each kernel alone on every SM, 20 launches back to back per graph",
                         "l2": f"weights {total_w / 1e6:.0f} MB > 126 MB L2 (no flush needed)",
                         "device_time": "CUDA events around the K replays, max over ranks",
                         "ramp": f"{ramp} untimed replays (~{RAMP_S} s) before the W warm-up steps"},
              "frac_of_hbm": round(value / ws / peak, 4), "frac_of_8tbs": round(value / ws / 8000.0, 4),
              "roofline": {"bound": "hbm", "kernel": "head_argmax", "achieved": round(achieved, 1),
                           "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                           "traffic": round(HEAD_TRAFFIC_BYTES_PER_ROW * head_rows),
                           "traffic_source": "ncu dram__bytes_read+write of the head kernel at vocab 151936, scaled by rows",
                           "algorithmic_bytes": alg["head_argmax"], "us": round(head_ms * 1000, 2)},
              "kernels": kernels,
              "cpu_baseline": cpu,
              "e2e": {"value": round(total_w / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                      "us_per_step": round(e2e_ms * 1000, 2), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
              "gpu_launches": step.LAUNCHES_PER_STEP * args.steps,
              "extras": extras,
              "clocks": clocks})
    if ws > 1:
        step.release()
        dist.destroy_process_group()
    return 0


def check_unsharded(step, shape, x, h, drafts, rank, torch, dist):
    """At N > 1: the merged argmax ids and accept record of the sharded step against
    a one-GPU VerifyStep over the full (same seeded) model on rank 0, same inputs;
    y to fp32 rounding (the all-reduce sums the k shards in another order)."""
    from thunderllamax_b200.verify import VerifyStep

    step.replay()
    torch.cuda.synchronize()
    got = torch.cat([step.out_idx, step.accept_out]).cpu()
    y = step.y.clone()
    ok = torch.ones(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.float64, device="cuda")
    if rank == 0:
        full = VerifyStep(shape, seed=0)
        full.set_inputs(x.cuda(), h.cuda(), drafts=drafts.cuda())
        full.launch()
        torch.cuda.synchronize()
        ref = torch.cat([full.out_idx, full.accept_out]).cpu()
        ok[0] = int(torch.equal(ref, got))
        err[0] = float(((y - full.y).abs().amax(dim=1) / full.y.norm(dim=1)).max())
        del full
        torch.cuda.empty_cache()
    dist.broadcast(ok, 0)
    dist.broadcast(err, 0)
    # every rank's merged ids must equal rank 0's (they merge the same gathered keys)
    mine = got.cuda().to(torch.int64)
    lo, hi = mine.clone(), mine.clone()
    dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    return {"ids_and_accept_equal": bool(ok.item()) and bool(torch.equal(lo, hi)),
            "y_max_err_over_row_norm": float(err.item()),
            "reference": "one-GPU VerifyStep over the full seeded model on rank 0, same inputs and drafts"}


def profile_gemv(which: str, vocab: int, ffn: int) -> int:
    """A small driver for ncu: one of the verify step's three GEMVs alone (the bench's
    seeded model at --vocab / --ffn, inputs N(0, 1) bf16), launched four times
    eagerly (three warm-up launches, then the one to capture), then exit."""
    import numpy as np
    import torch
    from thunderllamax_b200 import synth
    from thunderllamax_b200.verify import VerifyShape, VerifyStep

    step = VerifyStep(VerifyShape(vocab=vocab, ffn=ffn), seed=0)
    rng = np.random.default_rng(2323)
    rows = [torch.from_numpy(synth.bf16_normal(rng, (step.shape.rows, step.shape.dim)).view(np.int16))
            .cuda().view(torch.bfloat16) for _ in range(2)]
    step.set_inputs(rows[0], rows[1])
    step.launch()                                  # every input the chosen kernel reads
    fn = {"gate_up": step.launch_ffn_gate_up, "down": step.launch_ffn_down, "head": step.launch_head_argmax}[which]
    for _ in range(4):
        fn()
    torch.cuda.synchronize()
    bad = {k: w.error() for k, w in step.ws.items() if w.error()}
    print(json.dumps({"profile_gemv": which, "vocab": vocab, "ffn": ffn, "ok": not bad, "errors": bad}))
    return 0 if not bad else 1


def profile_layer(which: str) -> int:
    """A small driver for ncu: four eager launches of the MoE verify layer (config 4:
    router, gate/up, act image, down per layer), of the prefill FFN (config 5: token
    staging, gate/up, act staging, down) or of the W4A8 gate/up (token quantiser,
    staging, gate/up), seeded as in the bench, then exit."""
    import numpy as np
    import torch
    from thunderllamax_b200 import synth

    rng = np.random.default_rng(4321)
    if which == "moe":
        from thunderllamax_b200 import moe

        step = moe.MoeVerifyStep(moe.MoeShape(), seed=0)
        s = step.shape
        h = torch.from_numpy(synth.bf16_normal(rng, (s.positions, s.hidden)).view(np.int16)).cuda()
        step.set_inputs(h.view(torch.bfloat16), torch.zeros((s.positions, s.hidden), device="cuda"))
        errs = lambda: [step.ws.error()]                            # noqa: E731
    elif which == "prefill":
        from thunderllamax_b200 import prefill

        step = prefill.PrefillFFN(prefill.PrefillShape(), seed=0)
        s = step.shape
        step.x.copy_(torch.from_numpy(synth.bf16_normal(rng, (s.tokens, s.dim)).view(np.int16)).cuda()
                     .view(torch.bfloat16))
        errs = lambda: [step.ws.error(), step.ws_down.error()]     # noqa: E731
    else:
        from thunderllamax_b200 import prefill

        ffn = prefill.PrefillFFN(prefill.PrefillShape(), seed=0)
        s = ffn.shape
        x16 = torch.from_numpy(synth.bf16_normal(rng, (s.tokens, s.dim)).view(np.int16)).cuda() \
            .view(torch.bfloat16).to(torch.float16)
        xq = torch.empty((s.tokens, s.dim), dtype=torch.int8, device="cuda")
        sx = torch.empty((s.tokens, s.dim // 128), dtype=torch.float32, device="cuda")
        rs = torch.empty_like(sx, dtype=torch.int32)
        lut = prefill.lut8()

        class W4a8GateUp:
            def launch(self):
                prefill.act_quant_q8(x16, xq=xq, sx=sx, rs=rs)
                prefill.w4a8_gate_up(ffn.w["gate"], ffn.w["up"], xq, sx, s.ffn, ffn.ws, act=ffn.act, lut=lut)

        step = W4a8GateUp()
        errs = lambda: [ffn.ws.error()]                              # noqa: E731
    for _ in range(4):
        step.launch()
    torch.cuda.synchronize()
    bad = [e for e in errs() if e]
    print(json.dumps({"profile_layer": which, "ok": not bad, "errors": bad}))
    return 0 if not bad else 1


def profile_attention(pos: int) -> int:
    """A small driver for ncu: the attention split kernel alone at context `pos`
    (11 rows, ctx 100352, random int8 cache and scales, qw16 N(0, 1) / 16)."""
    import torch
    from thunderllamax_b200 import ops

    rows, ctx = 11, 100352
    if not 0 <= pos <= ctx - rows:
        raise SystemExit(f"--profile-attention POS must be in [0, {ctx - rows}]")
    kv = torch.randint(1, 256, (8, ctx, 256), dtype=torch.uint8, device="cuda")
    sc = (torch.rand((8, ctx, 8), device="cuda") * 0.02 + 0.01).half()
    qw16 = (torch.randn((rows, 24, 256), device="cuda") / 16).half()
    pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
    at = ops.Attention(rows, ctx)
    for _ in range(2):
        at.split(kv, sc, qw16, pos_t)
    torch.cuda.synchronize()
    print(json.dumps({"profile_attention": pos, "ok": True}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-port baseline")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE layer (config 4) measurement")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill contraction (config 5) measurement")
    ap.add_argument("--no-extras", action="store_true", help="skip the aq3k8v11 / acceptsel11k measurements")
    # smaller shapes for profiler captures only; the benchmark line uses the defaults
    ap.add_argument("--profile-attention", type=int, default=None, metavar="POS",
                    help="profiling case: one warm-up and one tlx_attn_split launch at context POS, then exit")
    ap.add_argument("--profile-gemv", choices=["gate_up", "down", "head"], default=None,
                    help="profiling case: one verify GEMV alone (a full step first, then four launches), then exit")
    ap.add_argument("--profile-layer", choices=["moe", "prefill", "w4a8"], default=None,
                    help="profiling case: four eager MoE-layer, prefill-FFN or W4A8 gate/up launches, then exit")
    ap.add_argument("--vocab", type=int, default=151936, help="head rows (profiling cases only)")
    ap.add_argument("--ffn", type=int, default=17408, help="FFN rows, a multiple of 256 (profiling cases only)")
    args = ap.parse_args()
    if args.profile_attention is not None:
        return profile_attention(args.profile_attention)
    if args.profile_gemv is not None:
        return profile_gemv(args.profile_gemv, args.vocab, args.ffn)
    if args.profile_layer is not None:
        return profile_layer(args.profile_layer)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
