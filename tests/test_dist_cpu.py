"""Host-side multi-GPU plumbing on CPU: shard partitions and the two collectives
(all-reduce of down partials, all-gather of argmax keys) with world_size 2 over
gloo.  Each rank computes its shard with the oracle; the merged result must equal
the unsharded oracle (argmax ids bit-exact)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from thunderllamax_b200 import dist as tdist
from thunderllamax_b200 import synth


def test_partitions_cover_exactly():
    for n, w in ((68, 1), (68, 2), (68, 8), (5, 8), (1000, 3)):
        r = tdist.block_ranges(n, w)
        assert r[0][0] == 0 and r[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
    for n, w in ((151936, 8), (151936, 3), (100, 4), (7, 2)):
        r = tdist.row_ranges(n, w)
        assert r[0][0] == 0 and r[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        assert all(a[0] % 16 == 0 for a in r)


def key_of(v: float, idx: int) -> int:
    """The library's packed argmax key (common.cuh argmax_key), for the CPU test."""
    f = np.float32(v)
    if np.isnan(f):
        return 0
    u = int(np.array([f + np.float32(0.0)], np.float32).view(np.uint32)[0])
    u = (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)
    return (u << 32) | (0xFFFFFFFF - idx)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)
        H, F, V, m = 512, 1024, 3001, 11
        rg, ru = synth.iq3xxs_blocks(rng, F, H), synth.iq3xxs_blocks(rng, F, H)
        rd, rh = synth.q6k_blocks(rng, H, F), synth.q6k_blocks(rng, V, H)
        x = synth.bf16_bits_to_f32(synth.bf16_normal(rng, (m, H))).astype(np.float64)
        # this rank's shards, cut exactly as ShardedVerifyStep cuts them
        b0, b1 = tdist.block_ranges(F // 256, world)[rank]
        f0, f1 = 256 * b0, 256 * b1
        v0, v1 = tdist.row_ranges(V, world)[rank]
        g = oracle.matvec_f64(oracle.dequant_iq3xxs(tdist.shard_gguf_rows(rg, f0, f1), H), x)
        u = oracle.matvec_f64(oracle.dequant_iq3xxs(tdist.shard_gguf_rows(ru, f0, f1), H), x)
        gact = oracle.silu_f64(g) * u
        wd = oracle.dequant_q6k(tdist.shard_gguf_cols(rd, f0, f1, 210), f1 - f0)
        y = torch.from_numpy(oracle.matvec_f64(wd, gact))
        tdist.allreduce_partial(y)
        lg = oracle.head_logits_f64(x, tdist.shard_gguf_rows(rh, v0, v1)).astype(np.float32)
        u64 = [max(key_of(lg[t, i], v0 + i) for i in range(lg.shape[1])) for t in range(m)]
        keys = torch.tensor([k - (1 << 64) if k >= (1 << 63) else k for k in u64], dtype=torch.int64)
        # int64 holds the u64 key bit pattern; compare as unsigned after the gather
        local = keys.clone()
        all_keys = torch.zeros((world, m), dtype=torch.int64)
        tdist.gather_keys(local, all_keys)
        merged = [max(int(k) & 0xFFFFFFFFFFFFFFFF for k in all_keys[:, t]) for t in range(m)]
        idx = [0xFFFFFFFF - (k & 0xFFFFFFFF) for k in merged]
        if rank == 0:
            _, y_ref = oracle.ffn_f64(x, rg, ru, rd)
            lg_full = oracle.head_logits_f64(x, rh).astype(np.float32)
            idx_ref = [int(np.argmax(lg_full[t])) for t in range(m)]
            q.put((float(np.abs(y.numpy() - y_ref).max() / np.linalg.norm(y_ref)), idx, idx_ref))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_step_equals_unsharded_oracle():
    # spawned ranks re-import this module: give them the test's import paths
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    os.environ["PYTHONPATH"] = os.pathsep.join([root, here, os.path.join(here, "golden"),
                                                os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    try:
        err, idx, idx_ref = q.get(timeout=180)
    finally:
        for p_ in procs:
            p_.join(timeout=60)
    for p_ in procs:
        assert p_.exitcode == 0
    assert err < 1e-12
    assert idx == idx_ref


def _spawn(target, world=2, timeout=240):
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    os.environ["PYTHONPATH"] = os.pathsep.join([root, here, os.path.join(here, "golden"),
                                                os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p_ in procs:
        p_.start()
    out = []
    try:
        for _ in range(world):
            out.append(q.get(timeout=timeout))
    finally:
        for p_ in procs:
            p_.join(timeout=60)
    assert all(p_.exitcode == 0 for p_ in procs)
    return out


def _moe_worker(rank, world, port, q):
    # expert parallel: this rank's routed experts (+ shared and residual on rank 0),
    # summed by the all-reduce, equal the whole layer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        E, H, I, P = 16, 256, 256, 3
        Wr = rng.normal(0, 0.05, (E, H)).astype(np.float32)
        wsh = rng.normal(0, 0.05, H).astype(np.float32)
        gate = synth.iq4xs_blocks(rng, E * I, H).reshape(E, I, -1)
        up = synth.iq4xs_blocks(rng, E * I, H).reshape(E, I, -1)
        down = synth.iq4xs_blocks(rng, E * H, I).reshape(E, H, -1)
        sg_, su_, sd_ = synth.iq4xs_blocks(rng, I, H), synth.iq4xs_blocks(rng, I, H), synth.iq4xs_blocks(rng, H, I)
        h = rng.standard_normal((P, H))
        hres = rng.standard_normal((P, H))
        full = oracle.moe_verify_f64(h, Wr, wsh, gate, up, down, sg_, su_, sd_, hres=hres)
        e0, e1 = tdist.expert_ranges(E, world)[rank]
        part = np.zeros((P, H))
        for p in range(P):
            for r in range(8):
                if e0 <= full["ids"][p, r] < e1:
                    part[p] += full["gates"][p, r] * full["parts"][p, r]
        if rank == 0:
            shared = full["y"] - hres - np.einsum("pr,prh->ph", full["gates"], full["parts"])
            part += shared + hres
        y = torch.from_numpy(part)
        tdist.allreduce_partial(y)
        q.put((rank, float(np.abs(y.numpy() - full["y"]).max() / np.abs(full["y"]).max())))
    finally:
        dist.destroy_process_group()


def test_two_rank_expert_parallel_moe_equals_layer():
    for rank, err in _spawn(_moe_worker):
        assert err < 1e-12, (rank, err)


def _prefill_worker(rank, world, port, q):
    # tensor parallel prefill FFN: gate/up rows and down k split by 256-row blocks
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(12)
        T, H, F = 5, 256, 1024
        rg, ru = synth.iq3xxs_blocks(rng, F, H), synth.iq3xxs_blocks(rng, F, H)
        rd = synth.q6k_blocks(rng, H, F)
        x = synth.bf16_bits_to_f32(synth.bf16_normal(rng, (T, H))).astype(np.float64)
        b0, b1 = tdist.block_ranges(F // 256, world)[rank]
        f0, f1 = 256 * b0, 256 * b1
        g = oracle.matvec_f64(oracle.dequant_iq3xxs(tdist.shard_gguf_rows(rg, f0, f1), H), x)
        u = oracle.matvec_f64(oracle.dequant_iq3xxs(tdist.shard_gguf_rows(ru, f0, f1), H), x)
        wd = oracle.dequant_q6k(tdist.shard_gguf_cols(rd, f0, f1, 210), f1 - f0)
        y = torch.from_numpy(oracle.matvec_f64(wd, oracle.silu_f64(g) * u))
        tdist.allreduce_partial(y)
        _, y_ref = oracle.ffn_f64(x, rg, ru, rd)
        q.put((rank, float(np.abs(y.numpy() - y_ref).max() / np.abs(y_ref).max())))
    finally:
        dist.destroy_process_group()


def test_two_rank_tensor_parallel_prefill_equals_ffn():
    for rank, err in _spawn(_prefill_worker):
        assert err < 1e-12, (rank, err)


def test_four_rank_expert_and_tensor_parallel_partitions():
    # the same two sharded layers over four gloo ranks (the partitions at N = 4:
    # a quarter of the experts, one 256-row block of the FFN per rank)
    for rank, err in _spawn(_moe_worker, world=4):
        assert err < 1e-12, ("moe", rank, err)
    for rank, err in _spawn(_prefill_worker, world=4):
        assert err < 1e-12, ("prefill", rank, err)
