"""The sharded verify step on 2..8 GPUs against the oracle: FFN rows / k split,
vocabulary split, the partials and argmax keys exchanged over peer memory inside
the kernels (comm="peer") or by NCCL collectives plus a merge kernel
(comm="nccl"); every rank must hold the same ids, accept record and y.  World
sizes beyond the box's GPU count are skipped.  A single-GPU test drives the peer
kernels' bounded waits into their timeout (a flag nothing sets) and checks the
error word."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q, comm="peer", steps=3):
    import datetime

    import torch.distributed as dist

    import oracle
    from thunderllamax_b200 import dist as tdist
    from thunderllamax_b200 import ops, synth
    from thunderllamax_b200.verify import VerifyShape

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        rng = np.random.default_rng(7)
        s = VerifyShape(dim=1024, ffn=3072, vocab=7001, rows=11)
        rg, ru = synth.iq3xxs_blocks(rng, s.ffn, s.dim), synth.iq3xxs_blocks(rng, s.ffn, s.dim)
        rd, rh = synth.q6k_blocks(rng, s.dim, s.ffn), synth.q6k_blocks(rng, s.vocab, s.dim)
        xb, hb = synth.bf16_normal(rng, (s.rows, s.dim)), synth.bf16_normal(rng, (s.rows, s.dim))
        res = rng.standard_normal((s.rows, s.dim), dtype=np.float32)
        b0, b1 = tdist.block_ranges(s.ffn // 256, world)[rank]
        f0, f1 = 256 * b0, 256 * b1
        v0, v1 = tdist.row_ranges(s.vocab, world)[rank]
        w = {"gate": ops.pack_tiles("iq3_xxs", tdist.shard_gguf_rows(rg, f0, f1), s.dim),
             "up": ops.pack_tiles("iq3_xxs", tdist.shard_gguf_rows(ru, f0, f1), s.dim),
             "down": ops.pack_tiles("q6_k", tdist.shard_gguf_cols(rd, f0, f1, 210), f1 - f0),
             "head": ops.pack_tiles("q6_k", tdist.shard_gguf_rows(rh, v0, v1), s.dim)}
        step = tdist.ShardedVerifyStep(s, rank, world, weights=w, comm=comm)
        x64 = synth.bf16_bits_to_f32(xb).astype(np.float64)
        h64 = synth.bf16_bits_to_f32(hb).astype(np.float64)
        _, idx_ref, _ = oracle.head_argmax(h64, rh, "q6_k")
        drafts = idx_ref[:10].copy()
        drafts[5] = (drafts[5] + 1) % s.vocab
        step.set_inputs(torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16),
                        torch.from_numpy(hb.view(np.int16)).cuda().view(torch.bfloat16),
                        res=torch.from_numpy(res).cuda(), drafts=torch.from_numpy(drafts).cuda())
        step.capture()
        ys = []
        for _ in range(steps):       # several steps: the peer slots alternate by step parity
            step.replay()
            torch.cuda.synchronize()
            ys.append(step.y.clone())
        _, y_ref = oracle.ffn_f64(x64, rg, ru, rd, residual=res)
        y = step.y.cpu().numpy()
        err = float((np.abs(y - y_ref).max(axis=1) / np.linalg.norm(y_ref, axis=1)).max())
        same = all(torch.equal(ys[0], t) for t in ys[1:])
        werr = [w_.error() for w_ in step.ws.values()] + [int(step.finish_err.item())]
        out = (rank, err, step.out_idx.cpu().tolist(), idx_ref.tolist(), step.accept_out.cpu().tolist(),
               list(oracle.accept(idx_ref, drafts)), same, werr, y.tobytes())
        step.release()
        q.put(out)
    finally:
        dist.destroy_process_group()


WORLDS = [w for w in (2, 4, 8)]


@pytest.mark.parametrize("comm", ["peer", "nccl"])
@pytest.mark.parametrize("world", WORLDS)
def test_sharded_verify_step(world, comm):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    os.environ["PYTHONPATH"] = os.pathsep.join([root, here, os.path.join(here, "golden"),
                                                os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, comm)) for r in range(world)]
    for p_ in procs:
        p_.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=300))
    finally:
        for p_ in procs:
            p_.join(timeout=60)
    assert all(p_.exitcode == 0 for p_ in procs)
    for rank, err, idx, idx_ref, acc, acc_ref, same, werr, _ in results:
        assert err <= 2e-3 and err <= 1e-4, (rank, err)
        assert idx == idx_ref, rank
        assert acc == acc_ref, rank
        assert same, f"rank {rank}: y differs between steps"
        assert werr == [0, 0, 0, 0], (rank, werr)
    # every rank holds the same y (the partials are added in rank order everywhere)
    assert len({r[-1] for r in results}) == 1


def _moe_rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from thunderllamax_b200 import dist as tdist
    from thunderllamax_b200 import moe, synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        shape = moe.MoeShape(positions=5, experts=64, hidden=1024, inner=512)
        host = moe.synth_host(shape, 23)
        rng = np.random.default_rng(23)
        h = torch.from_numpy(synth.bf16_normal(rng, (shape.positions, shape.hidden)).view(np.int16)).cuda()
        h = h.view(torch.bfloat16)
        hres = torch.from_numpy(rng.standard_normal((shape.positions, shape.hidden)).astype(np.float32)).cuda()
        full = moe.MoeVerifyStep(shape, host=host)
        full.set_inputs(h, hres)
        full.launch()
        step = tdist.ShardedMoeVerifyStep(shape, rank, world, host=host, comm="peer")
        step.set_inputs(h, hres)
        step.capture()
        ys = []
        for _ in range(3):        # the parity slots alternate by step
            step.replay()
            torch.cuda.synchronize()
            ys.append(step.y.clone())
        ref = full.y
        err = float(((ys[-1] - ref).abs().amax(dim=1) / ref.norm(dim=1)).max())
        same = all(torch.equal(ys[0], t) for t in ys[1:])
        out = (rank, err, same, int(step.finish_err.item()), step.local.ws.error(), ys[-1].cpu().numpy().tobytes())
        step.release()
        q.put(out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_sharded_moe_peer_exchange(world):
    # expert-parallel MoE layer, the ranks' partials summed over peer memory: every rank
    # holds the unsharded layer's y to fp32 rounding, the same bits on every rank and
    # over repeated steps
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    os.environ["PYTHONPATH"] = os.pathsep.join([root, here, os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_moe_rank, args=(r, world, port, q)) for r in range(world)]
    for p_ in procs:
        p_.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=300))
    finally:
        for p_ in procs:
            p_.join(timeout=60)
    assert all(p_.exitcode == 0 for p_ in procs)
    for rank, err, same, ferr, werr, _ in results:
        assert err <= 1e-5, (rank, err)
        assert same, rank
        assert ferr == 0 and werr == 0, (rank, ferr, werr)
    assert len({r[-1] for r in results}) == 1


def test_peer_wait_times_out_into_error_word():
    # Failure detection without a GPU fault: rank 0 of a 2-rank step whose rank 1 never
    # runs.  Both buffers live on this GPU (nothing else runs on it); the down kernel
    # sends its partial and raises its flag, the head kernel then waits for rank 1's
    # argmax keys and the finish kernel for rank 1's down partial, which nothing sets:
    # the bounded waits give up, raise TLX_WS_ERR_PEER_TIMEOUT in their error words and
    # the kernels return (the context stays usable).
    import ctypes

    from thunderllamax_b200 import _lib, ops, synth

    ops.require_device()
    L = _lib.lib()
    m, dim, ffn, vocab = 11, 512, 512, 1000
    nb = int(L.tlx_peer_buffer_bytes(2, m, dim))
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        _lib.check(L.tlx_peer_buffer_alloc(nb, ctypes.byref(p)), "alloc")
        bufs.append(p.value)
    ptrs = (ctypes.c_void_p * 2)(*bufs)
    try:
        rng = np.random.default_rng(3)
        wd = ops.pack_tiles("q6_k", synth.q6k_blocks(rng, dim, ffn), ffn)
        wh = ops.pack_tiles("q6_k", synth.q6k_blocks(rng, vocab, dim), dim)
        img = ops.stage(torch.randn((m, ffn), device="cuda").half())
        ws_d = ops.Workspace.for_shape(ops.MODE_STORE, "q6_k", dim, ffn, m, "image")
        ws_h = ops.Workspace.for_shape(ops.MODE_ARGMAX, "q6_k", vocab, dim, m)
        h = torch.randn((m, dim), device="cuda").half()
        y = torch.zeros((m, dim), device="cuda")
        idx = torch.zeros(m, dtype=torch.int32, device="cuda")
        ferr = torch.zeros(1, dtype=torch.int32, device="cuda")
        s = ops._stream(h)
        _lib.check(L.tlx_gemv_peer(ops.qtype_id("q6_k"), ops._ptr(wd), None, ops._ptr(img.buf), _lib.TLX_DT_IMAGE,
                                   0, m, dim, ffn, 2, 0, ptrs, 0, ops._ptr(ws_d.buf), ws_d.nbytes, s), "gemv_peer")
        _lib.check(L.tlx_head_argmax_peer(ops.qtype_id("q6_k"), ops._ptr(wh), None, ops._ptr(h), _lib.TLX_DT_F16,
                                          dim, m, vocab, dim, 0, None, ops._ptr(idx), None, 0, None, 2, 0, ptrs, 0,
                                          ops._ptr(ws_h.buf), ws_h.nbytes, s), "head_argmax_peer")
        _lib.check(L.tlx_peer_finish(2, 0, ptrs, m, dim, None, 0, ops._ptr(y), dim, ops._ptr(ferr), s), "finish")
        torch.cuda.synchronize()
        assert ws_d.error() == 0
        assert ws_h.error() & 4, ws_h.error()          # TLX_WS_ERR_PEER_TIMEOUT (keys)
        assert int(ferr.item()) & 4, int(ferr.item())   # TLX_WS_ERR_PEER_TIMEOUT (down partial)
        # the context is still usable
        assert torch.equal(torch.ones(4, device="cuda").sum().cpu(), torch.tensor(4.0))
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            L.tlx_peer_buffer_free(b)
