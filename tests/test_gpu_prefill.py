"""GPU parity of the tcgen05 prefill contraction (BASELINE config 5 shapes, cut
down) against the numpy oracle on identical seeded inputs, through the C ABI.

The kernels round every dequantised weight to fp16 once (integer part times the
block scale); the gate/up act is fp32, and bf16 / fp32 tokens are staged to fp16
with a power-of-two scale per row (one fp16 rounding, none for bf16).  Contract:
max|err| <= 2e-3 * ||row||_2 per token row of the float64 oracle; a tighter
1e-3 bound (about two fp16 roundings of the largest products) is asserted too."""
import numpy as np
import pytest
import torch

import oracle
from thunderllamax_b200 import ops, prefill, synth

pytestmark = pytest.mark.gpu

CONTRACT = 2e-3
TIGHT = 1e-3


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()
    yield


def tokens(rng, m, k):
    bits = synth.bf16_normal(rng, (m, k))
    return torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16), \
        synth.bf16_bits_to_f32(bits).astype(np.float64)


def check_rows(got, ref, tol):
    err = np.abs(got.astype(np.float64) - ref).max(axis=1)
    norm = np.linalg.norm(ref, axis=1)
    assert (err <= tol * norm).all(), float((err / norm).max())


@pytest.mark.parametrize("m,n,k", [(256, 256, 512), (300, 128, 256), (1, 384, 768), (513, 256, 1024)])
def test_prefill_gate_up_iq3(m, n, k):
    rng = np.random.default_rng(m + n + k)
    rg, ru = synth.iq3xxs_blocks(rng, n, k), synth.iq3xxs_blocks(rng, n, k)
    x_t, x64 = tokens(rng, m, k)
    ws = prefill.PrefillWorkspace(m, k)
    act = prefill.gate_up("iq3_xxs", ops.pack_tiles("iq3_xxs", rg, k), ops.pack_tiles("iq3_xxs", ru, k), x_t, n, ws)
    torch.cuda.synchronize()
    assert ws.error() == 0
    g = oracle.matvec_f64(oracle.dequant_iq3xxs(rg, k), x64)
    u = oracle.matvec_f64(oracle.dequant_iq3xxs(ru, k), x64)
    ref = oracle.silu_f64(g) * u
    got = act.float().cpu().numpy()
    check_rows(got, ref, CONTRACT)
    check_rows(got, ref, TIGHT)


@pytest.mark.parametrize("qtype,m,n,k", [("q6_k", 256, 256, 512), ("q6_k", 300, 128, 1024), ("q6_k", 77, 256, 768)])
def test_prefill_gemm(qtype, m, n, k):
    rng = np.random.default_rng(7 + m + n)
    raw = synth.BLOCK_GEN[qtype](rng, n, k)
    bits = synth.bf16_normal(rng, (m, k))
    x16 = synth.bf16_bits_to_f32(bits).astype(np.float16)          # fp16 tokens (like the gate/up act)
    x_t = torch.from_numpy(x16).cuda()
    ws = prefill.PrefillWorkspace(m, k)
    y = prefill.gemm(qtype, ops.pack_tiles(qtype, raw, k), x_t, n, ws)
    torch.cuda.synchronize()
    assert ws.error() == 0
    ref = oracle.matvec_f64(oracle.dequant(qtype, raw, k), x16.astype(np.float64))
    got = y.cpu().numpy()
    check_rows(got, ref, CONTRACT)
    check_rows(got, ref, TIGHT)


def test_prefill_ffn_small_chain_and_repeat():
    shape = prefill.PrefillShape(tokens=260, dim=512, ffn=768)
    step = prefill.PrefillFFN(shape, seed=3)
    rng = np.random.default_rng(9)
    x_t, x64 = tokens(rng, shape.tokens, shape.dim)
    step.x.copy_(x_t)
    step.launch()
    torch.cuda.synchronize()
    y0 = step.y.clone()
    step.launch()
    torch.cuda.synchronize()
    assert torch.equal(step.y, y0)                                    # deterministic
    rg = ops.unpack_tiles_host("iq3_xxs", step.w["gate"].cpu().numpy(), shape.ffn, shape.dim, 2 * 98)
    ru = ops.unpack_tiles_host("iq3_xxs", step.w["up"].cpu().numpy(), shape.ffn, shape.dim, 2 * 98)
    rd = ops.unpack_tiles_host("q6_k", step.w["down"].cpu().numpy(), shape.dim, shape.ffn, 3 * 210)
    _, y_ref = oracle.ffn_f64(x64, rg, ru, rd)
    check_rows(step.y.cpu().numpy(), y_ref, CONTRACT)


def test_prefill_rejects_unsupported_formats():
    from thunderllamax_b200 import _lib
    x = torch.zeros((16, 256), dtype=torch.float16, device="cuda")
    ws = prefill.PrefillWorkspace(16, 256)
    w = torch.zeros(ops.tiled_bytes("iq3_xxs", 128, 256), dtype=torch.uint8, device="cuda")
    with pytest.raises(_lib.TLXError):
        prefill.gemm("iq3_xxs", w, x, 128, ws)          # single-matrix path is Q6_K
    with pytest.raises(_lib.TLXError):
        prefill.gate_up("q6_k", w, w, x, 128, ws)       # gate/up path is IQ3_XXS


def test_prefill_gemm_rows_beyond_fp16_range():
    # bf16 and fp32 rows whose values exceed the fp16 range (the gate/up act of
    # large-weight inputs does): staged with a power-of-two scale per row, multiplied
    # back in the epilogue; a row inside the fp16 range keeps scale 1
    rng = np.random.default_rng(91)
    m, n, k = 40, 256, 1024
    raw = synth.q6k_blocks(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x *= (10.0 ** rng.uniform(-2, 7, m)).astype(np.float32)[:, None]   # row scales 1e-2 .. 1e7
    x[0] *= 0
    bits = synth.f32_to_bf16_bits(x)
    w = ops.pack_tiles("q6_k", raw, k)
    W = oracle.dequant("q6_k", raw, k)
    for x_t, x64 in ((torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16),
                      synth.bf16_bits_to_f32(bits).astype(np.float64)),
                     (torch.from_numpy(x).cuda(), x.astype(np.float64))):
        ws = prefill.PrefillWorkspace(m, k)
        y = prefill.gemm("q6_k", w, x_t, n, ws)
        torch.cuda.synchronize()
        assert ws.error() == 0
        got = y.cpu().numpy()
        assert np.isfinite(got).all()
        assert np.array_equal(got[0], np.zeros(n, np.float32))
        check_rows(got[1:], oracle.matvec_f64(W, x64)[1:], TIGHT)


@pytest.mark.parametrize("mode,m,n,k", [("gate_up", 256, 256, 2048), ("gate_up", 300, 128, 4096),
                                        ("gemm", 300, 256, 4096), ("gemm", 77, 128, 8192)])
def test_prefill_split_tiles(mode, m, n, k):
    """Fewer tiles than SMs and a long k: each tile runs as k pieces on separate SMs,
    the last piece to finish sums the fp32 partials in piece order.  Two calls on the
    same workspace (the piece counters re-arm) give the same bits."""
    rng = np.random.default_rng(11 + m + n + k)
    x_t, x64 = tokens(rng, m, k)
    ws = prefill.PrefillWorkspace(m, k)
    if mode == "gate_up":
        rg, ru = synth.iq3xxs_blocks(rng, n, k), synth.iq3xxs_blocks(rng, n, k)
        wg, wu = ops.pack_tiles("iq3_xxs", rg, k), ops.pack_tiles("iq3_xxs", ru, k)
        run = lambda: prefill.gate_up("iq3_xxs", wg, wu, x_t, n, ws)      # noqa: E731
        ref = oracle.silu_f64(oracle.matvec_f64(oracle.dequant_iq3xxs(rg, k), x64)) * \
            oracle.matvec_f64(oracle.dequant_iq3xxs(ru, k), x64)
    else:
        raw = synth.q6k_blocks(rng, n, k)
        w = ops.pack_tiles("q6_k", raw, k)
        run = lambda: prefill.gemm("q6_k", w, x_t, n, ws)                 # noqa: E731
        ref = oracle.matvec_f64(oracle.dequant("q6_k", raw, k), x64)
    out0 = run().clone()
    out1 = run()
    torch.cuda.synchronize()
    assert ws.error() == 0
    assert torch.equal(out0, out1)
    got = out1.float().cpu().numpy()
    check_rows(got, ref, CONTRACT)
    check_rows(got, ref, TIGHT)
