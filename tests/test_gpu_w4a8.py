"""GPU parity of the W4A8 prefill tier (int8 tokens x linearised IQ3_XXS levels)
through the C ABI, against the numpy oracle (oracle/w4a8.py, pinned to the
reference's own numpy code by tests/test_oracle_w4a8.py) and against the
reference's own kernels compiled into oracle/_ref (p8q8x, p8w4ffn7) run on the
same device inputs.

The quantiser is integer work: bit-exact.  The gate/up contraction runs on the
fp16 tcgen05 path with one fp16 rounding per weight and per staged token value;
contract: max|err| <= 2e-3 * ||row||_2 per token row of the float64 oracle, with
the tighter 1e-3 asserted too."""
import os
import sys

import numpy as np
import pytest
import torch

import oracle
from thunderllamax_b200 import ops, prefill, synth

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import refkernels  # noqa: E402

pytestmark = pytest.mark.gpu

CONTRACT = 2e-3
TIGHT = 1e-3
K5, N5 = 5120, 17408   # config 5 (and the reference kernels' compiled shapes)


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()
    yield


def tokens16(rng, m, k, special=True):
    """fp16 tokens ~ N(0, 0.7^2), with (m >= 4) an all-zero chunk, a row of values
    below the quantiser's 1e-6 floor and a row near the fp16 range."""
    x = (rng.standard_normal((m, k)) * 0.7).astype(np.float16)
    if special and m >= 4:
        x[1, 128:256] = 0
        x[2] = (rng.standard_normal(k) * 1e-7).astype(np.float16)
        x[3] = np.clip(rng.standard_normal(k) * 1.5e4, -6e4, 6e4).astype(np.float16)
    return x


def check_rows(got, ref, tol):
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref).max(axis=1)
    norm = np.linalg.norm(ref, axis=1)
    assert (err <= tol * norm).all(), float((err / norm).max())


def quant_equal(xq, sx, rs, ref):
    oq, osx, ors = ref
    assert np.array_equal(xq.cpu().numpy(), oq)
    assert np.array_equal(sx.cpu().numpy().view(np.uint32), np.asarray(osx, dtype=np.float32).view(np.uint32))
    assert np.array_equal(rs.cpu().numpy(), ors)


@pytest.mark.parametrize("m,k", [(1, 128), (37, 640), (300, 5120), (2048, 5120)])
def test_act_quant_q8_bit_exact(m, k):
    rng = np.random.default_rng(m * 7 + k)
    x = tokens16(rng, m, k)
    xq, sx, rs = prefill.act_quant_q8(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    quant_equal(xq, sx, rs, oracle.act_quant_q8(x))


def test_act_quant_q8_row_strides():
    rng = np.random.default_rng(3)
    m, k = 19, 1024
    x = tokens16(rng, m, k)
    wide = torch.zeros((m, k + 64), dtype=torch.float16, device="cuda")
    wide[:, :k] = torch.from_numpy(x).cuda()
    xq_wide = torch.full((m, k + 32), -19, dtype=torch.int8, device="cuda")
    xq, sx, rs = prefill.act_quant_q8(wide[:, :k], xq=xq_wide[:, :k])
    torch.cuda.synchronize()
    quant_equal(xq, sx, rs, oracle.act_quant_q8(x))
    assert (xq_wide[:, k:] == -19).all()      # nothing written past k


def test_act_quant_q8_vs_reference_kernel():
    refkernels.require("p8q8x")
    rng = np.random.default_rng(11)
    m = 64
    x = tokens16(rng, m, K5)
    xd = torch.from_numpy(x).cuda()
    rq = torch.full((m, K5), -19, dtype=torch.int8, device="cuda")
    rsx = torch.full((m, K5 // 128), 7.7e31, dtype=torch.float32, device="cuda")
    rrs = torch.full((m, K5 // 128), 0x5A5A5A5A, dtype=torch.int32, device="cuda")
    refkernels.launch("p8q8x", m, 256, [xd, rq, rsx, rrs, xd, xd])   # the last two are never read
    xq, sx, rs = prefill.act_quant_q8(xd)
    torch.cuda.synchronize()
    assert torch.equal(xq, rq)
    assert torch.equal(sx.view(torch.int32), rsx.view(torch.int32))
    assert torch.equal(rs, rrs)
    quant_equal(xq, sx, rs, oracle.act_quant_q8(x))


@pytest.mark.parametrize("m,n,k", [(256, 256, 512), (300, 128, 256), (1, 384, 768), (513, 256, 1024)])
def test_w4a8_gate_up_vs_oracle(m, n, k):
    rng = np.random.default_rng(m + 3 * n + k)
    rg, ru = synth.iq3xxs_blocks(rng, n, k), synth.iq3xxs_blocks(rng, n, k)
    x = tokens16(rng, m, k)
    xq, sx, _ = prefill.act_quant_q8(torch.from_numpy(x).cuda())
    ws = prefill.PrefillWorkspace(m, k)
    act = prefill.w4a8_gate_up(ops.pack_tiles("iq3_xxs", rg, k), ops.pack_tiles("iq3_xxs", ru, k), xq, sx, n, ws)
    torch.cuda.synchronize()
    assert ws.error() == 0
    ref = oracle.w4a8_gate_up_f64(xq.cpu().numpy(), sx.cpu().numpy(), rg, ru)
    got = act.cpu().numpy()
    check_rows(got, ref, CONTRACT)
    check_rows(got, ref, TIGHT)


@pytest.fixture(scope="module")
def config5_weights():
    rng = np.random.default_rng(20261202)
    rg, ru = synth.iq3xxs_blocks(rng, N5, K5), synth.iq3xxs_blocks(rng, N5, K5)
    return rg, ru, ops.pack_tiles("iq3_xxs", rg, K5), ops.pack_tiles("iq3_xxs", ru, K5)


def test_w4a8_gate_up_vs_reference_kernel(config5_weights):
    """The reference's p8w4ffn7 (oracle/_ref) and the library on the same int8 tokens,
    the same IQ3_XXS weights (the reference's packed7 layout for its kernel, the tile
    layout for the library's) and the same codebook: both within the contract of the
    oracle on a seeded sample of rows, and within 2e-3 of each other over all rows."""
    refkernels.require("p8w4ffn7")
    rg, ru, tg, tu = config5_weights
    rng = np.random.default_rng(7)
    m = 128
    x = tokens16(rng, m, K5, special=False)
    xq, sx, _ = prefill.act_quant_q8(torch.from_numpy(x).cuda())
    lut = prefill.lut8()
    p7g = torch.from_numpy(refkernels.packed7_planes(rg, K5).view(np.uint8).reshape(-1)).cuda()
    p7u = torch.from_numpy(refkernels.packed7_planes(ru, K5).view(np.uint8).reshape(-1)).cuda()
    out16 = torch.full((m, N5), 7.7, dtype=torch.float16, device="cuda")
    refkernels.launch("p8w4ffn7", (m // 64) * (N5 // 64), 256, [p7g, p7u, lut, xq, sx, out16])
    ws = prefill.PrefillWorkspace(m, K5)
    act = prefill.w4a8_gate_up(tg, tu, xq, sx, N5, ws)
    torch.cuda.synchronize()
    assert ws.error() == 0
    rows = np.sort(rng.choice(N5, 256, replace=False))
    ref = oracle.w4a8_gate_up_f64(xq.cpu().numpy(), sx.cpu().numpy(), rg, ru, rows=rows)
    theirs = out16.float().cpu().numpy().astype(np.float64)
    ours = act.cpu().numpy().astype(np.float64)
    check_rows(theirs[:, rows], ref, CONTRACT)     # the oracle restates the reference kernel
    check_rows(ours[:, rows], ref, CONTRACT)
    check_rows(ours[:, rows], ref, TIGHT)
    assert np.isfinite(theirs).all()
    rel = np.linalg.norm(ours - theirs) / np.linalg.norm(theirs)
    assert rel <= 2e-3, rel


def test_w4a8_gate_up_config5_sampled(config5_weights):
    """BASELINE config 5's shape (2048 tokens, 5120 -> 17408) on the W4A8 tier: a
    seeded sample of 128 rows x all 2048 tokens against the float64 oracle."""
    rg, ru, tg, tu = config5_weights
    rng = np.random.default_rng(2048)
    m = 2048
    x = tokens16(rng, m, K5)
    xq, sx, _ = prefill.act_quant_q8(torch.from_numpy(x).cuda())
    ws = prefill.PrefillWorkspace(m, K5)
    act = prefill.w4a8_gate_up(tg, tu, xq, sx, N5, ws)
    torch.cuda.synchronize()
    assert ws.error() == 0
    rows = np.sort(rng.choice(N5, 128, replace=False))
    ref = oracle.w4a8_gate_up_f64(xq.cpu().numpy(), sx.cpu().numpy(), rg, ru, rows=rows)
    got = act[:, torch.from_numpy(rows).cuda()].cpu().numpy()
    check_rows(got, ref, CONTRACT)
    check_rows(got, ref, TIGHT)


def test_w4a8_wrappers_reject_mismatched_tables():
    from thunderllamax_b200._lib import TLXError

    m, k, n = 8, 512, 128
    x = torch.zeros((m, k), dtype=torch.float16, device="cuda")
    with pytest.raises(TLXError):
        prefill.act_quant_q8(x, sx=torch.empty((m, k // 256), dtype=torch.float32, device="cuda"))
    with pytest.raises(TLXError):
        prefill.act_quant_q8(x, rs=torch.empty((m, k // 128), dtype=torch.float32, device="cuda"))
    xq, sx, _ = prefill.act_quant_q8(x)
    w = torch.zeros(16, dtype=torch.uint8, device="cuda")     # never reached: the checks run first
    ws = prefill.PrefillWorkspace(m, k)
    with pytest.raises(TLXError):
        prefill.w4a8_gate_up(w, w, xq, sx[:, :2].contiguous(), n, ws)
    with pytest.raises(TLXError):
        prefill.w4a8_gate_up(w, w, xq, sx, n, ws, lut=torch.zeros(512, dtype=torch.int8, device="cuda"))
    torch.cuda.synchronize()


def test_act_quant_q8_reference_golden_rows_and_ties():
    """The reference's own quantiser outputs (tests/golden/golden_w4a8.npz: an all-zero
    chunk, values under the 1e-6 floor, values near the fp16 range, .5 ties), and rows
    whose every quotient is an exact half-integer (chunk maximum 127, so s = 1)."""
    gold = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_w4a8.npz"))
    xq, sx, rs = prefill.act_quant_q8(torch.from_numpy(gold["q8_x"]).cuda())
    torch.cuda.synchronize()
    quant_equal(xq, sx, rs, (gold["q8_xq"], gold["q8_sx"], gold["q8_rs"]))
    rng = np.random.default_rng(17)
    m, k = 64, 1024
    x = (rng.integers(-127, 127, (m, k)) + 0.5).astype(np.float16)    # exact half-integers
    x.reshape(m, k // 128, 128)[:, :, 0] = 127.0
    xq, sx, rs = prefill.act_quant_q8(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert (sx == 1.0).all()
    quant_equal(xq, sx, rs, oracle.act_quant_q8(x))
