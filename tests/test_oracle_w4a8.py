"""The W4A8 prefill tier on the CPU: the oracle (oracle/w4a8.py) against the golden
fixture made by the reference's own code (tests/golden/gen_golden_w4a8.py), the
restated packed7 layout the reference kernel reads, the device codebook the library
uploads, and the C ABI's host-side argument checks (no GPU)."""
import os
import sys

import numpy as np

import oracle
from thunderllamax_b200 import _lib, tables

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import refkernels  # noqa: E402

GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_w4a8.npz"))
K = 512


def test_quantiser_matches_reference_bit_for_bit():
    xq, sx, rs = oracle.act_quant_q8(GOLD["q8_x"])
    assert np.array_equal(xq, GOLD["q8_xq"])
    assert np.array_equal(sx.view(np.uint32), GOLD["q8_sx"].view(np.uint32))
    assert np.array_equal(rs, GOLD["q8_rs"])


def test_quantiser_edge_cases():
    xq, sx, rs = oracle.act_quant_q8(GOLD["q8_x"])
    # all-zero chunk: the 1e-6 floor, all levels 0
    assert sx[1, 1] == np.float32(1e-6) * np.float32(1.0 / 127.0) and not xq[1, 128:256].any()
    # a chunk whose maximum is 127: s = 1 and the .5 steps round to even
    assert sx[4, 0] == 1.0
    assert list(xq[4, 1:9]) == [-62, -62, -60, -60, -58, -58, -56, -56]
    assert (np.abs(xq.astype(np.int32)) <= 127).all()
    assert np.array_equal(rs, xq.astype(np.int32).reshape(8, 4, 128).sum(axis=2))
    # every chunk with a nonzero maximum above the floor reaches +-127
    big = np.abs(GOLD["q8_x"].astype(np.float32)).reshape(8, 4, 128).max(axis=2) > 1e-6
    assert (np.abs(xq.astype(np.int32)).reshape(8, 4, 128).max(axis=2)[big] == 127).all()


def test_codebook_matches_reference():
    assert np.array_equal(oracle.lut8_levels(), GOLD["lut8"])
    assert np.array_equal(tables.iq3xxs_levels_lut8(), GOLD["lut8"])      # what the library uploads
    assert set(np.unique(GOLD["lut8"])) == {1, 3, 5, 7, 9, 11, 13, 15}


def test_linearised_dequant_matches_reference_bit_for_bit():
    w = oracle.dequant_iq3xxs_lin(GOLD["lin_raw"], K)
    assert np.array_equal(w.view(np.uint32), GOLD["lin_w"].astype(np.float32).view(np.uint32))
    # the linearised weights track the IQ3_XXS ones (grid ~= 4.0507 * level, 62 -> 15 the worst)
    ref = oracle.dequant_iq3xxs(GOLD["lin_raw"], K)
    assert np.abs(w - ref).max() <= 0.021 * np.abs(ref).max()


def test_packed7_restatement_matches_reference_packer():
    p = refkernels.packed7_planes(GOLD["lin_raw"], K)
    assert np.array_equal(p.view(np.uint8).ravel(), GOLD["packed7"])


def test_w4a8_oracle_gate_up_small():
    rng = np.random.default_rng(5)
    from thunderllamax_b200 import synth

    rg, ru = synth.iq3xxs_blocks(rng, 8, K), synth.iq3xxs_blocks(rng, 8, K)
    x = (rng.standard_normal((3, K)) * 0.7).astype(np.float16)
    xq, sx, _ = oracle.act_quant_q8(x)
    act = oracle.w4a8_gate_up_f64(xq, sx, rg, ru)
    X = xq.astype(np.float64) * np.repeat(sx.astype(np.float64), 128, axis=1)
    g = X @ oracle.dequant_iq3xxs_lin(rg, K).astype(np.float64).T
    u = X @ oracle.dequant_iq3xxs_lin(ru, K).astype(np.float64).T
    assert np.allclose(act, g / (1 + np.exp(-g)) * u, rtol=1e-12, atol=0)
    sub = oracle.w4a8_gate_up_f64(xq, sx, rg, ru, rows=np.array([5, 2]))
    assert np.allclose(sub, act[:, [5, 2]], rtol=1e-12, atol=0)


def test_w4a8_entry_points_host_checks():
    # argument checks run on the host, before any CUDA call (no GPU needed)
    lib = _lib.lib()
    err_shape, err_align, err_ws, err_null = -1, -2, -5, -8
    a = 1 << 20   # an aligned stand-in address (never dereferenced)
    assert lib.tlx_act_quant_q8(None, 512, 4, 512, a, 512, a, a, None) == err_null
    assert lib.tlx_act_quant_q8(a, 512, 0, 512, a, 512, a, a, None) == err_shape
    assert lib.tlx_act_quant_q8(a, 512, 4, 500, a, 512, a, a, None) == err_shape       # k % 128
    assert lib.tlx_act_quant_q8(a, 256, 4, 512, a, 512, a, a, None) == err_align       # ldx < k
    assert lib.tlx_act_quant_q8(a + 2, 512, 4, 512, a, 512, a, a, None) == err_align   # x not 8-byte aligned
    assert lib.tlx_act_quant_q8(a, 512, 4, 512, a + 1, 512, a, a, None) == err_align   # xq not 4-byte aligned
    ws = int(lib.tlx_prefill_workspace_bytes(4, K))
    args = lambda **o: [o.get(n, v) for n, v in (("wg", a), ("wu", a), ("lut", a), ("xq", a), ("ldq", K),  # noqa: E731
                                                ("sx", a), ("m", 4), ("n", 256), ("k", K), ("act", a),
                                                ("lda", 256), ("ws", a), ("wsb", ws), ("s", None))]
    f = lib.tlx_prefill_w4a8_gate_up
    assert f(*args(lut=None)) == err_null
    assert f(*args(ws=None)) == err_null
    assert f(*args(n=200)) == err_shape            # n_rows % 128
    assert f(*args(k=384, ldq=384)) == err_shape   # k % 256
    assert f(*args(lda=128)) == err_shape          # ld_act < n_rows
    assert f(*args(ldq=516)) == err_align          # ldq % 8
    assert f(*args(lut=a + 2)) == err_align        # lut8 not 4-byte aligned
    assert f(*args(wg=a + 8)) == err_align         # weights not 16-byte aligned
    assert f(*args(wsb=1024)) == err_ws            # workspace smaller than the token image


def test_tier_weights_are_one_fp16_rounding_of_the_reference_weights():
    # the library's decode of a linearised weight: level * (2s+1) (exact in fp16, at most
    # 15 * 31), times fp16(d / 4), one fp16 rounding; the factor 4.0507 rides on the
    # staged token values.  Against the reference's weights (dq_lin, the golden fixture)
    # that is within 2^-11 relative, plus the fp32 rounding of the reference's own scale.
    raw = GOLD["lin_raw"]
    n, nb = raw.shape[0], K // 256
    blk = raw.reshape(n, nb, 98)
    d = np.ascontiguousarray(blk[..., 0:2]).view(np.float16)[..., 0]            # [n, nb]
    sw = np.ascontiguousarray(blk[..., 66:98]).view(np.uint32)                   # [n, nb, 8]
    m2 = (2 * (sw >> 28) + 1).astype(np.float16)                                 # 2s+1
    lv = GOLD["lut8"].reshape(256, 4)[blk[..., 2:66]].reshape(n, nb, 8, 32).astype(np.float16)
    prod = lv * m2[..., None]
    assert np.array_equal(prod.astype(np.float64), lv.astype(np.float64) * m2[..., None].astype(np.float64))
    a = prod * (d.astype(np.float32) * np.float32(0.25)).astype(np.float16)[..., None, None]
    ours = np.abs(a.astype(np.float64).reshape(n, K)) * 4.0507
    ref = np.abs(GOLD["lin_w"].astype(np.float64))
    assert (np.abs(ours - ref) <= ref * (2.0 ** -11 + 2.0 ** -21)).all()
