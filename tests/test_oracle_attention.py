"""CPU checks of the attention oracle (oracle/attention.py): the int8 cache round
trip is within half a quantisation step, rotary keeps the norm of each pair, and
the causal mask holds (keys after pos + t do not change row t)."""
import numpy as np

import oracle
from oracle.attention import HD, _norm_rope, _quant8


def test_quant8_round_trip():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(HD) * 2.0
    x[:32] = 0.0                                  # an all-zero group takes the fp16(1e-8) = 0 scale
    with np.errstate(all="raise"):                # no undefined cast on the way
        q, s = _quant8(x)
    back = (q.astype(np.float64) - 128) * np.repeat(s.astype(np.float64), 32)
    assert np.all(np.abs(back - x) <= np.repeat(s.astype(np.float64), 32) * 0.5 + 1e-12)
    # the reference kernel's 0 / 0 = NaN clamps to -127 through fmaxf (byte 1)
    assert s[0] == np.float16(1e-8) == 0 and (q[:32] == 1).all()


def test_quant8_underflowing_scale():
    # a group whose max|x| / 127 underflows fp16: non-zero entries saturate, zeros
    # go to byte 1 (0 / 0 -> NaN -> -127), exactly as the reference's clamp does
    x = np.zeros(HD)
    x[0], x[1] = 1e-7, -1e-7
    q, s = _quant8(x)
    assert s[0] == 0
    assert q[0] == 255 and q[1] == 1 and (q[2:32] == 1).all()


def test_rope_keeps_pair_norms():
    rng = np.random.default_rng(2)
    v = rng.standard_normal(HD)
    w = np.ones(HD, np.float32)
    ang = rng.uniform(0, 100, 32)
    a = _norm_rope(v, w, np.zeros(32))
    b = _norm_rope(v, w, ang)
    assert np.allclose(a[:32] ** 2 + a[32:64] ** 2, b[:32] ** 2 + b[32:64] ** 2)
    assert np.array_equal(a[64:], b[64:])


def test_causal_rows():
    rng = np.random.default_rng(3)
    T, pos, ctx = 4, 20, 64
    qw16 = (rng.standard_normal((T, 24, HD)) / 16).astype(np.float16)
    qrow = rng.standard_normal((T, 12288)).astype(np.float16)
    kv = rng.integers(1, 256, (8, ctx, HD), dtype=np.uint8)
    sc = rng.uniform(0.01, 0.03, (8, ctx, 8)).astype(np.float16)
    a = oracle.attn_decode(qw16, kv, sc, qrow, pos)
    kv2 = kv.copy()
    kv2[:, pos + 2:] = rng.integers(1, 256, (8, ctx - pos - 2, HD), dtype=np.uint8)
    b = oracle.attn_decode(qw16, kv2, sc, qrow, pos)
    assert np.array_equal(a[:2], b[:2]) and not np.array_equal(a[2:], b[2:])
