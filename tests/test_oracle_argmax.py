"""The oracle's argmax rule (the reference scan: best = -1e30, strict '>', lowest
index on ties) and h_argmax side effects, on CPU (engine/amx3.cu:117-142,
engine/h_argmax.cu:13-42)."""
import numpy as np

import oracle


def _scan(row):
    """The reference's scalar scan, written out."""
    best, bidx = -1e30, 0
    for i, v in enumerate(row):
        if v > best or (v == best and i < bidx):
            best, bidx = v, i
    return bidx


def test_argmax_rule_matches_the_scan():
    rng = np.random.default_rng(3)
    rows = [
        [1.0, 3.0, 3.0, np.nan],
        [np.nan] * 4,
        [-0.0, 0.0, -1.0, -2.0],
        [np.nan, -np.inf, -np.inf],          # no candidate -> 0
        [-np.inf, -5.0, np.nan, -5.0],
        [-1e31, -2e30, -5.0],
        [np.inf, 1.0, np.inf],
    ]
    for _ in range(20):
        r = rng.standard_normal(9)
        r[rng.integers(0, 9, 3)] = r[0]        # ties
        r[rng.integers(0, 9)] = np.nan
        rows.append(list(r))
    for row in rows:
        assert oracle.argmax_rows(np.array([row]))[1][0] == _scan(row), row


def test_h_argmax_side_effects():
    rng = np.random.default_rng(4)
    lg = rng.standard_normal(1000).astype(np.float16)
    hist = np.full(32, -1, dtype=np.int32)
    idx, hist2, pos2 = oracle.h_argmax(lg, hist, 5)
    assert idx == _scan(lg.astype(np.float64))
    assert pos2 == 6 and hist2[5] == idx
    assert (np.delete(hist2, 5) == -1).all() and (hist == -1).all()


def test_acceptsel11k_slot_table():
    # the reference's own table (engine/acceptsel11k.cu:5-6): rec m<5 slot m, m==5
    # rec6x ... m==10 rec11x; conv m<4 slot m, m==4 conv5x ... m==10 conv11x
    B, R, C = 2, 3, 2
    rec4 = np.arange(B * 5 * R, dtype=np.float32).reshape(B, 5, R)
    conv4 = -np.arange(B * 5 * C, dtype=np.float32).reshape(B, 5, C)
    rec_x = [np.full((B, R), 100 + 6 + i, np.float32) for i in range(6)]     # rec6x..rec11x
    conv_x = [np.full((B, C), -(100 + 5 + i), np.float32) for i in range(7)]  # conv5x..conv11x
    for m in range(11):
        r, c = oracle.acceptsel11k(rec4, conv4, m, conv_x, rec_x)
        want_r = rec4[:, m] if m < 5 else np.full((B, R), 100 + m + 1, np.float32)
        want_c = conv4[:, m] if m < 4 else np.full((B, C), -(100 + m + 1), np.float32)
        assert np.array_equal(r[:, 4], want_r) and np.array_equal(c[:, 4], want_c), m
        assert np.array_equal(np.delete(r, 4, axis=1), np.delete(rec4, 4, axis=1))
        assert np.array_equal(np.delete(c, 4, axis=1), np.delete(conv4, 4, axis=1))
    r, c = oracle.acceptsel11k(rec4, conv4, 11, conv_x, rec_x)   # out of range: no copy
    assert np.array_equal(r, rec4) and np.array_equal(c, conv4)
