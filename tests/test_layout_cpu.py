"""CPU checks of the C library: it loads, exports the header's symbols, and its
tile packer + the decoder arithmetic (restated here in numpy, lane by lane, the
way formats.cuh's q6_group / iq3_mma compute) reproduce the oracle's exact fp32
weights.  No GPU calls."""
import os
import re

import numpy as np
import pytest

import oracle
from oracle.dequant import _scale_min_k4
from thunderllamax_b200 import _lib, ops, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "tlx_verify.h")).read()
    return sorted(set(re.findall(r"^\s*(?:[\w\*]+\s+)+\**(tlx_\w+)\s*\(", src, re.M)))


def test_library_exports_every_header_symbol():
    lib = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 15
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    assert lib.tlx_version() >= 1


def test_error_strings_and_host_argument_checks():
    lib = _lib.lib()
    assert lib.tlx_error_string(-1).decode().startswith("unsupported")
    assert lib.tlx_tiled_bytes(14, 10, 300) == 0          # k not a multiple of 256
    assert lib.tlx_tiled_bytes(99, 16, 256) == 0          # unknown qtype
    assert lib.tlx_tiled_bytes(14, 17, 512) == 2 * 2 * 3360
    assert lib.tlx_gemv_workspace_bytes(0, 14, 16, 256, 17, 30) == 0   # m > 16
    assert lib.tlx_gemv_workspace_bytes(0, 14, 16, 256, 6, 0) == 0     # fp32 x: m <= 5


def test_peer_and_slot_table_host_checks():
    # the peer exchange and GDN slot-table entry points reject bad arguments on the
    # host, before any CUDA call (no GPU needed)
    import ctypes

    lib = _lib.lib()
    err_null, err_shape, err_align = -8, -1, -2
    # slot table: 2 x 12 eight-byte addresses per GDN block
    assert lib.tlx_gdn_slots_bytes(48) == 48 * 2 * 12 * 8
    assert lib.tlx_gdn_slots_bytes(0) == 0 and lib.tlx_gdn_slots_bytes(-3) == 0
    six, seven = (ctypes.c_void_p * 6)(*([8] * 6)), (ctypes.c_void_p * 7)(*([8] * 7))
    assert lib.tlx_gdn_slots_init(None, 8, 8, seven, six, 48, 64, 32, None) == err_null
    assert lib.tlx_gdn_slots_init(8, 8, 8, seven, six, 0, 64, 32, None) == err_shape
    assert lib.tlx_gdn_slots_init(12, 8, 8, seven, six, 48, 64, 32, None) == err_align    # table not 8-byte aligned
    seven_null = (ctypes.c_void_p * 7)(*([8] * 6 + [None]))
    assert lib.tlx_gdn_slots_init(8, 8, 8, seven_null, six, 48, 64, 32, None) == err_null
    assert lib.tlx_acceptsel11k_flip(None, 8, 48, None) == err_null
    assert lib.tlx_acceptsel11k_flip(8, None, 48, None) == err_null
    assert lib.tlx_acceptsel11k_flip(8, 8, 0, None) == err_shape
    assert lib.tlx_acceptsel11k_flip(12, 8, 48, None) == err_align
    # peer exchange: world in 2..8, rank in range, buffers 256-byte aligned, m <= 16
    assert lib.tlx_peer_buffer_bytes(1, 11, 5120) == 0 and lib.tlx_peer_buffer_bytes(9, 11, 5120) == 0
    assert lib.tlx_peer_buffer_bytes(2, 17, 5120) == 0
    assert lib.tlx_peer_buffer_bytes(8, 11, 5120) == 4096 + 2 * 11 * 5120 * 4
    two = (ctypes.c_void_p * 2)(256, 512)
    misaligned = (ctypes.c_void_p * 2)(256, 520)
    assert lib.tlx_peer_publish(2, 0, None, 5, 2048, 256, 2048, None) == err_null
    assert lib.tlx_peer_publish(1, 0, two, 5, 2048, 256, 2048, None) == err_shape       # world < 2
    assert lib.tlx_peer_publish(2, 2, two, 5, 2048, 256, 2048, None) == err_shape       # rank out of range
    assert lib.tlx_peer_publish(2, 0, two, 17, 2048, 256, 2048, None) == err_shape      # m > 16
    assert lib.tlx_peer_publish(2, 0, two, 5, 2048, 256, 1024, None) == err_shape       # row stride < ny
    assert lib.tlx_peer_publish(2, 0, two, 5, 2048, None, 2048, None) == err_null
    assert lib.tlx_peer_publish(2, 0, misaligned, 5, 2048, 256, 2048, None) == err_align
    assert lib.tlx_peer_finish(2, 0, misaligned, 5, 2048, None, 0, 256, 2048, 256, None) == err_align


@pytest.mark.parametrize("qtype,gen,bb", [("q6_k", synth.q6k_blocks, 210), ("iq3_xxs", synth.iq3xxs_blocks, 98),
                                          ("iq4_xs", synth.iq4xs_blocks, 136), ("q4_k", synth.q4k_blocks, 144),
                                          ("q5_k", synth.q5k_blocks, 176), ("q8_0", synth.q8_0_blocks, 272)])
def test_pack_unpack_round_trip(qtype, gen, bb):
    rng = np.random.default_rng(1)
    for n in (1, 16, 37):
        raw = gen(rng, n, 512)
        t = ops.pack_tiles_host(qtype, raw, 512)
        assert t.size == ((n + 15) // 16) * 2 * 16 * bb
        back = ops.unpack_tiles_host(qtype, t, n, 512, raw.shape[1])
        assert np.array_equal(back, raw)


def _f16(x):
    return np.float32(np.float16(x))


def emulate_q6(tiled, n_rows, k):
    """Weights as the device decodes them: d * fp16((q-32)*sc) per (row, k)."""
    nb = k // 256
    T = (n_rows + 15) // 16
    W = np.zeros((T * 16, k), np.float32)
    ch = tiled.reshape(T, nb, 3360)
    for t in range(T):
        for b in range(nb):
            c = ch[t, b]
            d16 = c[3328:3360].view(np.float16).astype(np.float32).reshape(8, 2)
            for lane in range(32):
                g, q = lane >> 2, lane & 3
                w = np.array([c[((i >> 2) * 32 + lane) * 16 + (i & 3) * 4:][:4].view(np.uint32)[0]
                              for i in range(24)], dtype=np.uint64)
                sc = (c[3072 + lane * 8:3080 + lane * 8] ^ 0x80).view(np.int8).astype(np.float32)
                for gam in range(8):
                    W0, W1, W2 = (int(v) for v in w[3 * gam:3 * gam + 3])
                    magic = 0x64006400
                    # every field at mantissa offset 4 (value 1024 + 16q), one fma
                    # (1024 + 16q) * (sc/16) - 96 sc per formats.cuh q6_group
                    p = [(W0 & 0x03F003F0) | magic, ((W0 >> 6) & 0x03F003F0) | magic,
                         (W1 & 0x03F003F0) | magic, ((W1 >> 6) & 0x03F003F0) | magic,
                         (W2 & 0x03F003F0) | magic, ((W2 >> 6) & 0x03F003F0) | magic,
                         ((W0 << 4) & 0x00F000F0) | ((W2 << 8) & 0x03000300) | magic,
                         ((W1 << 4) & 0x00F000F0) | ((W2 << 6) & 0x03000300) | magic]
                    for pi, pv in enumerate(p):
                        mu, r = pi >> 2, pi & 3
                        m = 2 * gam + mu
                        rr = r & 1
                        row = t * 16 + g + 8 * rr
                        s = np.float64(sc[(gam >> 1) * 2 + rr])
                        for h in range(2):
                            half = (pv >> (16 * h)) & 0xFFFF
                            v = np.float64(np.frombuffer(np.uint16(half).tobytes(), np.float16)[0])
                            # fused multiply-add: exact product and sum, one fp16 rounding
                            a = _f16(v * (s / 16.0) - 96.0 * s)
                            kk = b * 256 + 64 * q + 4 * m + 2 * (r >> 1) + h
                            W[row, kk] = d16[g, rr] * a
    return W[:n_rows]


def emulate_iq3(tiled, n_rows, k):
    grid = oracle.iq3xxs_grid_u32()
    nb = k // 256
    T = (n_rows + 15) // 16
    W = np.zeros((T * 16, k), np.float32)
    ch = tiled.reshape(T, nb, 1568)
    for t in range(T):
        for b in range(nb):
            c = ch[t, b]
            d16 = c[1536:1568].view(np.float16).astype(np.float32).reshape(8, 2)
            for lane in range(32):
                g, q = lane >> 2, lane & 3
                sw = c[1024 + lane * 16:1040 + lane * 16].view(np.uint32).reshape(2, 2)
                for m in range(16):
                    cc, l, e = m >> 3, (m >> 1) & 3, m & 1
                    for rr in range(2):
                        idx = c[rr * 512 + lane * 16 + m]
                        G = int(grid[idx])
                        u = int(sw[rr, cc])
                        # formats.cuh iq3_word: parities of the four fields at once, the
                        # scale gathered from bits 19 + 4j by one multiply
                        y0 = u & 0x7777FFFF
                        y = y0 ^ (y0 >> 16)
                        y ^= y >> 2
                        y ^= y >> 1
                        sg = ((y << 19) & 0x88880000) | y0
                        gsc = (((u >> 19) & 0x1111) * 0x12481248) & 0xFFFFFFFF
                        ms = 2 * ((gsc >> 12) & 0xF) + 1
                        assert ms == 2 * ((gsc >> 28) & 0xF) + 1
                        for j in range(4):
                            mag = (G >> (8 * j)) & 0xFF
                            i = 2 * e + (j >> 1)           # sign pair of the field
                            # pair_signs: bit 15 (even weight) / 31 (odd weight) after one shift
                            mask = (sg << (15 - 4 * l - i)) & 0x80008000
                            neg = (mask >> (31 if j & 1 else 15)) & 1
                            a = float(mag * ms) * (-1.0 if neg else 1.0)
                            row = t * 16 + g + 8 * rr
                            kk = b * 256 + 64 * q + 4 * m + j
                            W[row, kk] = (d16[g, rr] * np.float32(0.25)) * np.float32(a)
    return W[:n_rows]


def emulate_q4k(tiled, n_rows, k):
    """Q4_K as the device decodes it (formats.cuh q4_load / q4_mma): the exact
    integers sc * v per weight and the sub-block mins, combined as d * (sc v) - dmin * mn
    (the kernel applies d and dmin to the sums; per weight this is the same value)."""
    nb = k // 256
    T = (n_rows + 15) // 16
    W = np.zeros((T * 16, k), np.float32)
    ch = tiled.reshape(T, nb, 2304)
    for t in range(T):
        for b in range(nb):
            c = ch[t, b]
            for lane in range(32):
                g, q = lane >> 2, lane & 3
                for rr in range(2):
                    row = g + 8 * rr
                    hdr = c[2048 + 16 * row:2064 + 16 * row]
                    d = np.float32(hdr[0:2].view(np.float16)[0])
                    dmin = np.float32(hdr[2:4].view(np.float16)[0])
                    sc, mn = _scale_min_k4(hdr[4:16][None])
                    qs = np.concatenate([c[((2 * rr + hf) * 32 + lane) * 16:][:16] for hf in range(2)])
                    for m in range(16):
                        s_ = 2 * q + (m >> 3)
                        for i in range(4):
                            byte = int(qs[4 * (m & 7) + i])
                            v = (byte & 0xF) if m < 8 else (byte >> 4)
                            a = np.float32(int(sc[0, s_]) * v)          # exact fp16 integer
                            kk = b * 256 + 64 * q + 4 * m + i
                            W[t * 16 + row, kk] = d * a - dmin * np.float32(int(mn[0, s_]))
    return W[:n_rows]


def emulate_q5k(tiled, n_rows, k):
    """Q5_K as the device decodes it (formats.cuh q4_load<true> / q4_mma<true>): the
    Q4_K nibble path plus the fifth bit, taken from the regrouped byte of word i with
    the multiply-and-shift spread q4_mma applies (bits 4 / 20 for the low nibbles,
    8 / 24 for the high ones), then d * (sc q) - dmin * mn."""
    nb = k // 256
    T = (n_rows + 15) // 16
    W = np.zeros((T * 16, k), np.float32)
    ch = tiled.reshape(T, nb, 2816)
    for t in range(T):
        for b in range(nb):
            c = ch[t, b]
            for lane in range(32):
                g, q = lane >> 2, lane & 3
                for rr in range(2):
                    row = g + 8 * rr
                    hdr = c[2560 + 16 * row:2576 + 16 * row]
                    d = np.float32(hdr[0:2].view(np.float16)[0])
                    dmin = np.float32(hdr[2:4].view(np.float16)[0])
                    sc, mn = _scale_min_k4(hdr[4:16][None])
                    qs = np.concatenate([c[((2 * rr + hf) * 32 + lane) * 16:][:16] for hf in range(2)])
                    hb = c[2048 + lane * 16 + rr * 8:][:8]
                    for m in range(16):
                        s_ = 2 * q + (m >> 3)
                        x = (int(hb[m & 7]) * 0x00100001) & 0xFFFFFFFF
                        if m < 8:
                            hw = [x & 0x00100010, (x >> 1) & 0x00100010]
                        else:
                            hw = [(x << 2) & 0x01000100, (x << 1) & 0x01000100]
                        for i in range(4):
                            byte = int(qs[4 * (m & 7) + i])
                            half = (hw[i >> 1] >> (16 * (i & 1))) & 0xFFFF
                            if m < 8:
                                v = (byte & 0xF) | (half & 0x10)          # v + 16 h
                            else:
                                v = ((byte >> 4) << 4 | (half & 0x100)) >> 4
                            a = np.float32(int(sc[0, s_]) * v)
                            kk = b * 256 + 64 * q + 4 * m + i
                            W[t * 16 + row, kk] = d * a - dmin * np.float32(int(mn[0, s_]))
    return W[:n_rows]


def emulate_q8(tiled, n_rows, k):
    """Q8_0 as the device decodes it (formats.cuh q8_load / q8_mma): fp16(d * q)."""
    nb = k // 256
    T = (n_rows + 15) // 16
    W = np.zeros((T * 16, k), np.float32)
    ch = tiled.reshape(T, nb, 4352)
    for t in range(T):
        for b in range(nb):
            c = ch[t, b]
            for lane in range(32):
                g, q = lane >> 2, lane & 3
                dd = c[4096 + 8 * lane:4104 + 8 * lane].view(np.float16)
                for rr in range(2):
                    row = g + 8 * rr
                    qs = np.concatenate([c[((4 * rr + j) * 32 + lane) * 16:][:16] for j in range(4)]).view(np.int8)
                    for m in range(16):
                        d = dd[2 * rr + (m >> 3)]
                        for i in range(4):
                            kk = b * 256 + 64 * q + 4 * m + i
                            W[t * 16 + row, kk] = np.float32(np.float16(np.float32(qs[4 * m + i]) * np.float32(d)))
    return W[:n_rows]


def test_q5k_tile_decode_matches_oracle_exactly():
    rng = np.random.default_rng(11)
    raw = synth.q5k_blocks(rng, 19, 512)
    got = emulate_q5k(ops.pack_tiles_host("q5_k", raw, 512), 19, 512)
    assert np.array_equal(got.view(np.uint32), oracle.dequant_q5k(raw, 512).view(np.uint32))


def test_q8_tile_decode_is_the_fp16_rounded_oracle():
    rng = np.random.default_rng(12)
    raw = synth.q8_0_blocks(rng, 21, 512)
    got = emulate_q8(ops.pack_tiles_host("q8_0", raw, 512), 21, 512)
    ref = oracle.dequant_q8_0(raw, 512).astype(np.float16).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q4k_tile_decode_matches_oracle_exactly():
    rng = np.random.default_rng(10)
    raw = synth.q4k_blocks(rng, 19, 512)
    got = emulate_q4k(ops.pack_tiles_host("q4_k", raw, 512), 19, 512)
    assert np.array_equal(got.view(np.uint32), oracle.dequant_q4k(raw, 512).view(np.uint32))


def test_q6_tile_decode_matches_oracle_exactly():
    rng = np.random.default_rng(7)
    raw = synth.q6k_blocks(rng, 19, 512)
    tiled = ops.pack_tiles_host("q6_k", raw, 512)
    got = emulate_q6(tiled, 19, 512)
    ref = oracle.dequant_q6k(raw, 512)
    assert np.array_equal(got, ref)


def test_q6_tile_decode_full_range_scales():
    # real checkpoints use int8 sub-scales in [-128, 127]: integer products in
    # (2048, 4096] round to even (<= 2^-11 relative), exact for |(q-32)*sc| <= 2048
    rng = np.random.default_rng(8)
    raw = synth.q6k_blocks(rng, 16, 256).reshape(16, 1, 210)
    raw[:, :, 192:208] = rng.integers(-128, 128, (16, 1, 16)).astype(np.int8).view(np.uint8)
    raw = raw.reshape(16, 210)
    got = emulate_q6(ops.pack_tiles_host("q6_k", raw, 256), 16, 256)
    ref = oracle.dequant_q6k(raw, 256)
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)
    assert rel.max() <= 2.0 ** -11
    d = raw[:, 208:210].copy().view(np.float16).astype(np.float32)
    small = np.abs(ref) <= 2048 * d
    assert np.array_equal(got[small], ref[small])


def test_iq3_tile_decode_matches_oracle_exactly():
    rng = np.random.default_rng(9)
    raw = synth.iq3xxs_blocks(rng, 21, 512)
    tiled = ops.pack_tiles_host("iq3_xxs", raw, 512)
    got = emulate_iq3(tiled, 21, 512)
    ref = oracle.dequant_iq3xxs(raw, 512)
    assert np.array_equal(got, ref)


def emulate_iq4(tiled, n_rows, k):
    """IQ4_XS weights as moe.cu decodes them: lane (g, q), mma m reads qs bytes
    2m, 2m+1 of its 32-byte slice; byte -> (kv[lo], kv[hi]) fp16 pair times the
    sub-block scale (ls - 32) in fp16, times d in fp32.  Also checks that the
    (lane, m, half) -> k map of the activation image covers every k once."""
    kv = oracle.iq4nl_kvalues().astype(np.float32)
    nb = k // 256
    T = (n_rows + 15) // 16
    W = np.zeros((T * 16, k), np.float32)
    hit = np.zeros((T * 16, k), np.int32)
    ch = tiled.reshape(T, nb, 2176)
    for t in range(T):
        for b in range(nb):
            c = ch[t, b]
            for lane in range(32):
                g, q = lane >> 2, lane & 3
                units = [c[(u * 32 + lane) * 16:(u * 32 + lane) * 16 + 16] for u in range(4)]
                for rr in range(2):
                    hd = c[2048 + g * 16 + rr * 8:2048 + g * 16 + rr * 8 + 8]
                    d = np.float32(hd[0:2].view(np.float16)[0])
                    sh = int(hd[2:4].view(np.uint16)[0])
                    sl = int(hd[4:8].view(np.uint32)[0])
                    qs = np.concatenate(units[2 * rr:2 * rr + 2])  # 32 bytes of sub-blocks 2q, 2q+1
                    for m in range(16):
                        hh = m >> 3
                        ls = ((sl >> (8 * q + 4 * hh)) & 15) | (((sh >> (4 * q + 2 * hh)) & 3) << 4)
                        s16 = np.float16(ls - 32)
                        k0 = 64 * q + 32 * hh + 2 * (m & 7)
                        for jb in range(2):
                            byte = int(qs[2 * m + jb])
                            for nib, dk in ((byte & 15, 0), (byte >> 4, 16)):
                                a = np.float16(np.float16(kv[nib]) * s16)
                                row = t * 16 + g + 8 * rr
                                kk = b * 256 + k0 + jb + dk
                                W[row, kk] = d * np.float32(a)
                                hit[row, kk] += 1
    assert (hit == 1).all()
    return W[:n_rows]


def test_iq4_tile_decode_matches_oracle():
    # exact where |kv * (ls - 32)| <= 2048; larger integer products round once in fp16
    rng = np.random.default_rng(10)
    raw = synth.iq4xs_blocks(rng, 18, 512)
    got = emulate_iq4(ops.pack_tiles_host("iq4_xs", raw, 512), 18, 512)
    ref = oracle.dequant_iq4xs(raw, 512)
    blk = raw.reshape(18, 2, 136)
    d = blk[..., 0:2].copy().view(np.float16).astype(np.float32)[..., 0]
    scale = np.repeat(d, 256, axis=1)
    small = np.abs(ref) <= 2048 * scale
    assert small.mean() > 0.5
    assert np.array_equal(got[small], ref[small])
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)
    assert rel.max() <= 2.0 ** -11


def test_moe_workspace_rejects_bad_shapes():
    lib = _lib.lib()
    assert lib.tlx_moe_workspace_bytes(9, 256, 2048, 512) == 0      # > 8 positions
    assert lib.tlx_moe_workspace_bytes(5, 4, 2048, 512) == 0        # fewer experts than top-8
    assert lib.tlx_moe_workspace_bytes(5, 256, 2000, 512) == 0      # hidden not a multiple of 256
    assert lib.tlx_moe_workspace_bytes(5, 256, 2048, 500) == 0      # inner not a multiple of 256
    assert lib.tlx_moe_workspace_bytes(5, 256, 2048, 512) > 0
