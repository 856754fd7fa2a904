"""Pin the numpy oracle to the reference's own ports (golden_v1.npz, made by
tests/golden/gen_golden.py from engine/mm/MM_P2_ports.py, MM_P0_d2_repack.py
and engine/pack_w4.py with gguf-py tables)."""
import numpy as np

import oracle
from inputs import cmb_inputs, router_inputs


def test_q6k_dequant_bit_exact(golden):
    got = oracle.dequant_q6k(golden["q6k_raw"], 512)
    assert np.array_equal(got.view(np.uint32), golden["q6k_ref"].view(np.uint32))


def test_iq4xs_dequant_bit_exact(golden):
    got = oracle.dequant_iq4xs(golden["iq4xs_raw"], 512)
    assert np.array_equal(got.view(np.uint32), golden["iq4xs_ref"].view(np.uint32))


def test_iq3xxs_dequant_vs_upstream_and_reference(golden):
    got = oracle.dequant_iq3xxs(golden["iq3xxs_raw"], 512)
    # exact fp32 values == gguf-py (the port of ggml dequantize_row_iq3_xxs)
    assert np.array_equal(got.view(np.uint32), golden["iq3xxs_gguf_f32"].astype(np.float32).view(np.uint32))
    # the reference's own port rounds each weight to fp16 (engine/pack_w4.py:69)
    assert np.array_equal(got.astype(np.float16), golden["iq3xxs_ref_f16"].astype(np.float16))


def _rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.linalg.norm(b), 1e-30)


def test_moe_lanes_vs_reference_kernel_order(golden):
    H = 2048
    Wg = oracle.dequant_iq4xs(golden["gxup4_rows_g"], H)
    Wu = oracle.dequant_iq4xs(golden["gxup4_rows_u"], H)
    x = golden["gxup4_x"]
    act = oracle.silu_f64(oracle.matvec_f64(Wg, x[None])[0]) * oracle.matvec_f64(Wu, x[None])[0]
    assert _rel_err(act, golden["gxup4_ref"]) < 1e-5
    a = golden["gxdn_act"]
    y4 = oracle.matvec_f64(oracle.dequant_iq4xs(golden["gxdn_rows4"], 512), a[None])[0]
    y6 = oracle.matvec_f64(oracle.dequant_q6k(golden["gxdn_rows6"], 512), a[None])[0]
    # the reference stores these parts in fp16 (engine/mm/MM_P2_gx8e256dn.cu:43):
    # the f64 oracle must sit within one fp16 rounding (+ fp32 order noise) of it
    for y, ref in ((y4, golden["gxdn4_ref"]), (y6, golden["gxdn6_ref"])):
        ref = ref.astype(np.float64)
        assert np.isfinite(ref).all()
        bound = np.abs(ref) * 2.0 ** -11 + np.linalg.norm(ref) * 1e-6
        assert (np.abs(y - ref) <= bound).all()


def test_router_vs_reference(golden):
    Wr, wsh, h = router_inputs()
    ids, gates, sg, lg = oracle.router_top8(Wr, wsh, h)
    # logits: reference fp32 kernel order vs f64
    assert _rel_err(lg, golden["router_logits"]) < 1e-6
    # selected experts bit-exact (the f64 top-8 gaps are far above fp32 error)
    assert np.array_equal(ids, golden["router_ids"])
    np.testing.assert_allclose(gates, golden["router_gates"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(sg, golden["router_sg"], rtol=1e-5, atol=1e-7)


def test_combine_vs_reference(golden):
    gates, sg, part, shared = cmb_inputs()
    acc = (gates[:, :, None].astype(np.float64) * part.astype(np.float64)).sum(axis=1)
    acc += sg[:, None].astype(np.float64) * shared
    ref = golden["cmb_ref"].astype(np.float64)
    # reference rounds the fp32 sum to fp16 (MM_P2_ports.py:237-248)
    assert np.abs(acc - ref).max() <= np.abs(ref).max() * 2.0 ** -10


def test_accept_semantics():
    # engine/accept11k.cu:25-36 ladder / engine/mm/MM_P7_acc36.cu:18-24
    amds = np.array([5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15])
    assert oracle.accept(amds, [5, 6, 7, 8, 9, 10, 11, 12, 13, 14]) == (10, 15)
    assert oracle.accept(amds, [1, 6, 7, 8, 9, 10, 11, 12, 13, 14]) == (0, 5)
    assert oracle.accept(amds, [5, 6, 0, 8, 9, 10, 11, 12, 13, 14]) == (2, 7)
    assert oracle.accept(amds, [5, 6, 7], k=3) == (3, 8)
    assert oracle.accept(amds, [], k=0) == (0, 5)


def test_accept11k_side_effects():
    amds = np.arange(100, 111, dtype=np.int32)
    drafts = np.array([100, 101, 102, 0, 0, 0, 0, 0, 0, 0], np.int32)
    st = {"pos": 7, "cyc": 3, "cur": -1, "m_slot": -1, "tok_hist": np.zeros(32, np.int32),
          "m_hist": np.zeros(8, np.int32), "l_hist": np.array([0, 0, 0, 9, 0, 0, 0, 0], np.int32)}
    xA = np.arange(11 * 4, dtype=np.float32)
    st2, emit, h_seed, dhd = oracle.accept11k(amds, drafts, st, xA=xA, hd_d0=np.zeros(4), hd_d1=np.ones(4), dim=4)
    assert st2["pos"] == 7 + 3 + 1 and st2["cur"] == 103 and st2["m_slot"] == 3 and st2["cyc"] == 4
    assert list(st2["tok_hist"][7:11]) == [100, 101, 102, 103]
    assert st2["m_hist"][3] == 3
    assert list(emit[:3]) == [11, 3, 100] and emit[13] == 0 and emit[14] == 3 and emit[15] == 9
    assert list(h_seed) == [12, 13, 14, 15] and list(dhd) == [1, 1, 1, 1]


def test_argmax_tie_and_nan_rules():
    lg = np.array([[1.0, 3.0, 3.0, np.nan], [np.nan, np.nan, np.nan, np.nan], [-0.0, 0.0, -1, -2]])
    mx, idx = oracle.argmax_rows(lg)
    assert list(idx) == [1, 0, 0]


def test_q5k_dequant_bit_exact(golden):
    # the reference's numpy restatement (engine/chain_sim.py dequant_q5k_rows) and gguf-py
    got = oracle.dequant_q5k(golden["q5k_raw"], 5120)
    assert np.array_equal(got.view(np.uint32), golden["q5k_ref"].astype(np.float32).view(np.uint32))
    assert np.array_equal(got.view(np.uint32), golden["q5k_gguf_f32"].astype(np.float32).view(np.uint32))


def test_q8_0_dequant_bit_exact(golden):
    # the reference's numpy port (engine/mm/MM_P2_ports.py dq_q8_0) and gguf-py
    got = oracle.dequant_q8_0(golden["q8_0_raw"], 512)
    assert np.array_equal(got.view(np.uint32), golden["q8_0_ref"].astype(np.float32).view(np.uint32))
    assert np.array_equal(got.view(np.uint32), golden["q8_0_gguf_f32"].astype(np.float32).view(np.uint32))


def test_q4k_dequant_bit_exact(golden):
    # the reference's numpy port (engine/mm/mm_mtp_anchor.py dq_q4_k_np) and gguf-py
    got = oracle.dequant_q4k(golden["q4k_raw"], 512)
    assert np.array_equal(got.view(np.uint32), golden["q4k_ref"].astype(np.float32).view(np.uint32))
    assert np.array_equal(got.view(np.uint32), golden["q4k_gguf_f32"].astype(np.float32).view(np.uint32))
