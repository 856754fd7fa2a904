"""GPU parity: the CUDA path (through the C ABI) against the numpy oracle on
identical seeded inputs.

Contract (north star): outputs within max|err| <= 2e-3 * ||row||_2 of the
float64 oracle; argmax ids and accept results bit-exact.  The kernels are
fp32-accurate by construction (exact-integer fp16 dequant + fp32 scale), so a
100x tighter bound (2e-5 * ||row||) is asserted as well.
"""
import numpy as np
import pytest
import torch

import oracle
from thunderllamax_b200 import ops, synth

pytestmark = pytest.mark.gpu

CONTRACT = 2e-3
TIGHT = 2e-5


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()
    yield
    ops.set_max_ctas(0)


def x_tensor(rng, m, k, dtype):
    if dtype == torch.float32:
        x = rng.standard_normal((m, k), dtype=np.float32)
        return torch.from_numpy(x).cuda(), x.astype(np.float64)
    bits = synth.bf16_normal(rng, (m, k))
    x32 = synth.bf16_bits_to_f32(bits)
    if dtype == torch.bfloat16:
        return torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16), x32.astype(np.float64)
    x16 = x32.astype(np.float16)
    return torch.from_numpy(x16).cuda(), x16.astype(np.float64)


def check_rows(got, ref, tight=TIGHT):
    got = np.asarray(got, np.float64)
    for t in range(ref.shape[0]):
        nrm = np.linalg.norm(ref[t])
        err = np.abs(got[t] - ref[t]).max()
        assert err <= CONTRACT * nrm, (t, err, nrm)
        assert err <= tight * nrm, (t, err, nrm)


GEN = {"q6_k": synth.q6k_blocks, "iq3_xxs": synth.iq3xxs_blocks, "q4_k": synth.q4k_blocks,
       "q5_k": synth.q5k_blocks, "q8_0": synth.q8_0_blocks}


def check_vs_oracle(qtype, got, raw, k, x64, tight=TIGHT):
    """Every format decodes exactly except Q8_0, whose weights the kernel rounds to
    fp16(d q) as the reference's o-projection does (engine/k3aonw32_11.cu:100-101):
    Q8_0 is held to the contract against the exact weights and to the tight bound
    against the fp16-rounded ones."""
    W = oracle.dequant(qtype, raw, k)
    if qtype == "q8_0":
        check_rows(got, oracle.matvec_f64(W, x64), tight=CONTRACT)
        W = W.astype(np.float16).astype(np.float32)
    check_rows(got, oracle.matvec_f64(W, x64), tight=tight)


@pytest.mark.parametrize("qtype", ["q6_k", "iq3_xxs", "q4_k", "q5_k", "q8_0"])
@pytest.mark.parametrize("n,k,m,dtype", [
    (16, 256, 1, torch.bfloat16),
    (100, 512, 3, torch.bfloat16),
    (37, 2048, 16, torch.float16),
    (1000, 5120, 11, torch.bfloat16),
    (300, 1024, 5, torch.float32),
    (2048, 17408, 11, torch.bfloat16),
])
def test_gemv_vs_oracle(qtype, n, k, m, dtype):
    rng = np.random.default_rng(n * 7 + k + m)
    raw = GEN[qtype](rng, n, k)
    x, x64 = x_tensor(rng, m, k, dtype)
    w = ops.pack_tiles(qtype, raw, k)
    ws = ops.Workspace.for_shape(ops.MODE_STORE, qtype, n, k, m, dtype)
    y = ops.gemv(qtype, w, x, n, ws)
    torch.cuda.synchronize()
    assert ws.error() == 0
    check_vs_oracle(qtype, y.cpu().numpy(), raw, k, x64)


@pytest.mark.parametrize("qtype", ["q6_k", "iq3_xxs", "q4_k", "q5_k", "q8_0"])
def test_gemv_split_tiles_and_segments(qtype):
    # few CTAs + long k: tiles split across warps and k-segments, reduced by the
    # last arriving piece in fixed order; residual epilogue; results repeatable
    rng = np.random.default_rng(5)
    n, k, m = 333, 17408, 11
    raw = GEN[qtype](rng, n, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    res = rng.standard_normal((m, n), dtype=np.float32)
    W = oracle.dequant(qtype, raw, k)
    if qtype == "q8_0":
        W = W.astype(np.float16).astype(np.float32)    # the kernel's fp16(d q) weights
    ref = oracle.matvec_f64(W, x64) + res
    w = ops.pack_tiles(qtype, raw, k)
    for ctas in (5, 12, 0):
        ops.set_max_ctas(ctas)
        p = ops.plan(ops.MODE_STORE, qtype, n, k, m)
        ws = ops.Workspace.for_shape(ops.MODE_STORE, qtype, n, k, m)
        r = torch.from_numpy(res).cuda()
        y1 = ops.gemv(qtype, w, x, n, ws, residual=r)
        y2 = ops.gemv(qtype, w, x, n, ws, residual=r)
        torch.cuda.synchronize()
        assert ws.error() == 0
        assert p["segments"] > 1
        check_rows(y1.cpu().numpy(), ref)
        assert torch.equal(y1, y2), "not deterministic"
    ops.set_max_ctas(0)


def test_config1_single_iq3_linear_fp32():
    # W 17408x5120 IQ3_XXS, x 1x5120 fp32
    rng = np.random.default_rng(101)
    n, k = 17408, 5120
    raw = synth.iq3xxs_blocks(rng, n, k)
    x, x64 = x_tensor(rng, 1, k, torch.float32)
    ref = oracle.matvec_f64(oracle.dequant("iq3_xxs", raw, k), x64)
    w = ops.pack_tiles("iq3_xxs", raw, k)
    ws = ops.Workspace.for_shape(ops.MODE_STORE, "iq3_xxs", n, k, 1, torch.float32)
    y = ops.gemv("iq3_xxs", w, x, n, ws)
    torch.cuda.synchronize()
    check_rows(y.cpu().numpy(), ref, tight=1e-6)


@pytest.mark.parametrize("n,m", [(700, 11), (17408, 11), (50, 1)])
def test_ffn_gate_up_vs_oracle(n, m):
    rng = np.random.default_rng(n + m)
    k = 5120
    rg, ru = synth.iq3xxs_blocks(rng, n, k), synth.iq3xxs_blocks(rng, n, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    g = oracle.matvec_f64(oracle.dequant("iq3_xxs", rg, k), x64)
    u = oracle.matvec_f64(oracle.dequant("iq3_xxs", ru, k), x64)
    ref = oracle.silu_f64(g) * u
    wg, wu = ops.pack_tiles("iq3_xxs", rg, k), ops.pack_tiles("iq3_xxs", ru, k)
    ws = ops.Workspace.for_shape(ops.MODE_GATE_UP, "iq3_xxs", n, k, m)
    gact = ops.ffn_gate_up("iq3_xxs", wg, wu, x, n, ws)
    torch.cuda.synchronize()
    # silu(g)*u: relative error of the product ~ relative error of g and u
    check_rows(gact.cpu().numpy(), ref, tight=1e-4)


def test_ffn_config2_end_to_end():
    # BASELINE config 2 at reduced width (full size runs in the bench):
    # gate/up IQ3_XXS -> silu*up stored fp16 -> down Q6_K (fp32 out, residual)
    rng = np.random.default_rng(2)
    H, F, m = 1024, 2048, 11
    rg, ru = synth.iq3xxs_blocks(rng, F, H), synth.iq3xxs_blocks(rng, F, H)
    rd = synth.q6k_blocks(rng, H, F)
    x, x64 = x_tensor(rng, m, H, torch.bfloat16)
    res = rng.standard_normal((m, H), dtype=np.float32)
    gact_ref, y_ref = oracle.ffn_f64(x64, rg, ru, rd, residual=res)
    wg, wu, wd = (ops.pack_tiles("iq3_xxs", rg, H), ops.pack_tiles("iq3_xxs", ru, H), ops.pack_tiles("q6_k", rd, F))
    ws1 = ops.Workspace.for_shape(ops.MODE_GATE_UP, "iq3_xxs", F, H, m)
    ws2 = ops.Workspace.for_shape(ops.MODE_STORE, "q6_k", H, F, m, torch.float16)
    gact = ops.ffn_gate_up("iq3_xxs", wg, wu, x, F, ws1, out_dtype=torch.float16)
    y = ops.gemv("q6_k", wd, gact, H, ws2, residual=torch.from_numpy(res).cuda())
    # same chain through the activation image: gate/up writes gact as down's image
    img = ops.Image(m, F)
    ws3 = ops.Workspace.for_shape(ops.MODE_STORE, "q6_k", H, F, m, "image")
    ops.ffn_gate_up("iq3_xxs", wg, wu, x, F, ws1, gact=img)
    y_img = ops.gemv("q6_k", wd, img, H, ws3, residual=torch.from_numpy(res).cuda())
    torch.cuda.synchronize()
    check_rows(gact.float().cpu().numpy(), gact_ref, tight=1e-3)
    check_rows(y.cpu().numpy(), y_ref, tight=1e-4)
    assert torch.equal(y, y_img)


def test_staged_activation_image_matches_raw_path():
    rng = np.random.default_rng(12)
    n, k, m = 500, 2048, 11
    raw = synth.q6k_blocks(rng, n, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    w = ops.pack_tiles("q6_k", raw, k)
    y_raw = ops.gemv("q6_k", w, x, n, ops.Workspace.for_shape(ops.MODE_STORE, "q6_k", n, k, m))
    img = ops.stage(x)
    y_img = ops.gemv("q6_k", w, img, n, ops.Workspace.for_shape(ops.MODE_STORE, "q6_k", n, k, m, "image"))
    torch.cuda.synchronize()
    assert torch.equal(y_raw, y_img)
    check_rows(y_img.cpu().numpy(), oracle.matvec_f64(oracle.dequant("q6_k", raw, k), x64))


@pytest.mark.parametrize("qtype", ["q6_k", "iq3_xxs"])
@pytest.mark.parametrize("V,m,ctas", [(20000, 11, 0), (3001, 4, 3), (777, 16, 0)])
def test_head_argmax_bit_exact(qtype, V, m, ctas):
    rng = np.random.default_rng(V + m)
    k = 1024 if V > 10000 else 512
    raw = GEN[qtype](rng, V, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    mx_ref, idx_ref, lg = oracle.head_argmax(x64, raw, qtype, row_offset=1000)
    gap = oracle.min_top2_gap(lg)
    assert (gap > 1e-6 * np.abs(lg).max()).all(), "near-tie in this seed: choose another"
    ops.set_max_ctas(ctas)
    w = ops.pack_tiles(qtype, raw, k)
    ws = ops.Workspace.for_shape(ops.MODE_ARGMAX, qtype, V, k, m)
    keys = torch.empty(m, dtype=torch.int64, device="cuda")
    mx, idx = ops.head_argmax(qtype, w, x, V, ws, row_offset=1000, out_keys=keys)
    mx2, idx2 = ops.head_argmax(qtype, w, x, V, ws, row_offset=1000)
    torch.cuda.synchronize()
    ops.set_max_ctas(0)
    assert ws.error() == 0
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    assert torch.equal(idx, idx2) and torch.equal(mx, mx2)
    np.testing.assert_allclose(mx.cpu().numpy(), mx_ref, rtol=1e-5, atol=1e-5 * np.abs(mx_ref).max())


def test_head_argmax_with_accept():
    rng = np.random.default_rng(33)
    V, k, m = 5000, 512, 11
    raw = synth.q6k_blocks(rng, V, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    _, idx_ref, _ = oracle.head_argmax(x64, raw, "q6_k")
    w = ops.pack_tiles("q6_k", raw, k)
    ws = ops.Workspace.for_shape(ops.MODE_ARGMAX, "q6_k", V, k, m)
    for trial in range(6):
        drafts_np, j = synth.drafts_for(idx_ref, m - 1, V, rng)
        if trial == 0:
            drafts_np[:] = idx_ref[:m - 1]          # all accepted
        if trial == 1:
            drafts_np[0] = (idx_ref[0] + 1) % V     # none accepted
        drafts = torch.from_numpy(drafts_np).cuda()
        acc = torch.full((2,), -7, dtype=torch.int32, device="cuda")
        _, idx = ops.head_argmax("q6_k", w, x, V, ws, drafts=drafts, accept_out=acc)
        torch.cuda.synchronize()
        m_ref, bonus_ref = oracle.accept(idx_ref, drafts_np)
        assert acc.cpu().tolist() == [m_ref, bonus_ref]


def test_fused_head_matches_unfused_logits_path():
    # head8v11 (logits) + amx3 (argmax) vs the fused kernel, same weights
    rng = np.random.default_rng(44)
    V, k, m = 4099, 512, 11
    raw = synth.q6k_blocks(rng, V, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    w = ops.pack_tiles("q6_k", raw, k)
    ws1 = ops.Workspace.for_shape(ops.MODE_STORE, "q6_k", V, k, m)
    ws2 = ops.Workspace.for_shape(ops.MODE_ARGMAX, "q6_k", V, k, m)
    logits = ops.gemv("q6_k", w, x, V, ws1)
    amds = ops.argmax_rows(logits)
    _, idx = ops.head_argmax("q6_k", w, x, V, ws2)
    torch.cuda.synchronize()
    assert torch.equal(amds, idx)
    amds16 = ops.argmax_rows(logits.half())
    ref16 = np.argmax(logits.half().float().cpu().numpy(), axis=1)
    assert np.array_equal(amds16.cpu().numpy(), ref16)


def test_argmax_rows_ties_and_nan():
    nan, inf = float("nan"), float("inf")
    lg = torch.tensor([[1.0, 3.0, 3.0, nan], [nan] * 4, [-0.0, 0.0, -1.0, -2.0],
                       [nan, -inf, -inf, nan], [-inf, -5.0, nan, -5.0], [inf, 1.0, inf, 2.0]], device="cuda")
    for t in (lg, lg.half()):
        amds = ops.argmax_rows(t)
        torch.cuda.synchronize()
        assert amds.cpu().tolist() == list(oracle.argmax_rows(t.float().cpu().numpy())[1])


def test_h_argmax_side_effects():
    # the reference's vocabulary (248320 fp16 logits), ties planted above the maximum
    rng = np.random.default_rng(21)
    V = 248320
    lg = rng.standard_normal(V).astype(np.float16)
    top = rng.choice(V, 3, replace=False)
    lg[top] = np.float16(9.5)
    lg[rng.choice(V, 5, replace=False)] = np.float16(np.nan)
    hist = np.full(64, -1, dtype=np.int32)
    t_lg = torch.from_numpy(lg).cuda()
    tok = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    pos = torch.tensor([17], dtype=torch.int32, device="cuda")
    t_hist = torch.from_numpy(hist).cuda()
    ref_idx, ref_hist, ref_pos = oracle.h_argmax(lg, hist, 17)
    assert ref_idx == int(top.min())
    ops.h_argmax(t_lg, tok, pos, t_hist)
    # a second call appends at the advanced position (a row with no candidate -> 0)
    empty = torch.full((V,), float("-inf"), dtype=torch.float16, device="cuda")
    ops.h_argmax(empty, tok, pos, t_hist)
    torch.cuda.synchronize()
    ref2_idx, ref_hist, ref_pos = oracle.h_argmax(empty.cpu().numpy(), ref_hist, ref_pos)
    assert ref2_idx == 0
    assert tok.item() == 0 and pos.item() == ref_pos == 19
    assert np.array_equal(t_hist.cpu().numpy(), ref_hist)
    assert ref_hist[17] == ref_idx


@pytest.mark.parametrize("nq,nk,nv,k,dtype", [(256, 128, 160, 512, torch.float16), (12288, 1024, 1024, 5120, torch.bfloat16)])
def test_aq3k8v11_vs_oracle(nq, nk, nv, k, dtype):
    # the attention q / k (IQ3_XXS) / v (Q4_K) projections over 11 rows, fp16 outputs
    rng = np.random.default_rng(nq + nv)
    m = 11
    rq, rk, rv = synth.iq3xxs_blocks(rng, nq, k), synth.iq3xxs_blocks(rng, nk, k), synth.q4k_blocks(rng, nv, k)
    x, x64 = x_tensor(rng, m, k, dtype)
    wq, wk, wv = ops.pack_tiles("iq3_xxs", rq, k), ops.pack_tiles("iq3_xxs", rk, k), ops.pack_tiles("q4_k", rv, k)
    proj = ops.AttnProjections(m, k, nq, nk, nv, dtype)
    q, kk, v = proj(wq, wk, wv, x)
    q2, kk2, v2 = proj(wq, wk, wv, x)
    torch.cuda.synchronize()
    assert proj.error() == 0
    for got, raw, qt in ((q, rq, "iq3_xxs"), (kk, rk, "iq3_xxs"), (v, rv, "q4_k")):
        ref = oracle.matvec_f64(oracle.dequant(qt, raw, k), x64)
        check_rows(got.float().cpu().numpy(), ref, tight=1e-3)   # fp16 outputs: one fp16 rounding
    assert torch.equal(q, q2) and torch.equal(kk, kk2) and torch.equal(v, v2)


def test_q4k_gemv_reads_a_staged_image():
    # a tlx_stage_activations image carries the sub-block sums the Q4_K min term reads
    rng = np.random.default_rng(31)
    n, k, m = 300, 1024, 11
    raw = synth.q4k_blocks(rng, n, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    w = ops.pack_tiles("q4_k", raw, k)
    img = ops.stage(x)
    y = ops.gemv("q4_k", w, img, n, ops.Workspace.for_shape(ops.MODE_STORE, "q4_k", n, k, m, "image"))
    torch.cuda.synchronize()
    check_rows(y.cpu().numpy(), oracle.matvec_f64(oracle.dequant("q4_k", raw, k), x64))


@pytest.mark.parametrize("nqkv,ngate,k,dtype", [(320, 192, 512, torch.float16), (10240, 6144, 5120, torch.float16),
                                                (10240, 6144, 5120, torch.bfloat16)])
def test_q5g8v11_vs_oracle(nqkv, ngate, k, dtype):
    # the GDN qkv (Q5_K) and gate (IQ3_XXS) projections over 11 rows, fp16 outputs
    rng = np.random.default_rng(nqkv + ngate)
    m = 11
    rqkv, rg = synth.q5k_blocks(rng, nqkv, k), synth.iq3xxs_blocks(rng, ngate, k)
    x, x64 = x_tensor(rng, m, k, dtype)
    wqkv, wg = ops.pack_tiles("q5_k", rqkv, k), ops.pack_tiles("iq3_xxs", rg, k)
    proj = ops.GdnProjections(m, k, nqkv, ngate, dtype)
    qkv, gate = proj(wqkv, wg, x)
    qkv2, gate2 = proj(wqkv, wg, x)
    torch.cuda.synchronize()
    assert proj.error() == 0
    for got, raw, qt in ((qkv, rqkv, "q5_k"), (gate, rg, "iq3_xxs")):
        ref = oracle.matvec_f64(oracle.dequant(qt, raw, k), x64)
        check_rows(got.float().cpu().numpy(), ref, tight=1e-3)   # fp16 outputs: one fp16 rounding
    assert torch.equal(qkv, qkv2) and torch.equal(gate, gate2)


@pytest.mark.parametrize("qtype", ["iq3_xxs", "q8_0"])
def test_gdn_o_projection_reference_shape(qtype):
    # op38nw32_11 (IQ3_XXS) / k3aonw32_11 (Q8_0): attn_out [11][5120] = W z, z [11][6144]
    # fp16, through the reference-named programs
    from thunderllamax_b200 import engine0
    rng = np.random.default_rng(61 if qtype == "q8_0" else 62)
    m, n, k = 11, 5120, 6144
    raw = GEN[qtype](rng, n, k)
    z, z64 = x_tensor(rng, m, k, torch.float16)
    w = ops.pack_tiles(qtype, raw, k)
    progs = engine0.load_progs(rows=m, vocab=4096)
    out = torch.empty((m, n), dtype=torch.float16, device="cuda")
    if qtype == "q8_0":
        progs["k3aonw32_11"](w, z.reshape(-1), out.reshape(-1))
    else:
        progs["op38nw32_11"](w, None, z.reshape(-1), out.reshape(-1))
    torch.cuda.synchronize()
    check_vs_oracle(qtype, out.float().cpu().numpy(), raw, k, z64, tight=1e-3)


def test_q5k_gemv_reads_a_staged_image():
    rng = np.random.default_rng(32)
    n, k, m = 300, 1024, 11
    raw = synth.q5k_blocks(rng, n, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    w = ops.pack_tiles("q5_k", raw, k)
    img = ops.stage(x)
    y = ops.gemv("q5_k", w, img, n, ops.Workspace.for_shape(ops.MODE_STORE, "q5_k", n, k, m, "image"))
    torch.cuda.synchronize()
    check_rows(y.cpu().numpy(), oracle.matvec_f64(oracle.dequant("q5_k", raw, k), x64))


def _sel_buffers(B, R, C, seed):
    rng = np.random.default_rng(seed)
    rec4 = rng.standard_normal((B, 5, R)).astype(np.float32)
    conv4 = rng.standard_normal((B, 5, C)).astype(np.float32)
    rec_x = [rng.standard_normal((B, R)).astype(np.float32) for _ in range(6)]
    conv_x = [rng.standard_normal((B, C)).astype(np.float32) for _ in range(7)]
    return rec4, conv4, rec_x, conv_x


@pytest.mark.parametrize("B,R,C", [(3, 1000, 100), (2, 1001, 37)])   # vector and scalar copies
def test_acceptsel11k_every_m(B, R, C):
    rec4, conv4, rec_x, conv_x = _sel_buffers(B, R, C, B + R)
    for m in list(range(11)) + [11, -1]:
        t_rec, t_conv = torch.from_numpy(rec4).cuda(), torch.from_numpy(conv4).cuda()
        m_slot = torch.tensor([m], dtype=torch.int32, device="cuda")
        ops.acceptsel11k(t_rec, t_conv, m_slot, [torch.from_numpy(x).cuda() for x in conv_x],
                         [torch.from_numpy(x).cuda() for x in rec_x], n_blocks=B, rec_elems=R, conv_elems=C)
        torch.cuda.synchronize()
        want_r, want_c = oracle.acceptsel11k(rec4, conv4, m, conv_x, rec_x)
        assert np.array_equal(t_rec.cpu().numpy(), want_r), m
        assert np.array_equal(t_conv.cpu().numpy(), want_c), m


def test_acceptsel11k_reference_size():
    # 48 blocks x (786432 + 30720) fp32: ~157 MB read and written, compared bitwise
    # on the device against torch copies
    B, R, C = ops.GDN_BLOCKS, ops.GDN_REC, ops.GDN_CONV
    g = torch.Generator(device="cuda").manual_seed(5)
    rec4 = torch.randn((B, 5, R), device="cuda", generator=g)
    conv4 = torch.randn((B, 5, C), device="cuda", generator=g)
    rec_x = [torch.randn((B, R), device="cuda", generator=g) for _ in range(6)]
    conv_x = [torch.randn((B, C), device="cuda", generator=g) for _ in range(7)]
    for m in (2, 7):
        want_r, want_c = rec4.clone(), conv4.clone()
        want_r[:, 4] = rec4[:, m] if m < 5 else rec_x[m - 5]
        want_c[:, 4] = conv4[:, m] if m < 4 else conv_x[m - 4]
        got_r, got_c = rec4.clone(), conv4.clone()
        ops.acceptsel11k(got_r, got_c, torch.tensor([m], dtype=torch.int32, device="cuda"), conv_x, rec_x)
        torch.cuda.synchronize()
        assert torch.equal(got_r, want_r) and torch.equal(got_c, want_c), m


def test_accept_kernels():
    amds_np = np.arange(100, 111, dtype=np.int32)
    amds = torch.from_numpy(amds_np).cuda()
    for drafts_np in (amds_np[:10].copy(), np.array([100, 101, 0, 0, 0, 0, 0, 0, 0, 0], np.int32),
                      np.zeros(10, np.int32)):
        mb, eb = ops.accept(amds, torch.from_numpy(drafts_np).cuda())
        torch.cuda.synchronize()
        m_ref, b_ref = oracle.accept(amds_np, drafts_np)
        assert mb.item() == m_ref and eb.cpu().tolist() == [m_ref, b_ref]


def test_accept11k_side_effects():
    from thunderllamax_b200 import engine0

    amds_np = np.arange(100, 111, dtype=np.int32)
    drafts_np = np.array([100, 101, 102, 0, 0, 0, 0, 0, 0, 0], np.int32)
    dim = 64
    xA = np.arange(11 * dim, dtype=np.float32)
    st = {"pos": 7, "cyc": 3, "cur": -1, "m_slot": -1, "tok_hist": np.zeros(32, np.int32),
          "m_hist": np.zeros(8, np.int32), "l_hist": np.array([0, 0, 0, 9, 0, 0, 0, 0], np.int32)}
    st_ref, emit_ref, h_ref, dhd_ref = oracle.accept11k(amds_np, drafts_np, st, xA=xA, hd_d0=np.zeros(dim),
                                                        hd_d1=np.ones(dim), dim=dim)
    out = engine0.run_accept11k(amds_np, drafts_np, st, xA, np.zeros(dim, np.float32), np.ones(dim, np.float32), dim)
    assert out["pos"] == st_ref["pos"] and out["cur"] == st_ref["cur"] and out["cyc"] == st_ref["cyc"]
    assert np.array_equal(out["tok_hist"], st_ref["tok_hist"]) and np.array_equal(out["m_hist"], st_ref["m_hist"])
    assert np.array_equal(out["emit"][:16], emit_ref[:16])
    assert np.array_equal(out["h_seed"], h_ref) and np.array_equal(out["dhd_seed"], dhd_ref)


def test_argmax_merge_across_shards():
    # vocab sharding: per-shard fused heads with row offsets, merged keys == global
    rng = np.random.default_rng(55)
    V, k, m, S = 6000, 512, 11, 4
    raw = synth.q6k_blocks(rng, V, k)
    x, x64 = x_tensor(rng, m, k, torch.bfloat16)
    _, idx_ref, _ = oracle.head_argmax(x64, raw, "q6_k")
    keys = torch.empty((S, m), dtype=torch.int64, device="cuda")
    bounds = np.linspace(0, V, S + 1).astype(int)
    for s in range(S):
        lo, hi = bounds[s], bounds[s + 1]
        w = ops.pack_tiles("q6_k", raw[lo:hi], k)
        ws = ops.Workspace.for_shape(ops.MODE_ARGMAX, "q6_k", hi - lo, k, m)
        ops.head_argmax("q6_k", w, x, hi - lo, ws, row_offset=int(lo), out_keys=keys[s])
    drafts_np = idx_ref[:10].copy()
    drafts_np[4] = (drafts_np[4] + 1) % V
    acc = torch.empty(2, dtype=torch.int32, device="cuda")
    _, idx = ops.argmax_merge(keys, drafts=torch.from_numpy(drafts_np).cuda(), accept_out=acc)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    assert acc.cpu().tolist() == list(oracle.accept(idx_ref, drafts_np))


@pytest.mark.parametrize("qtype", ["q6_k", "iq3_xxs"])
def test_device_packer_matches_host_packer(qtype):
    rng = np.random.default_rng(66)
    raw = GEN[qtype](rng, 45, 768)
    host = ops.pack_tiles_host(qtype, raw, 768)
    dev = ops.pack_tiles(qtype, raw, 768).cpu().numpy()
    assert np.array_equal(host, dev)


def test_host_argument_errors_raise():
    rng = np.random.default_rng(0)
    raw = synth.q6k_blocks(rng, 32, 256)
    w = ops.pack_tiles("q6_k", raw, 256)
    x, _ = x_tensor(rng, 2, 256, torch.bfloat16)
    small = ops.Workspace(256)
    with pytest.raises(ops.TLXError):
        ops.gemv("q6_k", w, x, 32, small)
    ws = ops.Workspace.for_shape(ops.MODE_STORE, "q6_k", 32, 256, 2)
    with pytest.raises(ops.TLXError):
        ops.gemv("q6_k", w, x[:, 1:], 32, ws)        # misaligned activations


@pytest.mark.parametrize("ffn_ctas", [None, 0, 20])
def test_verify_step_pipeline_vs_oracle(ffn_ctas):
    # the graph-captured verify step (stage -> gate/up -> gact image -> down; stage ->
    # head argmax + accept) at reduced width against the oracle: the FFN chain beside
    # the head (default split, a small FFN budget) and all three GEMVs in sequence (0)
    from thunderllamax_b200.verify import VerifyShape, VerifyStep

    rng = np.random.default_rng(99)
    s = VerifyShape(dim=1024, ffn=2048, vocab=7001, rows=11)
    rg, ru = synth.iq3xxs_blocks(rng, s.ffn, s.dim), synth.iq3xxs_blocks(rng, s.ffn, s.dim)
    rd, rh = synth.q6k_blocks(rng, s.dim, s.ffn), synth.q6k_blocks(rng, s.vocab, s.dim)
    w = {"gate": ops.pack_tiles("iq3_xxs", rg, s.dim), "up": ops.pack_tiles("iq3_xxs", ru, s.dim),
         "down": ops.pack_tiles("q6_k", rd, s.ffn), "head": ops.pack_tiles("q6_k", rh, s.dim)}
    step = VerifyStep(s, weights=w, ffn_ctas=ffn_ctas)
    x, x64 = x_tensor(rng, s.rows, s.dim, torch.bfloat16)
    h, h64 = x_tensor(rng, s.rows, s.dim, torch.bfloat16)
    res = rng.standard_normal((s.rows, s.dim), dtype=np.float32)
    _, y_ref = oracle.ffn_f64(x64, rg, ru, rd, residual=res)
    _, idx_ref, _ = oracle.head_argmax(h64, rh, "q6_k")
    drafts_np = idx_ref[:10].copy()
    drafts_np[7] = (drafts_np[7] + 3) % s.vocab
    step.set_inputs(x, h, res=torch.from_numpy(res).cuda(), drafts=torch.from_numpy(drafts_np).cuda())
    step.capture()
    for _ in range(3):
        step.replay()
    torch.cuda.synchronize()
    check_rows(step.y.cpu().numpy(), y_ref, tight=1e-4)
    assert np.array_equal(step.out_idx.cpu().numpy(), idx_ref)
    assert step.accept_out.cpu().tolist() == list(oracle.accept(idx_ref, drafts_np))
    assert not any(step.workspace_errors().values())


def test_verify_step_host_path_copies_every_call():
    # step_host (H2D inputs, graph replay, D2H of the accept record and argmax ids)
    # returns what the device path returns, and picks up new contents of the same
    # pinned buffers on every call
    from thunderllamax_b200.verify import VerifyShape, VerifyStep

    rng = np.random.default_rng(7)
    s = VerifyShape(dim=1024, ffn=2048, vocab=5003, rows=11)
    w = {"gate": ops.pack_tiles("iq3_xxs", synth.iq3xxs_blocks(rng, s.ffn, s.dim), s.dim),
         "up": ops.pack_tiles("iq3_xxs", synth.iq3xxs_blocks(rng, s.ffn, s.dim), s.dim),
         "down": ops.pack_tiles("q6_k", synth.q6k_blocks(rng, s.dim, s.ffn), s.ffn)}
    rh = synth.q6k_blocks(rng, s.vocab, s.dim)
    w["head"] = ops.pack_tiles("q6_k", rh, s.dim)
    step = VerifyStep(s, weights=w)
    xp = torch.empty((s.rows, s.dim), dtype=torch.bfloat16).pin_memory()
    hp = torch.empty_like(xp).pin_memory()
    dp = torch.empty(s.n_drafts, dtype=torch.int32).pin_memory()
    outp = torch.empty(2 + s.rows, dtype=torch.int32).pin_memory()
    for trial in range(3):
        x, _ = x_tensor(rng, s.rows, s.dim, torch.bfloat16)
        h, h64 = x_tensor(rng, s.rows, s.dim, torch.bfloat16)
        _, idx_ref, _ = oracle.head_argmax(h64, rh, "q6_k")
        drafts_np = idx_ref[:s.n_drafts].copy()
        drafts_np[trial + 2] = (drafts_np[trial + 2] + 1) % s.vocab
        xp.copy_(x.cpu())
        hp.copy_(h.cpu())
        dp.copy_(torch.from_numpy(drafts_np))
        step.step_host(xp, hp, dp, outp)
        torch.cuda.current_stream().synchronize()
        assert np.array_equal(outp[2:].numpy(), idx_ref)
        assert outp[:2].tolist() == list(oracle.accept(idx_ref, drafts_np))
        # the device path on the same inputs gives the same record
        step.set_inputs(x, h, drafts=torch.from_numpy(drafts_np).cuda())
        step.replay()
        torch.cuda.synchronize()
        assert step.accept_out.cpu().tolist() == outp[:2].tolist()


def test_verify_step_packed_host_path():
    # step_host_packed: one H2D copy of x | h | drafts and one D2H copy of (m, bonus,
    # ids) per step, new contents of the same pinned buffers on every call, against the
    # oracle and the device views
    from thunderllamax_b200.verify import VerifyShape, VerifyStep

    rng = np.random.default_rng(17)
    s = VerifyShape(dim=1024, ffn=2048, vocab=5003, rows=11)
    w = {"gate": ops.pack_tiles("iq3_xxs", synth.iq3xxs_blocks(rng, s.ffn, s.dim), s.dim),
         "up": ops.pack_tiles("iq3_xxs", synth.iq3xxs_blocks(rng, s.ffn, s.dim), s.dim),
         "down": ops.pack_tiles("q6_k", synth.q6k_blocks(rng, s.dim, s.ffn), s.ffn)}
    rh = synth.q6k_blocks(rng, s.vocab, s.dim)
    w["head"] = ops.pack_tiles("q6_k", rh, s.dim)
    step = VerifyStep(s, weights=w)
    inp, outp, views = step.host_buffers()
    assert inp.is_pinned() and outp.is_pinned()
    assert inp.numel() == 2 * s.rows * s.dim * 2 + s.n_drafts * 4 and outp.numel() == 2 + s.rows
    for trial in range(3):
        x, _ = x_tensor(rng, s.rows, s.dim, torch.bfloat16)
        h, h64 = x_tensor(rng, s.rows, s.dim, torch.bfloat16)
        _, idx_ref, _ = oracle.head_argmax(h64, rh, "q6_k")
        drafts_np = idx_ref[:s.n_drafts].copy()
        drafts_np[trial + 4] = (drafts_np[trial + 4] + 1) % s.vocab
        views["x"].copy_(x.cpu())
        views["h"].copy_(h.cpu())
        views["drafts"].copy_(torch.from_numpy(drafts_np))
        step.step_host_packed(inp, outp)
        torch.cuda.current_stream().synchronize()
        assert np.array_equal(outp[2:].numpy(), idx_ref)
        assert outp[:2].tolist() == list(oracle.accept(idx_ref, drafts_np))
        assert torch.equal(step.x.cpu(), x.cpu())
        assert torch.equal(step.drafts.cpu(), torch.from_numpy(drafts_np))


@pytest.mark.parametrize("qtype,n,k,rows,cols", [("q6_k", 20000, 512, (8704, 17408), None),
                                                 ("iq3_xxs", 20000, 512, (16, 8208), None),
                                                 ("q6_k", 512, 17408, None, (8704, 17408)),
                                                 ("q6_k", 300, 2048, (0, 300), (256, 1024))])
def test_synth_tiled_slices_one_model(qtype, n, k, rows, cols):
    # a shard of the seeded model (rows and / or a 256-aligned column range) equals the
    # same slice of the whole matrix, across the 8192-row generation chunks
    from thunderllamax_b200.verify import synth_tiled
    r0, r1 = rows if rows else (0, n)
    k0, k1 = cols if cols else (0, k)
    whole = synth.matrix_rows(qtype, n, k, 99)
    bb = synth.BLOCK_BYTES[qtype]
    ref = np.ascontiguousarray(whole[r0:r1, (k0 // 256) * bb:(k1 // 256) * bb])
    got = synth_tiled(qtype, n, k, 99, rows=rows, cols=cols)
    assert torch.equal(got, ops.pack_tiles(qtype, ref, k1 - k0))
