"""Split-KV int8 attention (tlx_attn_pre / tlx_attn_decode) against the float64
oracle (oracle/attention.py) and against the reference's own spk_pre11 /
spk_a11 / spk_c11 kernels (oracle/_ref cubins, built with the reference's
compile-time shapes) on the same device inputs.

Contract: ao within 2e-3 * ||row||_2 of the oracle per token row (6144 values);
the kernel's fp16 P and fp16 output put it inside 1e-3 * ||row||_2 as well.  The
pre step's qw16 and cache bytes follow the reference kernel's arithmetic
(reduction order, fp16 roundings) and are compared with it bit for bit."""
import numpy as np
import pytest
import torch

import oracle
import refkernels
from thunderllamax_b200 import ops

pytestmark = pytest.mark.gpu
CONTRACT, TIGHT = 2e-3, 1e-3
REF_CTX, REF_S, REF_ROWS = 100352, 256, 11


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()


def inputs(rng, T):
    qrow = rng.standard_normal((T, 12288)).astype(np.float16)
    krow = rng.standard_normal((T, 1024)).astype(np.float16)
    vrow = rng.standard_normal((T, 1024)).astype(np.float16)
    qnw = (1.0 + 0.2 * rng.standard_normal(256)).astype(np.float32)
    knw = (1.0 + 0.2 * rng.standard_normal(256)).astype(np.float32)
    return qrow, krow, vrow, qnw, knw


def random_cache(rng, ctx, upto):
    """Cache rows 0 .. upto-1 filled with random int8 codes and scales of the size a
    normed k / v row quantises to."""
    kv = np.full((8, ctx, 256), 128, dtype=np.uint8)
    sc = np.zeros((8, ctx, 8), dtype=np.float16)
    kv[:, :upto] = rng.integers(1, 256, (8, upto, 256), dtype=np.uint8)
    sc[:, :upto] = rng.uniform(0.012, 0.03, (8, upto, 8)).astype(np.float16)
    return kv, sc


def dev(*arrs):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def check_rows(got, ref, tol):
    got = np.asarray(got, np.float64)
    for t in range(ref.shape[0]):
        nrm = np.linalg.norm(ref[t])
        err = np.abs(got[t] - ref[t]).max()
        assert err <= tol * nrm, (t, err, nrm)


def run_lib(rows, ctx, qrow, krow, vrow, qnw, knw, kv, sc, pos):
    at = ops.Attention(rows, ctx)
    q_t, k_t, v_t, qn_t, kn_t, fr_t = dev(qrow, krow, vrow, qnw, knw, oracle.rope_freqs())
    kv_t, sc_t = dev(kv, sc)
    pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
    qw16 = at.pre(q_t, k_t, v_t, qn_t, kn_t, fr_t, pos_t, kv_t, sc_t)
    ao = at.decode(kv_t, sc_t, qw16, q_t, pos_t)
    ao2 = at.decode(kv_t, sc_t, qw16, q_t, pos_t)
    torch.cuda.synchronize()
    assert at.error() == 0
    assert torch.equal(ao, ao2)                     # deterministic
    return qw16.cpu().numpy(), kv_t.cpu().numpy(), sc_t.cpu().numpy(), ao.cpu().numpy()


@pytest.mark.parametrize("rows,pos,ctx", [(11, 0, 512), (11, 1, 512), (11, 63, 512), (11, 500, 1024),
                                          (11, 4085, 4096), (1, 777, 1024), (3, 64, 256), (16, 1000, 2048)])
def test_attention_vs_oracle(rows, pos, ctx):
    rng = np.random.default_rng(rows * 1000 + pos)
    qrow, krow, vrow, qnw, knw = inputs(rng, rows)
    kv, sc = random_cache(rng, ctx, pos)
    qw16, kv_lib, sc_lib, ao = run_lib(rows, ctx, qrow, krow, vrow, qnw, knw, kv, sc, pos)
    # the oracle's pre step on its own copy of the cache
    kv_o, sc_o = kv.copy(), sc.copy()
    qw16_o = oracle.attn_pre(qrow, krow, vrow, qnw, knw, oracle.rope_freqs(), pos, kv_o, sc_o)
    # one fp16 rounding of the normed value may differ (fp32 kernel vs float64 oracle);
    # the rotary mixes it into its pair, so bound it by the head vector's magnitude
    d = np.abs(qw16.astype(np.float64) - qw16_o.astype(np.float64))
    scale = np.abs(qw16_o.astype(np.float64)).max(axis=2, keepdims=True)
    assert (d <= scale * 2.0 ** -9).all()
    new = slice(pos, pos + rows)
    assert np.array_equal(kv_lib[:, :pos], kv[:, :pos]) and np.array_equal(kv_lib[:, pos + rows:], kv[:, pos + rows:])
    diff = np.abs(kv_lib[:, new].astype(np.int64) - kv_o[:, new].astype(np.int64))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-3                            # rounding ties only
    assert np.allclose(sc_lib[:, new].astype(np.float64), sc_o[:, new].astype(np.float64), rtol=2e-3)
    # the attention itself on the library's cache and qw16 (so only the decode differs)
    ref = oracle.attn_decode(qw16, kv_lib, sc_lib, qrow, pos)
    check_rows(ao.astype(np.float64), ref, CONTRACT)
    check_rows(ao.astype(np.float64), ref, TIGHT)


def test_attention_long_context_vs_oracle():
    rows, ctx, pos = 11, REF_CTX, 100000
    rng = np.random.default_rng(5)
    qrow, krow, vrow, qnw, knw = inputs(rng, rows)
    kv, sc = random_cache(rng, ctx, pos)
    qw16, kv_lib, sc_lib, ao = run_lib(rows, ctx, qrow, krow, vrow, qnw, knw, kv, sc, pos)
    ref = oracle.attn_decode(qw16, kv_lib, sc_lib, qrow, pos)
    check_rows(ao.astype(np.float64), ref, CONTRACT)
    check_rows(ao.astype(np.float64), ref, TIGHT)


@pytest.mark.parametrize("pos", [0, 3000, 99000])
def test_attention_vs_reference_kernels(pos):
    for k in ("spk_pre11", "spk_a11", "spk_c11"):
        refkernels.require(k)
    rows, ctx = REF_ROWS, REF_CTX
    rng = np.random.default_rng(77 + pos)
    qrow, krow, vrow, qnw, knw = inputs(rng, rows)
    kv, sc = random_cache(rng, ctx, pos)
    q_t, k_t, v_t, qn_t, kn_t, fr_t = dev(qrow, krow, vrow, qnw, knw, oracle.rope_freqs())
    pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
    # reference chain: spk_pre11 (grid 24 x 256), spk_a11 (grid 4 * S x 1024), spk_c11 (grid 24 x 256)
    kv_r, sc_r = dev(kv, sc)
    qw = torch.zeros((rows, 24, 256), dtype=torch.float32, device="cuda")
    qw16_r = torch.zeros((rows, 24, 256), dtype=torch.float16, device="cuda")
    refkernels.launch("spk_pre11", 24, 256, [q_t, k_t, v_t, qn_t, kn_t, fr_t, kv_r, sc_r, pos_t, qw, qw16_r])
    R = 6 * rows
    pm = torch.zeros(4 * REF_S * R, dtype=torch.float32, device="cuda")
    ps = torch.zeros_like(pm)
    pa = torch.zeros(4 * REF_S * R * 256, dtype=torch.float32, device="cuda")
    refkernels.launch("spk_a11", 4 * REF_S, 1024, [kv_r, sc_r, qw16_r, pos_t, pm, ps, pa])
    ao_r = torch.zeros((rows, 6144), dtype=torch.float16, device="cuda")
    refkernels.launch("spk_c11", 24, 256, [pm, ps, pa, q_t, ao_r])
    # library
    at = ops.Attention(rows, ctx)
    kv_l, sc_l = dev(kv, sc)
    qw16_l = at.pre(q_t, k_t, v_t, qn_t, kn_t, fr_t, pos_t, kv_l, sc_l)
    ao_l = at.decode(kv_l, sc_l, qw16_l, q_t, pos_t)
    torch.cuda.synchronize()
    assert at.error() == 0
    # the pre step follows the reference kernel's arithmetic: bit-exact
    assert torch.equal(qw16_l.view(torch.int16), qw16_r.view(torch.int16))
    assert torch.equal(kv_l, kv_r)
    assert torch.equal(sc_l.view(torch.int16), sc_r.view(torch.int16))
    # the attention: different tile order and accumulation, same contract
    ref = ao_r.float().cpu().numpy().astype(np.float64)
    check_rows(ao_l.float().cpu().numpy(), ref, CONTRACT)
    check_rows(ao_l.float().cpu().numpy(), ref, TIGHT)


def test_attention_rejects_bad_arguments():
    lib = ops._lib.lib()
    assert lib.tlx_attn_workspace_bytes(0) == 0 and lib.tlx_attn_workspace_bytes(17) == 0
    at = ops.Attention(11, 256)
    kv, sc = at.new_cache()
    x = torch.zeros(16, dtype=torch.float16, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.tlx_attn_decode(kv.data_ptr(), sc.data_ptr(), x.data_ptr(), x.data_ptr(), pos.data_ptr(), 11, 256,
                             x.data_ptr(), at.ws.buf.data_ptr(), 16, None)
    assert rc == -5      # TLX_ERR_WORKSPACE
    rc = lib.tlx_attn_decode(kv.data_ptr(), sc.data_ptr(), x.data_ptr(), x.data_ptr(), pos.data_ptr(), 0, 256,
                             x.data_ptr(), at.ws.buf.data_ptr(), at.ws.nbytes, None)
    assert rc == -1      # TLX_ERR_SHAPE


def test_engine0_spk_programs():
    # the reference-named programs with the reference's argument lists
    from thunderllamax_b200 import engine0
    rows, ctx, pos = 11, 1024, 300
    rng = np.random.default_rng(9)
    qrow, krow, vrow, qnw, knw = inputs(rng, rows)
    kv, sc = random_cache(rng, ctx, pos)
    q_t, k_t, v_t, qn_t, kn_t, fr_t = dev(qrow, krow, vrow, qnw, knw, oracle.rope_freqs())
    pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
    progs = engine0.load_progs(rows=rows, vocab=4096)
    kv_p, sc_p = dev(kv, sc)
    qw = torch.zeros((rows, 24, 256), dtype=torch.float32, device="cuda")
    qw16 = torch.zeros((rows, 24, 256), dtype=torch.float16, device="cuda")
    R = 6 * rows
    pm, ps = (torch.zeros(4 * 256 * R, device="cuda") for _ in range(2))
    pa = torch.zeros(16, device="cuda")
    ao = torch.zeros(rows * 6144, dtype=torch.float16, device="cuda")
    progs["spk_pre11"](q_t, k_t, v_t, qn_t, kn_t, fr_t, kv_p, sc_p, pos_t, qw, qw16, global_size=24)
    progs["spk_a11"](kv_p, sc_p, qw16, pos_t, pm, ps, pa)
    progs["spk_c11"](pm, ps, pa, q_t, ao)
    _, kv_l, sc_l, ao_l = run_lib(rows, ctx, qrow, krow, vrow, qnw, knw, kv, sc, pos)
    torch.cuda.synchronize()
    assert np.array_equal(kv_p.cpu().numpy(), kv_l)
    assert np.array_equal(ao.view(rows, 6144).cpu().numpy().view(np.int16), ao_l.view(np.int16))


def test_attention_all_zero_groups():
    # an all-zero 32-dim group quantises with scale fp16(1e-8) = 0; the reference's
    # fmaxf / fminf clamp turns 0 / 0 into -127, byte 1 (engine/spk_preqh.cu:77-83).
    # K head 1 is zero for every row (its RMS norm is then 0 as well) and V groups 0
    # and 5 of head 2 are zero; the cache bytes must match the oracle (and the
    # reference kernel, when its cubin is built) bit for bit, and decoding a cache
    # with zero scales stays finite.
    rows, ctx, pos = 11, REF_CTX, 700
    rng = np.random.default_rng(31)
    qrow, krow, vrow, qnw, knw = inputs(rng, rows)
    krow[:, 256:512] = 0
    vrow[:, 512:544] = 0
    vrow[:, 512 + 160:512 + 192] = 0
    kv, sc = random_cache(rng, ctx, pos)
    qw16, kv_lib, sc_lib, ao = run_lib(rows, ctx, qrow, krow, vrow, qnw, knw, kv, sc, pos)
    new = slice(pos, pos + rows)
    assert (kv_lib[1, new] == 1).all() and (sc_lib[1, new] == 0).all()
    assert (kv_lib[4 + 2, new, 0:32] == 1).all() and (kv_lib[4 + 2, new, 160:192] == 1).all()
    kv_o, sc_o = kv.copy(), sc.copy()
    oracle.attn_pre(qrow, krow, vrow, qnw, knw, oracle.rope_freqs(), pos, kv_o, sc_o)
    assert np.array_equal(kv_lib[1, new], kv_o[1, new]) and np.array_equal(kv_lib[6, new], kv_o[6, new])
    assert np.isfinite(ao.astype(np.float64)).all()
    ref = oracle.attn_decode(qw16, kv_lib, sc_lib, qrow, pos)
    check_rows(ao.astype(np.float64), ref, CONTRACT)
    if refkernels.have("spk_pre11"):
        q_t, k_t, v_t, qn_t, kn_t, fr_t = dev(qrow, krow, vrow, qnw, knw, oracle.rope_freqs())
        kv_r, sc_r = dev(kv, sc)
        pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
        qw = torch.zeros((rows, 24, 256), dtype=torch.float32, device="cuda")
        qw16_r = torch.zeros((rows, 24, 256), dtype=torch.float16, device="cuda")
        refkernels.launch("spk_pre11", 24, 256, [q_t, k_t, v_t, qn_t, kn_t, fr_t, kv_r, sc_r, pos_t, qw, qw16_r])
        torch.cuda.synchronize()
        assert np.array_equal(kv_r.cpu().numpy(), kv_lib)
        assert np.array_equal(sc_r.cpu().numpy().view(np.int16), sc_lib.view(np.int16))
