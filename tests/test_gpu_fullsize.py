"""BASELINE configs 2, 3 and 5 at their stated sizes, through the C ABI, against
the float64 oracle on the same seeded inputs.

* Config 3: the 151936 x 5120 Q6_K head fused with argmax and greedy accept.
  Drafts follow the configuration's recipe (j ~ U{0..10} from the seed; drafts
  before j equal the oracle argmax of their row, later ones uniform ids), and
  every j in 0..10 is run as well so that the accepted length takes every value.
  Argmax ids and accept records are compared bit for bit.
* Configs 2 + 3: the whole verify step (VerifyStep, one CUDA graph) on the same
  seeded model the bench times: y within the contract, ids and accept exact.
* Config 5: the 2048-token prefill FFN (tcgen05) on the same FFN weights; 128
  seeded FFN rows of act and 128 output rows of y are recomputed in float64
  (all 2048 tokens each).

The model is the bench's: synth.matrix_rows with VerifyStep(seed=0)'s seeds.
"""
import numpy as np
import pytest
import torch

import oracle
from thunderllamax_b200 import ops, synth
from thunderllamax_b200.verify import VerifyShape, VerifyStep

pytestmark = pytest.mark.gpu

CONTRACT = 2e-3
SEED = 0                       # VerifyStep(seed=0): gate 1, up 2, down 3, head 4
HEAD_SEEDS = (3031, 3032, 3033)
STEP_SEED = 2323


@pytest.fixture(scope="module")
def model():
    ops.require_device()
    s = VerifyShape()
    raw = {"gate": synth.matrix_rows(s.ffn_q, s.ffn, s.dim, SEED + 1),
           "up": synth.matrix_rows(s.ffn_q, s.ffn, s.dim, SEED + 2),
           "down": synth.matrix_rows(s.down_q, s.dim, s.ffn, SEED + 3),
           "head": synth.matrix_rows(s.head_q, s.vocab, s.dim, SEED + 4)}
    tiled = {"gate": ops.pack_tiles(s.ffn_q, raw["gate"], s.dim), "up": ops.pack_tiles(s.ffn_q, raw["up"], s.dim),
             "down": ops.pack_tiles(s.down_q, raw["down"], s.ffn),
             "head": ops.pack_tiles(s.head_q, raw["head"], s.dim)}
    return s, raw, tiled


def bf16_rows(rng, m, k):
    bits = synth.bf16_normal(rng, (m, k))
    x = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    return x, synth.bf16_bits_to_f32(bits).astype(np.float64)


@pytest.fixture(scope="module")
def head_cases(model):
    """H rows of every head case (three seeds for config 3, one for the verify
    step) and their float64 logits over the full vocabulary, in one oracle pass."""
    s, raw, _ = model
    cases = []
    for seed in HEAD_SEEDS + (STEP_SEED,):
        rng = np.random.default_rng(seed)
        if seed == STEP_SEED:
            bf16_rows(rng, s.rows, s.dim)           # the step draws x first, then h
        cases.append(bf16_rows(rng, s.rows, s.dim))
    X = np.concatenate([c[1] for c in cases], axis=0)
    lg = oracle.head_logits_f64(X, raw["head"], s.head_q)
    out = {}
    for i, seed in enumerate(HEAD_SEEDS + (STEP_SEED,)):
        L = lg[i * s.rows:(i + 1) * s.rows]
        mx, idx = oracle.argmax_rows(L)
        out[seed] = {"h": cases[i][0], "h64": cases[i][1], "mx": mx, "idx": idx, "gap": oracle.min_top2_gap(L),
                     "scale": np.abs(L).max()}
    return out


def recipe_drafts(idx_ref, n_drafts, vocab, rng, j=None):
    """Config 3's drafts; with j given, the first j drafts are the argmax and draft j
    (if any) is moved off it, so the accepted length is exactly j."""
    if j is None:
        return synth.drafts_for(idx_ref, n_drafts, vocab, rng)
    drafts = rng.integers(0, vocab, n_drafts).astype(np.int32)
    drafts[:j] = idx_ref[:j]
    if j < n_drafts and drafts[j] == idx_ref[j]:
        drafts[j] = (drafts[j] + 1) % vocab
    return drafts, j


def test_config3_full_size_head_argmax_accept(model, head_cases):
    s, _, tiled = model
    V, m = s.vocab, s.rows
    ws = ops.Workspace.for_shape(ops.MODE_ARGMAX, s.head_q, V, s.dim, m)
    seen = set()
    for seed in HEAD_SEEDS:
        c = head_cases[seed]
        # the fp32 kernel and the float64 oracle pick the same row whenever the top-1 /
        # top-2 gap exceeds fp32 accumulation error (~1e-6 of the logit scale)
        assert (c["gap"] > 1e-6 * c["scale"]).all(), "near-tie in this seed: choose another"
        rng = np.random.default_rng(seed + 7)
        draft_sets = [recipe_drafts(c["idx"], s.n_drafts, V, rng)] + \
                     [recipe_drafts(c["idx"], s.n_drafts, V, rng, j) for j in range(s.n_drafts + 1)]
        for drafts_np, _ in draft_sets:
            acc = torch.full((2,), -7, dtype=torch.int32, device="cuda")
            keys = torch.zeros(m, dtype=torch.int64, device="cuda")
            mx, idx = ops.head_argmax(s.head_q, tiled["head"], c["h"], V, ws, out_keys=keys,
                                      drafts=torch.from_numpy(drafts_np).cuda(), accept_out=acc)
            torch.cuda.synchronize()
            assert ws.error() == 0
            assert np.array_equal(idx.cpu().numpy(), c["idx"])
            m_ref, bonus_ref = oracle.accept(c["idx"], drafts_np)
            assert acc.cpu().tolist() == [m_ref, bonus_ref]
            seen.add(m_ref)
            np.testing.assert_allclose(mx.cpu().numpy(), c["mx"], rtol=1e-5, atol=1e-6 * c["scale"])
    assert seen == set(range(s.n_drafts + 1))


def test_config23_verify_step_full_size(model, head_cases):
    s, raw, tiled = model
    step = VerifyStep(s, weights=tiled)
    rng = np.random.default_rng(STEP_SEED)
    x, x64 = bf16_rows(rng, s.rows, s.dim)
    c = head_cases[STEP_SEED]
    bf16_rows(rng, s.rows, s.dim)                   # h (drawn in head_cases with this stream)
    res = rng.standard_normal((s.rows, s.dim), dtype=np.float32)
    drafts_np, _ = recipe_drafts(c["idx"], s.n_drafts, s.vocab, rng)
    step.set_inputs(x, c["h"], res=torch.from_numpy(res).cuda(), drafts=torch.from_numpy(drafts_np).cuda())
    step.replay()
    step.replay()                                   # a second replay: same bits
    torch.cuda.synchronize()
    for nm, e in step.workspace_errors().items():
        assert e == 0, nm
    _, y_ref = oracle.ffn_f64(x64, raw["gate"], raw["up"], raw["down"], residual=res)
    y = step.y.cpu().numpy().astype(np.float64)
    for t in range(s.rows):
        nrm = np.linalg.norm(y_ref[t])
        err = np.abs(y[t] - y_ref[t]).max()
        # gact is carried as fp16 (the reference's gact3 is fp16 too): one fp16 rounding
        assert err <= CONTRACT * nrm and err <= 1e-4 * nrm, (t, err, nrm)
    assert np.array_equal(step.out_idx.cpu().numpy(), c["idx"])
    assert step.accept_out.cpu().tolist() == list(oracle.accept(c["idx"], drafts_np))


def test_config5_prefill_full_size_sampled_rows(model):
    from thunderllamax_b200 import prefill

    s, raw, tiled = model
    p = prefill.PrefillShape()
    assert (p.dim, p.ffn) == (s.dim, s.ffn)
    step = prefill.PrefillFFN(p, weights={k: tiled[k] for k in ("gate", "up", "down")})
    rng = np.random.default_rng(555)
    x, x64 = bf16_rows(rng, p.tokens, p.dim)
    step.x.copy_(x)
    step.launch()
    torch.cuda.synchronize()
    assert step.ws.error() == 0 and step.ws_down.error() == 0
    act = step.act.float().cpu().numpy().astype(np.float64)
    y = step.y.cpu().numpy().astype(np.float64)
    n_s = 128
    # gate/up: 128 seeded FFN rows (act columns) over all tokens
    rows = np.sort(rng.choice(p.ffn, n_s, replace=False))
    g = x64 @ oracle.dequant(p.ffn_q, raw["gate"][rows], p.dim).astype(np.float64).T
    u = x64 @ oracle.dequant(p.ffn_q, raw["up"][rows], p.dim).astype(np.float64).T
    act_ref = oracle.silu_f64(g) * u
    # down: 128 seeded output rows over all tokens, from the kernel's own fp16 act
    outs = np.sort(rng.choice(p.dim, n_s, replace=False))
    y_ref = act @ oracle.dequant(p.down_q, raw["down"][outs], p.ffn).astype(np.float64).T
    for got, ref, full in ((act[:, rows], act_ref, p.ffn), (y[:, outs], y_ref, p.dim)):
        # ||row||_2 of the whole output row estimated from its sampled part
        nrm = np.linalg.norm(ref, axis=1) * np.sqrt(full / n_s)
        err = np.abs(got - ref).max(axis=1)
        # fp16 dequantised weights and fp16 act: well inside the 2e-3 contract
        assert (err <= 1e-3 * nrm).all(), (err / nrm).max()
