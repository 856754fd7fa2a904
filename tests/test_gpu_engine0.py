"""The drop-in verify programs of engine0.load_progs(), called the way the
reference engine calls its kernels: buffers only, in the reference's argument
order (engine/mtp.py:1127-1128 ffn8v11r7 -> down8nw32v11r7, :1159-1161 head8v11
-> amx3, :749-752 accept11k), at a reduced shape, against the float64 oracle.
"""
import numpy as np
import pytest
import torch

import oracle
from thunderllamax_b200 import engine0, ops, synth

pytestmark = pytest.mark.gpu

DIM, FFN, VOCAB, ROWS = 1024, 2048, 7001, 11


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()


def test_engine0_verify_programs_chain():
    rng = np.random.default_rng(1127)
    rg, ru = synth.iq3xxs_blocks(rng, FFN, DIM), synth.iq3xxs_blocks(rng, FFN, DIM)
    rd, rh = synth.q6k_blocks(rng, DIM, FFN), synth.q6k_blocks(rng, VOCAB, DIM)
    xb, hb = synth.bf16_normal(rng, (ROWS, DIM)), synth.bf16_normal(rng, (ROWS, DIM))
    # the reference engine carries activations as fp16 (hhx, xh) and the residual as fp32
    x16 = synth.bf16_bits_to_f32(xb).astype(np.float16)
    h16 = synth.bf16_bits_to_f32(hb).astype(np.float16)
    hh = rng.standard_normal((ROWS, DIM)).astype(np.float32)

    P = engine0.Bufs()
    P.pack("wg", "iq3_xxs", rg, DIM)
    P.pack("wu", "iq3_xxs", ru, DIM)
    P.pack("wd", "q6_k", rd, FFN)
    P.pack("wh", "q6_k", rh, DIM)
    P.up("gridf", oracle.iq3xxs_grid_u32())
    P.up("hhx", x16)
    P.up("xh", h16)
    P.up("hh", hh)
    P.alloc("gact", 2 * ROWS * FFN, torch.float16)
    P.alloc("y", 4 * ROWS * DIM, torch.float32)
    P.alloc("logits", 2 * ROWS * VOCAB, torch.float16)
    P.alloc("amds", 4 * ROWS, torch.int32)
    P.alloc("amds_f", 4 * ROWS, torch.int32)
    d = P.d

    progs = engine0.load_progs(dim=DIM, ffn=FFN, vocab=VOCAB, rows=ROWS)
    progs["ffn8v11"](d["wg"], d["wu"], d["gridf"], d["hhx"], d["gact"], global_size=(FFN // 4, 1, 1))
    progs["down8nw32_11"](d["wd"], d["gridf"], d["gact"], d["hh"], d["y"], global_size=(DIM // 32, 1, 1))
    progs["head8v11"](d["wh"], d["xh"], d["logits"])
    progs["amx3"](d["logits"], d["amds"])
    progs["head_argmax"](d["wh"], d["xh"], d["amds_f"])
    torch.cuda.synchronize()

    x64, h64 = x16.astype(np.float64), h16.astype(np.float64)
    gact_ref, y_ref = oracle.ffn_f64(x64, rg, ru, rd, residual=hh)
    gact = P.down("gact", (ROWS, FFN), np.float16).astype(np.float64)
    y = P.down("y", (ROWS, DIM), np.float32).astype(np.float64)
    for got, ref, tight in ((gact, gact_ref, 1e-3), (y, y_ref, 1e-4)):
        for t in range(ROWS):
            nrm = np.linalg.norm(ref[t])
            err = np.abs(got[t] - ref[t]).max()
            assert err <= 2e-3 * nrm and err <= tight * nrm, (t, err, nrm)

    _, idx_ref, lg = oracle.head_argmax(h64, rh, "q6_k")
    assert (oracle.min_top2_gap(lg) > 1e-3 * np.abs(lg).max()).all(), "near-tie in this seed"
    # fused head: bit-exact ids; head8v11 (fp16 logits, as the reference) + amx3: the
    # argmax of the fp16-rounded logits, which here equals the exact one
    assert np.array_equal(P.down("amds_f"), idx_ref)
    logits16 = P.down("logits", (ROWS, VOCAB), np.float16)
    assert np.array_equal(P.down("amds"), oracle.argmax_rows(logits16.astype(np.float64))[1])
    assert np.array_equal(P.down("amds"), idx_ref)

    # accept11k on the fused head's ids, drafts per the head+accept configuration
    drafts, j = synth.drafts_for(idx_ref, ROWS - 1, VOCAB, np.random.default_rng(5))
    ring = engine0.dring_views(P, 10)
    ring.copy_(torch.from_numpy(drafts))
    xA = rng.standard_normal((ROWS, DIM)).astype(np.float32)
    hd0, hd1 = rng.standard_normal(DIM).astype(np.float32), rng.standard_normal(DIM).astype(np.float32)
    state = {"pos": 40, "cyc": 3, "cur": 0, "m_slot": 0, "tok_hist": np.full(128, -1, np.int32),
             "m_hist": np.zeros(16, np.int32), "l_hist": np.arange(16, dtype=np.int32) + 100}
    P.up("xA", xA)
    for nm, v in (("m_slot", 0), ("cyc_slot", state["cyc"]), ("pos_slot", state["pos"]), ("cur_slot", 0)):
        P.up(nm, np.array([v], np.int32))
    P.up("m_hist", state["m_hist"])
    P.up("l_hist", state["l_hist"])
    P.up("tok_hist", state["tok_hist"])
    P.alloc("h_seed", 4 * DIM, torch.float32)
    P.alloc("dhd_seed", 4 * DIM, torch.float32)
    P.up("hd_d0", hd0)
    P.up("hd_d1", hd1)
    P.alloc("emit", 4 * 26, torch.int32).zero_()
    progs["accept11k"](d["amds_f"], *[d[f"dring{i}"] for i in range(10)], d["xA"], d["m_slot"], d["m_hist"],
                       d["cyc_slot"], d["pos_slot"], d["cur_slot"], d["tok_hist"], d["h_seed"], d["hd_d0"],
                       d["hd_d1"], d["dhd_seed"], d["emit"], d["l_hist"], global_size=(1, 1, 1))
    torch.cuda.synchronize()
    st, emit, h_seed, dhd_seed = oracle.accept11k(idx_ref, drafts, state, xA=xA, hd_d0=hd0, hd_d1=hd1, dim=DIM)
    assert int(d["pos_slot"].item()) == st["pos"] and int(d["cur_slot"].item()) == st["cur"]
    assert int(d["m_slot"].item()) == st["m_slot"] and int(d["cyc_slot"].item()) == st["cyc"]
    assert np.array_equal(P.down("tok_hist"), st["tok_hist"])
    assert np.array_equal(P.down("m_hist"), st["m_hist"])
    assert np.array_equal(P.down("emit")[:16], emit[:16])
    assert np.array_equal(P.down("h_seed"), h_seed)
    assert np.array_equal(P.down("dhd_seed"), dhd_seed)
