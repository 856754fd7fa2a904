"""The library's accept / argmax / state-select kernels against the reference's own
CUDA kernels (engine/accept11k.cu, engine/acceptsel11k.cu, engine/h_argmax.cu,
engine/amx3.cu, engine/mm/MM_P7_acc36.cu, compiled unchanged into oracle/_ref by
oracle/build_ref.py) on the same device inputs: every output bit-exact."""
import numpy as np
import pytest
import torch

import refkernels
from thunderllamax_b200 import engine0, ops

pytestmark = pytest.mark.gpu
VOCAB_REF = 248320   # the vocabulary compiled into amx3 / h_argmax
DIM_REF = 5120       # the row width compiled into accept11k


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()


def logit_rows(rng, rows):
    x = rng.standard_normal((rows, VOCAB_REF)).astype(np.float16)
    for r in range(rows):
        kind = r % 6
        if kind == 1:      # exact tie of the maximum at two indices
            a, b = sorted(rng.choice(VOCAB_REF, 2, replace=False))
            x[r, a] = x[r, b] = np.float16(9.0)
        elif kind == 2:    # NaN and -inf never win; +inf does
            x[r, rng.choice(VOCAB_REF, 50)] = np.nan
            x[r, rng.choice(VOCAB_REF, 50)] = -np.inf
            x[r, 12345] = np.inf
        elif kind == 3:    # no candidate at all -> 0
            x[r] = -np.inf
            x[r, rng.choice(VOCAB_REF, 20)] = np.nan
        elif kind == 4:    # maximum at the last index, fp16 max value
            x[r, -1] = np.float16(65504.0)
        elif kind == 5:    # every entry equal -> lowest index
            x[r] = np.float16(-3.5)
    return torch.from_numpy(x).cuda()


def test_amx3_matches_reference():
    refkernels.require("amx3")
    rows = 12
    logits = logit_rows(np.random.default_rng(1), rows)
    ref = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    refkernels.launch("amx3", rows, 256, [logits, ref])
    got = ops.argmax_rows(logits)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


def test_h_argmax_matches_reference():
    refkernels.require("h_argmax")
    logits = logit_rows(np.random.default_rng(2), 6)
    for r in range(6):
        outs = []
        for impl in ("ref", "lib"):
            tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
            pos = torch.tensor([37 + r], dtype=torch.int32, device="cuda")
            hist = torch.full((64,), -2, dtype=torch.int32, device="cuda")
            row = logits[r].contiguous()
            if impl == "ref":
                refkernels.launch("h_argmax", 1, 256, [row, tok, pos, hist])
            else:
                ops.h_argmax(row, tok, pos, hist)
                torch.cuda.synchronize()
            outs.append((tok.cpu().numpy(), pos.cpu().numpy(), hist.cpu().numpy()))
        for a, b in zip(*outs):
            assert np.array_equal(a, b), r


def test_acc36_matches_reference():
    refkernels.require("acc36")
    rng = np.random.default_rng(3)
    for K in (0, 1, 2, 8, 10):
        for trial in range(6):
            amds = rng.integers(0, 1000, K + 1).astype(np.int32)
            drafts = amds[:K].copy()
            if K and trial % 3:
                j = int(rng.integers(0, K))
                drafts[j] += 1
            a, d = torch.from_numpy(amds).cuda(), torch.from_numpy(drafts if K else np.zeros(1, np.int32)).cuda()
            mb_r, eb_r = torch.full((1,), -1, dtype=torch.int32, device="cuda"), torch.full((2,), -1, dtype=torch.int32,
                                                                                             device="cuda")
            refkernels.launch("acc36", 1, 256, [a, d, mb_r, eb_r, K])
            mb, eb = ops.accept(a, d, K)
            torch.cuda.synchronize()
            assert torch.equal(mb, mb_r) and torch.equal(eb, eb_r), (K, trial)


def accept11k_state(rng, m_target):
    amds = rng.integers(0, 150000, 11).astype(np.int32)
    drafts = amds[:10].copy()
    if m_target < 10:
        drafts[m_target] = (drafts[m_target] + 1) % 150000
    return {
        "amds": amds, "ring": drafts,
        "xA": rng.standard_normal(11 * DIM_REF).astype(np.float32),
        "m_slot": np.array([-1], np.int32), "m_hist": np.full(32, -1, np.int32),
        "cyc_slot": np.array([7], np.int32), "pos_slot": np.array([1000 + m_target], np.int32),
        "cur_slot": np.array([-1], np.int32), "tok_hist": np.full(2048, -3, np.int32),
        "h_seed": np.zeros(DIM_REF, np.float32), "hd_d0": rng.standard_normal(DIM_REF).astype(np.float32),
        "hd_d1": rng.standard_normal(DIM_REF).astype(np.float32), "dhd_seed": np.zeros(DIM_REF, np.float32),
        "emit": np.full(32, -5, np.int32), "l_hist": np.arange(32, dtype=np.int32) + 100,
    }


def test_accept11k_matches_reference():
    refkernels.require("accept11k")
    prog = engine0.load_progs_small_accept(DIM_REF)
    names = ["xA", "m_slot", "m_hist", "cyc_slot", "pos_slot", "cur_slot", "tok_hist", "h_seed", "hd_d0", "hd_d1",
             "dhd_seed", "emit", "l_hist"]
    for m_target in range(11):
        st = accept11k_state(np.random.default_rng(40 + m_target), m_target)
        results = []
        for impl in ("ref", "lib"):
            t = {k: torch.from_numpy(v.copy()).cuda() for k, v in st.items()}
            drings = [t["ring"][j:j + 1] for j in range(10)]
            args = [t["amds"], *drings, *[t[n] for n in names]]
            if impl == "ref":
                refkernels.launch("accept11k", 1, 256, args)
            else:
                prog(*args)
                torch.cuda.synchronize()
            results.append({n: t[n].cpu().numpy() for n in names})
        for n in names:
            assert np.array_equal(results[0][n].view(np.uint32), results[1][n].view(np.uint32)), (m_target, n)
        assert int(results[1]["m_slot"][0]) == m_target


def test_acceptsel11k_matches_reference():
    # full reference size: [48][5] x (786432 + 30720) fp32 slots + 13 scratch buffers
    refkernels.require("acceptsel11k")
    B, R, C = ops.GDN_BLOCKS, ops.GDN_REC, ops.GDN_CONV
    g = torch.Generator(device="cuda").manual_seed(5)
    rec4 = torch.randn((B, 5, R), device="cuda", generator=g)
    conv4 = torch.randn((B, 5, C), device="cuda", generator=g)
    rec_x = [torch.randn((B, R), device="cuda", generator=g) for _ in range(6)]
    conv_x = [torch.randn((B, C), device="cuda", generator=g) for _ in range(7)]
    for m in (0, 3, 4, 5, 9, 10):
        m_slot = torch.tensor([m], dtype=torch.int32, device="cuda")
        r_ref, c_ref = rec4.clone(), conv4.clone()
        refkernels.launch("acceptsel11k", B, 256, [r_ref, c_ref, m_slot, *conv_x, *rec_x])
        r_lib, c_lib = rec4.clone(), conv4.clone()
        ops.acceptsel11k(r_lib, c_lib, m_slot, conv_x, rec_x)
        torch.cuda.synchronize()
        assert torch.equal(r_lib.view(torch.int32), r_ref.view(torch.int32)), m
        assert torch.equal(c_lib.view(torch.int32), c_ref.view(torch.int32)), m
        del r_ref, c_ref, r_lib, c_lib
