"""GPU parity of the n-gram drafter (tlx_lookup) against the oracle and against
the reference's own lookup{K+1}_nw32 kernels (oracle/_ref cubins) on the same
device buffers: l_hist and the draft ring bit-exact."""
import numpy as np
import pytest
import torch

import oracle
import refkernels
from test_oracle_lookup import planted_history
from thunderllamax_b200 import ops

pytestmark = pytest.mark.gpu
SENTINEL = -7


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()


def run_lib(lk, h, pos, cyc=3, hist_cap=None):
    cap = hist_cap or len(h)
    hist = torch.zeros(max(cap, 1), dtype=torch.int32, device="cuda")
    hist[:len(h)] = torch.from_numpy(h).cuda()
    pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
    cyc_t = torch.tensor([cyc], dtype=torch.int32, device="cuda")
    drafts = torch.full((lk.k,), SENTINEL, dtype=torch.int32, device="cuda")
    l_hist = torch.zeros(16, dtype=torch.int32, device="cuda")
    lk(hist, pos_t, cyc_t, drafts, l_hist)
    torch.cuda.synchronize()
    return int(l_hist[cyc]), drafts.cpu().numpy(), l_hist.cpu().numpy()


def check(lh, d, ref, k):
    lh_ref, d_ref = ref
    assert lh == lh_ref
    if d_ref is None:
        assert (d == SENTINEL).all()
    else:
        assert np.array_equal(d, d_ref)


@pytest.mark.parametrize("k", sorted(ops.LOOKUP_SCAN_END))
def test_lookup_vs_oracle(k):
    lk = ops.Lookup(k)
    rng = np.random.default_rng(200 + k)
    for trial in range(30):
        n = int(rng.integers(1, 3000))
        h = planted_history(rng, n, int(rng.integers(2, 20)), int(rng.integers(0, 6)))
        pos = int(rng.integers(0, n + 1))
        if trial % 2 == 0 and n > 60:
            a = int(rng.integers(0, n - 40))
            h[n - 8:n] = h[a:a + 8]
            pos = n
        lh, d, _ = run_lib(lk, h, pos)
        check(lh, d, oracle.lookup_ngram(h, pos, k, lk.scan_end), k)


@pytest.mark.parametrize("k", sorted(ops.LOOKUP_SCAN_END))
def test_lookup_vs_reference_kernel(k):
    name = f"lookup{k + 1}_nw32"
    refkernels.require(name)
    lk = ops.Lookup(k)
    rng = np.random.default_rng(300 + k)
    for trial in range(12):
        n = int(rng.integers(20, 5000))
        h = planted_history(rng, n, int(rng.integers(2, 30)), int(rng.integers(0, 8)))
        pos = n if trial % 3 else int(rng.integers(0, n + 1))
        if trial % 2 == 0 and n > 60:
            a = int(rng.integers(0, n - 40))
            h[n - 8:n] = h[a:a + 8]
        hist = torch.from_numpy(h).cuda()
        pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
        cyc_t = torch.tensor([5], dtype=torch.int32, device="cuda")
        cur_t = torch.zeros(1, dtype=torch.int32, device="cuda")
        ring = torch.full((k,), SENTINEL, dtype=torch.int32, device="cuda")
        l_hist = torch.zeros(16, dtype=torch.int32, device="cuda")
        # the reference: one 1024-thread CTA (the nw32 launch law)
        refkernels.launch(name, 1, 1024, [hist, pos_t, cur_t, *[ring[j:j + 1] for j in range(k)], l_hist, cyc_t])
        ref_l, ref_ring = int(l_hist[5]), ring.cpu().numpy()
        lh, d, _ = run_lib(lk, h, pos, cyc=5)
        assert lh == ref_l and np.array_equal(d, ref_ring), (trial, n, pos, lh, ref_l)


def test_lookup_long_history_and_rearm():
    # a 200K-token history over ~200 CTAs; the winner near the start, then near the end
    lk = ops.Lookup(10)
    rng = np.random.default_rng(7)
    n = 200_000
    h = rng.integers(0, 50_000, n).astype(np.int32)
    h[n - 8:n] = h[1000:1008]
    lh, d, _ = run_lib(lk, h, n)
    ref = oracle.lookup_ngram(h, n, 10, 19)
    assert ref[0] == 9
    check(lh, d, ref, 10)
    h[150_000:150_008] = h[n - 8:n]
    lh, d, _ = run_lib(lk, h, n)
    ref = oracle.lookup_ngram(h, n, 10, 19)
    assert np.array_equal(ref[1], h[150_008:150_018])
    check(lh, d, ref, 10)
    # shorter pos on the same buffer capacity: CTAs past pos only join the handshake
    lh, d, _ = run_lib(lk, h, 5000, hist_cap=n)
    check(lh, d, oracle.lookup_ngram(h, 5000, 10, 19), 10)


def test_lookup_pos_beyond_buffer_writes_nothing():
    lk = ops.Lookup(10)
    h = np.arange(100, dtype=np.int32)
    lh, d, l_hist = run_lib(lk, h, 101)
    assert (l_hist == 0).all() and (d == SENTINEL).all()
    # and the workspace is re-armed for the next call
    h[92:100] = h[10:18]
    lh, d, _ = run_lib(lk, h, 100)
    check(lh, d, oracle.lookup_ngram(h, 100, 10, 19), 10)


def test_engine0_lookup11_program():
    from thunderllamax_b200 import engine0
    progs = engine0.load_progs(rows=11, vocab=4096)
    P = engine0.Bufs()
    ring = engine0.dring_views(P, 10)
    h = np.arange(1000, 1300, dtype=np.int32)
    h[292:300] = h[40:48]
    hist = torch.from_numpy(h).cuda()
    pos_t = torch.tensor([300], dtype=torch.int32, device="cuda")
    cyc_t = torch.tensor([2], dtype=torch.int32, device="cuda")
    l_hist = torch.zeros(8, dtype=torch.int32, device="cuda")
    progs["lookup11_nw32"](hist, pos_t, torch.zeros(1, dtype=torch.int32, device="cuda"),
                           *[P.d[f"dring{i}"] for i in range(10)], l_hist, cyc_t, global_size=1, local_size=1024)
    torch.cuda.synchronize()
    assert int(l_hist[2]) == 9
    assert np.array_equal(ring.cpu().numpy(), h[48:58])
