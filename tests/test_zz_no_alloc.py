"""The allocation-free head argmax (tlx_head_argmax_noalloc) against the
workspace-taking entry point (tlx_head_argmax), through the C ABI.

The no-alloc variant exists for callers that cannot call cudaMalloc where they
run the head (fixed-pool runtimes, budget-less plug-ins, loops that cannot take
cudaMalloc's implicit synchronisation).  It keeps its scratch in an array inside
the library, so this checks that (a) it gives the same ids, maxima, keys and
accept record as the regular entry point, call after call, with the array's
previous contents left in place, and (b) it refuses shapes whose scratch would
not fit.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from thunderllamax_b200 import _lib, ops, synth
from thunderllamax_b200.verify import synth_tiled

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 24 << 20


def noalloc_fn():
    L = _lib.lib()
    fn = L.tlx_head_argmax_noalloc
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    fn.argtypes = [i32, vp, vp, vp, i32, i64, i32, i64, i64, i64, vp, vp, vp, vp, i32, vp, vp]
    fn.restype = i32
    return fn


def noalloc_error():
    """The scratch error word of the last no-alloc call on this device."""
    fn = _lib.lib().tlx_head_argmax_noalloc_error
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    v = ctypes.c_uint32(0xFFFFFFFF)
    rc = fn(ctypes.byref(v), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.lib().tlx_error_string(rc).decode()
    return int(v.value)


def p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def run_noalloc(qtype, w, x, n_rows, row_offset, drafts):
    m, k = x.shape
    out = {"max": torch.full((m,), -1.0, device="cuda"), "idx": torch.full((m,), -1, dtype=torch.int32, device="cuda"),
           "keys": torch.zeros(m, dtype=torch.int64, device="cuda"),
           "acc": torch.full((2,), -1, dtype=torch.int32, device="cuda")}
    dt = {torch.bfloat16: 30, torch.float16: 1, torch.float32: 0}[x.dtype]
    grid = ops.grid("cuda") if qtype == "iq3_xxs" else None
    rc = noalloc_fn()(ops.qtype_id(qtype), p(w), p(grid), p(x), dt, x.stride(0), m, n_rows, k, row_offset,
                      p(out["max"]), p(out["idx"]), p(out["keys"]), p(drafts), int(drafts.numel()), p(out["acc"]),
                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.lib().tlx_error_string(rc).decode()
    return out


def run_regular(qtype, w, x, n_rows, row_offset, drafts, ws):
    m = x.shape[0]
    keys = torch.zeros(m, dtype=torch.int64, device="cuda")
    acc = torch.full((2,), -1, dtype=torch.int32, device="cuda")
    mx, idx = ops.head_argmax(qtype, w, x, n_rows, ws, row_offset=row_offset, out_keys=keys, drafts=drafts,
                              accept_out=acc)
    return {"max": mx, "idx": idx, "keys": keys, "acc": acc}


@pytest.mark.parametrize("qtype,vocab,k,ctas", [("q6_k", 20011, 1024, 0), ("iq3_xxs", 9000, 512, 0),
                                                ("q6_k", 151936, 5120, 0), ("q6_k", 20011, 1024, 37)])
def test_noalloc_head_matches_workspace_entry_point(qtype, vocab, k, ctas):
    # ctas = 37: both entry points run under the same tlx_set_max_ctas cap (a smaller
    # grid, so more tiles split across CTAs), reset afterwards
    ops.require_device()
    ops.set_max_ctas(ctas)
    try:
        _compare(qtype, vocab, k)
    finally:
        ops.set_max_ctas(0)


def _compare(qtype, vocab, k):
    m = 11
    rng = np.random.default_rng(vocab + k)
    if vocab * k > 50_000_000:
        w = synth_tiled(qtype, vocab, k, seed=77)
    else:
        w = ops.pack_tiles(qtype, synth.BLOCK_GEN[qtype](rng, vocab, k), k)
    ws = ops.Workspace.for_shape(ops.MODE_ARGMAX, qtype, vocab, k, m)
    assert ws.nbytes <= SCRATCH_BYTES
    for call in range(2):
        xb = synth.bf16_normal(rng, (m, k))
        x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
        ref = run_regular(qtype, w, x, vocab, 500, torch.zeros(m - 1, dtype=torch.int32, device="cuda"), ws)
        torch.cuda.synchronize()
        drafts = ref["idx"][:m - 1].clone()
        if call == 1:
            drafts[3] = (drafts[3] + 1) % (vocab + 500)   # accept stops at 3
        ref = run_regular(qtype, w, x, vocab, 500, drafts, ws)
        got = run_noalloc(qtype, w, x, vocab, 500, drafts)
        torch.cuda.synchronize()
        assert noalloc_error() == 0 and ws.error() == 0
        assert torch.equal(got["idx"], ref["idx"]), (call, got["idx"], ref["idx"])
        assert torch.equal(got["keys"], ref["keys"])
        np.testing.assert_allclose(got["max"].cpu().numpy(), ref["max"].cpu().numpy(), rtol=1e-6, atol=0)
        assert got["acc"].tolist() == ref["acc"].tolist() == ([m - 1, int(ref["idx"][m - 1])] if call == 0
                                                              else [3, int(ref["idx"][3])])


def test_noalloc_rejects_shapes_beyond_its_scratch():
    # Both refusals happen on the host before any pointer is used or any kernel is
    # launched (the weight buffer below is far smaller than either shape).
    ops.require_device()
    rng = np.random.default_rng(0)
    w = ops.pack_tiles("q6_k", synth.q6k_blocks(rng, 16, 256), 256)
    x = torch.zeros((11, 256), dtype=torch.bfloat16, device="cuda")
    d = torch.zeros(10, dtype=torch.int32, device="cuda")
    out = torch.empty(11, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # k = 2^20: the staged activation image alone (32 MB) exceeds the 24 MB scratch
    k = 1 << 20
    assert _lib.lib().tlx_gemv_workspace_bytes(ops.MODE_ARGMAX, 14, 16, k, 11, 30) > SCRATCH_BYTES
    rc = noalloc_fn()(14, p(w), None, p(x), 30, k, 11, 16, k, 0, None, p(out), None, p(d), 10, None, stream)
    assert rc == -5, _lib.lib().tlx_error_string(rc).decode()   # TLX_ERR_WORKSPACE
    # more than 16 columns: refused as a shape error
    rc = noalloc_fn()(14, p(w), None, p(x), 30, 256, 17, 16, 256, 0, None, p(out), None, p(d), 10, None, stream)
    assert rc != 0
