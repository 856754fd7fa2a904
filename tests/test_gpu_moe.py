"""GPU parity of the MoE verify layer against the numpy
oracle (oracle.moe_verify_f64, the restatement of rt8e256 -> shexp8 ->
gx8e256up4 -> gx8e256dn -> cmbz2048) on identical seeded inputs, through the C
ABI (tlx_moe_verify).

Contract: router ids bit-exact; outputs within max|err| <= 2e-3 * ||row||_2 of
the float64 oracle.  The expert matvecs run on fp16 activations (bf16 h is exact
in fp16; act = silu(g) * u is rounded to fp16 once, under a power-of-two scale per
pair) with fp16 products of the integer IQ4 levels and sub-scales, so a tighter
2e-4 * ||row|| bound is asserted as well."""
import numpy as np
import pytest
import torch

import oracle
from thunderllamax_b200 import moe, ops, synth

pytestmark = pytest.mark.gpu

CONTRACT = 2e-3
TIGHT = 2e-4


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()
    yield


def inputs(shape, seed):
    rng = np.random.default_rng(seed + 100)
    bits = synth.bf16_normal(rng, (shape.positions, shape.hidden))
    h64 = synth.bf16_bits_to_f32(bits).astype(np.float64)
    hres = rng.standard_normal((shape.positions, shape.hidden)).astype(np.float32)
    h_t = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    return h_t, h64, torch.from_numpy(hres).cuda(), hres


def router_gap(logits):
    """Smallest gap between consecutive values among each position's top 9 (the
    selection and its order are decided by these gaps; fp32 logits are ~1e-6 off)."""
    s = -np.sort(-logits, axis=1)[:, :9]
    return float(np.min(s[:, :-1] - s[:, 1:]))


def check_y(y, ref_y, tol):
    err = np.abs(y.astype(np.float64) - ref_y).max(axis=1)
    norm = np.linalg.norm(ref_y, axis=1)
    assert (err <= tol * norm).all(), (err / norm).max()


def oracle_of(host, h64, hres=None):
    return oracle.moe_verify_f64(h64, host["wr"], host["wsh"], host["gate"], host["up"], host["down"],
                                 host["sgate"], host["sup"], host["sdown"], hres=hres)


def run(shape, seed, **kw):
    host = moe.synth_host(shape, seed)
    h_t, h64, hres_t, hres = inputs(shape, seed)
    ref = oracle_of(host, h64, hres)
    step = moe.MoeVerifyStep(shape, host=host, **kw)
    step.set_inputs(h_t, hres_t)
    step.launch()
    torch.cuda.synchronize()
    return host, step, ref, (h_t, hres_t)


@pytest.mark.parametrize("shape,seed", [
    (moe.MoeShape(positions=5, experts=32, hidden=512, inner=256), 1),
    (moe.MoeShape(positions=1, experts=16, hidden=256, inner=256), 2),
    (moe.MoeShape(positions=8, experts=8, hidden=512, inner=512), 3),      # top-8 of 8: every expert
    (moe.MoeShape(positions=3, experts=64, hidden=1024, inner=768), 4),
])
def test_moe_small_shapes(shape, seed):
    _, step, ref, _ = run(shape, seed)
    assert router_gap(ref["logits"]) > 1e-5
    assert np.array_equal(step.ids.cpu().numpy(), ref["ids"])
    assert np.abs(step.gates.cpu().numpy() - ref["gates"]).max() < 1e-5
    assert np.abs(step.sg.cpu().numpy() - ref["sg"]).max() < 1e-6
    y = step.y.cpu().numpy()
    check_y(y, ref["y"], CONTRACT)
    check_y(y, ref["y"], TIGHT)
    assert step.ws.error() == 0


def test_moe_config4_full_shape():
    shape = moe.MoeShape()          # 5 positions, 256 experts, 2048 -> 512 -> 2048, top-8 + shared
    _, step, ref, _ = run(shape, 7)
    assert router_gap(ref["logits"]) > 1e-5
    assert np.array_equal(step.ids.cpu().numpy(), ref["ids"])
    assert np.abs(step.gates.cpu().numpy() - ref["gates"]).max() < 1e-5
    y = step.y.cpu().numpy()
    check_y(y, ref["y"], CONTRACT)
    check_y(y, ref["y"], TIGHT)
    # the layer's contribution alone (without the residual) is also within the bound
    hres = step.hres.cpu().numpy().astype(np.float64)
    check_y((y - hres).astype(np.float32), ref["y"] - hres, CONTRACT)
    u = len(set(ref["ids"].reshape(-1).tolist()))
    assert step.touched_bytes() == shape.router_bytes() + (u + 1) * shape.expert_bytes()
    assert step.ws.error() == 0


def test_moe_repeat_and_graph_replay_bitwise():
    shape = moe.MoeShape(positions=5, experts=64, hidden=1024, inner=512)
    _, step, ref, (h_t, hres_t) = run(shape, 11)
    y0 = step.y.clone()
    for _ in range(3):                      # counters re-arm: repeated launches agree bitwise
        step.launch()
    torch.cuda.synchronize()
    assert torch.equal(step.y, y0)
    step.capture()
    step.y.zero_()
    for _ in range(4):
        step.replay()
    torch.cuda.synchronize()
    assert torch.equal(step.y, y0)
    # new inputs through the same graph
    rng = np.random.default_rng(5)
    bits = synth.bf16_normal(rng, (shape.positions, shape.hidden))
    step.set_inputs(torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16))
    step.replay()
    torch.cuda.synchronize()
    ref2 = oracle_of(step.host, synth.bf16_bits_to_f32(bits).astype(np.float64), hres_t.cpu().numpy())
    assert np.array_equal(step.ids.cpu().numpy(), ref2["ids"])
    check_y(step.y.cpu().numpy(), ref2["y"], CONTRACT)


def test_moe_expert_parallel_partition_sums_to_full():
    # two expert ranges on one GPU, as two EP ranks would run them: the shared expert
    # and the residual on the first; the partial outputs sum to the full layer
    shape = moe.MoeShape(positions=5, experts=64, hidden=1024, inner=512)
    host = moe.synth_host(shape, 13)
    h_t, h64, hres_t, hres = inputs(shape, 13)
    ref = oracle_of(host, h64, hres)
    parts = []
    for e0, e1, shared in ((0, 24, True), (24, 64, False)):
        st = moe.MoeVerifyStep(shape, host=host, e0=e0, e1=e1, shared=shared)
        st.set_inputs(h_t, hres_t)
        st.launch()
        torch.cuda.synchronize()
        assert np.array_equal(st.ids.cpu().numpy(), ref["ids"])      # router replicated
        parts.append(st.y.cpu().numpy().astype(np.float64))
    check_y((parts[0] + parts[1]).astype(np.float32), ref["y"], TIGHT)


def test_moe_rank_without_local_experts_writes_zero():
    shape = moe.MoeShape(positions=2, experts=16, hidden=256, inner=256)
    host = moe.synth_host(shape, 17)
    h_t, h64, _, _ = inputs(shape, 17)
    ref = oracle_of(host, h64)
    used = set(ref["ids"].reshape(-1).tolist())
    free = [e for e in range(16) if e not in used]
    if not free:
        pytest.skip("every expert routed")
    st = moe.MoeVerifyStep(shape, host=host, e0=free[0], e1=free[0] + 1, shared=False)
    st.set_inputs(h_t)
    st.y.fill_(123.0)
    st.launch()
    torch.cuda.synchronize()
    assert (st.y.cpu().numpy() == 0).all()
