"""The MoE oracle (oracle.moe_verify_f64) against a direct per-(position, rank)
recomputation that dequantises each routed expert afresh, on seeded config-4
style inputs at a small size (CPU only).  Positions that share an expert must get
that expert's weights, never another's (the combine follows
engine/mm/MM_P34_cmbz2048.cu:20-27: ranks ascending, then the shared expert, then
the residual)."""
import numpy as np

import oracle
from thunderllamax_b200 import moe, synth


def test_moe_oracle_matches_direct_recomputation():
    shape = moe.MoeShape(positions=5, experts=16, hidden=256, inner=256)
    host = moe.synth_host(shape, 3)
    rng = np.random.default_rng(4)
    h = synth.bf16_bits_to_f32(synth.bf16_normal(rng, (5, 256))).astype(np.float64)
    hres = rng.standard_normal((5, 256))
    ref = oracle.moe_verify_f64(h, host["wr"], host["wsh"], host["gate"], host["up"], host["down"],
                                host["sgate"], host["sup"], host["sdown"], hres=hres)
    ids, gates, sg, _ = oracle.router_top8(host["wr"], host["wsh"], h)
    assert len(set(ids.reshape(-1).tolist())) < ids.size      # some experts are shared by positions

    def ffn(g, u, d, x):
        Wg = oracle.dequant_iq4xs(g, 256).astype(np.float64)
        Wu = oracle.dequant_iq4xs(u, 256).astype(np.float64)
        Wd = oracle.dequant_iq4xs(d, 256).astype(np.float64)
        return Wd @ (oracle.silu_f64(Wg @ x) * (Wu @ x))

    for p in range(5):
        acc = np.zeros(256)
        for r in range(8):
            e = ids[p, r]
            acc += gates[p, r] * ffn(host["gate"][e], host["up"][e], host["down"][e], h[p])
        acc += sg[p] * ffn(host["sgate"], host["sup"], host["sdown"], h[p])
        assert np.array_equal(ref["y"][p], hres[p] + acc)
    assert np.allclose(gates.sum(axis=1), 1.0)
