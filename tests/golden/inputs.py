"""Seeded inputs shared by gen_golden.py and the tests that read its fixtures.

Inputs too large to commit (the 256 x 2048 fp32 router, the combine parts)
are regenerated from these seeds; only the reference's outputs are stored.
"""
from __future__ import annotations

import numpy as np

ROUTER_SEED = 4242
CMB_SEED = 777


def router_inputs(seed: int = ROUTER_SEED, positions: int = 5):
    rng = np.random.default_rng(seed)
    Wr = rng.normal(0.0, 0.02, (256, 2048)).astype(np.float32)
    wsh = rng.normal(0.0, 0.02, 2048).astype(np.float32)
    h = rng.standard_normal((positions, 2048), dtype=np.float32)
    return Wr, wsh, h


def cmb_inputs(seed: int = CMB_SEED, positions: int = 5):
    rng = np.random.default_rng(seed)
    g = rng.uniform(0.0, 1.0, (positions, 8)).astype(np.float32)
    gates = (g / g.sum(axis=1, keepdims=True)).astype(np.float32)
    sg = rng.uniform(0.0, 1.0, positions).astype(np.float32)
    part = rng.standard_normal((positions, 8, 2048), dtype=np.float32).astype(np.float16)
    shared = rng.standard_normal((positions, 2048), dtype=np.float32)
    return gates, sg, part, shared
