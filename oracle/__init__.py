"""CPU oracle for the speculative-verify path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy, the reference's arithmetic for the
verify step (ggml block dequantisation, K-row matvec, SiLU-gated FFN, LM head
with per-row argmax, greedy draft acceptance, MoE router/experts/combine).
Every function cites the reference file:line it follows.

It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it.  The CUDA library in ``thunderllamax_b200`` never calls into it
and fails loudly when its extension is missing.

Parity is pinned: ``tests/test_oracle_golden.py`` checks these restatements
against golden vectors produced by the reference's own numpy ports
(``engine/mm/MM_P2_ports.py``, ``engine/mm/MM_P0_d2_repack.py``,
``engine/pack_w4.py``) with the ggml tables injected from gguf-py
(``tests/golden/gen_golden.py`` made them).
"""
from .tables import iq3xxs_grid_u32, iq3xxs_grid_bytes, ksigns_iq2xs, iq4nl_kvalues  # noqa: F401
from .dequant import (  # noqa: F401
    dequant_iq3xxs, dequant_q6k, dequant_iq4xs, dequant_q4k, dequant_q5k, dequant_q8_0, dequant,
)
from .path import (  # noqa: F401
    matvec_f64, ffn_f64, head_logits_f64, argmax_rows, h_argmax, acceptsel11k, lookup_ngram, head_argmax, accept, accept11k,
    router_top8, moe_verify_f64, silu_f64, min_top2_gap,
)
from .attention import attn_pre, attn_decode, rope_freqs, dequant_cache  # noqa: F401,E402
from .w4a8 import act_quant_q8, dequant_iq3xxs_lin, dequant_tokens, lut8_levels, w4a8_gate_up_f64  # noqa: F401,E402
