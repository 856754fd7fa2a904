"""Seeded synthetic inputs for the verify path (host side, numpy).

The reference is measured on a real 27B GGUF that is not available here, so
every benchmark and parity case runs on seeded synthetic data with the
shapes, byte layouts and value distributions of the benchmark configurations:

* IQ3_XXS blocks (98 B / 256 weights, ggml ``block_iq3_xxs``): fp16 ``d`` drawn
  U(1e-3, 1e-2); 64 grid-index bytes uniform over 0..255 (every byte is a
  valid index into the 256-entry grid); 8 scale/sign u32 words uniform over
  2^32 (4 x 7-bit sign fields + a 4-bit sub-scale).  Block layout as read by
  reference engine/pack_w1c.py:20-31 (GGUF order: d, qs[64], scales[32]).
* Q6_K blocks (210 B / 256 weights, ggml ``block_q6_K``): ql[128] and qh[64]
  bytes uniform (uniform 6-bit quants), sc[16] int8 U[-32, 31], fp16 ``d``
  U(1e-4, 1e-3).  Layout per reference engine/mm/MM_P2_ports.py:21-27.
* IQ4_XS blocks (136 B / 256 weights, ggml ``block_iq4_xs``): fp16 ``d``
  U(1e-3, 1e-2), scales_h u16 and scales_l bytes uniform, qs nibbles uniform.
  Layout per reference engine/mm/MM_P0_d2_repack.py:78-84.
* Activations: bf16 N(0, 1), stored as uint16 bit patterns (numpy has no
  bfloat16) and converted with round-to-nearest-even.
"""
from __future__ import annotations

import numpy as np

QK = 256
# bytes per 256 weights of a row (q8_0: eight 34-byte GGUF blocks)
BLOCK_BYTES = {"iq3_xxs": 98, "q6_k": 210, "iq4_xs": 136, "q4_k": 144, "q5_k": 176, "q8_0": 272}
GGML_TYPE = {"iq3_xxs": 18, "q6_k": 14, "iq4_xs": 23, "q4_k": 12, "q5_k": 13, "q8_0": 8}


def row_bytes(qtype: str, k: int) -> int:
    if k % QK:
        raise ValueError(f"k={k} is not a multiple of {QK}")
    return (k // QK) * BLOCK_BYTES[qtype]


def _f16_bytes(vals: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(vals.astype(np.float16)).view(np.uint8).reshape(vals.shape + (2,))


def iq3xxs_blocks(rng: np.random.Generator, n_rows: int, k: int) -> np.ndarray:
    nb = k // QK
    blk = np.empty((n_rows, nb, 98), dtype=np.uint8)
    blk[..., 0:2] = _f16_bytes(rng.uniform(1e-3, 1e-2, (n_rows, nb)))
    blk[..., 2:66] = rng.integers(0, 256, (n_rows, nb, 64), dtype=np.uint8)
    words = rng.integers(0, 1 << 32, (n_rows, nb, 8), dtype=np.uint64).astype(np.uint32)
    blk[..., 66:98] = np.ascontiguousarray(words).view(np.uint8).reshape(n_rows, nb, 32)
    return blk.reshape(n_rows, nb * 98)


def q6k_blocks(rng: np.random.Generator, n_rows: int, k: int) -> np.ndarray:
    nb = k // QK
    blk = np.empty((n_rows, nb, 210), dtype=np.uint8)
    blk[..., 0:192] = rng.integers(0, 256, (n_rows, nb, 192), dtype=np.uint8)
    blk[..., 192:208] = rng.integers(-32, 32, (n_rows, nb, 16)).astype(np.int8).view(np.uint8)
    blk[..., 208:210] = _f16_bytes(rng.uniform(1e-4, 1e-3, (n_rows, nb)))
    return blk.reshape(n_rows, nb * 210)


def iq4xs_blocks(rng: np.random.Generator, n_rows: int, k: int) -> np.ndarray:
    nb = k // QK
    blk = np.empty((n_rows, nb, 136), dtype=np.uint8)
    blk[..., 0:2] = _f16_bytes(rng.uniform(1e-3, 1e-2, (n_rows, nb)))
    blk[..., 2:136] = rng.integers(0, 256, (n_rows, nb, 134), dtype=np.uint8)
    return blk.reshape(n_rows, nb * 136)


def q4k_blocks(rng: np.random.Generator, n_rows: int, k: int) -> np.ndarray:
    """Q4_K blocks (d f16 | dmin f16 | scales[12] | qs[128]): random 6-bit scales and
    mins, d and dmin of the magnitude a trained checkpoint's v projection has."""
    nb = k // QK
    blk = np.empty((n_rows, nb, 144), dtype=np.uint8)
    blk[..., 0:2] = _f16_bytes(rng.uniform(1e-4, 1e-3, (n_rows, nb)))
    blk[..., 2:4] = _f16_bytes(rng.uniform(1e-4, 1e-3, (n_rows, nb)))
    blk[..., 4:144] = rng.integers(0, 256, (n_rows, nb, 140), dtype=np.uint8)
    return blk.reshape(n_rows, nb * 144)


def q5k_blocks(rng: np.random.Generator, n_rows: int, k: int) -> np.ndarray:
    """Q5_K blocks (d f16 | dmin f16 | scales[12] | qh[32] | qs[128]): random 6-bit
    scales and mins, uniform 5-bit quants, d and dmin as for Q4_K."""
    nb = k // QK
    blk = np.empty((n_rows, nb, 176), dtype=np.uint8)
    blk[..., 0:2] = _f16_bytes(rng.uniform(1e-4, 1e-3, (n_rows, nb)))
    blk[..., 2:4] = _f16_bytes(rng.uniform(1e-4, 1e-3, (n_rows, nb)))
    blk[..., 4:176] = rng.integers(0, 256, (n_rows, nb, 172), dtype=np.uint8)
    return blk.reshape(n_rows, nb * 176)


def q8_0_blocks(rng: np.random.Generator, n_rows: int, k: int) -> np.ndarray:
    """Q8_0 blocks (d f16 | qs[32] int8) for k weights per row: d of the magnitude
    an o-projection's 32-weight blocks have (max |w| / 127 for w ~ N(0, 0.02)),
    quants over the full int8 range (-128 included)."""
    nb = k // 32
    blk = np.empty((n_rows, nb, 34), dtype=np.uint8)
    blk[..., 0:2] = _f16_bytes(rng.uniform(2e-4, 8e-4, (n_rows, nb)))
    blk[..., 2:34] = rng.integers(0, 256, (n_rows, nb, 32), dtype=np.uint8)
    return blk.reshape(n_rows, nb * 34)


BLOCK_GEN = {"iq3_xxs": iq3xxs_blocks, "q6_k": q6k_blocks, "iq4_xs": iq4xs_blocks, "q4_k": q4k_blocks,
             "q5_k": q5k_blocks, "q8_0": q8_0_blocks}


# Seeded matrices are drawn in row chunks of this many rows, each chunk from its own
# generator (seed, chunk index): any row range of a model can be generated alone
# (a rank's vocabulary shard, a sampled test row) and equals those rows of the whole.
CHUNK_ROWS = 8192


def chunk_rng(seed: int, chunk: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence([int(seed), int(chunk)]))


def matrix_rows(qtype: str, n_rows: int, k: int, seed: int, r0: int = 0, r1: int | None = None) -> np.ndarray:
    """Rows [r0, r1) of the seeded synthetic (n_rows x k) GGUF matrix of `qtype`."""
    r1 = n_rows if r1 is None else r1
    if not 0 <= r0 <= r1 <= n_rows:
        raise ValueError(f"rows [{r0}, {r1}) outside [0, {n_rows})")
    out = np.empty((r1 - r0, row_bytes(qtype, k)), dtype=np.uint8)
    if r1 == r0:
        return out
    for c in range(r0 // CHUNK_ROWS, (r1 - 1) // CHUNK_ROWS + 1):
        c0, c1 = c * CHUNK_ROWS, min((c + 1) * CHUNK_ROWS, n_rows)
        raw = BLOCK_GEN[qtype](chunk_rng(seed, c), c1 - c0, k)
        a, b = max(c0, r0), min(c1, r1)
        out[a - r0:b - r0] = raw[a - c0:b - c0]
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_normal(rng: np.random.Generator, shape) -> np.ndarray:
    """bf16 N(0, 1) activations as uint16 bit patterns."""
    return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))


def drafts_for(amds: np.ndarray, n_drafts: int, vocab: int, rng: np.random.Generator):
    """Draft ids per the head+accept configuration: j ~ U{0..n_drafts}; the
    first j drafts equal the true argmax of their row, later ones are uniform
    random ids.  Returns (drafts int32[n_drafts], j)."""
    j = int(rng.integers(0, n_drafts + 1))
    drafts = rng.integers(0, vocab, n_drafts).astype(np.int32)
    drafts[:j] = amds[:j]
    return drafts, j
