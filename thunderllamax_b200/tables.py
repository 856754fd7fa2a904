"""ggml lookup tables for the device, read at run time from gguf-py.

The reference passes the IQ3_XXS grid to its kernels as a device buffer
(``gridf``, engine/engine0.py:108-112, taken from tinygrad's ggml_common); the
same table comes here from gguf-py (``gguf.quants.IQ3_XXS``), the upstream
llama.cpp Python port present in this image, and is never copied into source.
"""
from __future__ import annotations

import functools

import numpy as np


@functools.lru_cache(maxsize=None)
def iq3xxs_grid_u32() -> np.ndarray:
    from gguf import quants

    if quants.IQ3_XXS.grid is None:
        quants.IQ3_XXS.init_grid()
    g = np.asarray(quants.IQ3_XXS.grid, dtype=np.float32).reshape(256, 4).astype(np.uint8)
    return np.ascontiguousarray(g).view(np.uint32).reshape(256).copy()


LEVEL_STEP = 4.0507  # W4A8 tier: grid magnitude ~= step * level (engine/p8_w4ffn7.cu:42)


@functools.lru_cache(maxsize=None)
def iq3xxs_levels_lut8() -> np.ndarray:
    """int8[1024]: the W4A8 tier's linearised IQ3_XXS codebook, level
    clip(rint(g / 4.0507), 0, 15) of grid entry i, magnitude j at [4 i + j]
    (built by the reference at engine/pf_prefill.py:994)."""
    g = iq3xxs_grid_u32().view(np.uint8).astype(np.float32)
    return np.clip(np.rint(g / np.float32(LEVEL_STEP)), 0, 15).astype(np.int8)


@functools.lru_cache(maxsize=None)
def iq4nl_kvalues() -> np.ndarray:
    from gguf import quants

    return np.asarray(quants.IQ4_NL.kvalues, dtype=np.int8)
