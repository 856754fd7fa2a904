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


@functools.lru_cache(maxsize=None)
def iq4nl_kvalues() -> np.ndarray:
    from gguf import quants

    return np.asarray(quants.IQ4_NL.kvalues, dtype=np.int8)
