"""Launch reference kernels compiled by oracle/build_ref.py (oracle/_ref/*.cubin)
next to the library's, on the same device buffers (test infrastructure)."""
from __future__ import annotations

import ctypes
import os

import pytest

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
_modules = {}


def cubin_path(name: str) -> str:
    return os.path.join(REF_DIR, name + ".cubin")


def have(name: str) -> bool:
    return os.path.exists(cubin_path(name))


def require(name: str) -> None:
    if not have(name):
        pytest.skip(f"oracle/_ref/{name}.cubin not built (python oracle/build_ref.py with the reference tree)")


def launch(name: str, grid: int, block: int, args, stream=None) -> None:
    """args: device pointers (torch tensors) or Python ints passed as int32."""
    import torch
    from cuda.bindings import driver

    torch.cuda.init()
    torch.cuda.synchronize()
    if name not in _modules:
        err, mod = driver.cuModuleLoad(cubin_path(name).encode())
        assert err == driver.CUresult.CUDA_SUCCESS, err
        err, fn = driver.cuModuleGetFunction(mod, name.encode())
        assert err == driver.CUresult.CUDA_SUCCESS, err
        _modules[name] = (mod, fn)
    fn = _modules[name][1]
    vals, types = [], []
    for a in args:
        if isinstance(a, torch.Tensor):
            vals.append(a.data_ptr())
            types.append(ctypes.c_void_p)
        else:
            vals.append(int(a))
            types.append(ctypes.c_int)
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    err, = driver.cuLaunchKernel(fn, grid, 1, 1, block, 1, 1, 0, s, (tuple(vals), tuple(types)), 0)
    assert err == driver.CUresult.CUDA_SUCCESS, err
    torch.cuda.synchronize()


def packed7_planes(raw, k: int):
    """GGUF IQ3_XXS rows -> the packed7 units the reference's p8w4ffn7 reads
    (layout of engine/pack_w7.py:1-20; pinned by tests/test_oracle_w4a8.py against
    the reference's pack_tensor).  uint16 [n / 8][k / 128][32][8]: unit r * 4 + c of
    chunk 2b + h (256-k block b, half h) holds, for row r of the 8-row group, the
    four qs words 16h + 4c .. 16h + 4c + 3 of block b, then scale word 4h + c as two
    halves, then d of block b, then zero."""
    import numpy as np

    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    n, nb = raw.shape[0], k // 256
    assert n % 8 == 0
    blk = raw.reshape(n // 8, 8, nb, 98)                               # [group, r, b, byte]
    qs = np.ascontiguousarray(blk[..., 2:66]).view(np.uint16)          # [g, r, b, 32]
    sc = np.ascontiguousarray(blk[..., 66:98]).view(np.uint32)         # [g, r, b, 8]
    d = np.ascontiguousarray(blk[..., 0:2]).view(np.uint16)[..., 0]    # [g, r, b]
    out = np.zeros((n // 8, nb, 2, 8, 4, 8), dtype=np.uint16)          # [g, b, h, r, c, slot]
    out[..., 0:4] = qs.reshape(n // 8, 8, nb, 2, 4, 4).transpose(0, 2, 3, 1, 4, 5)
    w = sc.reshape(n // 8, 8, nb, 2, 4).transpose(0, 2, 3, 1, 4)
    out[..., 4] = (w & 0xFFFF).astype(np.uint16)
    out[..., 5] = (w >> 16).astype(np.uint16)
    out[..., 6] = d.transpose(0, 2, 1)[:, :, None, :, None]
    return out.reshape(n // 8, 2 * nb, 32, 8)
