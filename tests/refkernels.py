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
