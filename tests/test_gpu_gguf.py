"""GGUF -> HBM tile layout through the streaming loader (pinned staging, device
repack, two chunks in flight) equals the host packer, and the GEMVs read it."""
import numpy as np
import pytest
import torch

import oracle
from gguf_fixture import TENSORS, write_gguf
from test_gpu_parity import check_vs_oracle, x_tensor
from thunderllamax_b200 import gguf_loader as gl
from thunderllamax_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    ops.require_device()


@pytest.mark.parametrize("chunk", [1 << 12, 64 << 20])   # many small chunks / one chunk
def test_tiled_load_equals_host_pack(tmp_path, chunk):
    path = tmp_path / "m.gguf"
    data = write_gguf(path, seed=4)
    with gl.GGUFWeights(path) as g:
        for name, qt, rows, k in TENSORS:
            if not isinstance(qt, str):
                t = g.tensor(name)
                assert t.is_cuda and np.array_equal(t.cpu().numpy(), data[name])
                continue
            dev = g.tiled(name, chunk_bytes=chunk)
            host = ops.pack_tiles_host(qt, data[name], k)
            assert np.array_equal(dev.cpu().numpy(), host), name


def test_gemv_on_loaded_weights(tmp_path):
    path = tmp_path / "m.gguf"
    data = write_gguf(path, seed=5)
    rng = np.random.default_rng(6)
    with gl.GGUFWeights(path) as g:
        for name, qt, rows, k in TENSORS:
            if not isinstance(qt, str) or qt == "iq4_xs":
                continue
            w = g.tiled(name, chunk_bytes=1 << 13)
            x, x64 = x_tensor(rng, 11, k, torch.bfloat16)
            y = ops.gemv(qt, w, x, rows, ops.Workspace.for_shape(ops.MODE_STORE, qt, rows, k, 11))
            torch.cuda.synchronize()
            check_vs_oracle(qt, y.cpu().numpy(), data[name], k, x64)
