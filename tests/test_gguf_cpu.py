"""GGUF container reader (thunderllamax_b200.gguf_loader) against files written and
read by gguf-py, the upstream llama.cpp Python package."""
import numpy as np
import pytest

from gguf_fixture import TENSORS, write_gguf
from thunderllamax_b200 import gguf_loader as gl
from thunderllamax_b200._lib import TLXError


@pytest.mark.parametrize("alignment", [None, 64, 256])
def test_parse_matches_gguf_py(tmp_path, alignment):
    import gguf
    path = tmp_path / "m.gguf"
    data = write_gguf(path, seed=1, alignment=alignment)
    ds, infos = gl.parse_gguf(path)
    r = gguf.GGUFReader(str(path))
    assert r.alignment == (alignment or 32)
    assert set(infos) == {t.name for t in r.tensors}
    for t in r.tensors:
        typ, dims, off = infos[t.name]
        assert typ == int(t.tensor_type)
        assert dims == [int(d) for d in t.shape]
        assert ds + off == int(t.data_offset)
        raw = gl.read_raw(path, infos[t.name], ds)
        assert raw.size == int(t.n_bytes) == gl.tnbytes(int(np.prod(dims)), typ)
        assert np.array_equal(np.asarray(raw), np.ascontiguousarray(data[t.name]).view(np.uint8).reshape(-1))
    kv = gl.parse_gguf_kv(path)
    assert kv["test.u32"] == 7 and kv["test.i32"] == -5 and kv["test.f32"] == 1.5 and kv["test.bool"] is True
    assert kv["test.str"] == "héllo" and kv["test.arr_i"] == [1, 2, 3] and kv["test.arr_s"] == ["a", "bc"]
    assert kv["test.u64"] == 1 << 40 and kv["general.architecture"] == "qwen35"


def test_weights_view_shapes_and_types(tmp_path):
    path = tmp_path / "m.gguf"
    data = write_gguf(path, seed=2)
    with gl.GGUFWeights(path, device="cpu") as g:
        for name, qt, rows, k in TENSORS:
            if isinstance(qt, str):
                assert g.shape(name) == (rows, k)
                assert g.qtype(name) == qt
                assert np.array_equal(np.asarray(g.raw(name)).reshape(rows, -1), data[name])
            else:
                t = g.tensor(name)
                assert tuple(t.shape) == data[name].shape
                assert np.array_equal(t.numpy(), data[name])
        with pytest.raises(TLXError):
            g.qtype("blk.0.attn_norm.weight")
        with pytest.raises(TLXError):
            g.tensor("blk.0.ffn_down.weight")


def test_rejects_bad_files(tmp_path):
    path = tmp_path / "m.gguf"
    write_gguf(path, seed=3)
    blob = path.read_bytes()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + blob[4:])
    with pytest.raises(TLXError):
        gl.parse_gguf(bad)
    bad.write_bytes(blob[:200])              # cut inside the metadata
    with pytest.raises(TLXError):
        gl.parse_gguf(bad)
    with pytest.raises(TLXError):
        gl.tnbytes(100, 14)                  # not whole Q6_K blocks
    assert gl.tnbytes(512, 8) == 16 * 34 and gl.tnbytes(10, 0) == 40
