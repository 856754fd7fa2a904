"""GGUF container reader and B200 weight loader.

``parse_gguf`` / ``tnbytes`` / ``read_raw`` keep the reference loader's interface
(engine/engine0.py:26-59: ``parse_gguf(path) -> (data_start, infos)`` with
``infos[name] = (ggml_type, dims, offset)``), and ``parse_gguf_kv`` its metadata
reader (engine/api_server.py:224).  Beyond the reference it honours
``general.alignment`` (the GGUF default of 32 otherwise) and reads the file
through one memory map.

``GGUFWeights.tiled(name)`` streams a quantised 2-D tensor into HBM in the B200
tile layout: row chunks are copied from the map into pinned staging buffers, sent
to the device on a side stream and repacked there by ``tlx_pack_tiles_device``,
two chunks in flight, so disk / PCIe and the repack overlap.  The HBM footprint
equals the GGUF bytes (plus zero rows up to a multiple of 16).
"""
from __future__ import annotations

import mmap
import struct

import numpy as np
import torch

from . import _lib, ops
from ._lib import TLXError

# ggml type id -> (weights per block, bytes per block) for block formats, and bytes
# per element for plain ones (the GGUF format's own tables; engine/engine0.py:20-22)
QUANT = {2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 10: (256, 84), 11: (256, 110),
         12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292), 16: (256, 66), 17: (256, 74),
         18: (256, 98), 19: (256, 50), 20: (32, 18), 21: (256, 110), 22: (256, 82), 23: (256, 136),
         29: (256, 56), 39: (32, 17), 41: (128, 18)}
NATIVE = {0: 4, 1: 2, 24: 1, 25: 2, 26: 4, 27: 8, 28: 8, 30: 2}

# GGUF metadata value types: id -> (size, struct format); 8 = string, 9 = array
_VALUE = {0: (1, "B"), 1: (1, "b"), 2: (2, "H"), 3: (2, "h"), 4: (4, "I"), 5: (4, "i"), 6: (4, "f"), 7: (1, "?"),
          10: (8, "Q"), 11: (8, "q"), 12: (8, "d")}

# ggml type ids the tile GEMVs read
TILED_TYPES = {14: "q6_k", 18: "iq3_xxs", 12: "q4_k", 13: "q5_k", 8: "q8_0", 23: "iq4_xs"}


class _Cursor:
    def __init__(self, buf, pos=0):
        self.buf, self.pos = buf, pos

    def take(self, n):
        if self.pos + n > len(self.buf):
            raise TLXError("GGUF: truncated file")
        b = bytes(self.buf[self.pos:self.pos + n])
        self.pos += n
        return b

    def unpack(self, fmt):
        n = struct.calcsize(fmt)
        return struct.unpack("<" + fmt, self.take(n))[0]

    def string(self):
        return self.take(self.unpack("Q")).decode("utf-8")

    def value(self, t):
        if t == 8:
            return self.string()
        if t == 9:
            et, n = self.unpack("I"), self.unpack("Q")
            return [self.value(et) for _ in range(n)]
        if t not in _VALUE:
            raise TLXError(f"GGUF: unknown metadata type {t}")
        return self.unpack(_VALUE[t][1])


def _parse(buf):
    c = _Cursor(buf)
    if c.take(4) != b"GGUF":
        raise TLXError("not a GGUF file")
    version = c.unpack("I")
    if version < 2:
        raise TLXError(f"GGUF version {version} is not supported (v2 / v3 are)")
    n_tensors, n_kv = c.unpack("Q"), c.unpack("Q")
    kv = {}
    for _ in range(n_kv):
        key = c.string()
        kv[key] = c.value(c.unpack("I"))
    infos = {}
    for _ in range(n_tensors):
        name = c.string()
        nd = c.unpack("I")
        dims = [c.unpack("Q") for _ in range(nd)]
        t = c.unpack("I")
        off = c.unpack("Q")
        infos[name] = (t, dims, off)
    align = int(kv.get("general.alignment", 32))
    data_start = (c.pos + align - 1) // align * align
    return version, kv, infos, data_start


def _parse_file(path):
    with open(path, "rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as m:
        mv = memoryview(m)
        try:
            return _parse(mv)
        finally:
            mv.release()


def parse_gguf(path):
    """(data_start, {name: (ggml_type, dims, offset)}), dims innermost first."""
    _, _, infos, data_start = _parse_file(path)
    return data_start, infos


def parse_gguf_kv(path):
    """The metadata key/value pairs (arrays as lists)."""
    return _parse_file(path)[1]


def tnbytes(ne: int, t: int) -> int:
    """Bytes of ne elements of ggml type t."""
    if t in NATIVE:
        return NATIVE[t] * ne
    if t not in QUANT:
        raise TLXError(f"unknown ggml type {t}")
    a, b = QUANT[t]
    if ne % a:
        raise TLXError(f"{ne} elements is not a whole number of type-{t} blocks")
    return (ne // a) * b


def read_raw(path, info, data_start) -> np.ndarray:
    """The tensor's bytes (a read-only view of a memory map)."""
    t, dims, off = info
    ne = int(np.prod(dims)) if dims else 1
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    return mm[data_start + off:data_start + off + tnbytes(ne, t)]


class GGUFWeights:
    """One GGUF file, memory-mapped, with device loaders."""

    def __init__(self, path, device="cuda"):
        self.path, self.device = path, device
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        mv = memoryview(self._mm)
        try:
            self.version, self.kv, self.infos, self.data_start = _parse(mv)
        finally:
            mv.release()
        self._np = np.frombuffer(self._mm, dtype=np.uint8)

    def close(self):
        self._np = None
        try:
            self._mm.close()
        except BufferError:
            pass   # a raw() view is still alive; the map closes when it is collected
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def raw(self, name) -> np.ndarray:
        t, dims, off = self.infos[name]
        ne = int(np.prod(dims)) if dims else 1
        return self._np[self.data_start + off:self.data_start + off + tnbytes(ne, t)]

    def shape(self, name):
        """(rows, k) of a 2-D tensor: GGUF dims are innermost first."""
        t, dims, _ = self.infos[name]
        if len(dims) != 2:
            raise TLXError(f"{name}: {len(dims)}-D, a weight matrix is 2-D")
        return int(dims[1]), int(dims[0])

    def qtype(self, name) -> str:
        t = self.infos[name][0]
        if t not in TILED_TYPES:
            raise TLXError(f"{name}: ggml type {t} has no tile layout")
        return TILED_TYPES[t]

    def tensor(self, name) -> torch.Tensor:
        """A plain (f32 / f16 / bf16 / int) tensor on the device, GGUF dims reversed
        (row-major, the reference's reshape(*reversed(dims)))."""
        t, dims, _ = self.infos[name]
        dt = {0: torch.float32, 1: torch.float16, 30: torch.bfloat16, 24: torch.int8, 25: torch.int16,
              26: torch.int32, 27: torch.int64, 28: torch.float64}.get(t)
        if dt is None:
            raise TLXError(f"{name}: ggml type {t} is a block format (use tiled())")
        host = torch.from_numpy(self.raw(name).copy()).view(dt).reshape(*reversed([int(d) for d in dims]))
        return host.to(self.device)

    def tiled(self, name, chunk_bytes: int = 64 << 20) -> torch.Tensor:
        """The 2-D quantised tensor repacked into the tile layout in HBM."""
        qt = self.qtype(name)
        rows, k = self.shape(name)
        q = _lib.QTYPES[qt]
        if k % 256:
            raise TLXError(f"{name}: k = {k} is not a multiple of 256")
        row_bytes = tnbytes(k, self.infos[name][0])
        src = self.raw(name)
        out = torch.empty(ops.tiled_bytes(qt, rows, k), dtype=torch.uint8, device=self.device)
        per_tile = ops.tiled_bytes(qt, 16, k)
        step = max(16, (chunk_bytes // row_bytes) // 16 * 16)
        stream = torch.cuda.Stream(device=self.device)
        pinned = [torch.empty(step * row_bytes, dtype=torch.uint8).pin_memory() for _ in range(2)]
        staging = [torch.empty(step * row_bytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        done = [None, None]
        lib = _lib.lib()
        with torch.cuda.stream(stream):
            for i, r0 in enumerate(range(0, rows, step)):
                n = min(step, rows - r0)
                b = i & 1
                if done[b] is not None:
                    done[b].synchronize()          # the pinned / staging pair is free again
                pinned[b][:n * row_bytes].numpy()[:] = src[r0 * row_bytes:(r0 + n) * row_bytes]
                staging[b][:n * row_bytes].copy_(pinned[b][:n * row_bytes], non_blocking=True)
                dst = out[(r0 // 16) * per_tile:]
                rc = lib.tlx_pack_tiles_device(q, staging[b].data_ptr(), n, k, row_bytes, dst.data_ptr(),
                                               ctypes_stream(stream))
                _lib.check(rc, "pack_tiles_device")
                ev = torch.cuda.Event()
                ev.record(stream)
                done[b] = ev
        stream.synchronize()
        return out


def ctypes_stream(stream: torch.cuda.Stream):
    import ctypes
    return ctypes.c_void_p(stream.cuda_stream)


__all__ = ["parse_gguf", "parse_gguf_kv", "tnbytes", "read_raw", "GGUFWeights", "QUANT", "NATIVE", "TILED_TYPES"]
