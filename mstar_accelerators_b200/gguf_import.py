"""GGUF Q8_0 / Q4_0 tensor import: ggml-quantized checkpoints load straight into
the B200 block-quantized linears.

A GGUF file (the format of the reference's vendored ggml reader,
backends/pi/third_party/ggml/src/gguf.cpp:470-800, types in include/gguf.h:46-67)
is a header, key/value metadata, tensor infos, then the data section aligned to
``general.alignment`` (default 32). A Q8_0 or Q4_0 tensor's data is the ggml
block bytes themselves (34-byte {fp16 d; int8 qs[32]} / 18-byte {fp16 d;
uint8 qs[16]} blocks, ggml-common.h:194-199, 251-256), row after row, so the
import is a checked view of those bytes: they are exactly what the packers
(``mstar_b200_pack``) produce for the same weights, and they go to the device
unchanged as a ``BlockLinear``'s canonical blocks. F32 / F16 tensors are packed
on the device like any logical weight.

Checks, as ggml's reader makes them: magic ``GGUF``, version 2 or 3, a
power-of-two alignment, at most 4 dimensions, every tensor's data aligned and
inside the file, contiguous in order; unsupported ggml types raise.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

GGUF_MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32
# ggml tensor types this importer accepts: id -> (name, block elements, block bytes)
GGML_TYPES = {0: ("f32", 1, 4), 1: ("f16", 1, 2), 2: ("q4_0", 32, 18), 8: ("q8_0", 32, 34)}
# GGUF metadata value types (gguf.h:53-67): id -> struct format (None: string / array)
_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


class GGUFError(ValueError):
    pass


@dataclass(frozen=True)
class GGUFTensor:
    name: str
    shape: tuple[int, ...]   # logical, outermost first ([rows, width] for a matrix)
    ggml_type: int
    offset: int              # absolute file offset of the data
    nbytes: int

    @property
    def format(self) -> str:
        return GGML_TYPES[self.ggml_type][0]


class _Cursor:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt):
        size = struct.calcsize(fmt)
        if self.pos + size > len(self.buf):
            raise GGUFError("truncated GGUF header")
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += size
        return v

    def string(self):
        n = self.take("<Q")
        if self.pos + n > len(self.buf):
            raise GGUFError("truncated GGUF string")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8")
        self.pos += n
        return s

    def value(self, vtype):
        if vtype in _SCALARS:
            return self.take(_SCALARS[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, n = self.take("<I"), self.take("<Q")
            return [self.value(etype) for _ in range(n)]
        raise GGUFError(f"unknown GGUF value type {vtype}")


class GGUFFile:
    """A GGUF file mapped read-only; tensors are views of the mapping."""

    def __init__(self, path):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            self._map = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        c = _Cursor(self._map)
        if bytes(self._map[:4]) != GGUF_MAGIC:
            raise GGUFError("not a GGUF file")
        c.pos = 4
        self.version = c.take("<I")
        if self.version not in (2, 3):
            raise GGUFError(f"unsupported GGUF version {self.version}")
        n_tensors, n_kv = c.take("<Q"), c.take("<Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = c.string()
            self.metadata[key] = c.value(c.take("<I"))
        align = self.metadata.get("general.alignment", DEFAULT_ALIGNMENT)
        if not isinstance(align, int) or align <= 0 or align & (align - 1):
            raise GGUFError("alignment is not a power of 2")
        infos = []
        for _ in range(n_tensors):
            name = c.string()
            n_dims = c.take("<I")
            if n_dims > 4:
                raise GGUFError(f"tensor {name}: {n_dims} dimensions")
            ne = [c.take("<Q") for _ in range(n_dims)]
            gtype, offset = c.take("<I"), c.take("<Q")
            infos.append((name, ne, gtype, offset))
        data = -(-c.pos // align) * align
        self.data_offset = data
        self.tensors: dict[str, GGUFTensor] = {}
        expected = 0
        for name, ne, gtype, offset in infos:
            if gtype not in GGML_TYPES:
                raise GGUFError(f"tensor {name}: ggml type {gtype} is not imported (F32, F16, Q8_0, Q4_0)")
            _, per_block, block_bytes = GGML_TYPES[gtype]
            if ne and ne[0] % per_block:
                raise GGUFError(f"tensor {name}: row of {ne[0]} is not whole {per_block}-element blocks")
            nbytes = int(np.prod(ne, dtype=np.int64)) // per_block * block_bytes if ne else block_bytes
            if offset % align or offset != expected:
                raise GGUFError(f"tensor {name}: data offset {offset}, expected {expected}")
            expected += -(-nbytes // align) * align
            if data + offset + nbytes > len(self._map):
                raise GGUFError(f"tensor {name}: data runs past the end of the file")
            self.tensors[name] = GGUFTensor(name, tuple(int(n) for n in reversed(ne)), gtype, data + offset, nbytes)

    def raw(self, name: str) -> np.ndarray:
        """A copy of the tensor's bytes as uint8 [rows, bytes per row] (rows = 1 for a vector)."""
        t = self.tensors[name]
        arr = np.frombuffer(self._map, dtype=np.uint8, count=t.nbytes, offset=t.offset)
        rows = int(np.prod(t.shape[:-1], dtype=np.int64)) if len(t.shape) > 1 else 1
        out = arr.reshape(rows, -1).copy()
        del arr   # no view of the mapping outlives this call, so close() always succeeds
        return out

    def close(self):
        self._map.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def load_linear(gf: GGUFFile, name: str, *, bias=None, device="cuda", fmt: str = "q8_0"):
    """A BlockLinear from GGUF tensor ``name`` ([rows, width] logical). Q8_0 / Q4_0 data is
    used as the canonical blocks byte for byte; F32 / F16 weights are packed as ``fmt``."""
    import torch

    from .linear import BlockLinear
    t = gf.tensors[name]
    if len(t.shape) != 2:
        raise GGUFError(f"tensor {name}: a linear weight has 2 dimensions, not {len(t.shape)}")
    rows, width = t.shape
    raw = torch.from_numpy(gf.raw(name))
    if t.format in ("q8_0", "q4_0"):
        return BlockLinear(blocks=raw.to(device), fmt=t.format, rows=rows, width=width, bias=bias)
    dtype = torch.float32 if t.format == "f32" else torch.float16
    weight = raw.view(dtype).reshape(rows, width).to(device=device, dtype=torch.float32)
    return BlockLinear(weight, fmt=fmt, bias=bias)
