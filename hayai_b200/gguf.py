"""GGUF tensor ingestion: real model files into the resident uploads.

The host side of the reference's GGUF catalog for the FFN path: the header and tensor
directory parser (crates/hayai-model/src/gguf.rs:24-121 ``parse_header_bytes``), tensor byte
sizes (gguf.rs:240-284 ``tensor_nbytes``), tensor byte ranges (gguf.rs:189-213) and
``load_quant_matrix`` (crates/hayai-model/src/gguf_stream.rs:298-309), which yields a
``QuantMatrix`` with ``ncols = dims[0]`` (contiguous) and ``nrows`` = the product of the other
dimensions.  The file is memory-mapped; a tensor's bytes are a zero-copy view until they are
uploaded (``upload`` / ``load_ffn_layer``).

Validation follows the reference: bad magic, a version outside 1..4, counts larger than the
file, more than 4 dimensions or a zero dimension, an unknown type id, an element count, byte
size, absolute offset or byte range that overflows u64, duplicate names, a non-power-of-two
``general.alignment``, and tensor ranges past the end of the file are errors (``GgufError``).
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass, field

import numpy as np

from .engine import QuantMatrix

GGUF_MAGIC = 0x46554747  # "GGUF", little endian

# bytes per block and elements per block of every GGML type with a defined size (gguf.rs:256-282)
_BLOCKS = {0: (1, 4), 1: (1, 2), 30: (1, 2), 28: (1, 8), 27: (1, 8), 24: (1, 1), 25: (1, 2), 26: (1, 4),
           2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 36), 20: (32, 18),
           10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292),
           16: (256, 66), 17: (256, 74), 22: (256, 82), 18: (256, 98), 21: (256, 110), 19: (256, 50),
           29: (256, 56), 23: (256, 136), 34: (256, 54), 35: (256, 66)}


class GgufError(ValueError):
    """A malformed or unsupported GGUF file (the reference's GgufError)."""


@dataclass
class TensorInfo:
    name: str
    dims: list[int]
    type_id: int
    offset: int  # relative to the data section

    @property
    def ncols(self) -> int:
        return self.dims[0] if self.dims else 1

    @property
    def nrows(self) -> int:
        n = 1
        for d in self.dims[1:]:
            n *= d
        return n

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n


U64_MAX = (1 << 64) - 1


def tensor_nbytes(info: TensorInfo) -> int:
    """Bytes of a tensor: whole blocks of its type (gguf.rs:240-284).  An element count or a
    byte size that does not fit in u64 is an error, as the reference's checked arithmetic
    makes it."""
    n = info.n_elements
    if n > U64_MAX:
        raise GgufError(f"tensor {info.name} element count overflow")
    if info.type_id not in _BLOCKS:
        raise GgufError(f"unsupported ggml type {info.type_id} for tensor {info.name}")
    qk, bs = _BLOCKS[info.type_id]
    nbytes = -(-n // qk) * bs
    if nbytes > U64_MAX:
        raise GgufError(f"tensor {info.name} byte size overflow")
    return nbytes


class _Reader:
    def __init__(self, data, pos: int = 0):
        self.data, self.pos = data, pos

    def need(self, n: int) -> None:
        if n < 0 or self.pos + n > len(self.data):
            raise GgufError("truncated GGUF header")

    def unpack(self, fmt: str):
        n = struct.calcsize(fmt)
        self.need(n)
        v = struct.unpack_from("<" + fmt, self.data, self.pos)[0]
        self.pos += n
        return v

    def string(self) -> str:
        n = self.unpack("Q")
        self.need(n)
        s = bytes(self.data[self.pos:self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    _SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}

    def value(self, ty: int, depth: int = 0):
        """One metadata value (gguf.rs:633-672)."""
        if depth > 32:
            raise GgufError("metadata array nesting too deep")
        if ty in self._SCALAR:
            return self.unpack(self._SCALAR[ty])
        if ty == 8:
            return self.string()
        if ty == 9:
            elem, n = self.unpack("I"), self.unpack("Q")
            if n > len(self.data) - self.pos:
                raise GgufError("truncated GGUF metadata array length")
            return [self.value(elem, depth + 1) for _ in range(n)]
        raise GgufError(f"unknown metadata type {ty}")


@dataclass
class GgufFile:
    """A memory-mapped GGUF file: metadata, tensor directory, tensor byte views."""

    path: str
    version: int
    alignment: int
    metadata: dict
    tensors: list[TensorInfo]
    data_offset: int
    _map: object = field(repr=False, default=None)
    _index: dict = field(repr=False, default_factory=dict)

    @classmethod
    def open(cls, path: str | os.PathLike) -> "GgufFile":
        with open(path, "rb") as f:
            size = os.fstat(f.fileno()).st_size
            if size < 24:
                raise GgufError("truncated GGUF header")
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            with memoryview(mm) as view:
                g = cls._parse(str(path), view)
        except BaseException:
            mm.close()
            raise
        g._map = mm
        return g

    @classmethod
    def _parse(cls, path: str, data) -> "GgufFile":
        r = _Reader(data)
        if r.unpack("I") != GGUF_MAGIC:
            raise GgufError("bad GGUF magic")
        version = r.unpack("I")
        if not 1 <= version <= 4:
            raise GgufError(f"unsupported GGUF version {version}")
        n_tensors, n_kv = r.unpack("Q"), r.unpack("Q")
        remaining = len(data) - r.pos
        if n_kv > remaining // 8 + 1:
            raise GgufError("metadata count exceeds file size")
        if n_tensors > remaining // 8 + 1:
            raise GgufError("tensor count exceeds file size")
        metadata = {}
        for _ in range(n_kv):
            key = r.string()
            metadata[key] = r.value(r.unpack("I"))
        tensors, index = [], {}
        for i in range(n_tensors):
            name = r.string()
            n_dims = r.unpack("I")
            if n_dims > 4:
                raise GgufError(f"tensor {name} has {n_dims} dims")
            dims = [r.unpack("Q") for _ in range(n_dims)]
            if any(d == 0 for d in dims):
                raise GgufError(f"tensor {name} has a zero dimension")
            info = TensorInfo(name, dims, r.unpack("I"), r.unpack("Q"))
            # sizes are validated while parsing, so no later computation can overflow (gguf.rs:85-87)
            tensor_nbytes(info)
            if name in index:
                raise GgufError(f"duplicate tensor name {name}")
            index[name] = i
            tensors.append(info)
        alignment = metadata.get("general.alignment", 32)
        if not isinstance(alignment, int) or alignment <= 0 or alignment & (alignment - 1):
            raise GgufError(f"invalid general.alignment {alignment} (must be a non-zero power of two)")
        data_offset = -(-r.pos // alignment) * alignment
        # no absolute offset or byte range may wrap u64 (gguf.rs:105-115)
        for t in tensors:
            start = data_offset + t.offset
            if start > U64_MAX:
                raise GgufError(f"tensor {t.name} absolute offset overflow")
            if start + tensor_nbytes(t) > U64_MAX:
                raise GgufError(f"tensor {t.name} byte range overflow")
        g = cls(path, version, alignment, metadata, tensors, data_offset)
        g._index = index
        return g

    # ------------------------------------------------------------------ tensors
    def tensor(self, name: str) -> TensorInfo:
        if name not in self._index:
            raise GgufError(f"missing tensor {name}")
        return self.tensors[self._index[name]]

    def has(self, name: str) -> bool:
        return name in self._index

    def tensor_range(self, info: TensorInfo) -> tuple[int, int]:
        """Absolute (start, nbytes) of a tensor inside the file (gguf.rs:198-213)."""
        start, n = self.data_offset + info.offset, tensor_nbytes(info)
        if start + n > len(self._map):
            raise GgufError(f"tensor {info.name} data out of bounds")
        return start, n

    def tensor_bytes(self, info: TensorInfo) -> np.ndarray:
        start, n = self.tensor_range(info)
        return np.frombuffer(self._map, dtype=np.uint8, count=n, offset=start)

    def load_quant_matrix(self, name: str) -> QuantMatrix:
        """gguf_stream.rs:298-309: the tensor as a GGUF-layout matrix (a copy of its bytes)."""
        info = self.tensor(name)
        return QuantMatrix(info.name, info.ncols, info.nrows, info.type_id, self.tensor_bytes(info).copy())

    def f32(self, name: str) -> np.ndarray:
        """An F32 tensor (norm weights) as a float32 array."""
        info = self.tensor(name)
        if info.type_id != 0:
            raise GgufError(f"tensor {name} is type {info.type_id}, not F32")
        return self.tensor_bytes(info).view(np.float32).copy()

    def upload(self, engine, name: str):
        """Resident upload of a quantized tensor straight from the mapped file."""
        info = self.tensor(name)
        return engine.upload(info.type_id, info.nrows, info.ncols, self.tensor_bytes(info))

    def load_ffn_layer(self, engine, layer: int):
        """The FFN of block `layer` (llama tensor names, as the reference's catalog looks them up,
        crates/hayai-core/src/stream_infer.rs): resident gate, up, down and the f32 ffn_norm."""
        p = f"blk.{layer}."
        g, u, d = (self.upload(engine, p + n) for n in ("ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"))
        norm = self.f32(p + "ffn_norm.weight") if self.has(p + "ffn_norm.weight") else None
        return g, u, d, norm

    def close(self) -> None:
        """Unmap the file.  While arrays returned by ``tensor_bytes`` are alive the mapping
        stays open (it is released when the last of them goes)."""
        if self._map is not None:
            try:
                self._map.close()
            except BufferError:
                pass
            self._map = None
