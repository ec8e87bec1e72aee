"""GGUF format facts used on the quantized-matmul path.

Mirrors ``GgufDtype`` (rce-ingest-gguf/src/parser.rs:228, tags :308-338),
``tensor_byte_size`` (rce-ingest-gguf/src/dequant.rs:18-58) and the block
geometry of ``quant_info`` (rce-ingest-gguf/src/quant.rs:22-217) for the five
formats this library implements (Q8_0, Q4_0, Q4_K, Q5_K, Q6_K), and the GGUF
file reader (``GgufFile``, after ``GgufFile::parse``, parser.rs:446).
"""
from __future__ import annotations

from enum import IntEnum


class GgufDtype(IntEnum):
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2K = 10
    Q3K = 11
    Q4K = 12
    Q5K = 13
    Q6K = 14
    BF16 = 30

    # the reference spells it Q4K; keep the common alias too
    @classmethod
    def parse(cls, v) -> "GgufDtype":
        if isinstance(v, str):
            s = v.upper().replace("_K", "K")
            return cls[s]
        return cls(int(v))


Q4_K = GgufDtype.Q4K

#: values per block and bytes per block (tensor_byte_size, dequant.rs:18-58:
#: every format a GGUF file may hold beside the five this library computes
#: with, so that any tensor's byte range can be located)
BLOCK = {GgufDtype.Q4_0: 32, GgufDtype.Q8_0: 32, GgufDtype.Q4K: 256, GgufDtype.F32: 1, GgufDtype.F16: 1,
         GgufDtype.BF16: 1, GgufDtype.Q4_1: 32, GgufDtype.Q5_0: 32, GgufDtype.Q5_1: 32, GgufDtype.Q8_1: 32,
         GgufDtype.Q2K: 256, GgufDtype.Q3K: 256, GgufDtype.Q5K: 256, GgufDtype.Q6K: 256}
BLOCK_BYTES = {GgufDtype.Q4_0: 18, GgufDtype.Q8_0: 34, GgufDtype.Q4K: 144, GgufDtype.F32: 4, GgufDtype.F16: 2,
               GgufDtype.BF16: 2, GgufDtype.Q4_1: 20, GgufDtype.Q5_0: 22, GgufDtype.Q5_1: 24, GgufDtype.Q8_1: 36,
               GgufDtype.Q2K: 84, GgufDtype.Q3K: 110, GgufDtype.Q5K: 176, GgufDtype.Q6K: 210}

SUPPORTED = (GgufDtype.Q4_0, GgufDtype.Q8_0, GgufDtype.Q4K, GgufDtype.Q5K, GgufDtype.Q6K)


def tensor_byte_size(dtype, numel: int) -> int:
    """Bytes of a tensor of ``numel`` values (ceil-divided into blocks)."""
    dt = GgufDtype.parse(dtype)
    blk = BLOCK[dt]
    return (numel + blk - 1) // blk * BLOCK_BYTES[dt]


def row_bytes(dtype, n_cols: int) -> int:
    dt = GgufDtype.parse(dtype)
    return n_cols // BLOCK[dt] * BLOCK_BYTES[dt]


# ---- GGUF file reader (GgufFile::parse, rce-ingest-gguf/src/parser.rs:446-553) ------------
#
# Layout (GGUF v2/v3, little endian): magic "GGUF", u32 version, u64 tensor
# count, u64 metadata count; metadata entries (string key, u32 type tag,
# value); tensor infos (string name, u32 n_dims <= 8, u64 dims (ne0
# first), u32 dtype tag, u64 offset relative to the data section); the data
# section starts at the next multiple of `general.alignment` (u32 or u64
# metadata; 32 when absent).  Strings are a u64 length and UTF-8 bytes.

import mmap as _mmap
import struct as _struct
from dataclasses import dataclass as _dataclass, field as _field
from typing import Any as _Any, List as _List, Optional as _Optional

GGUF_MAGIC = b"GGUF"
MIN_VERSION, MAX_VERSION = 2, 3
MAX_DIMS = 8

# metadata value type tags and their fixed-width struct codes
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_U64: "<Q", T_I64: "<q", T_F64: "<d"}


class GgufParseError(ValueError):
    """A malformed or unsupported GGUF header (the reference's ParseError)."""


class _Cursor:
    def __init__(self, data):
        self.data = memoryview(data)
        self.pos = 0

    def take(self, n: int) -> memoryview:
        if n < 0 or self.pos + n > len(self.data):
            raise GgufParseError(f"unexpected end of data at offset {self.pos} (need {n} bytes)")
        b = self.data[self.pos:self.pos + n]
        self.pos += n
        return b

    def scalar(self, code: str):
        return _struct.unpack(code, self.take(_struct.calcsize(code)))[0]

    def string(self) -> str:
        n = self.scalar("<Q")
        off = self.pos
        try:
            return bytes(self.take(n)).decode("utf-8")
        except UnicodeDecodeError as e:
            raise GgufParseError(f"invalid UTF-8 string at offset {off}: {e}") from None

    def value(self, tag: int):
        if tag in _SCALAR:
            return self.scalar(_SCALAR[tag])
        if tag == T_BOOL:
            return self.scalar("<B") != 0
        if tag == T_STRING:
            return self.string()
        if tag == T_ARRAY:
            et = self.scalar("<I")
            n = self.scalar("<Q")
            return [self.value(et) for _ in range(n)]
        raise GgufParseError(f"unknown metadata value type {tag} at offset {self.pos}")


@_dataclass
class GgufTensorInfo:
    name: str
    dims: _List[int]   # ne0 first (the row length of a 2-D weight)
    dtype_tag: int
    offset: int        # relative to the data section

    @property
    def numel(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def dtype(self):
        try:
            return GgufDtype(self.dtype_tag)
        except ValueError:
            return self.dtype_tag  # a tag this library does not name

    @property
    def nbytes(self) -> int:
        if self.dtype not in BLOCK:
            raise GgufParseError(f"{self.name}: byte size of dtype tag {self.dtype_tag} unknown")
        return tensor_byte_size(self.dtype, self.numel)


@_dataclass
class GgufFile:
    """Header, metadata and tensor layout of a GGUF file; `data` is the whole
    file (bytes or an mmap), kept for tensor_bytes()."""
    version: int
    metadata: dict
    tensors: _List[GgufTensorInfo]
    data_offset: int
    alignment: int
    data: _Any = _field(default=None, repr=False)

    @classmethod
    def parse(cls, data) -> "GgufFile":
        cur = _Cursor(data)
        magic = bytes(cur.take(4))
        if magic != GGUF_MAGIC:
            raise GgufParseError(f"invalid magic: expected GGUF, got {magic!r}")
        version = cur.scalar("<I")
        if not MIN_VERSION <= version <= MAX_VERSION:
            raise GgufParseError(f"unsupported version {version} (supported: {MIN_VERSION}..={MAX_VERSION})")
        n_tensors = cur.scalar("<Q")
        n_kv = cur.scalar("<Q")
        meta = {}
        for _ in range(n_kv):
            key = cur.string()
            meta[key] = cur.value(cur.scalar("<I"))
        tensors = []
        for _ in range(n_tensors):
            name = cur.string()
            nd = cur.scalar("<I")
            if nd > MAX_DIMS:
                raise GgufParseError(f"tensor {name}: {nd} dimensions (at most {MAX_DIMS})")
            dims = [cur.scalar("<Q") for _ in range(nd)]
            tag = cur.scalar("<I")
            tensors.append(GgufTensorInfo(name, dims, tag, cur.scalar("<Q")))
        align = meta.get("general.alignment", 32)
        if not isinstance(align, int) or isinstance(align, bool) or align <= 0:
            align = 32
        data_offset = (cur.pos + align - 1) // align * align
        return cls(version, meta, tensors, data_offset, align, data)

    @classmethod
    def open(cls, path) -> "GgufFile":
        """Parse the file at `path` through a read-only mmap (the tensor bytes
        stay in the page cache until a weight is registered)."""
        with open(path, "rb") as f:
            mm = _mmap.mmap(f.fileno(), 0, access=_mmap.ACCESS_READ)
        return cls.parse(mm)

    def tensor(self, name: str) -> _Optional[GgufTensorInfo]:
        for t in self.tensors:
            if t.name == name:
                return t
        return None

    def tensor_bytes(self, t: GgufTensorInfo) -> memoryview:
        """The tensor's bytes, a view of the file (bounds-checked)."""
        start = self.data_offset + t.offset
        end = start + t.nbytes
        if end > len(self.data):
            raise GgufParseError(f"{t.name}: out of bounds [{start}, {end}) > file length {len(self.data)}")
        return memoryview(self.data)[start:end]

    # convenience accessors (parser.rs:554-620)
    def get(self, key: str, default=None):
        return self.metadata.get(key, default)

    def architecture(self) -> _Optional[str]:
        return self.metadata.get("general.architecture")

    def block_count(self) -> _Optional[int]:
        a = self.architecture()
        return self.metadata.get(f"{a}.block_count") if a else None


def build_gguf(metadata, tensors, alignment: int = 32, version: int = 3) -> bytes:
    """A whole GGUF file: `metadata` as (key, type tag, value) triples (values
    as Python objects; arrays as (element tag, list)), `tensors` as (name,
    dims ne0-first, dtype tag, bytes); each tensor at an offset aligned to
    `alignment` (recorded as general.alignment when not 32)."""
    out = bytearray()
    meta = list(metadata)
    if alignment != 32 and not any(k == "general.alignment" for k, _, _ in meta):
        meta.append(("general.alignment", T_U32, alignment))

    def put_str(s: str) -> None:
        b = s.encode("utf-8")
        out.extend(_struct.pack("<Q", len(b)))
        out.extend(b)

    def put_value(tag: int, v) -> None:
        if tag in _SCALAR:
            out.extend(_struct.pack(_SCALAR[tag], v))
        elif tag == T_BOOL:
            out.extend(_struct.pack("<B", 1 if v else 0))
        elif tag == T_STRING:
            put_str(v)
        elif tag == T_ARRAY:
            et, items = v
            out.extend(_struct.pack("<IQ", et, len(items)))
            for it in items:
                put_value(et, it)
        else:
            raise ValueError(f"unknown metadata type {tag}")

    out.extend(GGUF_MAGIC)
    out.extend(_struct.pack("<IQQ", version, len(tensors), len(meta)))
    for k, tag, v in meta:
        put_str(k)
        out.extend(_struct.pack("<I", tag))
        put_value(tag, v)
    offs, off = [], 0
    for _, _, _, data in tensors:
        offs.append(off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    for (name, dims, tag, _), o in zip(tensors, offs):
        put_str(name)
        out.extend(_struct.pack("<I", len(dims)))
        for d in dims:
            out.extend(_struct.pack("<Q", d))
        out.extend(_struct.pack("<IQ", tag, o))
    start = (len(out) + alignment - 1) // alignment * alignment
    out.extend(b"\0" * (start - len(out)))
    for (_, _, _, data), o in zip(tensors, offs):
        out.extend(b"\0" * (start + o - len(out)))
        out.extend(bytes(data))
    return bytes(out)
