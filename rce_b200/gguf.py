"""GGUF format facts used on the quantized-matmul path.

Mirrors ``GgufDtype`` (rce-ingest-gguf/src/parser.rs:228, tags :308-338),
``tensor_byte_size`` (rce-ingest-gguf/src/dequant.rs:18-58) and the block
geometry of ``quant_info`` (rce-ingest-gguf/src/quant.rs:22-217) for the three
formats this library implements.
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

#: values per block and bytes per block
BLOCK = {GgufDtype.Q4_0: 32, GgufDtype.Q8_0: 32, GgufDtype.Q4K: 256, GgufDtype.F32: 1, GgufDtype.F16: 1}
BLOCK_BYTES = {GgufDtype.Q4_0: 18, GgufDtype.Q8_0: 34, GgufDtype.Q4K: 144, GgufDtype.F32: 4, GgufDtype.F16: 2}

SUPPORTED = (GgufDtype.Q4_0, GgufDtype.Q8_0, GgufDtype.Q4K)


def tensor_byte_size(dtype, numel: int) -> int:
    """Bytes of a tensor of ``numel`` values (ceil-divided into blocks)."""
    dt = GgufDtype.parse(dtype)
    blk = BLOCK[dt]
    return (numel + blk - 1) // blk * BLOCK_BYTES[dt]


def row_bytes(dtype, n_cols: int) -> int:
    dt = GgufDtype.parse(dtype)
    return n_cols // BLOCK[dt] * BLOCK_BYTES[dt]
