"""Seeded synthetic GGUF weights and activations for benchmarks and tests.

The value distributions follow the benchmark configurations of this path:
  Q8_0: 32 int8 codes uniform in [-127, 127], fp16 scale d = |N(0,1)| * 0.01;
  Q4_0: 32 nibbles uniform in 0..15 (value n - 8), fp16 d = |N(0,1)| * 0.02;
  Q4_K: fp16 d and dmin = |N(0,1)| * 0.01, the 12 packed scale bytes and the
        128 nibble bytes uniform (so every 6-bit scale/min and every nibble
        is uniform);
  Q5_K: as Q4_K, with the 32 fifth-bit bytes uniform;
  Q6_K: fp16 d = |N(0,1)| * 0.01, the 16 int8 scales uniform in [-128, 127],
        the 192 code bytes uniform (every 6-bit code uniform in 0..63);
  activations: f32 N(0,1).
Everything is generated from numpy's PCG64 with the given seed, so a (seed,
shape) pair always produces the same bytes.  The fp16 fields are
round-to-nearest-even conversions (numpy's float16 cast).
"""
from __future__ import annotations

import numpy as np

from .gguf import GgufDtype

DEFAULT_SCALE = {GgufDtype.Q8_0: 0.01, GgufDtype.Q4_0: 0.02, GgufDtype.Q4K: 0.01, GgufDtype.Q5K: 0.01,
                 GgufDtype.Q6K: 0.01}


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(v.shape + (2,))


def q8_0(n_rows: int, n_cols: int, rng: np.random.Generator, scale: float = 0.01) -> np.ndarray:
    nb = n_cols // 32
    blocks = np.empty((n_rows, nb, 34), dtype=np.uint8)
    d = np.abs(rng.standard_normal((n_rows, nb), dtype=np.float32)) * np.float32(scale)
    blocks[:, :, 0:2] = _f16_bytes(d)
    blocks[:, :, 2:] = rng.integers(-127, 128, size=(n_rows, nb, 32), dtype=np.int8).view(np.uint8)
    return blocks.reshape(-1)


def q4_0(n_rows: int, n_cols: int, rng: np.random.Generator, scale: float = 0.02) -> np.ndarray:
    nb = n_cols // 32
    blocks = np.empty((n_rows, nb, 18), dtype=np.uint8)
    d = np.abs(rng.standard_normal((n_rows, nb), dtype=np.float32)) * np.float32(scale)
    blocks[:, :, 0:2] = _f16_bytes(d)
    blocks[:, :, 2:] = rng.integers(0, 256, size=(n_rows, nb, 16), dtype=np.uint8)
    return blocks.reshape(-1)


def q4_k(n_rows: int, n_cols: int, rng: np.random.Generator, scale: float = 0.01) -> np.ndarray:
    nsb = n_cols // 256
    blocks = np.empty((n_rows, nsb, 144), dtype=np.uint8)
    d = np.abs(rng.standard_normal((n_rows, nsb), dtype=np.float32)) * np.float32(scale)
    dmin = np.abs(rng.standard_normal((n_rows, nsb), dtype=np.float32)) * np.float32(scale)
    blocks[:, :, 0:2] = _f16_bytes(d)
    blocks[:, :, 2:4] = _f16_bytes(dmin)
    blocks[:, :, 4:] = rng.integers(0, 256, size=(n_rows, nsb, 140), dtype=np.uint8)
    return blocks.reshape(-1)


def q5_k(n_rows: int, n_cols: int, rng: np.random.Generator, scale: float = 0.01) -> np.ndarray:
    nsb = n_cols // 256
    blocks = np.empty((n_rows, nsb, 176), dtype=np.uint8)
    d = np.abs(rng.standard_normal((n_rows, nsb), dtype=np.float32)) * np.float32(scale)
    dmin = np.abs(rng.standard_normal((n_rows, nsb), dtype=np.float32)) * np.float32(scale)
    blocks[:, :, 0:2] = _f16_bytes(d)
    blocks[:, :, 2:4] = _f16_bytes(dmin)
    blocks[:, :, 4:] = rng.integers(0, 256, size=(n_rows, nsb, 172), dtype=np.uint8)
    return blocks.reshape(-1)


def q6_k(n_rows: int, n_cols: int, rng: np.random.Generator, scale: float = 0.01) -> np.ndarray:
    nsb = n_cols // 256
    blocks = np.empty((n_rows, nsb, 210), dtype=np.uint8)
    blocks[:, :, :208] = rng.integers(0, 256, size=(n_rows, nsb, 208), dtype=np.uint8)
    d = np.abs(rng.standard_normal((n_rows, nsb), dtype=np.float32)) * np.float32(scale)
    blocks[:, :, 208:210] = _f16_bytes(d)
    return blocks.reshape(-1)


def weights(dtype, n_rows: int, n_cols: int, rng, scale=None) -> np.ndarray:
    dt = GgufDtype.parse(dtype)
    s = DEFAULT_SCALE[dt] if scale is None else scale
    if dt == GgufDtype.Q8_0:
        return q8_0(n_rows, n_cols, rng, s)
    if dt == GgufDtype.Q4_0:
        return q4_0(n_rows, n_cols, rng, s)
    if dt == GgufDtype.Q4K:
        return q4_k(n_rows, n_cols, rng, s)
    if dt == GgufDtype.Q5K:
        return q5_k(n_rows, n_cols, rng, s)
    if dt == GgufDtype.Q6K:
        return q6_k(n_rows, n_cols, rng, s)
    raise ValueError(f"no generator for {dt}")


def activations(m: int, k: int, rng) -> np.ndarray:
    return rng.standard_normal((m, k), dtype=np.float32)


def pattern_bytes(n_bytes: int, mul: int, add: int) -> np.ndarray:
    """The reference tests' byte fill ((i * mul + add) & 0xFF)."""
    i = np.arange(n_bytes, dtype=np.int64)
    return ((i * mul + add) & 0xFF).astype(np.uint8)


def patch_f16(buf: np.ndarray, block_bytes: int, offset: int, value: float) -> None:
    """Overwrite the fp16 field at ``offset`` of every block with ``value``."""
    b = buf.reshape(-1, block_bytes)
    b[:, offset:offset + 2] = np.array([value], dtype=np.float16).view(np.uint8)


# ---- device-side generation (torch), same distributions ---------------------

def device_weights(dtype, n_rows: int, n_cols: int, gen, device, scale=None):
    """GGUF bytes generated directly in device memory (a uint8 CUDA tensor),
    for benchmark-sized weights; same distributions as the host generators."""
    import torch

    dt = GgufDtype.parse(dtype)
    s = DEFAULT_SCALE[dt] if scale is None else scale
    if dt == GgufDtype.Q6K:
        nb = n_rows * n_cols // 256
        raw = torch.randint(0, 256, (nb, 210), dtype=torch.uint8, device=device, generator=gen)
        d = (torch.randn(nb, device=device, generator=gen).abs() * s).to(torch.float16)
        raw[:, 208:210] = d.view(torch.uint8).view(nb, 2)
        return raw.view(-1)
    if dt in (GgufDtype.Q4K, GgufDtype.Q5K):
        nb, bb = n_rows * n_cols // 256, (144 if dt == GgufDtype.Q4K else 176)
    elif dt == GgufDtype.Q8_0:
        nb, bb = n_rows * n_cols // 32, 34
    else:
        nb, bb = n_rows * n_cols // 32, 18
    raw = torch.randint(0, 256, (nb, bb), dtype=torch.uint8, device=device, generator=gen)
    if dt == GgufDtype.Q8_0:  # codes uniform in [-127, 127]
        q = torch.randint(-127, 128, (nb, 32), dtype=torch.int8, device=device, generator=gen)
        raw[:, 2:] = q.view(torch.uint8)
    d = (torch.randn(nb, device=device, generator=gen).abs() * s).to(torch.float16)
    raw[:, 0:2] = d.view(torch.uint8).view(nb, 2)
    if dt in (GgufDtype.Q4K, GgufDtype.Q5K):
        dmin = (torch.randn(nb, device=device, generator=gen).abs() * s).to(torch.float16)
        raw[:, 2:4] = dmin.view(torch.uint8).view(nb, 2)
    return raw.view(-1)
