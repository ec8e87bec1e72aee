"""Fixtures of the reference's own unit tests for this path, rebuilt byte for
byte, plus the seeded configuration cases.

Each builder returns (weight_bytes u8, dtype, n_rows, n_cols, activations f32
[t, k]).  Activations are evaluated in binary32 with libm's sinf/cosf through
the oracle library, as Rust's f32::sin / f32::cos are on this platform.
"""
from __future__ import annotations

import numpy as np

import oracle as O
from rce_b200 import synth

Q4_0, Q8_0, Q4_K = O.GGUF_Q4_0, O.GGUF_Q8_0, O.GGUF_Q4_K


def vm_bit_exact_q4_0():
    """qmm_executes_through_rce_vm_bit_exact (rce-op-qmm/src/lib.rs:2267-2333):
    Q4_0, N=5, K=64, bytes (i*11+1)&0xFF, every block's d = 0.125,
    a = ((i as f32 * 0.05) - 1.0).sin()."""
    n, k = 5, 64
    w = synth.pattern_bytes(n * (k // 32) * 18, 11, 1)
    synth.patch_f16(w, 18, 0, 0.125)
    a = O.test_activations("sin", 0.05, -1.0, k)
    return w, Q4_0, n, k, a.reshape(1, k)


def q4_k_dequant_dot():
    """q4_k_matmul_matches_dequant_then_dot (lib.rs:2428-2464): K=512, N=5,
    bytes (i*17+3)&0xFF, d = 0.0625, dmin = 0.03125,
    a = ((i as f32 * 0.021) + 0.5).cos()."""
    n, k = 5, 512
    w = synth.pattern_bytes(n * (k // 256) * 144, 17, 3)
    synth.patch_f16(w, 144, 0, 0.0625)
    synth.patch_f16(w, 144, 2, 0.03125)
    a = O.test_activations("cos", 0.021, 0.5, k)
    return w, Q4_K, n, k, a.reshape(1, k)


def q4_0_dequant_dot():
    """q4_0_matmul_matches_dequant_then_dot (lib.rs:2466-2500): K=128, N=6,
    bytes (i*11+1)&0xFF, d = 0.125, a = ((i as f32 * 0.05) - 1.0).sin()."""
    n, k = 6, 128
    w = synth.pattern_bytes(n * (k // 32) * 18, 11, 1)
    synth.patch_f16(w, 18, 0, 0.125)
    a = O.test_activations("sin", 0.05, -1.0, k)
    return w, Q4_0, n, k, a.reshape(1, k)


def batched_q4_k():
    """mm_batched_byte_identical_to_per_row_for_q5k_and_q4k, Q4_K leg
    (lib.rs:2575-2616): K=512, N=6, T=4, bytes (i*31+7)&0xFF, d = 0.0625,
    dmin = 0.03125, a[t*k + i] = ((i as f32 * 0.011) - 0.5).sin() over all
    T*K positions."""
    n, k, t = 6, 512, 4
    w = synth.pattern_bytes(n * (k // 256) * 144, 31, 7)
    synth.patch_f16(w, 144, 0, 0.0625)
    synth.patch_f16(w, 144, 2, 0.03125)
    a = O.test_activations("sin", 0.011, -0.5, t * k)
    return w, Q4_K, n, k, a.reshape(t, k)


def router_gate_q8_0(n_experts: int, d_model: int):
    """synth_gate of rce-op-moe's tests (rce-op-moe/src/lib.rs:119-141): Q8_0
    [n_experts, d_model]; row r's blocks have scale 0.0625 + r*0.01 (f32, then
    f16) and q = 64 where r == (blk*32 + i) % n_experts, else 0."""
    bpr = d_model // 32
    b = np.zeros((n_experts, bpr, 34), dtype=np.uint8)
    for r in range(n_experts):
        scale = np.float32(0.0625) + np.float32(r) * np.float32(0.01)
        b[r, :, 0:2] = np.array([scale], dtype=np.float16).view(np.uint8)
        for blk in range(bpr):
            for i in range(32):
                if r == (blk * 32 + i) % n_experts:
                    b[r, blk, 2 + i] = 64
    return b.reshape(-1)


REFERENCE_CASES = {
    "vm_bit_exact_q4_0": vm_bit_exact_q4_0,
    "q4_k_dequant_dot": q4_k_dequant_dot,
    "q4_0_dequant_dot": q4_0_dequant_dot,
    "batched_q4_k": batched_q4_k,
}


def seeded_case(dtype: int, n_rows: int, n_cols: int, m: int, seed: int):
    """A case drawn from the benchmark configurations' distributions."""
    rng = np.random.default_rng(seed)
    w = synth.weights(dtype, n_rows, n_cols, rng)
    x = synth.activations(m, n_cols, rng)
    return w, dtype, n_rows, n_cols, x


# (name, dtype, n_rows, n_cols, m, seed): the benchmark configurations at the
# sizes the oracle finishes in well under a second.  seed follows the config.
SEEDED_CASES = [
    ("cfg0_q8_0_gemv", Q8_0, 4096, 4096, 1, 0),
    ("cfg1_q4_0_up", Q4_0, 11008, 4096, 1, 1),
    ("cfg1_q4_0_down", Q4_0, 4096, 11008, 1, 1),
    ("cfg2_q4_k_m1", Q4_K, 14336, 4096, 1, 2),
    ("cfg2_q4_k_m16_rows512", Q4_K, 512, 4096, 16, 2),
    ("cfg3_q4_k_kv", Q4_K, 1024, 4096, 1, 3),
    ("cfg3_q4_k_down_rows256", Q4_K, 256, 14336, 2, 3),
]
