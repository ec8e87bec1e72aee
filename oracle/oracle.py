"""ctypes binding of the C oracle (qmm_oracle.c) -- TEST INFRASTRUCTURE ONLY.

The C file restates the reference's Rust CPU path bit for bit (see the
file:line citations there).  This module adds numpy conveniences and two
independent restatements used to pin it:

* ``unpack_q8_0/unpack_q4_0/unpack_q4_k`` decode GGUF bytes into the
  unpacked operands of the spec kernels (q, d) / (q, s, o) with numpy
  integer arithmetic (rce-vm-backend-cpu/src/ml/kquant.rs:371-398 for the
  K-quant unpacking, nn.rs:477-517 for Q8_0/Q4_0's operands);
* ``py_mm_1d`` is a pure-Python, per-operation np.float32 restatement of
  mm_1d for tiny shapes.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

GGUF_F32 = 0
GGUF_F16 = 1
GGUF_Q4_0 = 2
GGUF_Q8_0 = 8
GGUF_Q4_K = 12
GGUF_Q5_K = 13
GGUF_Q6_K = 14

BLOCK = {GGUF_Q4_0: 32, GGUF_Q8_0: 32, GGUF_Q4_K: 256, GGUF_Q5_K: 256, GGUF_Q6_K: 256}
BLOCK_BYTES = {GGUF_Q4_0: 18, GGUF_Q8_0: 34, GGUF_Q4_K: 144, GGUF_Q5_K: 176, GGUF_Q6_K: 210}

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libqmm_oracle.so")
_lib = None
_lock = threading.Lock()

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)
_sz = ctypes.c_size_t


def build() -> str:
    """Compile the oracle with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            src = os.path.join(_HERE, "qmm_oracle.c")
            if not os.path.exists(_LIB_PATH) or (
                os.path.exists(src) and os.path.getmtime(src) > os.path.getmtime(_LIB_PATH)
            ):
                build()
            L = ctypes.CDLL(_LIB_PATH)
            L.oracle_f16_to_f32.restype = ctypes.c_float
            L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
            L.oracle_round_to_f16.restype = ctypes.c_float
            L.oracle_round_to_f16.argtypes = [ctypes.c_float]
            L.oracle_f32_to_f16_bits.restype = ctypes.c_uint16
            L.oracle_f32_to_f16_bits.argtypes = [ctypes.c_float]
            L.oracle_q4k_get_scale_min.argtypes = [_u8p, ctypes.c_int, _u8p, _u8p]
            L.oracle_tensor_byte_size.restype = _sz
            L.oracle_tensor_byte_size.argtypes = [ctypes.c_int, _sz]
            L.oracle_dequant.restype = ctypes.c_int
            L.oracle_dequant.argtypes = [_u8p, _sz, ctypes.c_int, _sz, _f32p]
            L.oracle_mm_1d_rows.restype = ctypes.c_int
            L.oracle_mm_1d_rows.argtypes = [_f32p, _u8p, ctypes.c_int, _sz, _sz, _sz, _sz, _f32p, ctypes.c_int]
            L.oracle_mm_1d.restype = ctypes.c_int
            L.oracle_mm_1d.argtypes = [_f32p, _u8p, ctypes.c_int, _sz, _sz, _f32p, ctypes.c_int]
            L.oracle_mm_batched.restype = ctypes.c_int
            L.oracle_mm_batched.argtypes = [_f32p, _sz, _u8p, ctypes.c_int, _sz, _sz, _f32p, ctypes.c_int]
            L.oracle_moe_softmax_topk.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p, _f32p]
            L.oracle_moe_router.restype = ctypes.c_int
            L.oracle_moe_router.argtypes = [_f32p, _u8p, ctypes.c_int, ctypes.c_int, _sz, ctypes.c_int,
                                            ctypes.c_int, _i32p, _f32p]
            L.oracle_moe_combine.argtypes = [_f32p, ctypes.c_int, _f32p, _sz, _f32p]
            L.oracle_silu.restype = ctypes.c_float
            L.oracle_silu.argtypes = [ctypes.c_float]
            L.oracle_moe_ffn.restype = ctypes.c_int
            L.oracle_moe_ffn.argtypes = [_f32p, _sz, _sz, _sz, _f32p, ctypes.c_int, ctypes.c_int,
                                         _u8p, _u8p, _u8p, _sz, _sz, _sz, ctypes.c_int, _f32p, ctypes.c_int]
            L.oracle_sigmoid.restype = ctypes.c_float
            L.oracle_sigmoid.argtypes = [ctypes.c_float]
            L.oracle_moe_shared_expert.restype = ctypes.c_int
            L.oracle_moe_shared_expert.argtypes = [_f32p, _sz, _sz, _sz, _f32p, _u8p, _u8p, _u8p, ctypes.c_int,
                                                   _f32p, ctypes.c_int]
            L.oracle_quantize_block.argtypes = [_f32p, ctypes.c_int, _i32p, _f32p]
            L.oracle_spec_matmul_q.argtypes = [_f32p, _sz, _i32p, _f32p, _sz, _sz, ctypes.c_int, _f32p]
            L.oracle_spec_matmul_q4k.argtypes = [_f32p, _sz, _i32p, _f32p, _f32p, _sz, _sz, _f32p]
            L.oracle_test_activations.argtypes = [ctypes.c_int, ctypes.c_float, ctypes.c_float, _sz, _f32p]
            _lib = L
    return _lib


def _p(arr, t):
    return arr.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(b):
    if isinstance(b, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(b), dtype=np.uint8)
    return np.ascontiguousarray(b, dtype=np.uint8)


def f16_to_f32(h: int) -> float:
    return lib().oracle_f16_to_f32(int(h) & 0xFFFF)


def round_to_f16(x: float) -> float:
    return lib().oracle_round_to_f16(float(x))


def f32_to_f16_bits(x: float) -> int:
    return lib().oracle_f32_to_f16_bits(float(x))


def q4k_get_scale_min(scales, j: int):
    s = _u8(scales)
    sc = ctypes.c_uint8()
    m = ctypes.c_uint8()
    lib().oracle_q4k_get_scale_min(_p(s, _u8p), int(j), ctypes.byref(sc), ctypes.byref(m))
    return sc.value, m.value


def tensor_byte_size(dtype: int, numel: int) -> int:
    return int(lib().oracle_tensor_byte_size(int(dtype), int(numel)))


def dequant(wbytes, dtype: int, n: int) -> np.ndarray:
    b = _u8(wbytes)
    blk = BLOCK[dtype]
    out = np.zeros(((n + blk - 1) // blk) * blk, dtype=np.float32)
    rc = lib().oracle_dequant(_p(b, _u8p), b.size, int(dtype), int(n), _p(out, _f32p))
    if rc != 0:
        raise ValueError(f"oracle dequant: unsupported dtype {dtype}")
    return out[:n]


def mm_1d(a, wbytes, dtype: int, n_rows: int, n_cols: int, nthreads: int = 1) -> np.ndarray:
    a = _f32(a)
    b = _u8(wbytes)
    out = np.zeros(n_rows, dtype=np.float32)
    rc = lib().oracle_mm_1d(_p(a, _f32p), _p(b, _u8p), int(dtype), n_rows, n_cols, _p(out, _f32p), int(nthreads))
    if rc != 0:
        raise ValueError(f"oracle mm_1d failed rc={rc}")
    return out


def mm_1d_rows(a, wbytes, dtype, n_rows, n_cols, row0, row1, nthreads=1) -> np.ndarray:
    """Rows [row0,row1) of mm_1d; returns an array of length row1-row0."""
    a = _f32(a)
    b = _u8(wbytes)
    out = np.zeros(n_rows, dtype=np.float32)
    rc = lib().oracle_mm_1d_rows(_p(a, _f32p), _p(b, _u8p), int(dtype), n_rows, n_cols, row0, row1,
                                 _p(out, _f32p), int(nthreads))
    if rc != 0:
        raise ValueError(f"oracle mm_1d_rows failed rc={rc}")
    return out[row0:row1].copy()


def mm_batched(a, t_rows: int, wbytes, dtype: int, n_rows: int, n_cols: int, nthreads: int = 1) -> np.ndarray:
    a = _f32(a)
    b = _u8(wbytes)
    out = np.zeros(t_rows * n_rows, dtype=np.float32)
    rc = lib().oracle_mm_batched(_p(a, _f32p), t_rows, _p(b, _u8p), int(dtype), n_rows, n_cols,
                                 _p(out, _f32p), int(nthreads))
    if rc != 0:
        raise ValueError(f"oracle mm_batched failed rc={rc}")
    return out.reshape(t_rows, n_rows)


def moe_softmax_topk(logits, top_k: int, normalize: bool = True):
    lg = _f32(logits)
    idx = np.zeros(top_k, dtype=np.int32)
    w = np.zeros(top_k, dtype=np.float32)
    lib().oracle_moe_softmax_topk(_p(lg, _f32p), lg.size, top_k, int(bool(normalize)), _p(idx, _i32p), _p(w, _f32p))
    return idx, w


def moe_router(x, gate_bytes, gate_dtype: int, n_experts: int, top_k: int, normalize: bool = True):
    x = _f32(x)
    b = _u8(gate_bytes)
    idx = np.zeros(top_k, dtype=np.int32)
    w = np.zeros(top_k, dtype=np.float32)
    rc = lib().oracle_moe_router(_p(x, _f32p), _p(b, _u8p), int(gate_dtype), n_experts, x.size, top_k,
                                 int(bool(normalize)), _p(idx, _i32p), _p(w, _f32p))
    if rc != 0:
        raise ValueError("oracle moe_router failed")
    return idx, w


def moe_combine(weights, outs) -> np.ndarray:
    w = _f32(weights)
    o = _f32(outs)
    k, d = o.shape
    out = np.zeros(d, dtype=np.float32)
    lib().oracle_moe_combine(_p(w, _f32p), k, _p(o, _f32p), d, _p(out, _f32p))
    return out


def silu(x: float) -> float:
    return lib().oracle_silu(float(x))


def moe_ffn(x, router_logits, top_k, gate, up, down, dtype, d_ff, nthreads=1) -> np.ndarray:
    """gate/up/down: uint8 arrays [E, bytes_per_expert]."""
    x = _f32(x)
    t_rows, d_model = x.shape
    lg = _f32(router_logits)
    gate, up, down = _u8(gate), _u8(up), _u8(down)
    n_experts = lg.shape[1]
    out = np.zeros((t_rows, d_model), dtype=np.float32)
    rc = lib().oracle_moe_ffn(_p(x, _f32p), t_rows, d_model, d_ff, _p(lg, _f32p), n_experts, top_k,
                              _p(gate, _u8p), _p(up, _u8p), _p(down, _u8p),
                              gate.size // n_experts, up.size // n_experts, down.size // n_experts,
                              int(dtype), _p(out, _f32p), int(nthreads))
    if rc != 0:
        raise ValueError("oracle moe_ffn failed")
    return out


def sigmoid(x: float) -> float:
    return lib().oracle_sigmoid(float(x))


def moe_shared_expert(x, out, gate_inp, gate, up, down, dtype, n_ff, nthreads=1) -> np.ndarray:
    """out + sigmoid(gate_inp . x) * SwiGLU(x) with the shared expert's weights
    (moe_ffn_forward, rce-qwen36-moe/src/lib.rs:694-705); returns a new array."""
    x = _f32(x)
    t_rows, d_model = x.shape
    res = np.array(_f32(out), dtype=np.float32, copy=True)
    gi = _f32(gate_inp)
    gate, up, down = _u8(gate), _u8(up), _u8(down)
    rc = lib().oracle_moe_shared_expert(_p(x, _f32p), t_rows, d_model, n_ff, _p(gi, _f32p), _p(gate, _u8p),
                                        _p(up, _u8p), _p(down, _u8p), int(dtype), _p(res, _f32p), int(nthreads))
    if rc != 0:
        raise ValueError("oracle moe_shared_expert failed")
    return res


def quantize_block(x, q4: bool):
    x = _f32(x)
    assert x.size == 32
    q = np.zeros(32, dtype=np.int32)
    d = ctypes.c_float()
    lib().oracle_quantize_block(_p(x, _f32p), int(bool(q4)), _p(q, _i32p), ctypes.byref(d))
    return q, d.value


def spec_matmul_q(x, q, d, q4: bool) -> np.ndarray:
    x = _f32(x)
    q = np.ascontiguousarray(q, dtype=np.int32)
    d = _f32(d)
    m, k = x.shape
    n = q.shape[0]
    out = np.zeros((m, n), dtype=np.float32)
    lib().oracle_spec_matmul_q(_p(x, _f32p), m, _p(q, _i32p), _p(d, _f32p), n, k, int(bool(q4)), _p(out, _f32p))
    return out


def spec_matmul_q4k(x, q, s, o) -> np.ndarray:
    x = _f32(x)
    q = np.ascontiguousarray(q, dtype=np.int32)
    s, o = _f32(s), _f32(o)
    m, k = x.shape
    n = q.shape[0]
    out = np.zeros((m, n), dtype=np.float32)
    lib().oracle_spec_matmul_q4k(_p(x, _f32p), m, _p(q, _i32p), _p(s, _f32p), _p(o, _f32p), n, k, _p(out, _f32p))
    return out


def test_activations(kind: str, c1: float, c0: float, n: int) -> np.ndarray:
    """The reference tests' activation vectors, e.g. ((i as f32 * 0.05) - 1.0).sin()."""
    out = np.zeros(n, dtype=np.float32)
    lib().oracle_test_activations(0 if kind == "sin" else 1, float(c1), float(c0), n, _p(out, _f32p))
    return out


# ---- independent numpy unpacking of the GGUF formats -------------------------

def _f16(lo, hi):
    return (lo.astype(np.uint16) | (hi.astype(np.uint16) << 8)).view(np.float16).astype(np.float32)


def unpack_q8_0(wbytes, n_rows, n_cols):
    """Q8_0 bytes -> q [n][k] int32, d [n][k/32] f32 (operands of matmul_q8_0)."""
    b = _u8(wbytes).reshape(n_rows, n_cols // 32, 34)
    d = _f16(b[:, :, 0], b[:, :, 1])
    q = b[:, :, 2:].view(np.int8).astype(np.int32).reshape(n_rows, n_cols)
    return q, d


def unpack_q4_0(wbytes, n_rows, n_cols):
    """Q4_0 bytes -> q [n][k] in -8..7, d [n][k/32] (low nibbles are positions
    0..15 of the block, high nibbles 16..31)."""
    b = _u8(wbytes).reshape(n_rows, n_cols // 32, 18)
    d = _f16(b[:, :, 0], b[:, :, 1])
    qs = b[:, :, 2:].astype(np.int32)
    q = np.concatenate([(qs & 15) - 8, (qs >> 4) - 8], axis=2).reshape(n_rows, n_cols)
    return q, d


def unpack_q4_k(wbytes, n_rows, n_cols):
    """Q4_K bytes -> q [n][k] in 0..15, s = d*sc and o = dmin*m [n][k/32] (f32,
    each product exact), following kquant.rs unpack/unpack_scale (:295-302,
    :371-398) with independent numpy integer code."""
    nsb = n_cols // 256
    b = _u8(wbytes).reshape(n_rows, nsb, 144)
    d = _f16(b[:, :, 0], b[:, :, 1])
    dmin = _f16(b[:, :, 2], b[:, :, 3])
    sc_b = b[:, :, 4:16].astype(np.int32)
    sc = np.zeros((n_rows, nsb, 8), dtype=np.int32)
    mn = np.zeros((n_rows, nsb, 8), dtype=np.int32)
    for j in range(8):
        if j < 4:
            sc[:, :, j] = sc_b[:, :, j] & 63
            mn[:, :, j] = sc_b[:, :, j + 4] & 63
        else:
            sc[:, :, j] = (sc_b[:, :, j + 4] & 15) | ((sc_b[:, :, j - 4] >> 6) << 4)
            mn[:, :, j] = (sc_b[:, :, j + 4] >> 4) | ((sc_b[:, :, j] >> 6) << 4)
    qs = b[:, :, 16:].astype(np.int32).reshape(n_rows, nsb, 4, 32)
    q = np.concatenate([qs & 15, qs >> 4], axis=3).reshape(n_rows, n_cols)
    s = (d[:, :, None] * sc.astype(np.float32)).astype(np.float32).reshape(n_rows, nsb * 8)
    o = (dmin[:, :, None] * mn.astype(np.float32)).astype(np.float32).reshape(n_rows, nsb * 8)
    return q, s, o


def unpack_q5_k(wbytes, n_rows, n_cols):
    """Q5_K bytes -> q [n][k] in 0..31, s = d*sc and o = dmin*m [n][k/32]
    (the operands of the spec's matmul_q5_k), decoded independently: Q4_K's
    nibbles and scales (block bytes 0..15 and 48..175), the fifth bit of
    value 64 g + 32 h + l from bit 2g + h of qh[l] (bytes 16..47)."""
    nsb = n_cols // 256
    b = _u8(wbytes).reshape(n_rows, nsb, 176)
    as_q4k = np.concatenate([b[:, :, :16], b[:, :, 48:]], axis=2).reshape(-1)
    q4, s, o = unpack_q4_k(as_q4k, n_rows, n_cols)
    qh = b[:, :, 16:48].astype(np.int32)
    hi = np.zeros((n_rows, nsb, 256), dtype=np.int32)
    for g in range(4):
        for h in range(2):
            hi[:, :, 64 * g + 32 * h:64 * g + 32 * h + 32] = (qh >> (2 * g + h)) & 1
    return q4 + 16 * hi.reshape(n_rows, n_cols), s, o


def unpack_q6_k(wbytes, n_rows, n_cols):
    """Q6_K bytes -> q [n][k] in -32..31 and s = d*sc [n][k/16] (f32, each
    product exact), the operands of the spec's matmul_q6_k
    (spec/RCE-SPEC.md, tensor.matmul_q6_k; kquant.rs:67-150), decoded with
    independent numpy integer code: element 128 o + 32 q + l of a block takes
    its low four bits from ql[64 o + 32 (q & 1) + l] (low nibble for q < 2)
    and its high two from bits 2q of qh[32 o + l]."""
    nsb = n_cols // 256
    b = _u8(wbytes).reshape(n_rows, nsb, 210).astype(np.int32)
    ql, qh = b[:, :, :128], b[:, :, 128:192]
    sc = b[:, :, 192:208]
    sc = np.where(sc >= 128, sc - 256, sc)
    d = _f16(b[:, :, 208].astype(np.uint8), b[:, :, 209].astype(np.uint8))
    q = np.zeros((n_rows, nsb, 256), dtype=np.int32)
    for o in range(2):
        for qq in range(4):
            c0 = 64 * o + 32 * (qq & 1)
            lo = ql[:, :, c0:c0 + 32]
            lo = (lo & 15) if qq < 2 else (lo >> 4)
            hi = (qh[:, :, 32 * o:32 * o + 32] >> (2 * qq)) & 3
            q[:, :, 128 * o + 32 * qq:128 * o + 32 * qq + 32] = (lo | (hi << 4)) - 32
    s = (d[:, :, None] * sc.astype(np.float32)).astype(np.float32).reshape(n_rows, nsb * 16)
    return q.reshape(n_rows, n_cols), s


def py_mm_1d(a, wbytes, dtype, n_rows, n_cols):
    """Pure-Python per-operation np.float32 restatement of mm_1d (tiny shapes)."""
    f = np.float32
    a = _f32(a)
    out = np.zeros(n_rows, dtype=np.float32)
    if dtype == GGUF_Q8_0:
        q, d = unpack_q8_0(wbytes, n_rows, n_cols)
        for j in range(n_rows):
            sumf = f(0)
            for b in range(n_cols // 32):
                sub = f(0)
                for t in range(32):
                    sub = f(sub + f(f(q[j, b * 32 + t]) * a[b * 32 + t]))
                sumf = f(sumf + f(d[j, b] * sub))
            out[j] = sumf
    elif dtype == GGUF_Q4_0:
        q, d = unpack_q4_0(wbytes, n_rows, n_cols)
        for j in range(n_rows):
            sumf = f(0)
            for b in range(n_cols // 32):
                sub = f(0)
                for t in range(16):
                    sub = f(sub + f(f(q[j, b * 32 + t]) * a[b * 32 + t]))
                    sub = f(sub + f(f(q[j, b * 32 + t + 16]) * a[b * 32 + t + 16]))
                sumf = f(sumf + f(d[j, b] * sub))
            out[j] = sumf
    elif dtype in (GGUF_Q4_K, GGUF_Q5_K):
        q, s, o = (unpack_q4_k if dtype == GGUF_Q4_K else unpack_q5_k)(wbytes, n_rows, n_cols)
        for j in range(n_rows):
            sumf = f(0)
            for g in range(n_cols // 64):
                u1 = a1 = u2 = a2 = f(0)
                for t in range(32):
                    p1, p2 = 64 * g + t, 64 * g + 32 + t
                    u1 = f(u1 + f(f(q[j, p1]) * a[p1]))
                    a1 = f(a1 + a[p1])
                    u2 = f(u2 + f(f(q[j, p2]) * a[p2]))
                    a2 = f(a2 + a[p2])
                acc = f(f(s[j, 2 * g] * u1) - f(o[j, 2 * g] * a1))
                acc = f(acc + f(s[j, 2 * g + 1] * u2))
                acc = f(acc - f(o[j, 2 * g + 1] * a2))
                sumf = f(sumf + acc)
            out[j] = sumf
    elif dtype == GGUF_Q6_K:
        # the spec's matmul_q6_k order: per half of a super-block, l = 0..31,
        # positions l, l+32, l+64, l+96; y += (s * q) * x from +0.0
        q, s = unpack_q6_k(wbytes, n_rows, n_cols)
        for j in range(n_rows):
            sumf = f(0)
            for sb in range(n_cols // 256):
                for o in range(2):
                    for l in range(32):
                        for qq in range(4):
                            t = 256 * sb + 128 * o + 32 * qq + l
                            sumf = f(sumf + f(f(s[j, t // 16] * f(q[j, t])) * a[t]))
            out[j] = sumf
    else:
        raise ValueError(dtype)
    return out
