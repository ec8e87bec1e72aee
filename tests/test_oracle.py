"""The oracle, pinned against the reference's own tests for this path.

The reference (Rust) cannot be built here, so the C restatement is checked
against every known answer and invariant its tests hold, plus two
independent restatements (the spec kernels' order and a pure-Python loop).
"""
import hashlib

import numpy as np
import pytest

import oracle as O
import refcases

Q4_0, Q8_0, Q4_K = O.GGUF_Q4_0, O.GGUF_Q8_0, O.GGUF_Q4_K


def test_tensor_byte_size_known_answers():
    # rce-ingest-gguf/src/dequant.rs:707-737
    assert O.tensor_byte_size(O.GGUF_F32, 100) == 400
    assert O.tensor_byte_size(Q4_K, 256) == 144
    assert O.tensor_byte_size(Q4_K, 257) == 288
    assert O.tensor_byte_size(Q8_0, 32) == 34
    assert O.tensor_byte_size(Q4_0, 33) == 36


def test_dequant_q8_0_roundtrip_const_scale():
    # rce-ingest-gguf/src/dequant.rs:747-765
    b = np.zeros(34, dtype=np.uint8)
    b[0:2] = np.array([1.0], dtype=np.float16).view(np.uint8)
    for i in range(32):
        b[2 + i] = np.uint8(np.int8(np.int64(i * 2).astype(np.int8)).view(np.uint8))
    out = O.dequant(b, Q8_0, 32)
    want = np.array([np.float32(np.int8(i * 2)) for i in range(32)], dtype=np.float32)
    assert np.array_equal(out, want)


def test_f16_decode_exact():
    # every finite binary16 value decodes to the same f32 as numpy's exact cast
    h = np.arange(0, 1 << 16, dtype=np.uint32)
    h = h[((h >> 10) & 0x1F) != 0x1F].astype(np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([O.f16_to_f32(int(v)) for v in h[::97]], dtype=np.float32)
    assert np.array_equal(got, want[::97])


def test_round_to_f16_matches_numpy_rne():
    rng = np.random.default_rng(7)
    xs = np.concatenate([rng.standard_normal(500).astype(np.float32) * (10.0 ** rng.integers(-6, 5, 500)).astype(np.float32),
                         np.array([65519.0, 65520.0, 1e-8, -3e-6], dtype=np.float32)]).astype(np.float32)
    for x in xs:
        want = np.float32(np.float16(x))
        assert np.float32(O.round_to_f16(float(x))) == want or (np.isinf(want) and abs(x) >= 65520)


@pytest.mark.parametrize("name", ["q4_k_dequant_dot", "q4_0_dequant_dot"])
def test_matmul_matches_dequant_then_dot(name):
    # q4_k_/q4_0_matmul_matches_dequant_then_dot (rce-op-qmm/src/lib.rs:2428-2500):
    # rel err < 1e-5 against dequantize_to_f32 -> scalar dot
    w, dt, n, k, x = refcases.REFERENCE_CASES[name]()
    got = O.mm_1d(x[0], w, dt, n, k)
    deq = O.dequant(w, dt, n * k).reshape(n, k)
    for j in range(n):
        acc = np.float32(0)
        for i in range(k):
            acc = np.float32(acc + np.float32(x[0, i] * deq[j, i]))
        rel = abs(got[j] - acc) / max(abs(acc), 1e-6)
        assert rel < 1e-5, (j, got[j], acc, rel)


def test_q8_0_matches_dequant_then_dot():
    rng = np.random.default_rng(11)
    n, k = 7, 256
    w, _, _, _, x = refcases.seeded_case(Q8_0, n, k, 1, 11)
    got = O.mm_1d(x[0], w, Q8_0, n, k)
    deq = O.dequant(w, Q8_0, n * k).reshape(n, k)
    want = (deq.astype(np.float64) @ x[0].astype(np.float64))
    assert np.allclose(got, want, rtol=1e-5, atol=1e-5)
    del rng


def test_mm_batched_byte_identical_to_per_row():
    # mm_batched_byte_identical_to_per_row_for_q5k_and_q4k (lib.rs:2575-2616)
    w, dt, n, k, x = refcases.batched_q4_k()
    t = x.shape[0]
    got = O.mm_batched(x, t, w, dt, n, k)
    for r in range(t):
        assert np.array_equal(got[r].view(np.uint32), O.mm_1d(x[r], w, dt, n, k).view(np.uint32))


def test_vm_fixture_python_restatement_bit_exact():
    # the fixture of qmm_executes_through_rce_vm_bit_exact (lib.rs:2267-2333)
    w, dt, n, k, x = refcases.vm_bit_exact_q4_0()
    got = O.mm_1d(x[0], w, dt, n, k)
    want = O.py_mm_1d(x[0], w, dt, n, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("dt", [Q8_0, Q4_0, Q4_K])
def test_python_restatement_bit_exact(dt):
    n, k = 3, 512
    w, _, _, _, x = refcases.seeded_case(dt, n, k, 1, 5)
    got = O.mm_1d(x[0], w, dt, n, k)
    want = O.py_mm_1d(x[0], w, dt, n, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("dt", [Q8_0, Q4_0, Q4_K])
def test_spec_order_kernel_bit_exact(dt):
    # spec/RCE-SPEC.md:2517-2533: matmul_q8_0 / matmul_q4_0 / matmul_q4_k
    # (rce-vm-backend-cpu/src/ml/nn.rs:477-517, ml/kquant.rs:81-150) equal
    # rce-op-qmm's kernels on every element (spec/checker/tests/lift_llama.rs:91-160)
    n, k, m = 24, 1024, 3
    w, _, _, _, x = refcases.seeded_case(dt, n, k, m, 13)
    got = O.mm_batched(x, m, w, dt, n, k)
    if dt == Q4_K:
        q, s, o = O.unpack_q4_k(w, n, k)
        want = O.spec_matmul_q4k(x, q, s, o)
    elif dt == Q8_0:
        q, d = O.unpack_q8_0(w, n, k)
        want = O.spec_matmul_q(x, q, d, q4=False)
    else:
        q, d = O.unpack_q4_0(w, n, k)
        want = O.spec_matmul_q(x, q, d, q4=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_dequant_equals_spec_values():
    # dequant_q4_k's value at t is s*q - o with s = d*sc, o = dmin*m (GT-10)
    n, k = 4, 768
    w, _, _, _, _ = refcases.seeded_case(Q4_K, n, k, 1, 17)
    q, s, o = O.unpack_q4_k(w, n, k)
    want = (np.repeat(s, 32, axis=1) * q.astype(np.float32)).astype(np.float32) - np.repeat(o, 32, axis=1)
    assert np.array_equal(O.dequant(w, Q4_K, n * k).reshape(n, k), want.astype(np.float32))
    for dt, unpack in ((Q8_0, O.unpack_q8_0), (Q4_0, O.unpack_q4_0)):
        w, _, _, _, _ = refcases.seeded_case(dt, n, k, 1, 19)
        q, d = unpack(w, n, k)
        want = (q.astype(np.float32) * np.repeat(d, 32, axis=1)).astype(np.float32)
        assert np.array_equal(O.dequant(w, dt, n * k).reshape(n, k), want)


def test_scale_packing_is_a_bijection():
    # q4_k_get_scale_min inverts kquant's pack_scales (kquant.rs:284-302)
    rng = np.random.default_rng(3)
    for _ in range(200):
        sc = rng.integers(0, 64, 8)
        mn = rng.integers(0, 64, 8)
        s = np.zeros(12, dtype=np.uint8)
        for j in range(4):
            s[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
            s[j + 4] = (mn[j] & 63) | ((mn[j + 4] >> 4) << 6)
            s[j + 8] = (sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4)
        for j in range(8):
            assert O.q4k_get_scale_min(s, j) == (sc[j], mn[j])


def test_threads_do_not_change_results():
    w, dt, n, k, x = refcases.seeded_case(Q4_K, 333, 512, 1, 23)
    a = O.mm_1d(x[0], w, dt, n, k, nthreads=1)
    b = O.mm_1d(x[0], w, dt, n, k, nthreads=7)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_unsupported_dtype_reports_error():
    with pytest.raises(ValueError):
        O.mm_1d(np.zeros(32, np.float32), np.zeros(64, np.uint8), 6, 1, 32)


# ---- MoE router / combine (rce-op-moe/src/lib.rs:140-204) --------------------

def test_router_returns_top_k_sorted():
    gate = refcases.router_gate_q8_0(8, 64)
    x = O.test_activations("sin", 0.013, 0.0, 64)
    idx, w = O.moe_router(x, gate, Q8_0, 8, 2, True)
    assert len(idx) == 2 and abs(float(w.sum()) - 1.0) < 1e-5
    assert w[0] >= w[1] and np.all((w >= 0) & (w <= 1)) and idx[0] != idx[1]


def test_router_top1_matches_top_k_with_k_eq_1():
    gate = refcases.router_gate_q8_0(16, 64)
    x = O.test_activations("cos", 0.017, 0.0, 64)
    logits = O.mm_1d(x, gate, Q8_0, 16, 64)
    idx, w = O.moe_router(x, gate, Q8_0, 16, 1, True)
    assert idx[0] == int(np.argmax(logits)) and abs(w[0] - 1.0) < 1e-6


def test_combine_weights_correctly():
    outs = np.stack([np.full(32, 1.0), np.full(32, 2.0), np.full(32, 3.0)]).astype(np.float32)
    got = O.moe_combine(np.array([0.5, 0.3, 0.2], np.float32), outs)
    assert np.all(np.abs(got - 1.7) < 1e-5)


def test_unnormalized_weights_can_sum_below_one():
    gate = refcases.router_gate_q8_0(32, 64)
    x = O.test_activations("sin", 0.013, 0.0, 64)
    _, w = O.moe_router(x, gate, Q8_0, 32, 2, False)
    assert 0.0 < float(w.sum()) < 1.0


def test_moe_ffn_equals_explicit_composition():
    rng = np.random.default_rng(4)
    e, d, f, t, k = 4, 256, 512, 3, 2
    from rce_b200 import synth
    gate = np.stack([synth.q4_k(f, d, rng) for _ in range(e)])
    up = np.stack([synth.q4_k(f, d, rng) for _ in range(e)])
    down = np.stack([synth.q4_k(d, f, rng) for _ in range(e)])
    x = rng.standard_normal((t, d), dtype=np.float32)
    logits = rng.standard_normal((t, e), dtype=np.float32)
    got = O.moe_ffn(x, logits, k, gate, up, down, Q4_K, f)
    for i in range(t):
        idx, wt = O.moe_softmax_topk(logits[i], k, True)
        outs = []
        for ex in idx:
            g = O.mm_1d(x[i], gate[ex], Q4_K, f, d)
            u = O.mm_1d(x[i], up[ex], Q4_K, f, d)
            h = np.array([O.silu(float(v)) for v in g], np.float32) * u
            outs.append(O.mm_1d(h.astype(np.float32), down[ex], Q4_K, d, f))
        assert np.array_equal(got[i], O.moe_combine(wt, np.stack(outs)))


def test_sigmoid_two_branches():
    # sigmoid (rce-qwen36-moe/src/lib.rs:465-467): 1 / (1 + e^-x) for x >= 0,
    # e^x / (1 + e^x) below, each step in binary32 (the exponential within
    # one unit in the last place of numpy's)
    for x in [0.0, 0.25, 3.5, 20.0, -0.25, -3.5, -20.0, -90.0]:
        xf = np.float32(x)
        if xf >= 0:
            want = np.float32(1.0) / (np.float32(1.0) + np.exp(-xf))
        else:
            e = np.exp(xf)
            want = e / (np.float32(1.0) + e)
        got = np.float32(O.sigmoid(x))
        assert abs(int(got.view(np.int32)) - int(np.float32(want).view(np.int32))) <= 1, x


def test_shared_expert_equals_explicit_composition():
    # moe_ffn_forward's shared expert (rce-qwen36-moe/src/lib.rs:694-705)
    rng = np.random.default_rng(5)
    d, f, t = 256, 512, 3
    from rce_b200 import synth
    sg, su, sd = synth.q4_k(f, d, rng), synth.q4_k(f, d, rng), synth.q4_k(d, f, rng)
    gi = (rng.standard_normal(d) * 0.1).astype(np.float32)
    x = rng.standard_normal((t, d), dtype=np.float32)
    base = rng.standard_normal((t, d), dtype=np.float32)
    got = O.moe_shared_expert(x, base, gi, sg, su, sd, Q4_K, f)
    for i in range(t):
        g = O.mm_1d(x[i], sg, Q4_K, f, d)
        u = O.mm_1d(x[i], su, Q4_K, f, d)
        h = np.array([O.silu(float(v)) for v in g], np.float32) * u
        sh = O.mm_1d(h.astype(np.float32), sd, Q4_K, d, f)
        acc = np.float32(0.0)
        for j in range(d):
            acc = np.float32(acc + np.float32(gi[j] * x[i, j]))
        alpha = np.float32(O.sigmoid(float(acc)))
        assert np.array_equal(got[i], (base[i] + alpha * sh).astype(np.float32))


# ---- quantize_block (rce-vm-backend-cpu/src/ml/nn.rs:541-563) ---------------

def test_quantize_block_known_answers():
    x = np.arange(32, dtype=np.float32) - 16.0  # amax 16 at x[0] = -16
    q, d = O.quantize_block(x, q4=False)
    assert d == np.float32(np.float16(np.float32(16.0) / np.float32(127.0)))
    assert q[0] == -127 and q[16] == 0
    q4, d4 = O.quantize_block(x, q4=True)
    assert d4 == 2.0 and q4[0] == -8 and q4[16] == 0 and q4.max() <= 7


def test_quantize_block_round_trip_error():
    rng = np.random.default_rng(9)
    for _ in range(50):
        x = rng.standard_normal(32).astype(np.float32)
        q, d = O.quantize_block(x, q4=False)
        assert np.max(np.abs(q * d - x)) <= 0.51 * abs(d) + 1e-3 * np.max(np.abs(x))


# ---- the committed golden vectors ------------------------------------------

def test_golden_reference_cases(golden):
    for name, build in refcases.REFERENCE_CASES.items():
        w, dt, n, k, x = build()
        assert np.array_equal(w, golden[f"{name}__w"])
        assert np.array_equal(x, golden[f"{name}__x"])
        y = O.mm_batched(x, x.shape[0], w, dt, n, k)
        assert np.array_equal(y.view(np.uint32), golden[f"{name}__y"].view(np.uint32))
        deq = O.dequant(w, dt, n * k).reshape(n, k)
        assert np.array_equal(deq.view(np.uint32), golden[f"{name}__deq"].view(np.uint32))


@pytest.mark.parametrize("case", refcases.SEEDED_CASES, ids=[c[0] for c in refcases.SEEDED_CASES])
def test_golden_seeded_cases(golden, case):
    name, dt, n, k, m, seed = case
    w, _, _, _, x = refcases.seeded_case(dt, n, k, m, seed)
    assert hashlib.sha256(w.tobytes()).hexdigest().encode() == golden[f"{name}__wsha"].tobytes()
    assert hashlib.sha256(x.tobytes()).hexdigest().encode() == golden[f"{name}__xsha"].tobytes()
    rows = min(n, 256)
    y = np.stack([O.mm_1d_rows(x[t], w, dt, n, k, 0, rows) for t in range(m)])
    assert np.array_equal(y.view(np.uint32), golden[f"{name}__y"][:, :rows].view(np.uint32))


# ---- Q6_K (rce-op-qmm/src/lib.rs:1667-1705, dequant.rs:658-698) --------------

def _q6k_serial_fixture():
    """mm_1d_serial_matches_parallel's Q6_K case (rce-op-qmm/src/lib.rs:
    3629-3665): k = 512, n = 7, bytes (i * 37 + 11) & 0xFF, every block's d
    patched to f16(0.05), a_i = sin(0.017 i - 0.3)."""
    k, n = 512, 7
    a = np.sin(np.arange(k, dtype=np.float32) * np.float32(0.017) - np.float32(0.3)).astype(np.float32)
    wb = ((np.arange(n * (k // 256) * 210, dtype=np.int64) * 37 + 11) & 0xFF).astype(np.uint8)
    blocks = wb.reshape(-1, 210)
    blocks[:, 208:210] = np.array([0.05], dtype=np.float16).view(np.uint8)
    return a, wb, n, k


def test_q6k_byte_size():
    assert O.tensor_byte_size(O.GGUF_Q6_K, 256) == 210
    assert O.tensor_byte_size(O.GGUF_Q6_K, 4096 * 14336) == 4096 * 14336 // 256 * 210


def test_q6k_python_restatement_bit_exact():
    # the C restatement of dot_row_q6_k against the spec-order pure-Python
    # one (tensor.matmul_q6_k: per half, l = 0..31, positions l, l+32, l+64,
    # l+96; y += (s * q) * x), bit for bit, on the reference test's fixture
    a, wb, n, k = _q6k_serial_fixture()
    got = O.mm_1d(a, wb, O.GGUF_Q6_K, n, k)
    want = O.py_mm_1d(a, wb, O.GGUF_Q6_K, n, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # serial (1 thread) == row-parallel (7 threads), as the reference asserts
    par = O.mm_1d(a, wb, O.GGUF_Q6_K, n, k, nthreads=7)
    assert np.array_equal(got.view(np.uint32), par.view(np.uint32))


def test_q6k_dequant_equals_spec_values():
    # dequant_q6_k's (d * sc) * q equals s * q of the independent unpacking
    # (s = d * sc exact), bit for bit, and the matmul agrees with
    # dequantise-then-dot to f32 rounding
    rng = np.random.default_rng(14)
    from rce_b200 import synth

    n, k = 24, 1024
    wb = synth.weights(O.GGUF_Q6_K, n, k, rng)
    deq = O.dequant(wb, O.GGUF_Q6_K, n * k).reshape(n, k)
    q, s = O.unpack_q6_k(wb, n, k)
    assert np.array_equal(deq.view(np.uint32), (np.repeat(s, 16, axis=1) * q.astype(np.float32)).view(np.uint32))
    x = synth.activations(1, k, rng)[0]
    got = O.mm_1d(x, wb, O.GGUF_Q6_K, n, k)
    want = deq.astype(np.float64) @ x.astype(np.float64)
    assert np.abs(got - want).max() / np.abs(want).max() < 1e-5


def test_q6k_code_layout_known_answers():
    # one block by hand: value 128 o + 32 q + l takes ql[64 o + 32 (q & 1) + l]
    # (low nibble for q < 2) and bits 2q of qh[32 o + l]; value = d * sc * (code - 32)
    blk = np.zeros(210, np.uint8)
    blk[208:210] = np.array([1.0], dtype=np.float16).view(np.uint8)
    blk[192:208] = np.arange(1, 17, dtype=np.int8).view(np.uint8)  # scale j = j + 1
    blk[5] = 0x3A          # ql[5]: low nibble 0xA -> value 5, high nibble 3 -> value 69
    blk[128 + 5] = 0b10_01_11_00  # qh[5]: value 5 hi 0, value 37 hi 3, value 69 hi 1, value 101 hi 2
    blk[64 + 32 + 7] = 0xF0  # ql[103]: high nibble 15 -> value 128 + 96 + 7 = 231
    blk[128 + 32 + 7] = 0xC0  # qh[39]: value 231 hi 3
    d = O.dequant(blk, O.GGUF_Q6_K, 256)
    assert d[5] == 1 * (0xA - 32)            # scale 0 (values 0..15) = 1
    assert d[37] == 3 * (((3 << 4) | 0) - 32)  # ql[37] = 0 low nibble, hi 3; scale 2 = 3
    assert d[69] == 5 * (((1 << 4) | 3) - 32)  # scale 4 = 5
    assert d[101] == 7 * (((2 << 4) | 0) - 32)  # scale 6 = 7
    assert d[231] == 15 * (((3 << 4) | 15) - 32)  # scale 14 = 15
    assert d[0] == 1 * (0 - 32)


# ---- Q5_K (rce-op-qmm/src/lib.rs:783-832, dequant.rs:606-656) ----------------

def test_q5k_restatements_bit_exact():
    # mm_1d_serial_matches_parallel's Q5_K case (lib.rs:3629-3665: k = 512,
    # n = 7, bytes (i * 37 + 11) & 0xFF, d and dmin patched to f16(0.05)):
    # the C restatement against the spec-order Python one (tensor.matmul_q5_k
    # = matmul_q4_k's order with codes 0..31), and serial == row-parallel
    k, n = 512, 7
    a = np.sin(np.arange(k, dtype=np.float32) * np.float32(0.017) - np.float32(0.3)).astype(np.float32)
    wb = ((np.arange(n * (k // 256) * 176, dtype=np.int64) * 37 + 11) & 0xFF).astype(np.uint8)
    blocks = wb.reshape(-1, 176)
    sc = np.array([0.05], dtype=np.float16).view(np.uint8)
    blocks[:, 0:2] = sc
    blocks[:, 2:4] = sc
    got = O.mm_1d(a, wb, O.GGUF_Q5_K, n, k)
    assert np.array_equal(got.view(np.uint32), O.py_mm_1d(a, wb, O.GGUF_Q5_K, n, k).view(np.uint32))
    assert np.array_equal(got.view(np.uint32), O.mm_1d(a, wb, O.GGUF_Q5_K, n, k, nthreads=7).view(np.uint32))


def test_q5k_dequant_equals_spec_values():
    from rce_b200 import synth

    rng = np.random.default_rng(13)
    n, k = 24, 1024
    wb = synth.weights(O.GGUF_Q5_K, n, k, rng)
    deq = O.dequant(wb, O.GGUF_Q5_K, n * k).reshape(n, k)
    q, s, o = O.unpack_q5_k(wb, n, k)
    spec = (np.repeat(s, 32, axis=1) * q.astype(np.float32)).astype(np.float32) - np.repeat(o, 32, axis=1)
    assert np.array_equal(deq.view(np.uint32), spec.astype(np.float32).view(np.uint32))
    assert q.min() >= 0 and q.max() == 31
    x = synth.activations(1, k, rng)[0]
    got = O.mm_1d(x, wb, O.GGUF_Q5_K, n, k)
    want = deq.astype(np.float64) @ x.astype(np.float64)
    assert np.abs(got - want).max() / np.abs(want).max() < 1e-5
