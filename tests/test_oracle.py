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
