"""GPU parity of the decode GEMV / matmul path against the oracle, through the
C-ABI (librce_qmm.so).

Tolerances (from the path's contract): dequantised values bit-exact; final
f32 outputs within a max normwise relative error of 1e-3 per output row
(max_i |got_i - want_i| / max_i |want_i|), and every element within
abs < 1e-4 or rel < 1e-3 (the reference's GPU tolerance idiom,
rce-op-qmm-metal/src/lib.rs:874).  The GEMV keeps ~22 significant bits of x
and exact weights, so it lands far inside both.
"""
import numpy as np
import pytest

import oracle as O
import refcases
import rce_b200 as R

pytestmark = pytest.mark.gpu

Q4_0, Q8_0, Q4_K = O.GGUF_Q4_0, O.GGUF_Q8_0, O.GGUF_Q4_K
NORM_TOL = 1e-3


def norm_rel_err(got, want):
    got = np.asarray(got, np.float64).reshape(-1, np.asarray(want).shape[-1])
    want = np.asarray(want, np.float64).reshape(got.shape)
    err = np.abs(got - want).max(axis=1)
    scale = np.maximum(np.abs(want).max(axis=1), 1e-30)
    return float((err / scale).max())


def assert_close(got, want, tol=NORM_TOL, elementwise=True):
    """Normwise bar always; the per-element idiom for the exact decode path
    (the fp16 prefill GEMM is held to the normwise bar only)."""
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert np.all(np.isfinite(got))
    e = norm_rel_err(got, want)
    assert e <= tol, f"normwise relative error {e:.3e} > {tol}"
    if elementwise:
        d = np.abs(got.astype(np.float64) - want.astype(np.float64))
        ok = (d < 1e-4) | (d <= 1e-3 * np.abs(want.astype(np.float64)))
        assert ok.all(), f"{(~ok).sum()} elements outside abs<1e-4||rel<1e-3; worst {d.max():.3e}"
    return e


def exact_path(ctx, m):
    """True when a batch of m tokens takes the exact decode path."""
    return ctx.prefill_min_tokens == 0 or m < ctx.prefill_min_tokens


def register(ctx, w, dt, n, k):
    return R.QuantWeight.from_owned_bytes(w, dt, n, k, ctx=ctx)


@pytest.mark.parametrize("name", list(refcases.REFERENCE_CASES))
def test_reference_fixtures(ctx, golden, name):
    w = golden[f"{name}__w"]
    x = golden[f"{name}__x"]
    dt, n, k, t = (int(v) for v in golden[f"{name}__shape"])
    qw = register(ctx, w, dt, n, k)
    got = R.mm_batched(x, t, qw).reshape(t, n)
    assert_close(got, golden[f"{name}__y"])
    # dequant_row: bit-exact with dequantize_to_f32
    for r in range(n):
        assert np.array_equal(qw.dequant_row(r).view(np.uint32), golden[f"{name}__deq"][r].view(np.uint32))
    # the device copy holds the GGUF bytes bit for bit
    assert np.array_equal(qw.read_device_bytes(), w)


def test_qmm_leaf_bit_identical_to_mm_1d(ctx, golden):
    # qmm_executes_through_rce_vm_bit_exact (rce-op-qmm/src/lib.rs:2267-2333)
    w = golden["vm_bit_exact_q4_0__w"]
    x = golden["vm_bit_exact_q4_0__x"][0]
    qw = register(ctx, w, Q4_0, 5, 64)
    leaf = R.QmmLeaf()
    leaf.register(1, qw)
    got = leaf.execute(1, "qmm", [x.reshape(1, 64)])
    want = R.mm_1d(x, qw)
    assert got.shape == (1, 5)
    assert np.array_equal(got[0].view(np.uint32), want.view(np.uint32))
    assert np.array_equal(R.CudaQmm().qmm_1d(x, qw).view(np.uint32), want.view(np.uint32))
    assert np.array_equal(R.mm_1d_serial(x, qw).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("case", refcases.SEEDED_CASES, ids=[c[0] for c in refcases.SEEDED_CASES])
def test_seeded_configs_against_golden(ctx, golden, case):
    name, dt, n, k, m, seed = case
    w, _, _, _, x = refcases.seeded_case(dt, n, k, m, seed)
    qw = register(ctx, w, dt, n, k)
    got = R.mm_batched(x, m, qw).reshape(m, n)
    e = assert_close(got, golden[f"{name}__y"], elementwise=exact_path(ctx, m))
    print(f"{name}: normwise rel err {e:.3e}")


@pytest.mark.parametrize("dt", [Q8_0, Q4_0, Q4_K])
def test_batched_is_bit_identical_to_per_row(ctx, dt):
    # mm_batched ≡ T × mm_1d bit for bit (rce-op-qmm/src/lib.rs:2575-2616)
    n, k, t = 200, 1024, 21
    w, _, _, _, x = refcases.seeded_case(dt, n, k, t, 31)
    qw = register(ctx, w, dt, n, k)
    saved = ctx.prefill_min_tokens
    ctx.prefill_min_tokens = 0  # every batch on the exact decode path
    try:
        got = R.mm_batched(x, t, qw).reshape(t, n)
        for r in range(t):
            assert np.array_equal(got[r].view(np.uint32), R.mm_1d(x[r], qw).view(np.uint32)), r
        again = R.mm_batched(x, t, qw).reshape(t, n)
        assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    finally:
        ctx.prefill_min_tokens = saved


@pytest.mark.parametrize("dt", [Q8_0, Q4_0, Q4_K])
@pytest.mark.parametrize("n", [1, 5, 16, 17, 33, 100])
def test_ragged_rows(ctx, dt, n):
    k = 512
    w, _, _, _, x = refcases.seeded_case(dt, n, k, 3, 100 + n)
    qw = register(ctx, w, dt, n, k)
    got = R.mm_batched(x, 3, qw).reshape(3, n)
    assert_close(got, O.mm_batched(x, 3, w, dt, n, k))


@pytest.mark.parametrize("dt,k", [(Q8_0, 32), (Q8_0, 96), (Q8_0, 288), (Q4_0, 32), (Q4_0, 160), (Q4_0, 11008),
                                  (Q4_K, 256), (Q4_K, 768), (Q4_K, 14336)])
def test_ragged_columns(ctx, dt, k):
    n = 48
    w, _, _, _, x = refcases.seeded_case(dt, n, k, 2, k)
    qw = register(ctx, w, dt, n, k)
    got = R.mm_batched(x, 2, qw).reshape(2, n)
    assert_close(got, O.mm_batched(x, 2, w, dt, n, k))


@pytest.mark.parametrize("dt", [Q8_0, Q4_0, Q4_K])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 9, 16, 17, 40])
def test_token_counts(ctx, dt, m):
    n, k = 96, 1024
    w, _, _, _, x = refcases.seeded_case(dt, n, k, m, 7 * m)
    qw = register(ctx, w, dt, n, k)
    got = R.mm_batched(x, m, qw).reshape(m, n)
    assert_close(got, O.mm_batched(x, m, w, dt, n, k), elementwise=exact_path(ctx, m))


@pytest.mark.parametrize("dt", [Q8_0, Q4_0, Q4_K])
def test_dequant_bit_exact_full(ctx, dt):
    n, k = 77, 2048
    w, _, _, _, _ = refcases.seeded_case(dt, n, k, 1, 55)
    qw = register(ctx, w, dt, n, k)
    dev = R.dequant_device(qw).cpu().numpy()
    assert np.array_equal(dev.view(np.uint32), O.dequant(w, dt, n * k).reshape(n, k).view(np.uint32))
    assert np.array_equal(qw.read_device_bytes(), w)


def test_activation_range_extremes(ctx):
    # power-of-two pre-scaling keeps tiny and huge activations exact enough
    n, k = 64, 1024
    for s in (1e-20, 1e-6, 1e4, 1e12):
        w, _, _, _, x = refcases.seeded_case(Q4_K, n, k, 1, 3)
        x = (x * np.float32(s)).astype(np.float32)
        qw = register(ctx, w, Q4_K, n, k)
        assert_close(R.mm_1d(x[0], qw), O.mm_1d(x[0], w, Q4_K, n, k))
    # a zero activation gives exact zeros
    assert np.all(R.mm_1d(np.zeros(k, np.float32), qw) == 0)


def test_sub_view_experts(ctx):
    e, n, k = 4, 48, 512
    rng = np.random.default_rng(8)
    from rce_b200 import synth
    stacked = np.concatenate([synth.q4_k(n, k, rng) for _ in range(e)])
    x = rng.standard_normal(k, dtype=np.float32)
    full = register(ctx, stacked, Q4_K, e * n, k)
    bpe = stacked.size // e
    for i in range(e):
        v = full.sub_view(i * bpe, bpe, n, k)
        want = O.mm_1d(x, stacked[i * bpe:(i + 1) * bpe], Q4_K, n, k)
        assert_close(R.mm_1d(x, v), want)
        assert np.array_equal(v.read_device_bytes(), stacked[i * bpe:(i + 1) * bpe])
    with pytest.raises(R.Unsupported):
        full.sub_view(8 * 144 * 2, 16 * 144 * 2, 16, k)  # starts at row 8


def test_errors_are_reported(ctx):
    from rce_b200 import _lib
    w = np.zeros(18 * 4, np.uint8)
    with pytest.raises(R.QmmError):
        R.QuantWeight.from_owned_bytes(w[:-1], Q4_0, 2, 64, ctx=ctx)  # wrong byte count
    with pytest.raises(R.QmmError):
        R.QuantWeight.from_owned_bytes(w, Q4_0, 4, 48, ctx=ctx)  # n_cols not a multiple of 32
    with pytest.raises(R.QmmError):
        R.QuantWeight.from_owned_bytes(np.zeros(144, np.uint8), Q4_K, 2, 128, ctx=ctx)  # K % 256 != 0
    with pytest.raises(R.Unsupported):
        R.QuantWeight.from_owned_bytes(np.zeros(64, np.uint8), 6, 1, 32, ctx=ctx)
    qw = register(ctx, np.zeros(18 * 2, np.uint8), Q4_0, 1, 64)
    with pytest.raises(ValueError):
        R.mm_1d(np.zeros(32, np.float32), qw)
    assert _lib.RCE_QMM_ERR_INVALID == 1


@pytest.mark.parametrize("dt,n,k,seed", [(Q8_0, 4096, 4096, 0), (Q4_0, 11008, 4096, 1), (Q4_0, 4096, 11008, 1),
                                         (Q4_K, 14336, 4096, 2), (Q4_K, 4096, 14336, 3)])
def test_full_size_decode_against_oracle(ctx, dt, n, k, seed):
    rng = np.random.default_rng(seed)
    from rce_b200 import synth
    w = synth.weights(dt, n, k, rng)
    x = synth.activations(1, k, rng)
    qw = register(ctx, w, dt, n, k)
    got = R.mm_1d(x[0], qw)
    want = O.mm_1d(x[0], w, dt, n, k, nthreads=8)
    e = assert_close(got, want)
    print(f"dtype {dt} {n}x{k}: normwise rel err {e:.3e}")


def test_device_path_and_strided_rows(ctx):
    import torch
    n, k, m = 300, 4096, 6
    w, _, _, _, x = refcases.seeded_case(Q4_K, n, k, m, 77)
    qw = register(ctx, w, Q4_K, n, k)
    assert exact_path(ctx, m)
    xb = torch.zeros((m, k + 64), dtype=torch.float32, device="cuda:0")
    xb[:, :k] = torch.from_numpy(x).cuda()
    out = torch.full((m, n + 3), float("nan"), device="cuda:0")
    R.mm_batched_device(xb[:, :k], qw, out[:, :n])
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert np.all(np.isnan(o[:, n:]))
    assert_close(o[:, :n], O.mm_batched(x, m, w, Q4_K, n, k))


def test_host_calls_replay_and_never_reuse_a_freed_weights_graph(ctx):
    # host-buffer decode calls are replayed from a per-thread cache of CUDA
    # graphs keyed by weight handle serial: repeated calls give the same bits,
    # a weight freed and another registered (often at the same handle
    # address) gets its own results, and growing the staging buffers (a
    # larger matrix) drops the cache without changing any result
    from rce_b200 import synth

    rng = np.random.default_rng(91)
    n, k = 512, 1024
    x = rng.standard_normal((1, k), dtype=np.float32)
    for _ in range(3):
        wb = synth.q4_k(n, k, rng)
        qw = register(ctx, wb, Q4_K, n, k)
        first = R.mm_1d(x[0], qw)
        assert_close(first, O.mm_batched(x, 1, wb, Q4_K, n, k))
        for _ in range(3):
            assert np.array_equal(R.mm_1d(x[0], qw).view(np.uint32), first.view(np.uint32))
        qw.close()
    big_b = synth.q4_k(4096, 4096, rng)
    big = register(ctx, big_b, Q4_K, 4096, 4096)
    xb = rng.standard_normal((2, 4096), dtype=np.float32)
    assert_close(R.mm_batched(xb, 2, big).reshape(2, 4096), O.mm_batched(xb, 2, big_b, Q4_K, 4096, 4096, nthreads=8))
    wb = synth.q4_k(n, k, rng)
    qw = register(ctx, wb, Q4_K, n, k)
    assert_close(R.mm_1d(x[0], qw), O.mm_batched(x, 1, wb, Q4_K, n, k))
