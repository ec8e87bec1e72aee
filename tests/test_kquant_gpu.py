"""Q5_K and Q6_K on the B200 against the oracle's restatements of
mm_1d_q5_k / dequant_q5_k (rce-op-qmm/src/lib.rs:783-832,
rce-ingest-gguf/src/dequant.rs:606-656) and mm_1d_q6_k / dequant_q6_k
(lib.rs:1667-1705, dequant.rs:658-698).  Q5_K runs through the cluster GEMV's
exact integer path (Q4_K's, with a fifth bit per code); Q6_K through its own
GEMV (qmm_q6k.cu); both through the tcgen05 GEMM from 16 tokens on.

Bars:
- the device copy of the GGUF bytes and the dequantised values: bit-exact;
- decode GEMV (batches below prefill_min_tokens): per output row
  max|got - want| / max|want| <= 1e-3 (Q5_K sums exactly; Q6_K sums the
  exact codes times the f32 activations in f32: both land near 1e-6); Q5_K
  also holds the element-wise idiom (abs < 1e-4 or rel < 1e-3) against the
  exact sum (the reference's own f32 sums do not hold it everywhere at the
  largest shapes); a batch gives, row for row, the bits of one-token calls;
- tensor-core GEMM (16 tokens and more): the same normwise bar over the whole
  output, and within 2.5e-4 of a model of its operands with exact
  accumulation (gemm_operand_model).
The allocation-free entry point's Q6_K case is in test_zz_no_alloc.py.
"""
import numpy as np
import pytest

import oracle as O
import rce_b200 as R
from rce_b200 import synth

pytestmark = pytest.mark.gpu

Q5_K, Q6_K = O.GGUF_Q5_K, O.GGUF_Q6_K
KQ = [Q5_K, Q6_K]


def _rel(got, want):
    got = np.asarray(got, np.float64).reshape(want.shape)
    return float((np.abs(got - want).max(axis=-1) / np.abs(want).max(axis=-1)).max())


@pytest.mark.parametrize("dt", KQ)
@pytest.mark.parametrize("n,k", [(16, 256), (37, 512), (300, 768), (1024, 4096)])
def test_register_read_back_and_dequant_bit_exact(ctx, dt, n, k):
    w = synth.weights(dt, n, k, np.random.default_rng(n + k))
    qw = R.QuantWeight.from_owned_bytes(w, dt, n, k, ctx=ctx)
    assert np.array_equal(qw.read_device_bytes(), w)
    deq = O.dequant(w, dt, n * k).reshape(n, k)
    for r in (0, n // 2, n - 1):
        assert np.array_equal(qw.dequant_row(r).view(np.uint32), deq[r].view(np.uint32))


@pytest.mark.parametrize("dt", KQ)
@pytest.mark.parametrize("n,k,m", [(16, 256, 1), (37, 512, 1), (300, 768, 2), (1024, 4096, 3), (4096, 14336, 1),
                                   (14336, 4096, 5), (200, 1024, 15)])
def test_decode_gemv_against_oracle(ctx, dt, n, k, m):
    rng = np.random.default_rng(1000 + n + m)
    w = synth.weights(dt, n, k, rng)
    x = synth.activations(m, k, rng)
    qw = R.QuantWeight.from_owned_bytes(w, dt, n, k, ctx=ctx)
    got = R.mm_batched(x, m, qw).reshape(m, n)
    want = O.mm_batched(x, m, w, dt, n, k, nthreads=8).reshape(m, n).astype(np.float64)
    err = _rel(got, want)
    print(f"dtype {dt} GEMV {n}x{k} m={m}: normwise {err:.2e}")
    assert np.all(np.isfinite(got))
    assert err <= 1e-3
    if dt == Q5_K:
        # the element-wise idiom, against the exact sum of the dequantised
        # weights times x (what the integer path computes): the reference's
        # own f32 sums miss it by up to ~1e-3 at these sizes (4096 x 14336:
        # 2 of 4096 outputs outside abs 1e-4 / rel 1e-3 of the exact value)
        exact = x.astype(np.float64) @ O.dequant(w, dt, n * k).reshape(n, k).astype(np.float64).T
        d = np.abs(got - exact)
        assert ((d < 1e-4) | (d <= 1e-3 * np.abs(exact))).all()
    # batch rows are the bits of one-token calls
    for t in (0, m - 1):
        one = R.mm_batched(x[t:t + 1], 1, qw)
        assert np.array_equal(one.view(np.uint32), got[t].view(np.uint32))
    assert ctx.device_error() == 0


def gemm_operand_model(dt, w, x, n, k):
    """The GEMM's operands with exact accumulation: x scaled by a power of two
    per token and rounded to fp16 (plus the fp16 rounding of the remainder for
    batches of up to 64 tokens); Q5_K weights d * (sc * q) - fp16(dmin * m)
    rounded once to fp16, Q6_K weights their exact f32 dequantised values
    rounded to fp16."""
    m = x.shape[0]
    if dt == Q5_K:
        q, sv, ov = O.unpack_q5_k(w, n, k)
        sv = np.repeat(sv.astype(np.float64), 32, axis=1)
        ov = np.repeat(ov.astype(np.float16).astype(np.float64), 32, axis=1)
        wm = (sv * q - ov).astype(np.float16).astype(np.float64)
    else:
        wm = O.dequant(w, dt, n * k).reshape(n, k).astype(np.float16).astype(np.float64)
    e = np.frexp(np.abs(x).max(axis=1, keepdims=True))[1]
    s = np.ldexp(np.float32(1.0), 14 - e).astype(np.float32)
    v = x * s
    hi = v.astype(np.float16)
    xm = hi.astype(np.float64)
    if m <= 64:
        xm = xm + (v - hi.astype(np.float32)).astype(np.float16).astype(np.float64)
    return (xm / s) @ wm.T


@pytest.mark.parametrize("dt", KQ)
@pytest.mark.parametrize("n,k,m", [(1024, 4096, 16), (2048, 4096, 128), (1024, 14336, 64), (512, 2048, 300),
                                   (2048, 4096, 384), (256, 1024, 520)])
def test_prefill_gemm_against_oracle(ctx, dt, n, k, m):
    rng = np.random.default_rng(2000 + m)
    w = synth.weights(dt, n, k, rng)
    x = synth.activations(m, k, rng)
    qw = R.QuantWeight.from_owned_bytes(w, dt, n, k, ctx=ctx)
    assert ctx.prefill_min_tokens == 16
    got = R.mm_batched(x, m, qw).reshape(m, n).astype(np.float64)
    want = O.mm_batched(x, m, w, dt, n, k, nthreads=8).reshape(m, n).astype(np.float64)
    scale = np.abs(want).max()
    tensor = np.abs(got - want).max() / scale
    model = gemm_operand_model(dt, w, x, n, k)
    vs_model = np.abs(got - model).max() / scale
    print(f"dtype {dt} GEMM {n}x{k} m={m}: max-norm {tensor:.2e}, vs the fp16-operand model {vs_model:.2e}")
    assert tensor <= 1e-3
    assert vs_model <= 2.5e-4
    assert ctx.device_error() == 0


@pytest.mark.parametrize("dt", KQ)
def test_unaligned_and_strided_activations(ctx, dt):
    import torch

    # x rows at an odd float offset (no 16-byte alignment): the scalar loads
    n, k, m = 512, 1024, 2
    rng = np.random.default_rng(78)
    w = synth.weights(dt, n, k, rng)
    qw = R.QuantWeight.from_owned_bytes(w, dt, n, k, ctx=ctx)
    big = torch.from_numpy(synth.activations(m, k + 3, rng)).cuda()
    x = big[:, 1:1 + k]
    got = R.mm_batched_device(x, qw)
    torch.cuda.synchronize()
    want = O.mm_batched(np.ascontiguousarray(x.cpu().numpy()), m, w, dt, n, k).reshape(m, n).astype(np.float64)
    assert _rel(got.cpu().numpy(), want) <= 1e-3


@pytest.mark.parametrize("dt", KQ)
def test_moe_with_kquant_experts(ctx, dt):
    import torch

    # experts of one K format through the grouped tensor-core path
    n_e, top_k, d_model, d_ff, t = 4, 2, 256, 512, 40
    rng = np.random.default_rng(79)
    gate = [synth.weights(dt, d_ff, d_model, rng) for _ in range(n_e)]
    up = [synth.weights(dt, d_ff, d_model, rng) for _ in range(n_e)]
    down = [synth.weights(dt, d_model, d_ff, rng) for _ in range(n_e)]
    x = synth.activations(t, d_model, rng)
    logits = rng.standard_normal((t, n_e)).astype(np.float32)
    want = O.moe_ffn(x, logits, top_k, np.stack(gate), np.stack(up), np.stack(down), dt, d_ff, nthreads=8)
    g = [R.QuantWeight.from_owned_bytes(b, dt, d_ff, d_model, ctx=ctx) for b in gate]
    u = [R.QuantWeight.from_owned_bytes(b, dt, d_ff, d_model, ctx=ctx) for b in up]
    d = [R.QuantWeight.from_owned_bytes(b, dt, d_model, d_ff, ctx=ctx) for b in down]
    got = R.moe_ffn_device(torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda(), top_k, g, u, d)
    torch.cuda.synchronize()
    err = np.abs(got.cpu().numpy() - want).max() / np.abs(want).max()
    print(f"MoE dtype {dt} grouped: max-norm {err:.2e}")
    assert err <= 1e-3
    assert ctx.device_error() == 0


def test_grouped_decode_q5k(ctx):
    import torch

    # Q5_K through the grouped GEMV (two weights sharing x, one launch):
    # each output the bits of its own call
    rng = np.random.default_rng(80)
    k = 2048
    ws = [synth.weights(Q5_K, n, k, rng) for n in (1024, 512)]
    qs = [R.QuantWeight.from_owned_bytes(w, Q5_K, n, k, ctx=ctx) for w, n in zip(ws, (1024, 512))]
    x = torch.from_numpy(synth.activations(3, k, rng)).cuda()
    outs = R.mm_multi_device(x, qs)
    singles = [R.mm_batched_device(x, q) for q in qs]
    torch.cuda.synchronize()
    for a, b in zip(outs, singles):
        assert np.array_equal(a.cpu().numpy().view(np.uint32), b.cpu().numpy().view(np.uint32))
