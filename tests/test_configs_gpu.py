"""Parity at the benchmark configurations' full sizes, through the default
routing of mm_batched (the decode GEMV below ctx.prefill_min_tokens tokens,
the tensor-core GEMM from there on), against the oracle (the reference's f32
CPU path restated bit for bit) on the whole output.

One bar for every configuration and both paths (the path's 1e-3
max-relative-error contract for final float outputs), per output row:
max_i |got_i - want_i| / max_i |want_i| <= 1e-3 for every token row.  The
exact decode path also keeps the reference's per-element idiom
(abs < 1e-4 or rel < 1e-3, rce-op-qmm-metal/src/lib.rs:874).

Configurations (weights and activations from rce_b200.synth with the
configuration's seed, numpy PCG64):
  configs[2]  Q4_K 14336 x 4096, seed 2, M = 1, 16, 128, 512 (all 14336 rows);
  configs[3]  the Llama-3-8B-shaped layer (q, k, v, o, gate, up, down), seed 3,
              batch 16 and batch 1 (every matrix shape);
  configs[4]  the Mixtral-shaped MoE FFN: 8 experts of Q4_K gate/up 14336 x
              4096 and down 4096 x 14336, 256 tokens, top-2, seed 4.
"""
import os

import numpy as np
import pytest

import oracle as O
import rce_b200 as R
from rce_b200 import synth

pytestmark = pytest.mark.gpu

Q4_K = O.GGUF_Q4_K
BAR = 1e-3
THREADS = os.cpu_count() or 1


def row_errors(got, want):
    """Per token row: max |got - want| / max |want|."""
    got = np.asarray(got, np.float64).reshape(np.asarray(want).shape)
    want = np.asarray(want, np.float64)
    return np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)


def check_rows(got, want, label, elementwise=False):
    assert np.all(np.isfinite(got)), label
    err = row_errors(got, want)
    print(f"{label}: per-row max-norm relative error worst {err.max():.3e}, median {np.median(err):.3e}")
    assert err.max() <= BAR, f"{label}: per-row error {err.max():.3e} > {BAR}"
    if elementwise:
        d = np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64))
        ok = (d < 1e-4) | (d <= 1e-3 * np.abs(np.asarray(want, np.float64)))
        assert ok.all(), f"{label}: {(~ok).sum()} elements outside abs<1e-4||rel<1e-3"
    return float(err.max())


@pytest.fixture(scope="module")
def cfg2(ctx):
    rng = np.random.default_rng(2)
    n, k = 14336, 4096
    w = synth.weights(Q4_K, n, k, rng)
    x = synth.activations(512, k, rng)
    return w, R.QuantWeight.from_owned_bytes(w, Q4_K, n, k, ctx=ctx), x


@pytest.mark.parametrize("m", [1, 16, 128, 512])
def test_config2_prefill_whole_output(ctx, cfg2, m):
    assert ctx.prefill_min_tokens == 16  # the default routing
    w, qw, x = cfg2
    n, k = qw.n_rows, qw.n_cols
    got = R.mm_batched(x[:m], m, qw).reshape(m, n)
    assert ctx.device_error() == 0
    want = O.mm_batched(x[:m], m, w, Q4_K, n, k, nthreads=THREADS)
    check_rows(got, want, f"configs[2] Q4_K 14336x4096 M={m}", elementwise=m < 16)


LAYER = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
         ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]


@pytest.fixture(scope="module")
def cfg3(ctx):
    rng = np.random.default_rng(3)
    mats = []
    for name, n, k in LAYER:
        w = synth.weights(Q4_K, n, k, rng)
        mats.append((name, n, k, w, R.QuantWeight.from_owned_bytes(w, Q4_K, n, k, ctx=ctx)))
    xs = {4096: synth.activations(16, 4096, rng), 14336: synth.activations(16, 14336, rng)}
    return mats, xs


@pytest.mark.parametrize("batch", [1, 16])
@pytest.mark.parametrize("name", [nm for nm, _, _ in LAYER])
def test_config3_decode_layer(ctx, cfg3, batch, name):
    mats, xs = cfg3
    _, n, k, w, qw = next(m for m in mats if m[0] == name)
    x = xs[k][:batch]
    got = R.mm_batched(x, batch, qw).reshape(batch, n)
    assert ctx.device_error() == 0
    want = O.mm_batched(x, batch, w, Q4_K, n, k, nthreads=THREADS)
    check_rows(got, want, f"configs[3] {name} {n}x{k} batch {batch}", elementwise=batch < 16)


def test_config4_moe_ffn_all_tokens(ctx):
    import torch

    n_e, d_model, d_ff, t, top_k = 8, 4096, 14336, 256, 2
    rng = np.random.default_rng(4)
    gate = [synth.weights(Q4_K, d_ff, d_model, rng) for _ in range(n_e)]
    up = [synth.weights(Q4_K, d_ff, d_model, rng) for _ in range(n_e)]
    down = [synth.weights(Q4_K, d_model, d_ff, rng) for _ in range(n_e)]
    x = synth.activations(t, d_model, rng)
    logits = rng.standard_normal((t, n_e)).astype(np.float32)
    g = [R.QuantWeight.from_owned_bytes(b, Q4_K, d_ff, d_model, ctx=ctx) for b in gate]
    u = [R.QuantWeight.from_owned_bytes(b, Q4_K, d_ff, d_model, ctx=ctx) for b in up]
    d = [R.QuantWeight.from_owned_bytes(b, Q4_K, d_model, d_ff, ctx=ctx) for b in down]
    got = R.moe_ffn_device(torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda(), top_k, g, u, d)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    want = O.moe_ffn(x, logits, top_k, np.stack(gate), np.stack(up), np.stack(down), Q4_K, d_ff, nthreads=THREADS)
    check_rows(got.cpu().numpy(), want, "configs[4] Mixtral MoE FFN 256 tokens top-2")
