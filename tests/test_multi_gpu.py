"""rce_qmm_mm_batched_device_multi: 1-4 weights sharing their activations in
one decode-GEMV launch (the grid splits the weights' tiles as one matrix).
Each output against the oracle's mm_batched (rce-op-qmm/src/lib.rs:545-565)
with the decode path's bars (normwise 1e-3 and per element abs < 1e-4 or
rel < 1e-3); each token's result independent of the batch (bit for bit);
batches on the GEMM path equal to per-weight mm_batched_device calls bit for
bit; mismatched weights rejected."""
import numpy as np
import pytest

import oracle as O
import rce_b200 as R
from rce_b200 import synth

pytestmark = pytest.mark.gpu


def _close(got, want, tol=1e-3):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert np.all(np.isfinite(got))
    err = np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)
    assert err.max() <= tol, f"normwise relative error {err.max():.3e}"
    d = np.abs(got - want)
    ok = (d < 1e-4) | (d <= 1e-3 * np.abs(want))
    assert ok.all(), f"{(~ok).sum()} elements outside abs<1e-4||rel<1e-3; worst {d.max():.3e}"


CASES = [
    (O.GGUF_Q4_K, [4096, 1024, 1024], 4096),       # attention q, k, v
    (O.GGUF_Q4_K, [14336, 14336], 4096),           # FFN gate, up
    (O.GGUF_Q4_K, [1000, 48, 16, 2000], 2048),     # ragged rows, four weights
    (O.GGUF_Q8_0, [700, 300], 1024),
    (O.GGUF_Q4_0, [512, 1536, 100], 3072),
]


@pytest.mark.parametrize("dt,ns,k", CASES, ids=[f"{c[0]}-{'x'.join(map(str, c[1]))}-{c[2]}" for c in CASES])
def test_multi_matches_oracle_and_is_batch_invariant(ctx, dt, ns, k):
    import torch

    rng = np.random.default_rng(sum(ns) + k + dt)
    wb = [synth.weights(dt, n, k, rng) for n in ns]
    ws = [R.QuantWeight.from_owned_bytes(b, dt, n, k, ctx=ctx) for b, n in zip(wb, ns)]
    t = 3
    x = synth.activations(t, k, rng)
    xd = torch.from_numpy(x).cuda()
    outs = R.mm_multi_device(xd, ws)
    singles = [R.mm_multi_device(xd[i:i + 1], ws) for i in range(t)]
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    for j, (b, n) in enumerate(zip(wb, ns)):
        got = outs[j].cpu().numpy()
        want = O.mm_batched(x, t, b, dt, n, k, nthreads=8).reshape(t, n)
        _close(got, want)
        for i in range(t):  # token i alone: the same bits
            assert np.array_equal(singles[i][j].cpu().numpy()[0], got[i])


def test_multi_gemm_path_equals_single_calls(ctx):
    import torch

    assert ctx.prefill_min_tokens == 16
    dt, ns, k = O.GGUF_Q4_K, [512, 256, 128], 1024
    rng = np.random.default_rng(5)
    ws = [R.QuantWeight.from_owned_bytes(synth.weights(dt, n, k, rng), dt, n, k, ctx=ctx) for n in ns]
    xd = torch.from_numpy(synth.activations(40, k, rng)).cuda()
    outs = R.mm_multi_device(xd, ws)
    for w, o in zip(ws, outs):
        assert np.array_equal(o.cpu().numpy(), R.mm_batched_device(xd, w).cpu().numpy())


def test_multi_rejects_mismatched_weights(ctx):
    import torch

    rng = np.random.default_rng(6)
    a = R.QuantWeight.from_owned_bytes(synth.weights(O.GGUF_Q4_K, 64, 512, rng), O.GGUF_Q4_K, 64, 512, ctx=ctx)
    b = R.QuantWeight.from_owned_bytes(synth.weights(O.GGUF_Q8_0, 64, 512, rng), O.GGUF_Q8_0, 64, 512, ctx=ctx)
    c = R.QuantWeight.from_owned_bytes(synth.weights(O.GGUF_Q4_K, 64, 768, rng), O.GGUF_Q4_K, 64, 768, ctx=ctx)
    x = torch.zeros((1, 512), device="cuda:0")
    with pytest.raises(R.QmmError):
        R.mm_multi_device(x, [a, b])  # dtype differs
    with pytest.raises(ValueError):
        R.mm_multi_device(x, [a, c])  # k differs
    with pytest.raises(ValueError):
        R.mm_multi_device(x, [a] * 5)
