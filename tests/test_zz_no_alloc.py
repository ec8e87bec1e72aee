"""rce_qmm_mm_batched_device_noalloc: the matmul for callers that may not
allocate device memory (an engine whose allocator owns the whole device, a
serving loop that forbids cudaMalloc after start-up).  Its tensor-core GEMM
keeps its workspace in one fixed device array instead of memory allocated on
first use; small batches run the decode GEMV, which needs none.

Each case calls the entry point through the C ABI twice in a row, on
different inputs (the second batch smaller than the first, so stale workspace
from the first call would show), and checks both outputs against the regular
entry point rce_qmm_mm_batched_device with the tolerance of the other parity
tests, and bit for bit (same kernels, same plan).

This file is named to be collected last, so a run that stops at the first
failure has run every other test before it.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
import refcases

pytestmark = pytest.mark.gpu

RCE_QMM_ERR_INVALID = 1


def _assert_close(got, want, tol=1e-3):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert np.all(np.isfinite(got))
    err = np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)
    assert err.max() <= tol, f"normwise relative error {err.max():.3e} > {tol}"
    d = np.abs(got - want)
    assert ((d < 1e-4) | (d <= 1e-3 * np.abs(want))).all()


def _noalloc(L, ctx, x, w, out, stream):
    return L.rce_qmm_mm_batched_device_noalloc(
        ctx.handle, ctypes.c_void_p(x.data_ptr()), x.stride(0), x.shape[0], w.handle,
        ctypes.c_void_p(out.data_ptr()), out.stride(0), ctypes.c_void_p(stream.cuda_stream))


# (dtype, n, k, first batch, second batch): decode-GEMV batches (below the
# default 16-token GEMM threshold), GEMM batches (the fixed workspace), and
# one case that crosses from the GEMM to the GEMV between the two calls
@pytest.mark.parametrize("dt,n,k,m1,m2", [
    (O.GGUF_Q4_K, 1024, 4096, 5, 1),
    (O.GGUF_Q6_K, 1024, 4096, 3, 2),
    (O.GGUF_Q4_K, 1024, 4096, 130, 17),
    (O.GGUF_Q8_0, 700, 4096, 64, 16),
    (O.GGUF_Q4_0, 512, 11008, 40, 7),
    (O.GGUF_Q5_K, 1024, 4096, 33, 20),
    (O.GGUF_Q6_K, 512, 4096, 48, 16),
    (O.GGUF_Q4_K, 4096, 14336, 512, 100),
])
def test_noalloc_matches_regular_entry_point(dt, n, k, m1, m2):
    import torch

    import rce_b200 as R
    from rce_b200 import _lib

    L = _lib.lib()
    ctx = R.default_context(0)
    wb, _, _, _, x = refcases.seeded_case(dt, n, k, max(m1, m2), 900 + m1)
    w = R.QuantWeight.from_owned_bytes(wb, dt, n, k, ctx=ctx)
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(77 + m2)
    saved = ctx.prefill_min_tokens
    ctx.prefill_min_tokens = 16  # the library's default GEMM threshold
    try:
        _two_calls(L, R, ctx, w, x, n, k, (m1, m2), rng, stream)
    finally:
        ctx.prefill_min_tokens = saved


def _two_calls(L, R, ctx, w, x, n, k, ms, rng, stream):
    import torch

    for call, m in enumerate(ms):
        xs = x[:m] if call == 0 else rng.standard_normal((m, k)).astype(np.float32)
        xd = torch.from_numpy(np.ascontiguousarray(xs)).cuda()
        want = R.mm_batched_device(xd, w).cpu().numpy()
        out = torch.full((m, n), float("nan"), device="cuda:0")
        rc = _noalloc(L, ctx, xd, w, out, stream)
        assert rc == 0, L.rce_qmm_last_error()
        torch.cuda.synchronize()
        code = ctypes.c_int()
        assert L.rce_qmm_device_error(ctx.handle, ctypes.byref(code), 1) == 0 and code.value == 0
        got = out.cpu().numpy()
        _assert_close(got, want)
        assert np.array_equal(got, want), f"call {call}: m={m} not bit-identical to the regular entry point"


def test_noalloc_rejects_batches_beyond_its_workspace():
    import torch

    import rce_b200 as R
    from rce_b200 import _lib

    L = _lib.lib()
    ctx = R.default_context(0)
    n, k = 256, 4096
    wb, _, _, _, _ = refcases.seeded_case(O.GGUF_Q4_K, n, k, 1, 5)
    w = R.QuantWeight.from_owned_bytes(wb, O.GGUF_Q4_K, n, k, ctx=ctx)
    stream = torch.cuda.current_stream()
    saved = ctx.prefill_min_tokens
    ctx.prefill_min_tokens = 16
    try:
        _check_limit(L, R, ctx, w, n, k, stream)
    finally:
        ctx.prefill_min_tokens = saved


def _check_limit(L, R, ctx, w, n, k, stream):
    import torch

    # 2047 tokens at k = 4096 fit the 16 MiB workspace; 2048 do not
    for m, ok in ((2047, True), (2048, False)):
        xd = torch.randn(m, k, device="cuda:0")
        out = torch.zeros(m, n, device="cuda:0")
        rc = _noalloc(L, ctx, xd, w, out, stream)
        if ok:
            assert rc == 0, L.rce_qmm_last_error()
            torch.cuda.synchronize()
            want = R.mm_batched_device(xd, w)
            assert torch.equal(out, want)
        else:
            assert rc == RCE_QMM_ERR_INVALID
            msg = L.rce_qmm_last_error()
            msg = msg.decode() if isinstance(msg, bytes) else str(msg)
            assert "workspace" in msg and "2047 tokens" in msg, msg


def _new_stream():
    """A CUDA stream created here, so that no earlier call of this library has
    used its handle (torch.cuda.Stream() recycles a fixed pool)."""
    import torch
    from cuda.bindings import runtime as cudart

    err, s = cudart.cudaStreamCreate()
    assert err == cudart.cudaError_t.cudaSuccess
    return torch.cuda.ExternalStream(int(s))


def test_noalloc_allocates_nothing():
    # The property the entry point exists for.  On a stream it has never seen,
    # the regular entry point allocates its GEMM workspace (cudaMalloc); this
    # one must leave the device's free memory as it was.  A first call warms
    # up (it loads the module holding the fixed array and looks the array's
    # address up); the measured call runs on a new stream.
    import torch

    import rce_b200 as R
    from rce_b200 import _lib

    L = _lib.lib()
    ctx = R.default_context(0)
    n, k, m = 1024, 4096, 130
    wb, _, _, _, x = refcases.seeded_case(O.GGUF_Q4_K, n, k, m, 61)
    w = R.QuantWeight.from_owned_bytes(wb, O.GGUF_Q4_K, n, k, ctx=ctx)
    assert m >= ctx.prefill_min_tokens  # the GEMM route, the one with a workspace
    xd = torch.from_numpy(x).cuda()
    out = torch.zeros((m, n), device="cuda:0")
    want = torch.zeros((m, n), device="cuda:0")
    # a batch whose regular workspace (8 MiB) shows in the free memory
    xc = torch.randn(1024, k, device="cuda:0")
    outc = torch.zeros((1024, n), device="cuda:0")
    assert _noalloc(L, ctx, xd, w, out, torch.cuda.current_stream()) == 0, L.rce_qmm_last_error()
    torch.cuda.synchronize()
    fresh = _new_stream()
    free0 = torch.cuda.mem_get_info()[0]
    assert _noalloc(L, ctx, xd, w, out, fresh) == 0, L.rce_qmm_last_error()
    assert _noalloc(L, ctx, xc, w, outc, fresh) == 0, L.rce_qmm_last_error()
    fresh.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    # the check can see an allocation: the regular entry point on another new
    # stream allocates that stream's workspace
    other = _new_stream()
    R.mm_batched_device(xd, w, out=want, stream=other)
    R.mm_batched_device(xc, w, out=outc, stream=other)
    other.synchronize()
    assert torch.cuda.mem_get_info()[0] < free1
    assert torch.equal(out, want)


def test_noalloc_gemm_against_oracle():
    # the GEMM route at 512 tokens checked directly against the oracle (the
    # reference's f32 CPU path), with the per-row bar of the GEMM tests
    import torch

    import rce_b200 as R
    from rce_b200 import _lib

    L = _lib.lib()
    ctx = R.default_context(0)
    dt, n, k, m = O.GGUF_Q4_K, 4096, 4096, 512
    wb, _, _, _, x = refcases.seeded_case(dt, n, k, m, 512)
    w = R.QuantWeight.from_owned_bytes(wb, dt, n, k, ctx=ctx)
    xd = torch.from_numpy(x).cuda()
    out = torch.full((m, n), float("nan"), device="cuda:0")
    assert _noalloc(L, ctx, xd, w, out, torch.cuda.current_stream()) == 0, L.rce_qmm_last_error()
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    want = O.mm_batched(x, m, wb, dt, n, k, nthreads=8).astype(np.float64)
    err = np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)
    assert np.all(np.isfinite(got)) and err.max() <= 1e-3, f"per-row error {err.max():.3e}"
