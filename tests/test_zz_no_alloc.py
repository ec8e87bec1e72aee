"""rce_qmm_mm_batched_device_noalloc: the decode matmul for callers that may
not allocate device memory (every batch through the decode GEMV, which needs
no device workspace).  Called through the C ABI and checked against the
regular device entry point, with the tolerance of the other parity tests, on
two calls in a row.

This file is named to be collected last, so a run that stops at the first
failure has run every other test before it.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
import refcases

pytestmark = pytest.mark.gpu


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


# shapes with few row blocks (clusters of one or two tiles) and batches above
# the GEMV's 4-token pass, one above the GEMM threshold
@pytest.mark.parametrize("dt,n,k,m", [(O.GGUF_Q4_K, 1024, 4096, 1), (O.GGUF_Q4_K, 1024, 4096, 5),
                                      (O.GGUF_Q8_0, 700, 4096, 3), (O.GGUF_Q4_0, 512, 11008, 17),
                                      (O.GGUF_Q6_K, 1024, 4096, 3), (O.GGUF_Q5_K, 1024, 4096, 5)])
def test_noalloc_matches_regular_entry_point(dt, n, k, m):
    import torch

    import rce_b200 as R
    from rce_b200 import _lib

    L = _lib.lib()
    ctx = R.default_context(0)
    wb, _, _, _, x = refcases.seeded_case(dt, n, k, m, 900 + m)
    w = R.QuantWeight.from_owned_bytes(wb, dt, n, k, ctx=ctx)
    xd = torch.from_numpy(x).cuda()
    stream = torch.cuda.current_stream()
    saved = ctx.prefill_min_tokens
    ctx.prefill_min_tokens = 0  # the regular entry point's decode path, which this one mirrors
    try:
        want = R.mm_batched_device(xd, w).cpu().numpy()
    finally:
        ctx.prefill_min_tokens = saved
    for call in range(2):
        out = torch.full((m, n), float("nan"), device="cuda:0")
        rc = _noalloc(L, ctx, xd, w, out, stream)
        assert rc == 0, L.rce_qmm_last_error()
        torch.cuda.synchronize()
        code = ctypes.c_int()
        assert L.rce_qmm_device_error(ctx.handle, ctypes.byref(code), 1) == 0 and code.value == 0
        _assert_close(out.cpu().numpy(), want)
        # the same GEMV with the same plan: bit for bit
        assert np.array_equal(out.cpu().numpy(), want)

