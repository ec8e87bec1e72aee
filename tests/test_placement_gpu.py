"""The cuda:op-qmm backend through the placement adapter on the B200: the
adapter picks it for a decode-sized Q4_K call, records the dispatch, and the
result is the library's mm_1d (rce-placement-adapter/src/lib.rs:418-480)."""
import numpy as np
import pytest

import oracle as O
import rce_b200 as R
from rce_b200 import placement as P
from rce_b200 import synth

pytestmark = pytest.mark.gpu


def test_adapter_dispatches_to_cuda(ctx):
    rng = np.random.default_rng(9)
    n, k = 4096, 4096
    w = synth.weights(O.GGUF_Q4_K, n, k, rng)
    x = synth.activations(1, k, rng)[0]
    qw = R.QuantWeight.from_owned_bytes(w, O.GGUF_Q4_K, n, k, ctx=ctx)
    ad = P.PlacementQmmAdapter.with_cuda()
    got = ad.qmm_1d(x, qw)
    assert np.array_equal(got, R.mm_1d(x, qw))
    ev = ad.transcript.events[0]
    assert ev.backend_id == "cuda:op-qmm" and ev.w_shape == [n, k, qw.nbytes(), P.QMM_DTYPE_Q4_K]
    want = O.mm_1d(x, w, O.GGUF_Q4_K, n, k, nthreads=8)
    assert np.abs(got - want).max() / np.abs(want).max() <= 1e-5


def test_split_experts_views(ctx):
    # split_experts (rce-qwen36-moe/src/lib.rs:217-223): expert e of a stacked
    # [4 * 256, 512] weight is the e-th quarter of its bytes
    rng = np.random.default_rng(10)
    stacked = synth.weights(O.GGUF_Q4_K, 4 * 256, 512, rng)
    full = R.QuantWeight.from_owned_bytes(stacked, O.GGUF_Q4_K, 4 * 256, 512, ctx=ctx)
    views = R.split_experts(full, 4, 256, 512)
    x = synth.activations(3, 512, rng)
    bpe = stacked.size // 4
    for e, v in enumerate(views):
        alone = R.QuantWeight.from_owned_bytes(stacked[e * bpe:(e + 1) * bpe], O.GGUF_Q4_K, 256, 512, ctx=ctx)
        assert np.array_equal(R.mm_batched(x, 3, v), R.mm_batched(x, 3, alone))
