"""Weights loaded from a GGUF file (QuantWeight.from_gguf, the reference's
QuantWeight::from_gguf, rce-op-qmm/src/lib.rs:173-209): the registered bytes
are the file's bytes, and the matmul of each matches the oracle; a wrong
declared shape, a missing tensor and a format this library does not compute
are errors."""
import numpy as np
import pytest

import oracle as O
import rce_b200 as R
from rce_b200 import gguf as G
from rce_b200 import synth

pytestmark = pytest.mark.gpu


def test_from_gguf_matmuls_match_oracle(ctx, tmp_path):
    rng = np.random.default_rng(12)
    # a Q4_K_M-style mix: Q4_K, Q6_K and Q5_K tensors beside Q8_0 / Q4_0
    shapes = {"blk.0.attn_q.weight": (O.GGUF_Q4_K, 256, 1024), "blk.0.attn_k.weight": (O.GGUF_Q8_0, 96, 1024),
              "blk.0.ffn_down.weight": (O.GGUF_Q4_0, 160, 512), "blk.0.attn_v.weight": (O.GGUF_Q6_K, 96, 1024),
              "blk.0.ffn_up.weight": (O.GGUF_Q5_K, 160, 512)}
    data = {name: synth.weights(dt, n, k, rng) for name, (dt, n, k) in shapes.items()}
    tensors = [(name, [k, n], dt, data[name]) for name, (dt, n, k) in shapes.items()]
    tensors.append(("output.weight", [256, 8], 11, rng.integers(0, 256, 8 * 110, dtype=np.uint8)))  # Q3_K
    p = tmp_path / "model.gguf"
    p.write_bytes(G.build_gguf([("general.architecture", G.T_STRING, "llama")], tensors))
    f = G.GgufFile.open(p)
    for name, (dt, n, k) in shapes.items():
        w = R.QuantWeight.from_gguf(f, name, n, k, ctx=ctx)
        assert w.dtype == dt and (w.n_rows, w.n_cols) == (n, k)
        assert np.array_equal(w.read_device_bytes(), data[name])
        x = synth.activations(1, k, rng)[0]
        got = np.asarray(R.mm_1d(x, w))[:n]
        want = O.mm_1d(x, data[name], dt, n, k, nthreads=8)
        err = np.abs(got - want).max() / np.abs(want).max()
        assert err <= 1e-5, (name, err)
    with pytest.raises(ValueError):
        R.QuantWeight.from_gguf(f, "blk.0.attn_q.weight", 128, 1024, ctx=ctx)  # numel differs
    with pytest.raises(ValueError):
        R.QuantWeight.from_gguf(f, "blk.9.attn_q.weight", 256, 1024, ctx=ctx)
    with pytest.raises(R.Unsupported):
        R.QuantWeight.from_gguf(f, "output.weight", 8, 256, ctx=ctx)
