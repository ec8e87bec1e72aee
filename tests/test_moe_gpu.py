"""The expert-grouped MoE FFN on the device (rce_qmm_moe_route_device,
rce_qmm_moe_ffn_device) against the oracle's restatement of moe_router /
moe_combine (rce-op-moe/src/lib.rs:35-110) and moe_ffn_forward
(rce-qwen36-moe/src/lib.rs:666-705).

Bars:
- routes: the same experts in the same rank order; weights within a few
  units in the last place (the device expf and the host libm exp may differ
  in the last bit);
- exact path (prefill_min_tokens = 0, every expert's rows through the
  decode GEMV): per token max|got - want| / max|want| <= 1e-5;
- default path (the grouped tensor-core GEMM: weights rounded to fp16,
  activations carried as two fp16 terms): max-norm error over the whole
  output <= 1e-3, and within 2.5e-4 of a model of those operands with exact
  accumulation (per-token relative L2 errors are printed);
- experts split into ranges: the ranges' outputs add up to the full output
  bit for bit (top-2).
"""
import numpy as np
import pytest

import oracle as O
import rce_b200 as R
from rce_b200 import synth

pytestmark = pytest.mark.gpu

Q4_K, Q8_0, Q4_0 = O.GGUF_Q4_K, O.GGUF_Q8_0, O.GGUF_Q4_0


def _setup(dt, n_experts, d_model, d_ff, t_rows, seed):
    rng = np.random.default_rng(seed)
    gate = [synth.weights(dt, d_ff, d_model, rng) for _ in range(n_experts)]
    up = [synth.weights(dt, d_ff, d_model, rng) for _ in range(n_experts)]
    down = [synth.weights(dt, d_model, d_ff, rng) for _ in range(n_experts)]
    x = synth.activations(t_rows, d_model, rng)
    logits = rng.standard_normal((t_rows, n_experts)).astype(np.float32)
    return gate, up, down, x, logits


def _device(ctx, dt, gate, up, down, d_model, d_ff):
    g = [R.QuantWeight.from_owned_bytes(b, dt, d_ff, d_model, ctx=ctx) for b in gate]
    u = [R.QuantWeight.from_owned_bytes(b, dt, d_ff, d_model, ctx=ctx) for b in up]
    d = [R.QuantWeight.from_owned_bytes(b, dt, d_model, d_ff, ctx=ctx) for b in down]
    return g, u, d


@pytest.mark.parametrize("n_experts,top_k,normalize", [(8, 2, True), (128, 8, True), (16, 4, False), (3, 1, True)])
def test_route_matches_oracle(n_experts, top_k, normalize):
    import torch

    rng = np.random.default_rng(40 + n_experts)
    logits = rng.standard_normal((300, n_experts)).astype(np.float32)
    idx, w = R.moe_route_device(torch.from_numpy(logits).cuda(), top_k, normalize)
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    for t in range(logits.shape[0]):
        ri, rw = O.moe_softmax_topk(logits[t], top_k, normalize)
        assert list(idx[t]) == list(ri), f"token {t}"
        np.testing.assert_allclose(w[t], rw, rtol=4e-7, atol=0)
    dec = R.decisions(torch.from_numpy(idx), torch.from_numpy(w))
    assert len(dec) == 300 and dec[0].expert_indices == list(idx[0])


def _ffn(ctx, dt, n_experts, top_k, d_model, d_ff, t_rows, seed, **kw):
    import torch

    gate, up, down, x, logits = _setup(dt, n_experts, d_model, d_ff, t_rows, seed)
    want = O.moe_ffn(x, logits, top_k, np.stack(gate), np.stack(up), np.stack(down), dt, d_ff, nthreads=8)
    g, u, d = _device(ctx, dt, gate, up, down, d_model, d_ff)
    got, idx, w = R.moe_ffn_device(torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda(), top_k, g, u, d,
                                   return_routes=True, **kw)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    return got.cpu().numpy(), want, (g, u, d, x, logits)


@pytest.mark.parametrize("dt", [Q4_K, Q8_0, Q4_0])
def test_ffn_exact_path_matches_oracle(ctx, dt):
    saved = ctx.prefill_min_tokens
    ctx.prefill_min_tokens = 0
    try:
        got, want, _ = _ffn(ctx, dt, 4, 2, 256, 512, 37, 7 + dt)
    finally:
        ctx.prefill_min_tokens = saved
    err = np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)
    print(f"MoE exact path dtype {dt}: per-token normwise {err.max():.3e}")
    assert err.max() <= 1e-5


def _fp16_operand_model(dt, gate, up, down, x, logits, top_k, d_model, d_ff):
    """The FFN as the tensor-core path computes it: each matmul's activation
    row scaled by a power of two and split into two fp16 terms (the rounding
    and the rounding of the remainder), the dequantised weights rounded to
    fp16, products accumulated exactly (f64), SwiGLU in f32."""
    Wg = [O.dequant(b, dt, d_ff * d_model).reshape(d_ff, d_model) for b in gate]
    Wu = [O.dequant(b, dt, d_ff * d_model).reshape(d_ff, d_model) for b in up]
    Wd = [O.dequant(b, dt, d_model * d_ff).reshape(d_model, d_ff) for b in down]
    h16 = lambda W: W.astype(np.float16).astype(np.float64)  # noqa: E731

    def r16(a):
        a = np.asarray(a, np.float32)
        e = np.frexp(np.abs(a).max(axis=-1, keepdims=True))[1]
        s = np.ldexp(np.float32(1.0), 14 - e).astype(np.float32)
        v = a * s
        hi = v.astype(np.float16)
        lo = (v - hi.astype(np.float32)).astype(np.float16)
        return (hi.astype(np.float64) + lo.astype(np.float64)) / s

    Wg, Wu, Wd = [h16(w) for w in Wg], [h16(w) for w in Wu], [h16(w) for w in Wd]
    out = np.zeros((x.shape[0], d_model))
    for t in range(x.shape[0]):
        idx, w = O.moe_softmax_topk(logits[t], top_k, True)
        for j in range(top_k):
            e = idx[j]
            xr = r16(x[t][None])[0]
            g = (Wg[e] @ xr).astype(np.float32)
            u = (Wu[e] @ xr).astype(np.float32)
            with np.errstate(over="ignore"):
                h = (g / (np.float32(1) + np.exp(-g))) * u
            out[t] += np.float64(w[j]) * (Wd[e] @ r16(h[None])[0])
    return out


@pytest.mark.parametrize("dt", [Q4_K, Q8_0])
def test_ffn_gemm_path_matches_oracle(ctx, dt):
    # 4 experts, 200 tokens x top-2: every expert gets far more than 16 rows
    assert ctx.prefill_min_tokens == 16
    d_model, d_ff = 512, 1024
    got, want, (g, u, d, x, logits) = _ffn(ctx, dt, 4, 2, d_model, d_ff, 200, 11 + dt)
    gate, up, down, _, _ = _setup(dt, 4, d_model, d_ff, 200, 11 + dt)
    scale = np.abs(want).max()
    tensor = np.abs(got.astype(np.float64) - want).max() / scale
    l2 = np.linalg.norm(got - want, axis=1) / np.linalg.norm(want, axis=1)
    model = _fp16_operand_model(dt, gate, up, down, x, logits, 2, d_model, d_ff)
    vs_model = np.abs(got - model).max() / scale
    print(f"MoE GEMM path dtype {dt}: max-norm {tensor:.3e}; per-token L2 median {np.median(l2):.3e}, "
          f"max {l2.max():.3e}; vs the fp16-operand model {vs_model:.3e}")
    assert tensor <= 1e-3
    # the tensor-core path is "fp16 weights, two-term activations, exact
    # accumulation" up to f32 accumulation and the last bit of exp inside
    # silu, which can flip the rounding of an intermediate
    assert vs_model <= 2.5e-4


def test_expert_ranges_add_up_bit_for_bit(ctx):
    import torch

    saved = ctx.prefill_min_tokens
    ctx.prefill_min_tokens = 0
    try:
        full, _, (g, u, d, x, logits) = _ffn(ctx, Q4_K, 4, 2, 256, 512, 23, 99)
        xd, ld = torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda()
        parts = [R.moe_ffn_device(xd, ld, 2, g, u, d, expert_range=r).cpu().numpy() for r in [(0, 1), (1, 3), (3, 4)]]
    finally:
        ctx.prefill_min_tokens = saved
    # each token's two routed experts: one range holds both, or two ranges one each
    assert np.array_equal(parts[0] + parts[1] + parts[2], full)


def test_ffn_mixtral_shape_token_subset(ctx):
    # configs[4]'s expert shape (gate/up 14336 x 4096, down 4096 x 14336,
    # Q4_K) with 4 experts and 8 tokens (the exact path), checked against the
    # oracle
    saved = ctx.prefill_min_tokens
    ctx.prefill_min_tokens = 0
    try:
        got, want, _ = _ffn(ctx, Q4_K, 4, 2, 4096, 14336, 8, 4)
    finally:
        ctx.prefill_min_tokens = saved
    err = np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)
    print(f"MoE Mixtral expert shape, 8 tokens: per-token normwise {err.max():.3e}")
    assert err.max() <= 1e-5


def test_bad_arguments_are_errors(ctx):
    import torch

    gate, up, down, x, logits = _setup(Q4_K, 2, 256, 512, 4, 3)
    g, u, d = _device(ctx, Q4_K, gate, up, down, 256, 512)
    xd, ld = torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda()
    with pytest.raises(R.QmmError):
        R.moe_ffn_device(xd, ld, 3, g, u, d)          # top_k > n_experts
    with pytest.raises(R.QmmError):
        R.moe_ffn_device(xd, ld, 1, g, d, u)          # up/down shapes swapped
    with pytest.raises(R.QmmError):
        R.moe_ffn_device(xd, ld, 1, g, u, d, expert_range=(1, 1))


def _bars(got, want, model):
    scale = np.abs(want).max()
    tensor = np.abs(got.astype(np.float64) - want).max() / scale
    vs_model = np.abs(got - model).max() / scale
    return tensor, vs_model


def test_ffn_grouped_many_experts_ragged(ctx):
    # 40 experts (two grouped launches each for gate/up and down: 32 experts
    # per launch), top-4 of 60 tokens: per-expert row counts from 0 to ~15,
    # below the 16-token GEMM threshold, all through the grouped tensor-core
    # path; four route slots per token keep the ordered combine kernel
    assert ctx.prefill_min_tokens == 16
    dt, n_e, k, d_model, d_ff, t = Q4_K, 40, 4, 256, 512, 60
    got, want, (g, u, d, x, logits) = _ffn(ctx, dt, n_e, k, d_model, d_ff, t, 31)
    gate, up, down, _, _ = _setup(dt, n_e, d_model, d_ff, t, 31)
    model = _fp16_operand_model(dt, gate, up, down, x, logits, k, d_model, d_ff)
    tensor, vs_model = _bars(got, want, model)
    print(f"MoE grouped, 40 experts top-4: max-norm {tensor:.3e}, vs the fp16-operand model {vs_model:.3e}")
    assert tensor <= 1e-3
    assert vs_model <= 2.5e-4


def test_ffn_grouped_expert_ranges_add_up(ctx):
    import torch

    # the grouped path per expert range: every (expert, token) output is the
    # same whichever launch computes it, so the ranges add up bit for bit
    full, _, (g, u, d, x, logits) = _ffn(ctx, Q8_0, 6, 2, 256, 512, 48, 5)
    xd, ld = torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda()
    parts = [R.moe_ffn_device(xd, ld, 2, g, u, d, expert_range=r).cpu().numpy() for r in [(0, 2), (2, 5), (5, 6)]]
    total = parts[0] + parts[1] + parts[2]
    print(f"grouped ranges: max |sum - full| = {np.abs(total - full).max():.3e}")
    assert np.array_equal(total, full)


def test_ffn_grouped_graph_replay(ctx):
    import torch

    # no host synchronisation inside the grouped call: it can be captured in
    # a CUDA graph and replayed on new inputs
    dt, n_e, d_model, d_ff, t = Q4_0, 4, 256, 512, 32
    gate, up, down, x, logits = _setup(dt, n_e, d_model, d_ff, t, 17)
    g, u, d = _device(ctx, dt, gate, up, down, d_model, d_ff)
    xd, ld = torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda()
    out = torch.empty((t, d_model), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        R.moe_ffn_device(xd, ld, 2, g, u, d, out=out, stream=s)  # sizes the workspace
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        R.moe_ffn_device(xd, ld, 2, g, u, d, out=out, stream=s)
    rng = np.random.default_rng(18)
    for _ in range(2):
        x2 = synth.activations(t, d_model, rng)
        l2 = rng.standard_normal((t, n_e)).astype(np.float32)
        xd.copy_(torch.from_numpy(x2))
        ld.copy_(torch.from_numpy(l2))
        graph.replay()
        torch.cuda.synchronize()
        eager = R.moe_ffn_device(xd, ld, 2, g, u, d)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), eager.cpu().numpy())
    want = O.moe_ffn(x2, l2, 2, np.stack(gate), np.stack(up), np.stack(down), dt, d_ff, nthreads=8)
    assert np.abs(out.cpu().numpy() - want).max() / np.abs(want).max() <= 1e-3
    assert ctx.device_error() == 0


# ---- moe_router with the gate weight (rce-op-moe/src/lib.rs:35-73, tests :140-204)

@pytest.mark.parametrize("n_e,top_k,norm,kind,c1", [(8, 2, True, "sin", 0.013), (16, 1, True, "cos", 0.017),
                                                    (32, 2, False, "sin", 0.013)])
def test_router_from_gate_weight_reference_fixtures(ctx, n_e, top_k, norm, kind, c1):
    import refcases

    gate = refcases.router_gate_q8_0(n_e, 64)
    x = O.test_activations(kind, c1, 0.0, 64)
    gw = R.QuantWeight.from_owned_bytes(gate, Q8_0, n_e, 64, ctx=ctx)
    dec = R.moe_router(x, gw, top_k, norm)
    ri, rw = O.moe_router(x, gate, Q8_0, n_e, top_k, norm)
    assert dec.expert_indices == list(ri)
    np.testing.assert_allclose(dec.expert_weights, rw, rtol=1e-5)
    w = np.array(dec.expert_weights)
    assert np.all((w >= 0) & (w <= 1)) and list(w) == sorted(w, reverse=True)
    assert len(set(dec.expert_indices)) == top_k
    if norm:
        assert abs(w.sum() - 1.0) < 1e-5
    else:
        assert 0.0 < w.sum() < 1.0


def _safe_margin(logits, top_k, rel=1e-3):
    """Tokens whose k-th and (k+1)-th largest logits differ by more than rel
    of the logits' spread (a route that rounding cannot flip)."""
    s = np.sort(logits, axis=1)[:, ::-1]
    spread = np.maximum(s[:, 0] - s[:, -1], 1e-30)
    return (s[:, top_k - 1] - s[:, top_k]) > rel * spread


def test_router_from_gate_weight_batches(ctx):
    import torch

    rng = np.random.default_rng(55)
    n_e, d, t, top_k = 8, 4096, 200, 2
    gate = synth.weights(Q4_K, n_e, d, rng)
    x = synth.activations(t, d, rng)
    gw = R.QuantWeight.from_owned_bytes(gate, Q4_K, n_e, d, ctx=ctx)
    want_logits = O.mm_batched(x, t, gate, Q4_K, n_e, d, nthreads=8)
    want = [O.moe_router(x[i], gate, Q4_K, n_e, top_k, True) for i in range(t)]
    saved = ctx.prefill_min_tokens
    try:
        for pmt in (0, saved):  # the exact decode path for every batch; then the default routing
            ctx.prefill_min_tokens = pmt
            idx, w, logits = R.moe_router_device(torch.from_numpy(x).cuda(), gw, top_k)
            idx, w, logits = idx.cpu().numpy(), w.cpu().numpy(), logits.cpu().numpy()
            if pmt == 0:  # per token, the exact path's bar
                err = np.abs(logits - want_logits).max(axis=1) / np.abs(want_logits).max(axis=1)
                assert err.max() <= 1e-5
            else:  # 200 tokens through the one-term fp16 GEMM: its bar over the whole output
                err = np.abs(logits - want_logits).max() / np.abs(want_logits).max()
                assert err <= 1e-3
            ok = np.ones(t, bool) if pmt == 0 else _safe_margin(want_logits, top_k)
            # a routing weight moves by at most w (1 - w) times the change of
            # the difference of two logits, i.e. by at most half of the
            # token's largest logit error
            lerr = np.abs(logits.astype(np.float64) - want_logits).max(axis=1)
            for i in np.nonzero(ok)[0]:
                assert list(idx[i]) == list(want[i][0]), f"token {i}"
                np.testing.assert_allclose(w[i], want[i][1], rtol=1e-5, atol=0.5 * lerr[i] + 1e-7)
            print(f"router prefill_min_tokens={pmt}: logits {err.max():.2e}, {ok.sum()} of {t} routes compared")
    finally:
        ctx.prefill_min_tokens = saved


def test_host_moe_ffn(ctx):
    import torch

    dt, n_e, top_k, d_model, d_ff, t = Q4_K, 4, 2, 256, 512, 37
    gate, up, down, x, logits = _setup(dt, n_e, d_model, d_ff, t, 71)
    g, u, d = _device(ctx, dt, gate, up, down, d_model, d_ff)
    # routed by given logits: the same results as the device entry point
    out, idx, w = R.moe_ffn(x, top_k, g, u, d, router_logits=logits, return_routes=True)
    dev, didx, dw = R.moe_ffn_device(torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda(), top_k, g, u, d,
                                     return_routes=True)
    assert np.array_equal(out, dev.cpu().numpy())
    assert np.array_equal(idx, didx.cpu().numpy()) and np.array_equal(w, dw.cpu().numpy())
    # routed by a gate weight, exact path: against the oracle's moe_router +
    # moe_ffn composition
    rw = synth.weights(Q8_0, n_e, d_model, np.random.default_rng(72))
    rq = R.QuantWeight.from_owned_bytes(rw, Q8_0, n_e, d_model, ctx=ctx)
    saved = ctx.prefill_min_tokens
    ctx.prefill_min_tokens = 0
    try:
        got, gidx, _ = R.moe_ffn(x, top_k, g, u, d, router_w=rq, return_routes=True)
    finally:
        ctx.prefill_min_tokens = saved
    want_logits = O.mm_batched(x, t, rw, Q8_0, n_e, d_model)
    want = O.moe_ffn(x, want_logits, top_k, np.stack(gate), np.stack(up), np.stack(down), dt, d_ff, nthreads=8)
    for i in range(t):
        assert list(gidx[i]) == list(O.moe_router(x[i], rw, Q8_0, n_e, top_k, True)[0])
    err = np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)
    assert err.max() <= 1e-5
    with pytest.raises(ValueError):
        R.moe_ffn(x, top_k, g, u, d)  # neither logits nor a gate weight


# ---- the shared expert of moe_ffn_forward (rce-qwen36-moe/src/lib.rs:684-705)

@pytest.mark.parametrize("exact", [True, False])
def test_ffn_with_shared_expert_matches_oracle(ctx, exact):
    import torch

    # routed experts (top-2 of 4) plus the always-on shared expert with its
    # sigmoid gate; the exact path against the oracle's moe_ffn_forward at
    # the exact path's bar, the default (tensor-core) path at the GEMM bar
    dt, n_e, d_model, d_ff, n_ff_s, t = Q4_K, 4, 512, 1024, 512, 40
    gate, up, down, x, logits = _setup(dt, n_e, d_model, d_ff, t, 61)
    rng = np.random.default_rng(62)
    sg = synth.weights(dt, n_ff_s, d_model, rng)
    su = synth.weights(dt, n_ff_s, d_model, rng)
    sd = synth.weights(dt, d_model, n_ff_s, rng)
    gate_inp = (rng.standard_normal(d_model) * 0.05).astype(np.float32)
    g, u, d = _device(ctx, dt, gate, up, down, d_model, d_ff)
    wsg = R.QuantWeight.from_owned_bytes(sg, dt, n_ff_s, d_model, ctx=ctx)
    wsu = R.QuantWeight.from_owned_bytes(su, dt, n_ff_s, d_model, ctx=ctx)
    wsd = R.QuantWeight.from_owned_bytes(sd, dt, d_model, n_ff_s, ctx=ctx)
    routed = O.moe_ffn(x, logits, 2, np.stack(gate), np.stack(up), np.stack(down), dt, d_ff, nthreads=8)
    want = O.moe_shared_expert(x, routed, gate_inp, sg, su, sd, dt, n_ff_s, nthreads=8)
    saved = ctx.prefill_min_tokens
    if exact:
        ctx.prefill_min_tokens = 0
    try:
        got = R.moe_ffn_device(torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda(), 2, g, u, d,
                               shared=(wsg, wsu, wsd, torch.from_numpy(gate_inp).cuda())).cpu().numpy()
    finally:
        ctx.prefill_min_tokens = saved
    assert ctx.device_error() == 0
    # the shared term matters: the output differs from the routed part alone
    assert np.abs(want - routed).max() > 1e-2 * np.abs(want).max()
    if exact:
        err = np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)
        print(f"MoE + shared expert, exact path: per-token normwise {err.max():.3e}")
        assert err.max() <= 1e-5
    else:
        tensor = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
        print(f"MoE + shared expert, tensor-core path: max-norm {tensor:.3e}")
        assert tensor <= 1e-3


def test_shared_expert_bad_arguments(ctx):
    import torch

    dt, d_model, n_ff_s = Q4_K, 256, 512
    rng = np.random.default_rng(63)
    wsg = R.QuantWeight.from_owned_bytes(synth.weights(dt, n_ff_s, d_model, rng), dt, n_ff_s, d_model, ctx=ctx)
    wsd = R.QuantWeight.from_owned_bytes(synth.weights(dt, d_model, n_ff_s, rng), dt, d_model, n_ff_s, ctx=ctx)
    x = torch.zeros((4, d_model), device="cuda")
    out = torch.zeros((4, d_model), device="cuda")
    gi = torch.zeros(d_model, device="cuda")
    with pytest.raises(R.QmmError):
        R.moe_shared_expert_device(x, wsg, wsd, wsd, gi, out)  # up with down's shape
    with pytest.raises(ValueError):
        R.moe_shared_expert_device(x, wsg, wsg, wsd, gi[:10], out)  # gate_inp of the wrong length
