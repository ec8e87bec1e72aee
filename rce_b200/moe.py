"""Expert-grouped MoE FFN on the device: the host mirror of the reference's
MoE pieces (rce-op-moe/src/lib.rs:35-110 moe_router / moe_combine;
rce-qwen36-moe/src/lib.rs:217-223 split_experts, :666-705 moe_ffn_forward)
over librce_qmm.so's rce_qmm_moe_route_device, rce_qmm_moe_router_device,
rce_qmm_moe_ffn_device and rce_qmm_moe_ffn.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

from ._lib import check, lib
from .qmm import QuantWeight, _check_weight, _stream_handle


@dataclass
class RouterDecision:
    """rce-op-moe's RouterDecision for one token: the selected experts in
    rank order and their (renormalised) weights."""
    expert_indices: List[int]
    expert_weights: List[float]


def split_experts(full: QuantWeight, n_expert: int, n_rows_per: int, n_cols_per: int) -> List[QuantWeight]:
    """Per-expert views of a stacked ``[n_expert, n_rows_per, n_cols_per]``
    weight (rce-qwen36-moe/src/lib.rs:217-223): expert e is the byte range
    ``[e * bpe, (e + 1) * bpe)`` with ``bpe = nbytes / n_expert``."""
    total = full.nbytes()
    if total % n_expert:
        raise ValueError(f"expert stack bytes {total} not divisible by n_expert {n_expert}")
    bpe = total // n_expert
    return [full.sub_view(e * bpe, bpe, n_rows_per, n_cols_per) for e in range(n_expert)]


def _f32_2d(t, name):
    import torch

    if t.dim() != 2 or t.dtype != torch.float32 or not t.is_cuda or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D CUDA float32 tensor with unit column stride")


def moe_route_device(logits, top_k: int, normalize: bool = True, stream=None) -> Tuple["object", "object"]:
    """moe_router on given logits [T, n_experts] (CUDA f32): returns
    (indices [T, top_k] int32, weights [T, top_k] f32), rank order per token."""
    import torch

    _f32_2d(logits, "logits")
    t_rows, n_experts = logits.shape
    idx = torch.empty((t_rows, top_k), dtype=torch.int32, device=logits.device)
    w = torch.empty((t_rows, top_k), dtype=torch.float32, device=logits.device)
    from .qmm import default_context

    ctx = default_context(logits.device.index)
    check(lib().rce_qmm_moe_route_device(ctx.handle, ctypes.c_void_p(logits.data_ptr()), logits.stride(0), t_rows,
                                         n_experts, top_k, 1 if normalize else 0, ctypes.c_void_p(idx.data_ptr()),
                                         ctypes.c_void_p(w.data_ptr()), _stream_handle(stream, logits.device)))
    return idx, w


def moe_router_device(x, router_w: QuantWeight, top_k: int, normalize: bool = True, stream=None):
    """moe_router with the router's quantized gate weight [n_experts, d_model]
    (rce-op-moe/src/lib.rs:35-73) for T tokens x [T, d_model] (CUDA f32): the
    logits router_w . x as mm_batched computes them, then softmax / top_k /
    renormalise.  Returns (indices [T, top_k] int32, weights [T, top_k] f32,
    logits [T, n_experts] f32)."""
    import torch

    _f32_2d(x, "x")
    _check_weight(router_w)
    t_rows = x.shape[0]
    n_experts = router_w.n_rows
    logits = torch.empty((t_rows, n_experts), dtype=torch.float32, device=x.device)
    idx = torch.empty((t_rows, top_k), dtype=torch.int32, device=x.device)
    w = torch.empty((t_rows, top_k), dtype=torch.float32, device=x.device)
    check(lib().rce_qmm_moe_router_device(router_w.ctx.handle, ctypes.c_void_p(x.data_ptr()), x.stride(0), t_rows,
                                          router_w.handle, top_k, 1 if normalize else 0,
                                          ctypes.c_void_p(logits.data_ptr()), logits.stride(0),
                                          ctypes.c_void_p(idx.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                          _stream_handle(stream, x.device)))
    return idx, w, logits


def moe_router(x, gate_w: QuantWeight, top_k: int, normalize: bool = True):
    """rce-op-moe's moe_router (lib.rs:35-73) on host activations: x of one
    token ([d_model]) gives one RouterDecision, x of T tokens ([T, d_model])
    a list of them."""
    import numpy as np
    import torch

    a = np.ascontiguousarray(x, dtype=np.float32)
    one = a.ndim == 1
    a2 = a.reshape(1, -1) if one else a
    dev = torch.device("cuda", gate_w.ctx.device)
    idx, w, _ = moe_router_device(torch.from_numpy(a2).to(dev), gate_w, top_k, normalize)
    dec = decisions(idx, w)
    return dec[0] if one else dec


def decisions(idx, w) -> List[RouterDecision]:
    """Host RouterDecision list from moe_route_device's tensors."""
    ii = idx.cpu().tolist()
    ww = w.cpu().tolist()
    return [RouterDecision(a, b) for a, b in zip(ii, ww)]


def _handles(ws: Sequence[Optional[QuantWeight]], lo: int, hi: int):
    arr = (ctypes.c_void_p * len(ws))()
    for e, w in enumerate(ws):
        if lo <= e < hi:
            _check_weight(w)
            arr[e] = w.handle
        else:
            arr[e] = None if w is None else w.handle
    return arr


def moe_shared_expert_device(x, gate: QuantWeight, up: QuantWeight, down: QuantWeight, gate_inp, out,
                             stream=None):
    """Add the always-on shared expert of moe_ffn_forward
    (rce-qwen36-moe/src/lib.rs:684-705) into out [T, d_model] (CUDA f32, in
    place): out[t] += sigmoid(gate_inp . x[t]) * W_down (silu(W_gate x[t]) *
    (W_up x[t])), gate_inp a CUDA f32 vector [d_model].  Returns out."""
    import torch

    _f32_2d(x, "x")
    _f32_2d(out, "out")
    t_rows, d_model = x.shape
    if tuple(out.shape) != (t_rows, d_model):
        raise ValueError("out must be [T, d_model]")
    if gate_inp.dtype != torch.float32 or not gate_inp.is_cuda or gate_inp.numel() != d_model \
            or not gate_inp.is_contiguous():
        raise ValueError("gate_inp must be a contiguous CUDA f32 vector of d_model values")
    check(lib().rce_qmm_moe_shared_expert_device(gate.ctx.handle, ctypes.c_void_p(x.data_ptr()), x.stride(0), t_rows,
                                                 gate.handle, up.handle, down.handle,
                                                 ctypes.c_void_p(gate_inp.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                                 out.stride(0), _stream_handle(stream, x.device)))
    return out


def moe_ffn_device(x, logits, top_k: int, gate: Sequence[QuantWeight], up: Sequence[QuantWeight],
                   down: Sequence[QuantWeight], expert_range: Optional[Tuple[int, int]] = None, out=None,
                   stream=None, return_routes: bool = False, shared=None):
    """The expert-grouped SwiGLU FFN over T tokens (x [T, d_model], router
    logits [T, n_experts], CUDA f32): route (softmax, top_k, renormalise),
    per routed expert y = W_down (silu(W_gate x) * (W_up x)), and combine in
    route order.  ``expert_range=(lo, hi)`` computes only the contributions
    of experts lo..hi-1 (the others add nothing; the weights of the others
    may be None), for experts placed across GPUs.  ``shared=(gate, up, down,
    gate_inp)`` then adds the sigmoid-gated shared expert
    (moe_shared_expert_device), completing moe_ffn_forward."""
    import torch

    _f32_2d(x, "x")
    _f32_2d(logits, "logits")
    t_rows, d_model = x.shape
    n_experts = logits.shape[1]
    if logits.shape[0] != t_rows:
        raise ValueError("logits must have one row per token")
    if not (len(gate) == len(up) == len(down) == n_experts):
        raise ValueError("gate/up/down need one weight per expert")
    lo, hi = expert_range if expert_range is not None else (0, n_experts)
    ctx = gate[lo].ctx
    if out is None:
        out = torch.empty((t_rows, d_model), dtype=torch.float32, device=x.device)
    idx = torch.empty((t_rows, top_k), dtype=torch.int32, device=x.device)
    w = torch.empty((t_rows, top_k), dtype=torch.float32, device=x.device)
    check(lib().rce_qmm_moe_ffn_device(ctx.handle, ctypes.c_void_p(x.data_ptr()), x.stride(0), t_rows,
                                       ctypes.c_void_p(logits.data_ptr()), logits.stride(0), n_experts, top_k, lo, hi,
                                       _handles(gate, lo, hi), _handles(up, lo, hi), _handles(down, lo, hi),
                                       ctypes.c_void_p(out.data_ptr()), out.stride(0), ctypes.c_void_p(idx.data_ptr()),
                                       ctypes.c_void_p(w.data_ptr()), _stream_handle(stream, x.device)))
    if shared is not None:
        sg, su, sd, sgi = shared
        moe_shared_expert_device(x, sg, su, sd, sgi, out, stream=stream)
    if return_routes:
        return out, idx, w
    return out


def moe_ffn(x, top_k: int, gate: Sequence[QuantWeight], up: Sequence[QuantWeight], down: Sequence[QuantWeight],
            router_logits=None, router_w: Optional[QuantWeight] = None,
            expert_range: Optional[Tuple[int, int]] = None, return_routes: bool = False):
    """The expert-grouped SwiGLU FFN on host buffers (rce_qmm_moe_ffn): x
    [T, d_model] f32, routed by router_logits [T, n_experts] or, without
    them, by the gate weight router_w (as moe_router).  Returns out [T,
    d_model] (and the routes (indices, weights) with return_routes)."""
    import numpy as np

    a = np.ascontiguousarray(x, dtype=np.float32)
    t_rows, d_model = a.shape
    n_experts = len(gate)
    if not (len(up) == len(down) == n_experts):
        raise ValueError("gate/up/down need one weight per expert")
    lo, hi = expert_range if expert_range is not None else (0, n_experts)
    lg = None
    if router_logits is not None:
        lg = np.ascontiguousarray(router_logits, dtype=np.float32)
        if lg.shape != (t_rows, n_experts):
            raise ValueError("router_logits must be [T, n_experts]")
    elif router_w is None:
        raise ValueError("moe_ffn needs router_logits or router_w")
    ctx = gate[lo].ctx
    out = np.empty((t_rows, d_model), dtype=np.float32)
    idx = np.empty((t_rows, top_k), dtype=np.int32)
    w = np.empty((t_rows, top_k), dtype=np.float32)
    f = ctypes.POINTER(ctypes.c_float)
    check(lib().rce_qmm_moe_ffn(ctx.handle, a.ctypes.data_as(f), t_rows,
                                None if lg is None else lg.ctypes.data_as(f),
                                None if router_w is None else router_w.handle, n_experts, top_k, lo, hi,
                                _handles(gate, lo, hi), _handles(up, lo, hi), _handles(down, lo, hi),
                                out.ctypes.data_as(f), idx.ctypes.data_as(ctypes.c_void_p),
                                w.ctypes.data_as(ctypes.c_void_p)))
    if return_routes:
        return out, idx, w
    return out
