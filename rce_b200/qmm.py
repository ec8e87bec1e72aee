"""Host-side mirror of the reference crate rce-op-qmm's operator API.

Same names, argument meaning and error behaviour as the Rust originals, with
the compute done by librce_qmm.so on a B200:

* ``QuantWeight``        rce-op-qmm/src/lib.rs:77-210
* ``mm_1d``              rce-op-qmm/src/lib.rs:216-270
* ``mm_1d_serial``       rce-op-qmm/src/lib.rs:281-304
* ``mm_batched``         rce-op-qmm/src/lib.rs:967-1023
* ``QmmLeaf``            rce-op-qmm/src/lib.rs:2075-2131 (an ``OpDispatch``
  leaf claiming ``Custom("qmm")``, rce-vm-backend-cpu/src/op_dispatch.rs:21-63)
* ``CudaQmm``            a ``QmmDispatch`` backend
  (rce-placement-adapter/src/lib.rs:130-134) with the ``PricedBackend`` id
  ``cuda:op-qmm``.

The reference panics on an unsupported dtype (lib.rs:268); here that is
``Unsupported``.  Debug-only shape assertions of the reference
(``debug_assert!``) are always checked here and raise ``ValueError``.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Dict, Optional

import numpy as np

from . import _lib
from ._lib import QmmError, Unsupported, check, lib
from .gguf import BLOCK, SUPPORTED, GgufDtype, row_bytes, tensor_byte_size

__all__ = [
    "Context", "QuantWeight", "mm_1d", "mm_1d_serial", "mm_batched", "mm_batched_device",
    "dequant_device", "QmmLeaf", "CudaQmm", "QmmError", "Unsupported", "default_context",
]


class Context:
    """One CUDA device (``rce_qmm_ctx``)."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().rce_qmm_ctx_create(int(device), ctypes.byref(h)))
        self._h = h
        self.device = int(device)
        n = ctypes.c_int()
        check(lib().rce_qmm_ctx_sm_count(self._h, ctypes.byref(n)))
        self.sm_count = n.value

    @property
    def handle(self):
        return self._h

    def synchronize(self) -> None:
        check(lib().rce_qmm_synchronize(self._h))

    @property
    def prefill_min_tokens(self) -> int:
        """Batches of at least this many tokens run the tensor-core prefill
        GEMM (fp16 operands); smaller ones the exact decode path; 0 = never."""
        n = ctypes.c_int()
        check(lib().rce_qmm_ctx_get_prefill_min_tokens(self._h, ctypes.byref(n)))
        return n.value

    @prefill_min_tokens.setter
    def prefill_min_tokens(self, n: int) -> None:
        check(lib().rce_qmm_ctx_set_prefill_min_tokens(self._h, int(n)))

    def device_error(self, clear: bool = True) -> int:
        """The kernel error word (0 = none): non-zero when a bounded wait
        inside a kernel expired; read it after synchronising the stream."""
        code = ctypes.c_int()
        check(lib().rce_qmm_device_error(self._h, ctypes.byref(code), int(bool(clear))))
        return code.value

    def close(self) -> None:
        if self._h is not None and self._h.value:
            lib().rce_qmm_ctx_destroy(self._h)
            self._h = None


_ctx_lock = threading.Lock()
_contexts: Dict[int, Context] = {}


def default_context(device: Optional[int] = None) -> Context:
    if device is None:
        try:
            import torch

            device = torch.cuda.current_device() if torch.cuda.is_available() else 0
        except Exception:  # torch missing: device 0
            device = 0
    with _ctx_lock:
        ctx = _contexts.get(device)
        if ctx is None:
            ctx = Context(device)
            _contexts[device] = ctx
    return ctx


def _f32_array(a, n: Optional[int] = None) -> np.ndarray:
    arr = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    if n is not None and arr.size != n:
        raise ValueError(f"activation len {arr.size} != k {n}")
    return arr


def _fptr(arr: np.ndarray):
    return arr.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _addr(arr: np.ndarray) -> int:
    """The array's data address (for the hot host calls, whose pointer
    arguments are declared void *: cheaper than a typed ctypes pointer)."""
    return arr.ctypes.data


class QuantWeight:
    """A weight in its native GGUF dtype, registered once on the device.

    Layout ``[n_rows = N_out][n_cols = K_in]`` row-major blocks, as GGUF stores
    it.  ``bytes()`` is a zero-copy view of the host bytes it was built from
    (the reference's ``Backing``); the device holds the same bytes repacked
    into the T16 tile layout (``read_device_bytes`` rebuilds them).
    """

    def __init__(self, handle, dtype: GgufDtype, n_rows: int, n_cols: int, ctx: Context,
                 host_bytes=None, parent: "QuantWeight" = None):
        self._h = handle
        self.dtype = GgufDtype(dtype)
        self.n_rows = int(n_rows)
        self.n_cols = int(n_cols)
        self.ctx = ctx
        self._host = host_bytes
        self._parent = parent  # keeps the parent's device storage alive

    # -- constructors ----------------------------------------------------
    @classmethod
    def from_owned_bytes(cls, data, dtype, n_rows: int, n_cols: int, ctx: Optional[Context] = None) -> "QuantWeight":
        """Register host GGUF bytes (QuantWeight::from_owned_bytes, lib.rs:123-139)."""
        dt = GgufDtype.parse(dtype)
        if dt not in SUPPORTED:
            raise Unsupported(_lib.RCE_QMM_ERR_UNSUPPORTED, f"dtype {dt.name} not supported by rce_b200")
        ctx = ctx or default_context()
        if isinstance(data, (bytes, bytearray, memoryview)):
            buf = np.frombuffer(data, dtype=np.uint8)
        else:
            buf = np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
        h = ctypes.c_void_p()
        check(lib().rce_qmm_weight_register(ctx.handle, buf.ctypes.data_as(ctypes.c_void_p), buf.size, int(dt),
                                            int(n_rows), int(n_cols), ctypes.byref(h)))
        return cls(h, dt, n_rows, n_cols, ctx, host_bytes=buf)

    @classmethod
    def from_device_bytes(cls, tensor, dtype, n_rows: int, n_cols: int, ctx: Optional[Context] = None,
                          stream=None) -> "QuantWeight":
        """Register GGUF bytes already on the device (a uint8 torch tensor)."""
        dt = GgufDtype.parse(dtype)
        ctx = ctx or default_context(tensor.device.index)
        h = ctypes.c_void_p()
        s = _stream_handle(stream, tensor.device)
        check(lib().rce_qmm_weight_register_device(ctx.handle, ctypes.c_void_p(tensor.data_ptr()), tensor.numel(),
                                                   int(dt), int(n_rows), int(n_cols), s, ctypes.byref(h)))
        return cls(h, dt, n_rows, n_cols, ctx)

    @classmethod
    def from_gguf(cls, gguf, name: str, n_rows: int, n_cols: int, ctx: Optional[Context] = None) -> "QuantWeight":
        """View tensor ``name`` of a parsed GGUF file (QuantWeight::from_gguf,
        lib.rs:173-209): checks the declared shape against numel and the byte
        range against the file, then registers the bytes (zero-copy on the
        host side: the bytes are a view of the file's mmap)."""
        t = gguf.tensor(name)
        if t is None:
            raise ValueError(f"tensor not found: {name}")
        if t.numel != n_rows * n_cols:
            raise ValueError(f"{name}: declared shape {n_rows}×{n_cols} = {n_rows * n_cols} ≠ tensor numel = {t.numel}")
        return cls.from_owned_bytes(gguf.tensor_bytes(t), t.dtype, n_rows, n_cols, ctx)

    # -- accessors -------------------------------------------------------
    @property
    def handle(self):
        return self._h

    def bytes(self) -> np.ndarray:
        """The tensor's GGUF bytes (host view when built from host bytes,
        otherwise rebuilt from the device)."""
        if self._host is not None:
            return self._host
        return self.read_device_bytes()

    def nbytes(self) -> int:
        return tensor_byte_size(self.dtype, self.n_rows * self.n_cols)

    def read_device_bytes(self) -> np.ndarray:
        out = np.empty(self.nbytes(), dtype=np.uint8)
        check(lib().rce_qmm_weight_read_bytes(self._h, out.ctypes.data_as(ctypes.c_void_p), out.size))
        return out

    def device_storage(self):
        p = ctypes.c_void_p()
        n = ctypes.c_size_t()
        check(lib().rce_qmm_weight_device_storage(self._h, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def sub_view(self, byte_offset_rel: int, byte_len: int, n_rows: int, n_cols: int) -> "QuantWeight":
        """QuantWeight::sub_view (lib.rs:99-118), e.g. one MoE expert of a
        stacked tensor; the view must start on a multiple of 16 rows."""
        if byte_offset_rel + byte_len > self.nbytes():
            raise ValueError(f"sub_view oob: {byte_offset_rel}+{byte_len} > {self.nbytes()}")
        h = ctypes.c_void_p()
        check(lib().rce_qmm_weight_sub_view(self._h, int(byte_offset_rel), int(byte_len), int(n_rows), int(n_cols),
                                            ctypes.byref(h)))
        host = None
        if self._host is not None:
            host = self._host[byte_offset_rel:byte_offset_rel + byte_len]
        return QuantWeight(h, self.dtype, n_rows, n_cols, self.ctx, host_bytes=host, parent=self)

    def dequant_row(self, row: int) -> np.ndarray:
        """QuantWeight::dequant_row (lib.rs:150-166): n_cols f32 values,
        bit-exact with dequantize_to_f32."""
        if not 0 <= row < self.n_rows:
            raise ValueError(f"row {row} ≥ n_rows {self.n_rows}")
        out = np.empty(self.n_cols, dtype=np.float32)
        check(lib().rce_qmm_dequant_row(self.ctx.handle, self._h, int(row), _fptr(out), out.size))
        return out

    def close(self) -> None:
        if self._h is not None and self._h.value:
            lib().rce_qmm_weight_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __repr__(self) -> str:
        return f"QuantWeight({self.dtype.name}, {self.n_rows}x{self.n_cols})"


def _check_weight(w: QuantWeight) -> None:
    if not isinstance(w, QuantWeight):
        raise TypeError("expected a QuantWeight")
    if w.dtype not in SUPPORTED:
        raise Unsupported(_lib.RCE_QMM_ERR_UNSUPPORTED, f"mm_1d: dtype {w.dtype!r} not yet supported by rce_b200")


def mm_1d(a, w: QuantWeight, out: Optional[np.ndarray] = None) -> np.ndarray:
    """``out[1, n] = a[1, k] · w[n, k]^T`` (mm_1d, lib.rs:216).  ``out`` (if
    given, f32 with at least n_rows elements) is written in place."""
    _check_weight(w)
    a = _f32_array(a, w.n_cols)
    if out is None:
        out = np.empty(w.n_rows, dtype=np.float32)
    if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < w.n_rows:
        raise ValueError("output buffer too small")
    check(lib().rce_qmm_mm_1d(w.ctx.handle, _addr(a), a.size, w.handle, _addr(out), out.size))
    return out


def mm_1d_serial(a, w: QuantWeight, out: Optional[np.ndarray] = None) -> np.ndarray:
    """mm_1d_serial (lib.rs:281): same results as ``mm_1d``."""
    _check_weight(w)
    a = _f32_array(a, w.n_cols)
    if out is None:
        out = np.empty(w.n_rows, dtype=np.float32)
    if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < w.n_rows:
        raise ValueError("output buffer too small")
    check(lib().rce_qmm_mm_1d_serial(w.ctx.handle, _fptr(a), a.size, w.handle, _fptr(out), out.size))
    return out


def mm_batched(a, t_rows: int, w: QuantWeight, out: Optional[np.ndarray] = None) -> np.ndarray:
    """``out[T, N] = a[T, K] · w[N, K]^T`` (mm_batched, lib.rs:967); ``a`` and
    ``out`` are row-major and flat or 2-D."""
    _check_weight(w)
    a = _f32_array(a, t_rows * w.n_cols)
    if out is None:
        out = np.empty(t_rows * w.n_rows, dtype=np.float32)
    if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < t_rows * w.n_rows:
        raise ValueError("output buffer too small")
    check(lib().rce_qmm_mm_batched(w.ctx.handle, _addr(a), int(t_rows), w.handle, _addr(out), out.size))
    return out


def _stream_handle(stream, device):
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(device)
    return ctypes.c_void_p(stream.cuda_stream)


def mm_batched_device(x, w: QuantWeight, out=None, stream=None):
    """Device-memory ``mm_batched``: ``x`` is a CUDA f32 tensor [T, K] (rows may
    be strided), ``out`` [T, N]; runs asynchronously on ``stream`` (default:
    torch's current stream)."""
    import torch

    _check_weight(w)
    if x.dim() == 1:
        x = x.view(1, -1)
    if x.dtype != torch.float32 or not x.is_cuda or x.stride(1) != 1:
        raise ValueError("x must be a CUDA float32 tensor with unit column stride")
    t_rows, k = x.shape
    if k != w.n_cols:
        raise ValueError(f"activation len {k} ≠ k {w.n_cols}")
    if out is None:
        out = torch.empty((t_rows, w.n_rows), dtype=torch.float32, device=x.device)
    if out.stride(-1) != 1:
        raise ValueError("out must have unit column stride")
    ldo = out.stride(0) if out.dim() == 2 else w.n_rows
    check(lib().rce_qmm_mm_batched_device(w.ctx.handle, ctypes.c_void_p(x.data_ptr()), x.stride(0), t_rows,
                                          w.handle, ctypes.c_void_p(out.data_ptr()), ldo,
                                          _stream_handle(stream, x.device)))
    return out


def mm_multi_device(x, weights, outs=None, stream=None):
    """Several ``mm_batched_device`` calls sharing ``x``, in one launch
    (``rce_qmm_mm_batched_device_multi``): 1-4 weights of one dtype and K,
    e.g. attention q, k, v or FFN gate, up.  Returns the list of outputs
    ([T, N_i] each; ``outs`` may supply them)."""
    import torch

    weights = list(weights)
    if not 1 <= len(weights) <= 4:
        raise ValueError("mm_multi_device takes 1 to 4 weights")
    for w in weights:
        _check_weight(w)
    if x.dim() == 1:
        x = x.view(1, -1)
    if x.dtype != torch.float32 or not x.is_cuda or x.stride(1) != 1:
        raise ValueError("x must be a CUDA float32 tensor with unit column stride")
    t_rows, k = x.shape
    for w in weights:
        if k != w.n_cols:
            raise ValueError(f"activation len {k} ≠ k {w.n_cols}")
    if outs is None:
        outs = [torch.empty((t_rows, w.n_rows), dtype=torch.float32, device=x.device) for w in weights]
    outs = list(outs)
    if len(outs) != len(weights) or any(o.stride(-1) != 1 for o in outs):
        raise ValueError("one output with unit column stride per weight")
    n = len(weights)
    hs = (ctypes.c_void_p * n)(*[w.handle for w in weights])
    ys = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
    lds = (ctypes.c_size_t * n)(*[o.stride(0) if o.dim() == 2 else w.n_rows for o, w in zip(outs, weights)])
    check(lib().rce_qmm_mm_batched_device_multi(weights[0].ctx.handle, ctypes.c_void_p(x.data_ptr()), x.stride(0),
                                                t_rows, hs, n, ys, lds, _stream_handle(stream, x.device)))
    return outs


def dequant_device(w: QuantWeight, row0: int = 0, row1: Optional[int] = None, out=None, stream=None):
    """Bit-exact dequantisation of rows [row0, row1) into a CUDA f32 tensor."""
    import torch

    row1 = w.n_rows if row1 is None else row1
    if out is None:
        out = torch.empty((row1 - row0, w.n_cols), dtype=torch.float32, device=f"cuda:{w.ctx.device}")
    check(lib().rce_qmm_dequant_device(w.ctx.handle, w.handle, int(row0), int(row1), ctypes.c_void_p(out.data_ptr()),
                                       out.stride(0), _stream_handle(stream, out.device)))
    return out


class QmmLeaf:
    """``OpDispatch`` leaf claiming ``Custom("qmm")`` (lib.rs:2075-2131): one
    row-vector × quantized-weight matmul per graph node, the weight selected by
    ``node_id``.  ``execute`` returns the ``[1, n]`` output and raises
    ``Unsupported`` where the reference returns InterpretError::Unsupported."""

    def __init__(self):
        self.weights: Dict[int, QuantWeight] = {}

    def register(self, node_id: int, w: QuantWeight) -> None:
        self.weights[int(node_id)] = w

    def handles(self):
        return ["qmm"]

    def execute(self, node_id: int, name: str, args) -> np.ndarray:
        if name != "qmm":
            raise Unsupported(_lib.RCE_QMM_ERR_UNSUPPORTED, f"QmmLeaf does not handle `{name}`")
        if not args:
            raise Unsupported(_lib.RCE_QMM_ERR_UNSUPPORTED, "qmm: arg 0 must be the activation tensor")
        w = self.weights.get(int(node_id))
        if w is None:
            raise Unsupported(_lib.RCE_QMM_ERR_UNSUPPORTED, f"qmm: no QuantWeight registered for node {node_id}")
        act = np.asarray(args[0])
        if act.dtype != np.float32:
            raise Unsupported(_lib.RCE_QMM_ERR_UNSUPPORTED, f"qmm: activation not f32: {act.dtype}")
        a = act.reshape(-1)
        if a.size != w.n_cols:
            raise Unsupported(_lib.RCE_QMM_ERR_UNSUPPORTED, f"qmm: activation len {a.size} ≠ k {w.n_cols}")
        out = np.empty(w.n_rows, dtype=np.float32)
        mm_1d(a, w, out)
        return out.reshape(1, w.n_rows)


class CudaQmm:
    """``PricedBackend`` + ``QmmDispatch`` for the placement adapter
    (rce-placement-adapter/src/lib.rs:130-134, 187-233): id ``cuda:op-qmm``;
    cost is infinite for dtypes it does not cover, as MetalQmm's
    (lib.rs:257-270), so ``pick_priced`` never routes those here."""

    ID = "cuda:op-qmm"

    def __init__(self, pj_per_flop: float = 0.05, pj_per_byte: float = 0.02, overhead_pj: float = 1.0e6):
        self.coeffs = (pj_per_flop, pj_per_byte, overhead_pj)

    def id(self) -> str:
        return self.ID

    def handles(self):
        return ["qmm"]

    def cost(self, op: str, shapes, dtype=None) -> float:
        if op != "qmm" or len(shapes) < 2:
            return float("inf")
        if dtype is not None and GgufDtype.parse(dtype) not in SUPPORTED:
            return float("inf")
        k = shapes[0][0]
        n = shapes[1][0]
        wbytes = shapes[1][2] if len(shapes[1]) > 2 else 0
        flops = 2 * n * k
        nbytes = wbytes + 4 * k + 4 * n  # qmm_1d_flops_bytes (lib.rs:142-146)
        a, b, c = self.coeffs
        return a * flops + b * nbytes + c

    def qmm_1d(self, a, w: QuantWeight) -> np.ndarray:
        return mm_1d(a, w)
