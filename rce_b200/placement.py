"""The ``cuda:op-qmm`` priced backend for the reference's placement layer, and
the pieces of that layer it plugs into, mirrored on the host.

The reference routes every ``qmm_1d(a, w)`` through
``PlacementQmmAdapter`` (rce-placement-adapter/src/lib.rs:330-480): each
registered backend prices the call (``PricedBackend::cost``), the cheapest
one that handles ``"qmm"`` wins (``pick_priced``,
rce-vm-scheduler/src/placement.rs:98-117), the decision is cached per
``(op, n_rows, n_cols, dtype_id)``, and every dispatch is appended to a
``DispatchTranscript`` whose FNV-1a digest lets replicas compare what ran
(rce-placement-adapter/src/trace.rs:59-142).  ``CudaQmm`` is the backend a
maintainer registers there (``PlacementQmmAdapter::register``, lib.rs:418)
to route quantized matmuls to the B200: its ``cost`` gates on the weight
format the way ``MetalQmm::cost`` does (lib.rs:255-272: INFINITY for a
format it has no kernel for, so the generalist CPU backend wins those) and
prices the call with ``qmm_1d_flops_bytes`` (lib.rs:140-146) through a cost
table; its ``qmm_1d`` runs ``rce_b200.mm_1d``.

The shape encoding (``[k]`` and ``[n_rows, n_cols, weight_bytes,
dtype_id]``), the dtype ids and the transcript's byte encoding are the
reference's wire format, kept identical so that a transcript written here
has the digest the reference computes for the same dispatches.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field
from enum import IntEnum
from typing import Dict, List, Optional, Sequence, Tuple

from .gguf import GgufDtype

# dtype slot of the weight shape (rce-placement-adapter/src/lib.rs:83-93)
QMM_DTYPE_UNKNOWN = 0
QMM_DTYPE_Q8_0 = 1
QMM_DTYPE_Q4_K = 2
QMM_DTYPE_Q5_K = 3
QMM_DTYPE_Q6_K = 4
QMM_DTYPE_Q4_0 = 5
QMM_DTYPE_Q5_0 = 6
QMM_DTYPE_Q4_1 = 7
QMM_DTYPE_Q1_0 = 8
QMM_DTYPE_Q2_0 = 9
QMM_DTYPE_Q3_K = 10

_DTYPE_IDS = {GgufDtype.Q8_0: QMM_DTYPE_Q8_0, GgufDtype.Q4K: QMM_DTYPE_Q4_K, GgufDtype.Q5K: QMM_DTYPE_Q5_K,
              GgufDtype.Q6K: QMM_DTYPE_Q6_K, GgufDtype.Q4_0: QMM_DTYPE_Q4_0}


def qmm_dtype_id(dtype) -> int:
    """qmm_dtype_id (lib.rs:108-123) for the formats this library knows;
    every other tag maps to QMM_DTYPE_UNKNOWN."""
    try:
        return _DTYPE_IDS.get(GgufDtype(int(dtype)), QMM_DTYPE_UNKNOWN)
    except ValueError:
        return QMM_DTYPE_UNKNOWN


def cuda_qmm_supports(dtype_id: int) -> bool:
    """True iff this library has a kernel for the format (Q8_0, Q4_0, Q4_K,
    Q5_K, Q6_K): the CUDA counterpart of metal_qmm_supports (lib.rs:96-103)."""
    return dtype_id in (QMM_DTYPE_Q8_0, QMM_DTYPE_Q4_0, QMM_DTYPE_Q4_K, QMM_DTYPE_Q5_K, QMM_DTYPE_Q6_K)


def qmm_1d_flops_bytes(n: int, k: int, weight_bytes: int) -> Tuple[int, int]:
    """(2 n k, weight bytes + 4 k + 4 n) of qmm_1d(a: [k], w: [n, k])
    (lib.rs:140-146)."""
    return 2 * n * k, weight_bytes + 4 * k + 4 * n


class EnergyBasis(IntEnum):
    """D.11 basis of a cost estimate; the value is its digest code."""
    EST = 0
    REPORTED = 1
    MEASURED = 2


@dataclass(frozen=True)
class LinearCoeffs:
    """pJ = a * flops + b * bytes + c (rce-placement/src/lib.rs:230-243)."""
    a_pj_per_flop: float
    b_pj_per_byte: float
    c_pj_overhead: float

    def estimate_pj(self, flops: int, bytes_: int) -> float:
        return self.a_pj_per_flop * float(flops) + self.b_pj_per_byte * float(bytes_) + self.c_pj_overhead


class CostTable:
    """Per-(op, backend) coefficients with a basis; missing cells take the
    fallback prior with basis EST (rce-placement/src/lib.rs:245-320)."""

    def __init__(self, fallback: LinearCoeffs):
        self.fallback = fallback
        self.cells: Dict[Tuple[str, str], Tuple[LinearCoeffs, EnergyBasis]] = {}

    def insert(self, op: str, backend: str, coeffs: LinearCoeffs, basis: EnergyBasis = EnergyBasis.EST) -> None:
        self.cells[(op, backend)] = (coeffs, basis)

    def lookup(self, op: str, backend: str) -> Tuple[LinearCoeffs, EnergyBasis]:
        return self.cells.get((op, backend), (self.fallback, EnergyBasis.EST))

    def estimate(self, op: str, backend: str, flops: int, bytes_: int) -> Tuple[float, EnergyBasis]:
        c, basis = self.lookup(op, backend)
        return c.estimate_pj(flops, bytes_), basis


# Analytical prior of the B200 backend for qmm, basis EST.  a: the tensor
# path's energy per flop (1000 W at the measured ~1.6 PFLOP/s dense fp16);
# b: HBM energy per byte (1000 W at the measured ~6.5 TB/s copy rate); c:
# the fixed cost of one host call (copy in, launch, copy out and
# synchronise: ~40 us at ~500 W).  The CPU cell is the reference's own
# prior (lib.rs:160-168).
CUDA_QMM_COEFFS = LinearCoeffs(a_pj_per_flop=0.6, b_pj_per_byte=0.15, c_pj_overhead=20_000_000.0)
CPU_QMM_COEFFS = LinearCoeffs(a_pj_per_flop=10.0, b_pj_per_byte=0.05, c_pj_overhead=500_000.0)


def default_qmm_cost_table() -> CostTable:
    """default_qmm_cost_table (lib.rs:148-170) with the cuda:op-qmm cell."""
    t = CostTable(LinearCoeffs(1.0, 0.0, 0.0))
    t.insert("qmm", "cpu:op-qmm", CPU_QMM_COEFFS, EnergyBasis.EST)
    t.insert("qmm", "cuda:op-qmm", CUDA_QMM_COEFFS, EnergyBasis.EST)
    return t


class CudaQmm:
    """PricedBackend + QmmDispatch of this library (id ``cuda:op-qmm``)."""

    def __init__(self, table: CostTable, ctx=None):
        self.table = table
        self.ctx = ctx

    def id(self) -> str:
        return "cuda:op-qmm"

    def handles(self) -> Sequence[str]:
        return ("qmm",)

    def cost(self, op: str, shapes: Sequence[Sequence[int]]) -> Tuple[float, EnergyBasis]:
        """shapes = [[k], [n_rows, n_cols, weight_bytes, dtype_id]]; INFINITY
        for another op or a format this library has no kernel for."""
        if op != "qmm" or len(shapes) < 2:
            return math.inf, EnergyBasis.EST
        w_shape = shapes[1]
        dtype_id = w_shape[3] if len(w_shape) > 3 else QMM_DTYPE_UNKNOWN
        if not cuda_qmm_supports(dtype_id):
            return math.inf, EnergyBasis.EST
        k = int(shapes[0][0])
        n_rows = int(w_shape[0])
        weight_bytes = int(w_shape[2]) if len(w_shape) > 2 else 0
        flops, nbytes = qmm_1d_flops_bytes(n_rows, k, weight_bytes)
        return self.table.estimate(op, self.id(), flops, nbytes)

    def execute(self, op: str, inputs) -> None:
        raise RuntimeError("CudaQmm: qmm dispatch uses qmm_1d, not execute (QuantWeight does not fit the Value model)")

    def qmm_1d(self, a, w):
        from .qmm import mm_1d

        return mm_1d(a, w)


def pick_priced(backends, op: str, shapes):
    """The cheapest backend that handles op (the first of equal costs), with
    its estimate, or None (rce-vm-scheduler/src/placement.rs:98-117)."""
    best = None
    for be in backends:
        if op not in be.handles():
            continue
        pj, basis = be.cost(op, shapes)
        if best is None or pj < best[1]:
            best = (be, pj, basis)
    return best


# ---- verifiable dispatch trace (rce-placement-adapter/src/trace.rs) --------

_TAG_OP, _TAG_A_SHAPE, _TAG_W_SHAPE, _TAG_BACKEND, _TAG_EST_PJ, _TAG_MEASURED = 1, 2, 3, 4, 5, 6
_FNV_OFFSET = 0xCBF29CE484222325
_FNV_PRIME = 0x100000001B3


@dataclass
class DispatchEvent:
    """One qmm_1d dispatch: op, activation shape [k], weight shape [n_rows,
    n_cols, weight_bytes, dtype_id], the chosen backend and its estimate."""
    op: str
    a_shape: List[int]
    w_shape: List[int]
    backend_id: str
    estimated_picojoules: float
    basis: EnergyBasis = EnergyBasis.EST

    def encode(self) -> bytes:
        """The event's canonical bytes: tagged fields, u64 little-endian
        lengths and values, length-prefixed UTF-8 strings, the estimate as
        its f64 bits, the basis as one byte."""
        def u64(v: int) -> bytes:
            return struct.pack("<Q", v & 0xFFFFFFFFFFFFFFFF)

        def s(v: str) -> bytes:
            b = v.encode()
            return u64(len(b)) + b

        out = bytes([_TAG_OP]) + s(self.op)
        out += bytes([_TAG_A_SHAPE]) + u64(len(self.a_shape)) + b"".join(u64(int(x)) for x in self.a_shape)
        out += bytes([_TAG_W_SHAPE]) + u64(len(self.w_shape)) + b"".join(u64(int(x)) for x in self.w_shape)
        out += bytes([_TAG_BACKEND]) + s(self.backend_id)
        out += bytes([_TAG_EST_PJ]) + struct.pack("<d", float(self.estimated_picojoules))
        out += bytes([_TAG_MEASURED, int(self.basis)])
        return out


@dataclass
class DispatchTranscript:
    """Ordered log of dispatch events with an FNV-1a digest over (position,
    event) pairs in append order."""
    events: List[DispatchEvent] = field(default_factory=list)

    def append(self, ev: DispatchEvent) -> int:
        self.events.append(ev)
        return len(self.events) - 1

    def __len__(self) -> int:
        return len(self.events)

    def digest(self) -> int:
        buf = b"".join(struct.pack("<Q", i) + ev.encode() for i, ev in enumerate(self.events))
        h = _FNV_OFFSET
        for b in buf:
            h ^= b
            h = (h * _FNV_PRIME) & 0xFFFFFFFFFFFFFFFF
        return h


@dataclass
class PlacementAdapterStats:
    calls: int = 0
    reading_calls: int = 0
    estimated_picojoules: float = 0.0
    calls_per_backend: Dict[str, int] = field(default_factory=dict)
    dispatch_cache_hits: int = 0
    dispatch_cache_misses: int = 0

    def record(self, backend_id: str, pj: float, basis: EnergyBasis) -> None:
        self.calls += 1
        self.estimated_picojoules += pj
        if basis in (EnergyBasis.REPORTED, EnergyBasis.MEASURED):
            self.reading_calls += 1
        self.calls_per_backend[backend_id] = self.calls_per_backend.get(backend_id, 0) + 1


class PlacementQmmAdapter:
    """The reference's adapter (lib.rs:330-480) with backends registered on
    the host: per call the cached or freshly picked backend, its estimate in
    stats and an event in the transcript, then the dispatch."""

    def __init__(self, table: Optional[CostTable] = None):
        self.table = table or default_qmm_cost_table()
        self.backends: List = []
        self.dispatchers: Dict[str, object] = {}
        self.dispatch_cache: Dict[Tuple[str, int, int, int], str] = {}
        self.stats = PlacementAdapterStats()
        self.transcript = DispatchTranscript()

    @classmethod
    def with_cuda(cls, ctx=None) -> "PlacementQmmAdapter":
        s = cls()
        s.register(CudaQmm(s.table, ctx))
        return s

    def register(self, backend) -> None:
        self.backends.append(backend)
        self.dispatchers[backend.id()] = backend

    def clear_dispatch_cache(self) -> None:
        self.dispatch_cache.clear()

    def route(self, k: int, n_rows: int, n_cols: int, weight_bytes: int, dtype_id: int):
        """The placement decision for one call, recorded in stats and the
        transcript: (backend_id, picojoules, basis)."""
        a_shape = [k]
        w_shape = [n_rows, n_cols, weight_bytes, dtype_id]
        key = ("qmm", n_rows, n_cols, dtype_id)
        cached = self.dispatch_cache.get(key)
        if cached is not None:
            self.stats.dispatch_cache_hits += 1
            flops, nbytes = qmm_1d_flops_bytes(n_rows, n_cols, weight_bytes)
            pj, basis = self.table.estimate("qmm", cached, flops, nbytes)
            be_id = cached
        else:
            self.stats.dispatch_cache_misses += 1
            picked = pick_priced(self.backends, "qmm", [a_shape, w_shape])
            if picked is None:
                raise RuntimeError("no priced backend handles `qmm`")
            be, pj, basis = picked
            be_id = be.id()
            self.dispatch_cache[key] = be_id
        self.stats.record(be_id, pj, basis)
        self.transcript.append(DispatchEvent("qmm", a_shape, w_shape, be_id, pj, basis))
        return be_id, pj, basis

    def qmm_1d(self, a, w):
        if len(a) != w.n_cols:
            raise ValueError(f"activation len {len(a)} != n_cols {w.n_cols}")
        be_id, _, _ = self.route(len(a), w.n_rows, w.n_cols, w.nbytes(), qmm_dtype_id(w.dtype))
        return self.dispatchers[be_id].qmm_1d(a, w)
