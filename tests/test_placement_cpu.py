"""The cuda:op-qmm priced backend and the host mirror of the placement pieces
it plugs into (rce_b200/placement.py), without a GPU: format gating and
pricing (rce-placement-adapter/src/lib.rs:128-146, 255-272), pick_priced
(rce-vm-scheduler/src/placement.rs:98-117), the adapter's dispatch cache and
stats, and the dispatch transcript's digest with the properties the
reference's own tests assert (rce-placement-adapter/src/trace.rs:170-290)."""
import math
import struct

import pytest

from rce_b200 import placement as P
from rce_b200.gguf import GgufDtype


def ev(be="cpu:op-qmm", w=(2048, 2048, 32, 1), pj=1.0e6, basis=P.EnergyBasis.EST, a=(2048,)):
    return P.DispatchEvent("qmm", list(a), list(w), be, pj, basis)


def test_dtype_ids_and_gating():
    assert P.qmm_dtype_id(GgufDtype.Q8_0) == P.QMM_DTYPE_Q8_0 == 1
    assert P.qmm_dtype_id(GgufDtype.Q4K) == 2 and P.qmm_dtype_id(GgufDtype.Q6K) == 4
    assert P.qmm_dtype_id(GgufDtype.Q4_0) == 5 and P.qmm_dtype_id(999) == P.QMM_DTYPE_UNKNOWN
    be = P.CudaQmm(P.default_qmm_cost_table())
    assert be.id() == "cuda:op-qmm" and tuple(be.handles()) == ("qmm",)
    for dt in (P.QMM_DTYPE_UNKNOWN, P.QMM_DTYPE_Q3_K, P.QMM_DTYPE_Q5_0, P.QMM_DTYPE_Q4_1):
        assert math.isinf(be.cost("qmm", [[4096], [4096, 4096, 100, dt]])[0])
    assert math.isinf(be.cost("matmul", [[4096], [4096, 4096, 100, 1]])[0])
    assert math.isinf(be.cost("qmm", [[4096]])[0])
    with pytest.raises(RuntimeError):
        be.execute("qmm", [])


def test_cost_is_the_linear_prior_of_flops_and_bytes():
    be = P.CudaQmm(P.default_qmm_cost_table())
    n, k, wb = 14336, 4096, 33030144
    flops, nbytes = P.qmm_1d_flops_bytes(n, k, wb)
    assert (flops, nbytes) == (2 * n * k, wb + 4 * k + 4 * n)
    pj, basis = be.cost("qmm", [[k], [n, k, wb, P.QMM_DTYPE_Q4_K]])
    c = P.CUDA_QMM_COEFFS
    assert pj == c.a_pj_per_flop * flops + c.b_pj_per_byte * nbytes + c.c_pj_overhead
    assert basis == P.EnergyBasis.EST


class CpuPrior:
    """A CPU backend priced with the reference's cpu:op-qmm cell (cost only)."""

    def __init__(self, table):
        self.table = table

    def id(self):
        return "cpu:op-qmm"

    def handles(self):
        return ("qmm",)

    def cost(self, op, shapes):
        flops, nbytes = P.qmm_1d_flops_bytes(shapes[1][0], shapes[0][0], shapes[1][2])
        return self.table.estimate(op, self.id(), flops, nbytes)


def test_pick_priced_routes_small_calls_to_cpu_and_large_ones_to_cuda():
    t = P.default_qmm_cost_table()
    backends = [CpuPrior(t), P.CudaQmm(t)]
    small = [[64], [64, 64, 64 * 64 // 32 * 34, P.QMM_DTYPE_Q8_0]]
    large = [[4096], [4096, 4096, 4096 * 4096 // 32 * 34, P.QMM_DTYPE_Q8_0]]
    unknown = [[4096], [4096, 4096, 1 << 20, P.QMM_DTYPE_Q3_K]]
    assert P.pick_priced(backends, "qmm", small)[0].id() == "cpu:op-qmm"
    assert P.pick_priced(backends, "qmm", large)[0].id() == "cuda:op-qmm"
    assert P.pick_priced(backends, "qmm", unknown)[0].id() == "cpu:op-qmm"  # gated out: the generalist wins
    assert P.pick_priced(backends, "softmax", small) is None


def test_adapter_caches_decisions_and_records_every_dispatch():
    t = P.default_qmm_cost_table()
    ad = P.PlacementQmmAdapter(t)
    ad.register(CpuPrior(t))
    ad.register(P.CudaQmm(t))
    wb = 4096 * 4096 // 256 * 144
    for _ in range(3):
        be, pj, basis = ad.route(4096, 4096, 4096, wb, P.QMM_DTYPE_Q4_K)
        assert be == "cuda:op-qmm" and basis == P.EnergyBasis.EST
    ad.route(64, 64, 64, 64 // 32 * 34 * 64, P.QMM_DTYPE_Q8_0)
    s = ad.stats
    assert (s.dispatch_cache_misses, s.dispatch_cache_hits) == (2, 2)
    assert s.calls == 4 and s.calls_per_backend == {"cuda:op-qmm": 3, "cpu:op-qmm": 1}
    assert len(ad.transcript) == 4
    assert [e.backend_id for e in ad.transcript.events] == ["cuda:op-qmm"] * 3 + ["cpu:op-qmm"]
    assert ad.transcript.events[0].w_shape == [4096, 4096, wb, P.QMM_DTYPE_Q4_K]


def _fnv1a(data: bytes) -> int:
    h = 0xCBF29CE484222325
    for b in data:
        h = ((h ^ b) * 0x100000001B3) % (1 << 64)
    return h


def test_digest_of_the_canonical_encoding():
    # the empty transcript is the FNV-1a offset basis; one event is the
    # FNV-1a of: u64 position, tag 1 + "qmm", tag 2 + [2048], tag 3 +
    # [2048, 2048, 32, 1], tag 4 + backend, tag 5 + f64 bits, tag 6 + basis
    assert P.DispatchTranscript().digest() == 0xCBF29CE484222325
    q = lambda v: struct.pack("<Q", v)  # noqa: E731
    raw = (q(0) + b"\x01" + q(3) + b"qmm" + b"\x02" + q(1) + q(2048) + b"\x03" + q(4) + q(2048) + q(2048) + q(32)
           + q(1) + b"\x04" + q(10) + b"cpu:op-qmm" + b"\x05" + struct.pack("<d", 1.0e6) + b"\x06\x00")
    t = P.DispatchTranscript()
    t.append(ev())
    assert t.digest() == _fnv1a(raw)


def test_transcript_properties_of_the_reference_tests():
    def build(*events):
        t = P.DispatchTranscript()
        for e in events:
            t.append(e)
        return t.digest()

    e1, e2 = ev(), ev("cuda:op-qmm", (5632, 2048, 64, 1), 5.0e5)
    assert build(e1, e2) == build(ev(), ev("cuda:op-qmm", (5632, 2048, 64, 1), 5.0e5))  # honest replicas agree
    assert build(ev("cuda:op-qmm")) != build(ev("cpu:op-qmm"))                       # backend swap
    assert build(e1, e2) != build(e1)                                                 # dropped event
    assert build(ev(pj=1.0e6)) != build(ev(pj=1.1e6))                                 # cost drift
    assert build(ev()) != build(ev(basis=P.EnergyBasis.REPORTED))                     # basis
    assert build(e1, e2) != build(e2, e1)                                             # order
    assert build(ev(w=(2048, 2048, 32, 1))) != build(ev(w=(2048, 2048, 32, 2)))       # dtype swap
