"""CPU-only checks of the boundary: the C-ABI library loads and exports every
symbol include/rce_qmm.h declares; host-side logic that needs no GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle as O
from rce_b200 import _lib, gguf, synth
from rce_b200.qmm import CudaQmm, QmmLeaf, Unsupported

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rce_qmm.h")


def header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rce_qmm_\w+)\s*\(", text)))


def test_header_declares_the_expected_surface():
    syms = header_symbols()
    for s in ["rce_qmm_mm_1d", "rce_qmm_mm_batched", "rce_qmm_weight_register", "rce_qmm_dequant_row",
              "rce_qmm_last_error", "rce_qmm_tensor_byte_size"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in header_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert set(header_symbols()) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_abi_version_and_pure_functions():
    L = _lib.lib()
    assert L.rce_qmm_abi_version() == 1
    for dt in (O.GGUF_Q4_0, O.GGUF_Q8_0, O.GGUF_Q4_K, O.GGUF_Q5_K, O.GGUF_Q6_K):
        for n in (1, 31, 32, 33, 255, 256, 257, 4096 * 4096):
            assert L.rce_qmm_tensor_byte_size(dt, n) == O.tensor_byte_size(dt, n) == gguf.tensor_byte_size(dt, n)
    assert L.rce_qmm_tensor_byte_size(6, 32) == 0


def test_bad_device_is_an_error_not_a_crash():
    L = _lib.lib()
    h = ctypes.c_void_p()
    rc = L.rce_qmm_ctx_create(-1, ctypes.byref(h))
    assert rc != 0 and L.rce_qmm_last_error()
    with pytest.raises(_lib.QmmError):
        _lib.check(rc)


def test_null_arguments_are_rejected():
    L = _lib.lib()
    assert L.rce_qmm_ctx_create(0, None) == _lib.RCE_QMM_ERR_INVALID
    assert L.rce_qmm_weight_free(None) == _lib.RCE_QMM_ERR_INVALID
    assert L.rce_qmm_mm_batched(None, None, 1, None, None, 0) == _lib.RCE_QMM_ERR_INVALID
    assert b"null" in L.rce_qmm_last_error()


def test_qmm_leaf_errors_match_reference():
    # QmmLeaf::execute's Unsupported paths (rce-op-qmm/src/lib.rs:2096-2124)
    leaf = QmmLeaf()
    assert leaf.handles() == ["qmm"]
    with pytest.raises(Unsupported, match="does not handle"):
        leaf.execute(1, "matmul", [np.zeros(4, np.float32)])
    with pytest.raises(Unsupported, match="no QuantWeight registered"):
        leaf.execute(1, "qmm", [np.zeros(4, np.float32)])
    with pytest.raises(Unsupported, match="arg 0"):
        leaf.execute(1, "qmm", [])


def test_cuda_qmm_cost_gates_formats():
    b = CudaQmm()
    assert b.id() == "cuda:op-qmm"
    assert b.cost("qmm", [[4096], [4096, 4096, 9437184]], dtype=12) < float("inf")
    assert b.cost("qmm", [[4096], [4096, 4096, 0]], dtype=gguf.GgufDtype.F16) == float("inf")
    assert b.cost("matmul", [[1], [1, 1]]) == float("inf")


def test_synth_is_deterministic_and_in_range():
    a = synth.q4_k(16, 512, np.random.default_rng(2))
    b = synth.q4_k(16, 512, np.random.default_rng(2))
    assert np.array_equal(a, b) and a.size == gguf.tensor_byte_size(12, 16 * 512)
    q8 = synth.q8_0(8, 256, np.random.default_rng(0))
    q, d = O.unpack_q8_0(q8, 8, 256)
    assert q.min() >= -127 and q.max() <= 127 and np.all(d >= 0)
    q4 = synth.q4_0(8, 256, np.random.default_rng(1))
    q, d = O.unpack_q4_0(q4, 8, 256)
    assert q.min() >= -8 and q.max() <= 7


def test_dtype_parse():
    assert gguf.GgufDtype.parse("Q4_K") == gguf.GgufDtype.Q4K == 12
    assert gguf.GgufDtype.parse(8) == gguf.GgufDtype.Q8_0
