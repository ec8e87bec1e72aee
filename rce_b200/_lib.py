"""ctypes binding of librce_qmm.so (include/rce_qmm.h).

The library is built in-tree (``rce_b200/_build/librce_qmm.so``) by
``rce_b200/build.py`` / ``__graft_entry__.build()``.  There is no fallback:
if the library is missing or cannot load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "librce_qmm.so")

RCE_QMM_OK = 0
RCE_QMM_ERR_INVALID = 1
RCE_QMM_ERR_UNSUPPORTED = 2
RCE_QMM_ERR_CUDA = 3
RCE_QMM_ERR_NOMEM = 4
RCE_QMM_ERR_TIMEOUT = 5

_lib = None
_lock = threading.Lock()

_c = ctypes
_vp = _c.c_void_p
_vpp = _c.POINTER(_c.c_void_p)
_f32p = _c.POINTER(_c.c_float)
_sz = _c.c_size_t
_i64 = _c.c_int64
_int = _c.c_int

# name -> (restype, argtypes); every symbol declared in include/rce_qmm.h.
SIGNATURES = {
    "rce_qmm_abi_version": (_int, []),
    "rce_qmm_last_error": (_c.c_char_p, []),
    "rce_qmm_tensor_byte_size": (_sz, [_int, _c.c_uint64]),
    "rce_qmm_ctx_create": (_int, [_int, _vpp]),
    "rce_qmm_ctx_destroy": (_int, [_vp]),
    "rce_qmm_ctx_sm_count": (_int, [_vp, _c.POINTER(_int)]),
    "rce_qmm_ctx_set_prefill_min_tokens": (_int, [_vp, _int]),
    "rce_qmm_ctx_get_prefill_min_tokens": (_int, [_vp, _c.POINTER(_int)]),
    "rce_qmm_weight_register": (_int, [_vp, _vp, _sz, _int, _i64, _i64, _vpp]),
    "rce_qmm_weight_register_device": (_int, [_vp, _vp, _sz, _int, _i64, _i64, _vp, _vpp]),
    "rce_qmm_weight_sub_view": (_int, [_vp, _sz, _sz, _i64, _i64, _vpp]),
    "rce_qmm_weight_free": (_int, [_vp]),
    "rce_qmm_weight_info": (_int, [_vp, _c.POINTER(_int), _c.POINTER(_i64), _c.POINTER(_i64), _c.POINTER(_sz)]),
    "rce_qmm_weight_device_storage": (_int, [_vp, _vpp, _c.POINTER(_sz)]),
    "rce_qmm_weight_read_bytes": (_int, [_vp, _vp, _sz]),
    # (the per-token host calls take plain addresses: building a typed
    # pointer costs several microseconds a call)
    "rce_qmm_mm_1d": (_int, [_vp, _vp, _sz, _vp, _vp, _sz]),
    "rce_qmm_mm_1d_serial": (_int, [_vp, _f32p, _sz, _vp, _f32p, _sz]),
    "rce_qmm_mm_batched": (_int, [_vp, _vp, _sz, _vp, _vp, _sz]),
    "rce_qmm_mm_batched_device": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _vp]),
    "rce_qmm_mm_batched_device_noalloc": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _vp]),
    "rce_qmm_mm_batched_device_multi": (_int, [_vp, _vp, _sz, _sz, _vp, _sz, _vp, _vp, _vp]),
    "rce_qmm_mm_batched_device_multi_gather": (_int, [_vp, _vp, _sz, _sz, _vp, _sz, _int, _int, _vp, _vp, _vp, _vp,
                                                      _c.c_uint, _vp, _vp]),
    "rce_qmm_mm_batched_device_multi_gather_bulk": (_int, [_vp, _vp, _sz, _sz, _vp, _sz, _int, _int, _vp, _vp, _vp,
                                                           _vp, _vp, _c.c_uint, _vp, _vp]),
    "rce_qmm_peer_unpack_bulk": (_int, [_vp, _vp, _sz, _vp, _sz, _sz, _i64, _i64, _i64, _int, _int, _c.c_uint, _vp,
                                        _vp]),
    "rce_qmm_dequant_row": (_int, [_vp, _vp, _i64, _f32p, _sz]),
    "rce_qmm_dequant_device": (_int, [_vp, _vp, _i64, _i64, _vp, _sz, _vp]),
    "rce_qmm_device_error": (_int, [_vp, _c.POINTER(_int), _int]),
    "rce_qmm_peer_alloc": (_int, [_vp, _sz, _c.POINTER(_vp), _vp]),
    "rce_qmm_peer_free": (_int, [_vp, _vp]),
    "rce_qmm_peer_open": (_int, [_vp, _vp, _c.POINTER(_vp)]),
    "rce_qmm_peer_close": (_int, [_vp, _vp]),
    "rce_qmm_mm_batched_device_gather": (_int, [_vp, _vp, _sz, _sz, _vp, _int, _int, _i64, _vp, _sz, _vp, _c.c_uint,
                                                 _vp, _vp]),
    "rce_qmm_peer_unpack": (_int, [_vp, _vp, _vp, _sz, _sz, _i64, _i64, _i64, _c.c_uint, _vp, _vp]),
    "rce_qmm_peer_epoch_advance": (_int, [_vp, _vp, _c.c_uint, _vp]),
    "rce_qmm_moe_route_device": (_int, [_vp, _vp, _sz, _sz, _int, _int, _int, _vp, _vp, _vp]),
    "rce_qmm_moe_ffn_device": (_int, [_vp, _vp, _sz, _sz, _vp, _sz, _int, _int, _int, _int, _vp, _vp, _vp, _vp,
                                       _sz, _vp, _vp, _vp]),
    "rce_qmm_moe_router_device": (_int, [_vp, _vp, _sz, _sz, _vp, _int, _int, _vp, _sz, _vp, _vp, _vp]),
    "rce_qmm_moe_ffn": (_int, [_vp, _vp, _sz, _vp, _vp, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _vp]),
    "rce_qmm_moe_shared_expert_device": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "rce_qmm_synchronize": (_int, [_vp]),
}


class QmmError(RuntimeError):
    """A librce_qmm call failed; ``code`` is the RCE_QMM_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"rce_qmm error {code}: {msg}")
        self.code = code


class Unsupported(QmmError):
    """The call's dtype or shape is outside this library (the reference
    panics or returns InterpretError::Unsupported there)."""


def lib():
    """Load librce_qmm.so once; raise if it is missing (no CPU fallback)."""
    global _lib
    loaded = _lib
    if loaded is not None:  # (no lock once loaded: this runs on every call)
        return loaded
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"librce_qmm.so not built ({LIB_PATH}); run `python -c 'import __graft_entry__ as g; g.build()'`"
                )
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != RCE_QMM_OK:
        msg = lib().rce_qmm_last_error().decode("utf-8", "replace")
        if rc == RCE_QMM_ERR_UNSUPPORTED:
            raise Unsupported(rc, msg)
        raise QmmError(rc, msg)
