"""Loader for libks_b200.so, the C-ABI operator library (include/ks_b200.h).

The library is built in-tree by ``kernelswift_b200.build`` (nvcc, sm_100a) and
loaded with ctypes.  There is no fallback: if the library is missing, every op
raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libks_b200.so")

KS_OK = 0
KS_ERR_INVALID = 1
KS_ERR_UNSUPPORTED = 2
KS_ERR_ALIGNMENT = 3
KS_ERR_CUDA = 4
KS_ERR_WORKSPACE = 5
KS_ERR_DEVICE = 6
KS_INT32 = 0
KS_INT64 = 1

_c_i32, _c_i64, _c_u64, _c_f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float
_vp, _sz = ctypes.c_void_p, ctypes.c_size_t

# name -> (restype, argtypes), mirroring include/ks_b200.h
SIGNATURES = {
    "ks_last_error": (ctypes.c_char_p, []),
    "ks_version": (ctypes.c_int, []),
    "ks_sinkhorn": (ctypes.c_int, [_vp, _vp, _c_i64, _c_i32, _c_i32, _c_f32, _vp]),
    "ks_sparse_attn": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64,
                                      _c_i64, _c_i64, _c_i64, _c_i64, _c_f32, _vp]),
    "ks_indexer_workspace_size": (_sz, [_c_i64, _c_i64, _c_i64]),
    "ks_indexer": (ctypes.c_int, [_vp, _vp, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64,
                                  _c_i64, _c_i32, _c_i64, _c_i32, _c_i32, _c_i32, _c_i64, _vp,
                                  _c_i32, _vp, _sz, _vp]),
    "ks_indexer_scores": (ctypes.c_int, [_vp, _vp, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                         _c_i64, _c_i64, _c_i32, _c_i64, _c_i32, _c_i32, _vp,
                                         _c_i64, _vp]),
    "ks_topk_rows": (ctypes.c_int, [_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32,
                                    _c_i32, _c_i64, _vp, _c_i32, _vp]),
    "ks_indexer_noalloc": (ctypes.c_int, [_vp, _vp, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                          _c_i64, _c_i64, _c_i32, _c_i64, _c_i32, _c_i32, _c_i32,
                                          _c_i64, _vp, _c_i32, _vp]),
    "ks_dsa": (ctypes.c_int, [_vp, _vp, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                              _c_i32, _c_i64, _c_i32, _c_i32, _c_i32, _c_i64, _vp, _vp, _c_i64, _vp,
                              _c_i64, _c_i64, _c_i64, _c_f32, _vp, _vp, _vp, _sz, _vp]),
    "ks_proj_rope": (ctypes.c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32, _vp,
                                    _c_i64, _c_f32, _c_i32, _vp]),
    "ks_quant_fp8_rows": (ctypes.c_int, [_vp, _vp, _vp, _c_i64, _c_i32, _vp]),
    "ks_indexer_fp8": (ctypes.c_int, [_vp, _vp, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64,
                                      _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i64, _vp, _c_i32,
                                      _vp, _sz, _vp]),
    "ks_indexer_fp8_scores": (ctypes.c_int, [_vp, _vp, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                             _c_i64, _c_i64, _c_i64, _c_i32, _c_i32, _vp, _c_i64,
                                             _vp]),
    "ks_device_status": (ctypes.c_int, [_vp]),
    "ks_selftest_wait_timeout": (ctypes.c_int, [_c_u64, _vp]),
}


class KsError(RuntimeError):
    """A libks_b200 call returned an error code."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_LIB = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m kernelswift_b200.build` "
                "(the operators have no fallback path)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(rc: int, what: str) -> None:
    if rc != KS_OK:
        msg = lib().ks_last_error().decode(errors="replace")
        raise KsError(rc, f"{what} failed (code {rc}): {msg}")
