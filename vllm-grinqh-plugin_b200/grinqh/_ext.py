"""Loading of the native libraries. There is no fallback: if the CUDA library or
the torch-op library is missing, importing the ops raises."""
from __future__ import annotations

import ctypes
import os
import threading

_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_DIR, "libgrinqh_b200.so")
OPS_PATH = os.path.join(_DIR, "_grinqh_ops.so")

_lock = threading.Lock()
_cabi = None
_ops_loaded = False

# C ABI status codes (include/grinqh_b200.h)
GRINQH_OK = 0
GRINQH_F16, GRINQH_BF16 = 0, 1
MODE_AUTO, MODE_DENSE, MODE_GRADED, MODE_UNION = 0, 1, 2, 3

_i64, _int, _ptr, _size = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
_fptr = ctypes.POINTER(ctypes.c_float)

# (name, restype, argtypes) for every entry point of include/grinqh_b200.h
SIGNATURES = {
    "grinqh_abi_version": (_int, []),
    "grinqh_status_string": (ctypes.c_char_p, [_int]),
    "grinqh_last_error": (ctypes.c_char_p, []),
    "grinqh_take_error_flags": (_int, [_ptr]),
    "grinqh_pack_words": (_int, [_ptr, _ptr, _i64, _i64, _int, _ptr]),
    "grinqh_pack_codes": (_int, [_ptr, _i64, _ptr, _i64, _i64, _int, _ptr]),
    "grinqh_unpack_checkpoint": (_int, [_ptr, _i64, _int, _i64, _i64, _i64, _i64, _ptr, _i64, _ptr]),
    "grinqh_allreduce_buffer_bytes": (ctypes.c_size_t, [_int, _i64]),
    "grinqh_allreduce_buffer_alloc": (_int, [ctypes.c_size_t, _ptr]),
    "grinqh_allreduce_buffer_free": (_int, [_ptr]),
    "grinqh_ipc_get_handle": (_int, [_ptr, _ptr]),
    "grinqh_ipc_open_handle": (_int, [_ptr, _ptr]),
    "grinqh_ipc_close_handle": (_int, [_ptr]),
    "grinqh_gemv_allreduce": (_int, [_ptr, _int, _i64, _ptr, _ptr, _ptr, _int, _int, _i64, _ptr, _ptr, _ptr,
                                     ctypes.c_size_t, _int, _int, _ptr, _i64, _int, _ptr]),
    "grinqh_allreduce_workspace_size": (_size, [_i64, _i64, _i64, _int, _int, _int]),
    "grinqh_gemm_allreduce": (_int, [_ptr, _int, _i64, _i64, _ptr, _ptr, _ptr, _int, _int, _i64, _fptr, _int,
                                     _ptr, _ptr, _size, _int, _int, _ptr, _i64, _ptr]),
    "grinqh_unpack": (_int, [_ptr, _ptr, _i64, _i64, _int, _ptr]),
    "grinqh_grade": (_int, [_ptr, _int, _i64, _i64, _fptr, _int, _ptr, _ptr, _ptr]),
    "grinqh_workspace_size": (_size, [_i64, _i64, _i64, _int, _int, _int]),
    "grinqh_gemm_or_gemv": (_int, [_ptr, _int, _i64, _i64, _ptr, _ptr, _ptr, _int, _int, _i64, _fptr, _int,
                                   _ptr, _ptr, _size, _ptr]),
    "grinqh_gemv_batch_union": (_int, [_ptr, _int, _i64, _i64, _ptr, _ptr, _ptr, _int, _int, _i64, _fptr,
                                       _ptr, _ptr, _size, _ptr]),
    "grinqh_prefill_gemm": (_int, [_ptr, _int, _i64, _i64, _ptr, _ptr, _ptr, _int, _int, _i64, _ptr, _ptr,
                                   _size, _ptr]),
    "grinqh_gemv_batch_union_masked": (_int, [_ptr, _int, _i64, _i64, _ptr, _ptr, _ptr, _int, _int, _i64, _fptr,
                                              _ptr, _ptr, _ptr, _size, _ptr]),
    "grinqh_rmsnorm_grade": (_int, [_ptr, _ptr, _ptr, _int, _i64, _i64, ctypes.c_float, _fptr, _int, _ptr, _ptr,
                                    _ptr, _ptr]),
    "grinqh_silu_mul_grade": (_int, [_ptr, _int, _i64, _i64, _fptr, _int, _ptr, _ptr, _ptr, _ptr]),
    "grinqh_gemv_noalloc": (_int, [_ptr, _int, _i64, _ptr, _ptr, _ptr, _int, _int, _i64, _fptr, _ptr, _ptr]),
}


def cabi() -> ctypes.CDLL:
    """The C ABI library with argument types declared."""
    global _cabi
    with _lock:
        if _cabi is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"GRINQH: native library {LIB_PATH} is missing; build it with "
                                  "`python -m grinqh._build` (nvcc for sm_100a)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _cabi = lib
    return _cabi


def load_ops() -> None:
    """Register torch.ops.grinqh.* (C++ op library)."""
    global _ops_loaded
    with _lock:
        if _ops_loaded:
            return
        if not os.path.exists(OPS_PATH):
            raise ImportError(f"GRINQH: op library {OPS_PATH} is missing; build it with `python -m grinqh._build`")
        import torch
        torch.ops.load_library(OPS_PATH)
        _ops_loaded = True


def check(status: int, what: str) -> None:
    if status != GRINQH_OK:
        lib = cabi()
        raise RuntimeError(f"GRINQH {what} failed ({lib.grinqh_status_string(status).decode()}): "
                           f"{lib.grinqh_last_error().decode()}")


def thresholds_arg(thresholds):
    t = (list(thresholds) + [0.0] * 4)[:4]
    return (ctypes.c_float * 4)(*[float(v) for v in t])
