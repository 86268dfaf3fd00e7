"""ctypes binding of libchpl.so (the C ABI declared in include/chpl.h).

The library is built in-tree (``python -m chpl_b200.build``).  Loading never
falls back to anything: a missing or unloadable libchpl.so raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libchpl.so")

CHPL_OK = 0
CHPL_ERR_INVALID = -1
CHPL_ERR_CUDA = -2
CHPL_ERR_TIMEOUT = -3
CHPL_ERR_WORKSPACE = -4
CHPL_ERR_UNSUPPORTED = -5
CHPL_ERR_SINGULAR = -6
CHPL_ERR_NCCL = -7
CHPL_ERR_NO_DEVICE = -8

CHPL_OP_N = 0
CHPL_OP_T = 1

CHPL_GEN_CHPL = 0
CHPL_GEN_PHILOX = 1

_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t
_int = ctypes.c_int
_uint = ctypes.c_uint
_dbl = ctypes.c_double
_vp = ctypes.c_void_p
_dp = ctypes.POINTER(ctypes.c_double)


class HplConfig(ctypes.Structure):
    _fields_ = [("N", _i64), ("NB", _i64), ("P", _int), ("Q", _int), ("moduli", _int), ("emulate", _int),
                ("fast", _int), ("chunk", _i64), ("lookahead", _int), ("agg", _int), ("reserve_sms", _int), ("trsm_mode", _int), ("panel_mode", _int),
                ("seed", _u64), ("threshold", _dbl), ("verbose", _int), ("generator", _int)]


class HplResult(ctypes.Structure):
    _fields_ = [("time_s", _dbl), ("tflops", _dbl), ("resid", _dbl), ("passed", _int), ("matgen_s", _dbl),
                ("phase_s", _dbl * 8), ("n_emulated", _i64), ("n_launches", _i64), ("gemm_launches", _i64),
                ("gemm_kernel_s", _dbl), ("gemm_int8_ops", _dbl), ("gemm_fp64eq_flops", _dbl), ("schedule", _int)]


# name -> (restype, argtypes); every function declared in include/chpl.h
SIGNATURES = {
    "chpl_last_error_string": (ctypes.c_char_p, []),
    "chpl_version": (ctypes.c_char_p, []),
    "chpl_device_status": (_int, [ctypes.POINTER(_int)]),
    "chpl_diag_bounded_wait": (_int, [_vp, _int, ctypes.c_uint64]),
    "chpl_host_alloc": (_int, [_sz, ctypes.POINTER(_vp)]),
    "chpl_host_free": (_int, [_vp]),
    "chpl_oz2_worksize": (_int, [_sz, _sz, _sz, _uint, _int, _int, ctypes.POINTER(_sz), ctypes.POINTER(_sz),
                                 ctypes.POINTER(_sz)]),
    "chpl_oz2_gemm": (_int, [_vp, _int, _int, _sz, _sz, _sz, _dp, _vp, _sz, _vp, _sz, _dp, _vp, _sz, _uint, _int,
                             _vp, _vp, _vp, _int, _int, _int, _int, _dp]),
    "chpl_oz2_gemm_noalloc": (_int, [_vp, _int, _int, _sz, _sz, _sz, _dp, _vp, _sz, _vp, _sz, _dp, _vp, _sz,
                                     _uint]),
    "chpl_oz2_split_rows": (_int, [_vp, _int, _sz, _sz, _vp, _sz, _uint, _vp, _sz, _sz, _vp, _vp]),
    "chpl_oz2_split_cols": (_int, [_vp, _int, _sz, _sz, _vp, _sz, _uint, _vp, _sz, _sz, _vp, _vp]),
    "chpl_oz2_split_tmp_bytes": (_sz, [_sz]),
    "chpl_oz2_products": (_int, [_vp, _sz, _sz, _sz, _uint, _vp, _sz, _vp, _sz, _sz, _vp, _sz]),
    "chpl_oz2_shift_bits": (_int, [_uint, _sz, ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "chpl_oz1_worksize": (_int, [_sz, _sz, _sz, ctypes.POINTER(_sz)]),
    "chpl_oz1_gemm": (_int, [_vp, _sz, _sz, _sz, _dbl, _vp, _sz, _vp, _sz, _dbl, _vp, _sz, _vp]),
    "chpl_matgen": (_int, [_vp, _vp, _sz, _sz, _sz, _i64, _i64, _i64, _u64]),
    "chpl_matgen_philox": (_int, [_vp, _vp, _sz, _sz, _sz, _i64, _i64, _i64, _u64]),
    "chpl_matgen_cyclic": (_int, [_vp, _vp, _sz, _i64, _i64, _int, _int, _int, _int, _u64]),
    "chpl_matgen_host": (_int, [_i64, _u64, _vp, _sz]),
    "chpl_laswp_work_bytes": (_sz, [_i64, _i64]),
    "chpl_laswp": (_int, [_vp, _vp, _sz, _i64, _i64, _i64, _vp, _i64, _vp]),
    "chpl_panel_getrf_work_bytes": (_sz, [_i64, _i64]),
    "chpl_panel_getrf_f64": (_int, [_vp, _i64, _i64, _vp, _sz, _vp, _vp, _vp]),
    "chpl_dgemm": (_int, [_vp, _i64, _i64, _i64, _dbl, _vp, _sz, _vp, _sz, _dbl, _vp, _sz]),
    "chpl_dtrsm_llnu": (_int, [_vp, _i64, _i64, _vp, _sz, _vp, _sz]),
    "chpl_dtrtri_llnu": (_int, [_vp, _i64, _vp, _sz, _vp, _sz]),
    "chpl_dtrsv_unn": (_int, [_vp, _i64, _vp, _sz, _vp, _vp]),
    "chpl_dgemv": (_int, [_vp, _i64, _i64, _dbl, _vp, _sz, _vp, _dbl, _vp]),
    "chpl_residual": (_int, [_vp, _i64, _u64, _vp, _dp]),
    "chpl_residual_matrix": (_int, [_vp, _i64, _vp, _sz, _vp, _dp]),
    "chpl_hpl_default_config": (None, [ctypes.POINTER(HplConfig)]),
    "chpl_hpl_run": (_int, [ctypes.POINTER(HplConfig), ctypes.POINTER(HplResult), _vp]),
    "chpl_hpl_run_host": (_int, [ctypes.POINTER(HplConfig), _vp, _sz, _int, ctypes.POINTER(HplResult), _vp]),
    "chpl_grid_unique_id": (_int, [_vp, _sz]),
    "chpl_grid_create": (_int, [_int, _int, _int, _vp, _sz, _dbl, ctypes.POINTER(_vp)]),
    "chpl_grid_run": (_int, [_vp, ctypes.POINTER(HplConfig), ctypes.POINTER(HplResult), _vp]),
    "chpl_grid_destroy": (_int, [_vp]),
    "chpl_grid_plan_exchange": (_int, [_i64, _i64, _vp, _i64, _int, _int, _vp, _vp, ctypes.POINTER(_int), _vp,
                                       ctypes.POINTER(_int), _vp, ctypes.POINTER(_int)]),
}

_lib = None


class ChplError(RuntimeError):
    def __init__(self, code: int, where: str, msg: str):
        super().__init__(f"{where} failed with status {code}: {msg}")
        self.code = code


def load() -> ctypes.CDLL:
    """Load libchpl.so (raises if it is missing: there is no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m chpl_b200.build` (no CPU fallback exists)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(code: int, where: str) -> None:
    if code != CHPL_OK:
        msg = load().chpl_last_error_string().decode(errors="replace")
        raise ChplError(code, where, msg)
