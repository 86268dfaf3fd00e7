"""Ozaki scheme II emulated DGEMM -- the GEMMul8 interface the reference calls.

``gemm`` / ``workSize`` mirror ``gemmul8::gemm<double, Backend::INT8>`` and
``gemmul8::workSize<false, Backend::INT8>`` (call sites src/chpl_single.cu:641-649,
367-369; src/chpl_p2.cu:1674-1683, 755-757): same argument order and meaning,
column-major FP64 operands given as device pointers (ints) or CUDA tensors, the
stream in place of the cuBLAS handle.  Everything runs in libchpl.so on the
GPU; there is no host implementation here.
"""
from __future__ import annotations

import ctypes

from . import _lib

OP_N = _lib.CHPL_OP_N
OP_T = _lib.CHPL_OP_T


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    return int(getattr(stream, "cuda_stream", stream))


def workSize(m: int, n: int, k: int, num_moduli: int, enable_skip_scalA: bool = False,
             enable_skip_scalB: bool = False) -> tuple[int, int, int]:
    """Bytes of `work` (all parts inside), of the A part and of the B part."""
    L = _lib.load()
    tot, wa, wb = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check(L.chpl_oz2_worksize(m, n, k, num_moduli, int(enable_skip_scalA), int(enable_skip_scalB),
                                   ctypes.byref(tot), ctypes.byref(wa), ctypes.byref(wb)), "chpl_oz2_worksize")
    return tot.value, wa.value, wb.value


work_size = workSize


def gemm(opA: int, opB: int, m: int, n: int, k: int, alpha: float, A, lda: int, B, ldb: int, beta: float, C,
         ldc: int, num_moduli: int, fastmode: bool, work, workA=None, workB=None, enable_skip_scalA: bool = False,
         enable_skip_scalB: bool = False, skip_scalA: bool = False, skip_scalB: bool = False, stream=None,
         timed: bool = False) -> list[float]:
    """C = alpha*op(A)*op(B) + beta*C (FP64, column-major) on the int8 tensor cores.

    Returns the four phase times [split, int8 GEMM + fused mod/CRT/unscale, 0, 0]
    in seconds when ``timed`` (the call then synchronizes), else [].
    """
    L = _lib.load()
    a = ctypes.c_double(alpha)
    b = ctypes.c_double(beta)
    ph = (ctypes.c_double * 4)() if timed else None
    rc = L.chpl_oz2_gemm(_stream(stream), opA, opB, m, n, k, ctypes.byref(a), _ptr(A), lda, _ptr(B), ldb,
                         ctypes.byref(b), _ptr(C), ldc, num_moduli, int(fastmode), _ptr(work), _ptr(workA),
                         _ptr(workB), int(enable_skip_scalA), int(enable_skip_scalB), int(skip_scalA),
                         int(skip_scalB), ph)
    _lib.check(rc, "chpl_oz2_gemm")
    return list(ph) if timed else []


def shift_bits(num_moduli: int, k: int) -> tuple[int, int]:
    L = _lib.load()
    a, b = ctypes.c_int(), ctypes.c_int()
    _lib.check(L.chpl_oz2_shift_bits(num_moduli, k, ctypes.byref(a), ctypes.byref(b)), "chpl_oz2_shift_bits")
    return a.value, b.value


def split_rows(opA: int, m: int, k: int, A, lda: int, num_moduli: int, res, ld_vec: int, ld_k: int, shift, tmp,
               stream=None) -> None:
    L = _lib.load()
    _lib.check(L.chpl_oz2_split_rows(_stream(stream), opA, m, k, _ptr(A), lda, num_moduli, _ptr(res), ld_vec, ld_k,
                                     _ptr(shift), _ptr(tmp)), "chpl_oz2_split_rows")


def split_cols(opB: int, k: int, n: int, B, ldb: int, num_moduli: int, res, ld_vec: int, ld_k: int, shift, tmp,
               stream=None) -> None:
    L = _lib.load()
    _lib.check(L.chpl_oz2_split_cols(_stream(stream), opB, k, n, _ptr(B), ldb, num_moduli, _ptr(res), ld_vec, ld_k,
                                     _ptr(shift), _ptr(tmp)), "chpl_oz2_split_cols")


def split_tmp_bytes(nvec: int) -> int:
    return int(_lib.load().chpl_oz2_split_tmp_bytes(nvec))


def products(m: int, n: int, k: int, num_moduli: int, ra, lda_vec: int, rb, ldb_vec: int, ld_k: int, P, ldp: int,
             stream=None) -> None:
    L = _lib.load()
    _lib.check(L.chpl_oz2_products(_stream(stream), m, n, k, num_moduli, _ptr(ra), lda_vec, _ptr(rb), ldb_vec, ld_k,
                                   _ptr(P), ldp), "chpl_oz2_products")
