"""CPU oracle for chpl_b200 -- test infrastructure, never the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or as the timed CPU baseline.  The shipped library never calls it.

``oracle.c`` (built into ``oracle/_build/liboracle.so`` by ``make -C oracle``
or ``__graft_entry__.build()``) restates the reference's arithmetic:

* ``elem`` / ``matgen``: ``chpl_elem`` of ``src/chpl_p2.cu:66-73``
  (SplitMix64 output, top 53 bits, minus 0.5), index ``i*(N+1)+j``.
* ``oz2_*``: the Ozaki scheme II emulated DGEMM that the reference calls
  through ``gemmul8::gemm<double, Backend::INT8>`` (``src/chpl_single.cu:641-649``,
  ``src/chpl_p2.cu:1674-1683``), restated from the published method.
* ``hpl_solve`` / ``laswp`` / ``hpl_residual``: LU with partial pivoting
  (``src/chpl_single.cu:658-727``), LAPACK row-interchange semantics
  (``src/chpl_single.cu:489-518``) and the HPL scaled residual
  (``src/chpl_single.cu:785-802``).

Parity pins: the reference's own generator (``chpl_elem``), swap resolution
(``resolve_seq``), residual reduction and chpl_single's Philox generator
kernel, cut verbatim out of the reference checkout and compiled into
``oracle/_ref/`` by ``oracle/ref_build.py`` (``tests/test_oracle_ref.py``);
SplitMix64 published known answers; exact CRT against Python big integers; LU
against LAPACK (scipy); GEMM against numpy FP64.  GEMMul8's own outputs are not
available (submodule absent), so kernel-level parity with GEMMul8 is unpinned;
the reference's own end-to-end check (HPL residual < 16,
``src/chpl_single.cu:931-948``) is the anchor there.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_dbl = ctypes.c_double
_ptr = ctypes.c_void_p


def build() -> str:
    """Compile oracle.c (gcc) into oracle/_build/liboracle.so, and oracle/_ref/
    from the reference's own source where the reference checkout is present."""
    src = os.path.join(_HERE, "oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    build_ref()
    return _SO


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_SO)
        L.orc_splitmix64.restype = ctypes.c_uint64
        L.orc_splitmix64.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.orc_hpl_residual_parts.restype = _dbl
        L.orc_hpl_residual_parts.argtypes = [_ptr, _ptr, _ptr, _ptr, _i64]
        L.orc_elem.restype = _dbl
        L.orc_elem.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.orc_matgen.argtypes = [_ptr, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_uint64]
        L.orc_oz2_moduli.argtypes = [ctypes.c_int, _ptr]
        L.orc_oz2_constants.argtypes = [ctypes.c_int, _ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _ptr]
        L.orc_oz2_shift_bits.argtypes = [ctypes.c_int, _i64, _ptr, _ptr]
        L.orc_oz2_row_shift.argtypes = [_ptr, _i64, ctypes.c_int, _i64, _i64, ctypes.c_int, _ptr]
        L.orc_oz2_col_shift.argtypes = [_ptr, _i64, ctypes.c_int, _i64, _i64, ctypes.c_int, _ptr]
        L.orc_oz2_split_rows.argtypes = [_ptr, _i64, ctypes.c_int, _i64, _i64, _ptr, ctypes.c_int, _ptr]
        L.orc_oz2_split_cols.argtypes = [_ptr, _i64, ctypes.c_int, _i64, _i64, _ptr, ctypes.c_int, _ptr]
        L.orc_int8_gemm.argtypes = [_ptr, _ptr, _i64, _i64, _i64, _ptr]
        L.orc_oz2_reconstruct.argtypes = [_ptr, _i64, _i64, ctypes.c_int, _ptr, _ptr, _dbl, _dbl,
                                          _ptr, _i64, ctypes.c_int]
        L.orc_oz2_gemm.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _i64, _i64, _dbl, _ptr, _i64,
                                   _ptr, _i64, _dbl, _ptr, _i64, ctypes.c_int, ctypes.c_int]
        L.orc_laswp.argtypes = [_ptr, _i64, _i64, _i64, _i64, _i64, _ptr]
        L.orc_hpl_solve.argtypes = [_ptr, _i64, _i64, _i64, ctypes.c_int, _ptr]
        L.orc_hpl_residual.restype = _dbl
        L.orc_hpl_residual.argtypes = [_ptr, _i64, _i64, _ptr]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def splitmix64(seed: int, idx: int) -> int:
    return int(lib().orc_splitmix64(seed, idx))


def matgen(m: int, n: int, seed: int = 42, row0: int = 0, col0: int = 0, ncg: int | None = None,
           lda: int | None = None) -> np.ndarray:
    """Column-major m x n block of the generated system (Fortran-ordered array)."""
    lda = m if lda is None else lda
    ncg = n if ncg is None else ncg
    A = np.zeros((lda, n), dtype=np.float64, order="F")
    lib().orc_matgen(_p(A), lda, m, n, row0, col0, ncg, seed)
    return A[:m, :]


def hpl_system(N: int, seed: int = 42) -> np.ndarray:
    """The N x (N+1) HPL system of src/chpl_p2.cu (b = column N)."""
    return matgen(N, N + 1, seed=seed, ncg=N + 1)


def oz2_moduli(L: int) -> list[int]:
    m = np.zeros(L, dtype=np.int32)
    if lib().orc_oz2_moduli(L, _p(m)):
        raise ValueError(f"unsupported number of moduli {L}")
    return [int(x) for x in m]


def oz2_constants(L: int) -> dict:
    mod = np.zeros(L, dtype=np.int32)
    y = np.zeros(L, dtype=np.int64)
    v = np.zeros(L, dtype=np.uint64)
    Mf = ctypes.c_double()
    lg = ctypes.c_double()
    hi = ctypes.c_uint64()
    lo = ctypes.c_uint64()
    if lib().orc_oz2_constants(L, _p(mod), _p(y), _p(v), ctypes.byref(Mf), ctypes.byref(lg),
                               ctypes.byref(hi), ctypes.byref(lo)):
        raise ValueError(L)
    return {"moduli": [int(x) for x in mod], "y": [int(x) for x in y], "v": [int(x) for x in v],
            "Mf": Mf.value, "log2M": lg.value, "M": (hi.value << 64) | lo.value}


def oz2_shift_bits(L: int, k: int) -> tuple[int, int]:
    a = ctypes.c_int()
    b = ctypes.c_int()
    if lib().orc_oz2_shift_bits(L, k, ctypes.byref(a), ctypes.byref(b)):
        raise ValueError((L, k))
    return a.value, b.value


def _f(a: np.ndarray) -> np.ndarray:
    return np.asfortranarray(a, dtype=np.float64)


def oz2_row_shift(A: np.ndarray, alpha: int, opA: int = 0) -> np.ndarray:
    A = _f(A)
    m, k = (A.shape[1], A.shape[0]) if opA else A.shape
    s = np.zeros(m, dtype=np.int32)
    lib().orc_oz2_row_shift(_p(A), A.shape[0], opA, m, k, alpha, _p(s))
    return s


def oz2_col_shift(B: np.ndarray, beta: int, opB: int = 0) -> np.ndarray:
    B = _f(B)
    k, n = (B.shape[1], B.shape[0]) if opB else B.shape
    s = np.zeros(n, dtype=np.int32)
    lib().orc_oz2_col_shift(_p(B), B.shape[0], opB, k, n, beta, _p(s))
    return s


def oz2_split_rows(A: np.ndarray, shift: np.ndarray, L: int, opA: int = 0) -> np.ndarray:
    """int8 residues [L, m, k] of op(A) (K-major rows)."""
    A = _f(A)
    m, k = (A.shape[1], A.shape[0]) if opA else A.shape
    r = np.zeros((L, m, k), dtype=np.int8)
    lib().orc_oz2_split_rows(_p(A), A.shape[0], opA, m, k, _p(np.ascontiguousarray(shift, np.int32)),
                             L, _p(r))
    return r


def oz2_split_cols(B: np.ndarray, shift: np.ndarray, L: int, opB: int = 0) -> np.ndarray:
    """int8 residues [L, n, k] of op(B) (K-major columns)."""
    B = _f(B)
    k, n = (B.shape[1], B.shape[0]) if opB else B.shape
    r = np.zeros((L, n, k), dtype=np.int8)
    lib().orc_oz2_split_cols(_p(B), B.shape[0], opB, k, n, _p(np.ascontiguousarray(shift, np.int32)),
                             L, _p(r))
    return r


def int8_gemm(Ar: np.ndarray, Br: np.ndarray) -> np.ndarray:
    """Exact int32 product of K-major residues: (m,k) x (n,k) -> (m,n) column-major."""
    m, k = Ar.shape
    n = Br.shape[0]
    C = np.zeros((m, n), dtype=np.int32, order="F")
    lib().orc_int8_gemm(_p(np.ascontiguousarray(Ar)), _p(np.ascontiguousarray(Br)), m, n, k, _p(C))
    return C


def oz2_gemm(A: np.ndarray, B: np.ndarray, C: np.ndarray, L: int, alpha: float = -1.0,
             beta: float = 1.0, opA: int = 0, opB: int = 0, mode: int = 1) -> np.ndarray:
    """alpha*op(A)op(B) + beta*C by the restated Ozaki-II method.

    mode 0: exact 128-bit CRT; mode 1: the 64-bit fixed-point CRT the GPU uses.
    """
    A = _f(A)
    B = _f(B)
    out = np.array(C, dtype=np.float64, order="F", copy=True)
    m, k = (A.shape[1], A.shape[0]) if opA else A.shape
    n = B.shape[0] if opB else B.shape[1]
    rc = lib().orc_oz2_gemm(opA, opB, m, n, k, alpha, _p(A), A.shape[0], _p(B), B.shape[0], beta,
                            _p(out), out.shape[0], L, mode)
    if rc:
        raise RuntimeError(f"orc_oz2_gemm failed ({rc})")
    return out


def laswp(A: np.ndarray, ipiv: np.ndarray, k1: int, k2: int, c0: int = 0, c1: int | None = None):
    A = np.asfortranarray(A)
    c1 = A.shape[1] if c1 is None else c1
    lib().orc_laswp(_p(A), A.shape[0], c0, c1, k1, k2, _p(np.ascontiguousarray(ipiv, np.int64)))
    return A


def hpl_solve(N: int, NB: int, L: int = 0, seed: int = 42):
    """Solve the generated system on the CPU; returns (x, ipiv, factored system)."""
    A = np.asfortranarray(hpl_system(N, seed))
    ipiv = np.zeros(N, dtype=np.int64)
    rc = lib().orc_hpl_solve(_p(A), N, N, NB, L, _p(ipiv))
    if rc:
        raise RuntimeError(f"orc_hpl_solve failed ({rc})")
    return A[:, N].copy(), ipiv, A


def hpl_residual(x: np.ndarray, N: int, seed: int = 42) -> float:
    A = np.asfortranarray(hpl_system(N, seed))
    return float(lib().orc_hpl_residual(_p(A), N, N, _p(np.ascontiguousarray(x, np.float64))))


def hpl_residual_parts(y: np.ndarray, rs: np.ndarray, b: np.ndarray, x: np.ndarray) -> float:
    """Scaled residual from per-row data (y = A x, rs = row sums of |A|, b, x):
    the reduction and formula of src/chpl_single.cu:790-801."""
    N = len(y)
    f = [np.ascontiguousarray(v, np.float64) for v in (y, rs, b, x)]
    return float(lib().orc_hpl_residual_parts(*[_p(v) for v in f], N))


# ---------------------------------------------------------------------------
# Ozaki scheme I (the reference's alternative engine, HPLS_BACKEND=ozaki)
# ---------------------------------------------------------------------------
OZ1_SLICES = 6


def _oz1_digits(x: np.ndarray) -> list[np.ndarray]:
    """Base-128 digits of entries in (-1, 1): t = rint(128 x) clamped to 127,
    x <- 128 x - t (ozsliceA/ozsliceB, src/chpl_single.cu:172-219).  The
    digits are integers in [-128, 127] held as float64."""
    out = []
    x = x.copy()
    for _ in range(OZ1_SLICES):
        t = np.minimum(np.rint(x * 128.0), 127.0)
        x = x * 128.0 - t
        out.append(t)
    return out


def oz1_gemm(A: np.ndarray, B: np.ndarray, C: np.ndarray, alpha: float = -1.0, beta: float = 1.0) -> np.ndarray:
    """C = alpha A B + beta C by Ozaki scheme I as the reference computes it
    (src/chpl_single.cu:147-236, 532-612): power-of-two row / column scales
    (ilogb(max) + 1), six base-128 digits, the anti-diagonals d = p + q < 6 of
    the digit products in exact integers, reconstruction
    sum_d P_d 128^-(d+2) in order d = 0..5, times 2^(ea_i + eb_j).  With
    alpha = -1, beta = 1 (the solver's update) or beta = 0 the result is bit
    for bit the GPU's (one rounding for alpha v + beta C either way)."""
    A = np.asarray(A, np.float64)
    B = np.asarray(B, np.float64)
    ea = np.frexp(np.max(np.abs(A), axis=1))[1].astype(np.int64)
    eb = np.frexp(np.max(np.abs(B), axis=0))[1].astype(np.int64)
    da = _oz1_digits(np.ldexp(A, -ea[:, None]))
    db = _oz1_digits(np.ldexp(B, -eb[None, :]))
    acc = np.zeros((A.shape[0], B.shape[1]))
    w = 2.0 ** -14
    for d in range(OZ1_SLICES):
        # every partial sum is an integer of magnitude < 6 k 2^14 < 2^53, so the
        # float64 product is the exact integer whatever order BLAS sums in
        P = np.hstack(da[:d + 1]) @ np.vstack(db[d::-1])
        acc = acc + P * w
        w *= 2.0 ** -7
    v = np.ldexp(acc, (ea[:, None] + eb[None, :]))
    if beta == 0.0:
        return alpha * v
    if alpha == -1.0 and beta == 1.0:
        return C - v
    return alpha * v + beta * C


# ---------------------------------------------------------------------------
# oracle/_ref: fragments of the reference's own source (oracle/ref_build.py)
# ---------------------------------------------------------------------------
_REF = os.path.join(_HERE, "_ref")
_ref_host = None


def build_ref() -> bool:
    """Build oracle/_ref/ when the reference checkout is present (False otherwise)."""
    from . import ref_build
    return ref_build.build()


def ref_host():
    """ctypes handle of oracle/_ref/libref_host.so (the reference's own
    generator, swap resolution and residual reduction), or None if it was
    never built (no reference checkout where the repository was built)."""
    global _ref_host
    if _ref_host is None:
        so = os.path.join(_REF, "libref_host.so")
        if not os.path.exists(so):
            return None
        L = ctypes.CDLL(so)
        L.ref_chpl_elem.restype = _dbl
        L.ref_chpl_elem.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.ref_matgen.restype = None
        L.ref_matgen.argtypes = [_ptr, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_uint64]
        L.ref_resolve_seq.restype = None
        L.ref_resolve_seq.argtypes = [_ptr, ctypes.c_longlong, ctypes.c_int, _ptr, _ptr, _ptr,
                                      ctypes.POINTER(ctypes.c_int)]
        L.ref_residual.restype = _dbl
        L.ref_residual.argtypes = [_ptr, _ptr, _ptr, _ptr, _i64]
        _ref_host = L
    return _ref_host


def ref_single_matgen_path() -> str | None:
    """Path of oracle/_ref/libref_single_matgen.so (chpl_single's own Philox
    generator kernel, sm_100a), or None if it was never built."""
    so = os.path.join(_REF, "libref_single_matgen.so")
    return so if os.path.exists(so) else None


def ref_oz1_path() -> str | None:
    """Path of oracle/_ref/libref_oz1.so (chpl_single's own Ozaki-I scale,
    slice and reconstruction kernels, sm_100a), or None if it was never built."""
    so = os.path.join(_REF, "libref_oz1.so")
    return so if os.path.exists(so) else None


def ref_resolve_seq(piv: np.ndarray, base: int) -> tuple[np.ndarray, dict]:
    """The reference's resolve_seq: (top, {row >= base+n: original row})."""
    L = ref_host()
    n = len(piv)
    p = np.ascontiguousarray(piv, np.int64)
    top = np.zeros(n, np.int64)
    bp = np.zeros(max(n, 1), np.int64)
    bs = np.zeros(max(n, 1), np.int64)
    nb = ctypes.c_int()
    L.ref_resolve_seq(_p(p), base, n, _p(top), _p(bp), _p(bs), ctypes.byref(nb))
    return top, {int(bp[i]): int(bs[i]) for i in range(nb.value)}


def hpl_residual_from(A: np.ndarray, x: np.ndarray) -> float:
    """Scaled residual for an explicit N x (N+1) system (numpy, any size)."""
    N = A.shape[0]
    Ax = A[:, :N] @ x
    b = A[:, N]
    eps = 2.0 ** -53
    return float(np.max(np.abs(Ax - b)) /
                 (eps * (np.max(np.sum(np.abs(A[:, :N]), axis=1)) * np.max(np.abs(x))
                         + np.max(np.abs(b))) * N))


def hpl_system_fast(N: int, seed: int = 42, threads: int | None = None) -> np.ndarray:
    """The N x (N+1) system, generated by the C oracle in parallel column slabs."""
    import concurrent.futures as cf
    threads = threads or os.cpu_count() or 1
    A = np.empty((N, N + 1), dtype=np.float64, order="F")
    nc = N + 1
    step = (nc + threads - 1) // threads
    L = lib()

    def work(c0):
        c1 = min(nc, c0 + step)
        if c1 > c0:
            L.orc_matgen(ctypes.c_void_p(A.ctypes.data + c0 * N * 8), N, N, c1 - c0, 0, c0, nc, seed)

    with cf.ThreadPoolExecutor(threads) as ex:
        list(ex.map(work, range(0, nc, step)))
    return A


def lapack_hpl_solve(A: np.ndarray):
    """Host FP64 blocked LU with partial pivoting (LAPACK dgetrf + dgetrs via
    scipy/OpenBLAS) of the N x (N+1) system; the CPU baseline of the hot path.
    Returns x.  The factorization overwrites A."""
    import scipy.linalg
    N = A.shape[0]
    lu, piv = scipy.linalg.lu_factor(A[:, :N], overwrite_a=True, check_finite=False)
    return scipy.linalg.lu_solve((lu, piv), A[:, N], check_finite=False)
