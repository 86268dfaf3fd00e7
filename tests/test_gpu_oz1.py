"""GPU tests of the Ozaki scheme I emulated DGEMM (the reference's
HPLS_BACKEND=ozaki engine, src/chpl_single.cu:147-236 and 532-612) through the
C ABI: bit for bit against the CPU restatement oracle.oz1_gemm for the
solver's update (alpha = -1, beta = 1) and for beta = 0, on ragged sizes, rows
and columns of zeros, rows spanning hundreds of binades and a C that aliases
B; then the accuracy of the scheme itself against FP64 and the size limits."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from chpl_b200 import _lib
from gpu_util import empty_bytes, from_dev, to_dev

pytestmark = pytest.mark.gpu


def _work(m, n, k):
    w = ctypes.c_size_t()
    _lib.check(_lib.load().chpl_oz1_worksize(m, n, k, ctypes.byref(w)), "chpl_oz1_worksize")
    return empty_bytes(w.value)


def _oz1(A, B, C, alpha=-1.0, beta=1.0, ldc_pad=0):
    L = _lib.load()
    m, k = A.shape
    n = B.shape[1]
    tA, lda = to_dev(A if A.size else np.zeros((max(m, 1), max(k, 1))), max(m, 1) + 3)
    tB, ldb = to_dev(B if B.size else np.zeros((max(k, 1), max(n, 1))))
    tC, ldc = to_dev(C, m + ldc_pad)
    w = _work(m, n, k)
    _lib.check(L.chpl_oz1_gemm(None, m, n, k, alpha, tA.data_ptr(), lda, tB.data_ptr(), ldb, beta, tC.data_ptr(), ldc,
                               w.data_ptr()), "chpl_oz1_gemm")
    torch.cuda.synchronize()
    return from_dev(tC, m, n)


def _same(a, b):
    return np.array_equal(a.view(np.uint64), b.view(np.uint64))


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 5, 3), (129, 257, 130), (1000, 300, 1024), (300, 1000, 4096),
                                   (2049, 64, 256), (100, 3000, 31), (513, 511, 2048)])
def test_oz1_bit_exact_vs_oracle(cuda, m, n, k):
    rng = np.random.default_rng(m + 3 * n + 7 * k)
    A = rng.uniform(-1, 1, (m, k))
    B = rng.uniform(-1, 1, (k, n))
    C = rng.uniform(-1, 1, (m, n))
    got = _oz1(A, B, C, ldc_pad=5)
    assert _same(got, oracle.oz1_gemm(A, B, C))
    got0 = _oz1(A, B, C, alpha=1.0, beta=0.0)
    assert _same(got0, oracle.oz1_gemm(A, B, C, alpha=1.0, beta=0.0))


def test_oz1_scales_zeros_and_wide_range(cuda):
    """Row / column scales are per row and column: rows 2^+-300 apart, a zero
    row of A and a zero column of B, and entries far below their row's
    maximum (lost below the sixth digit, as in the reference) all agree."""
    rng = np.random.default_rng(11)
    m, n, k = 300, 200, 777
    A = rng.standard_normal((m, k)) * np.ldexp(1.0, rng.integers(-300, 300, m))[:, None]
    B = rng.standard_normal((k, n)) * np.ldexp(1.0, rng.integers(-200, 200, n))[None, :]
    A[5] = 0.0
    B[:, 7] = 0.0
    A[9, ::3] *= 1e-20
    C = rng.standard_normal((m, n)) * np.abs(A).max(axis=1)[:, None] * np.abs(B).max(axis=0)[None, :]
    got = _oz1(A, B, C)
    assert _same(got, oracle.oz1_gemm(A, B, C))
    assert np.array_equal(got[5], C[5]) and np.array_equal(got[:, 7], C[:, 7])


def test_oz1_c_aliases_b_with_beta_zero(cuda):
    """B is cut into digits before C is written, so C may be B itself."""
    L = _lib.load()
    rng = np.random.default_rng(12)
    m = k = 640
    n = 300
    A = rng.uniform(-1, 1, (m, k))
    B = rng.uniform(-1, 1, (k, n))
    tA, lda = to_dev(A)
    tB, ldb = to_dev(B)
    w = _work(m, n, k)
    _lib.check(L.chpl_oz1_gemm(None, m, n, k, 1.0, tA.data_ptr(), lda, tB.data_ptr(), ldb, 0.0, tB.data_ptr(), ldb,
                               w.data_ptr()), "chpl_oz1_gemm")
    torch.cuda.synchronize()
    assert _same(from_dev(tB, m, n), oracle.oz1_gemm(A, B, None, alpha=1.0, beta=0.0))


def test_oz1_accuracy_against_fp64(cuda):
    """Six base-128 digits: each scaled entry is kept to 2^-42 and the dropped
    digit products are below 128^-7 of the row x column scale, so
    |C - A B| <= k 2^-40 2^(ea_i + eb_j) elementwise (with room to spare)."""
    rng = np.random.default_rng(13)
    m, n, k = 1500, 700, 4096
    A = rng.uniform(-1, 1, (m, k))
    B = rng.uniform(-1, 1, (k, n))
    got = _oz1(A, B, np.zeros((m, n)), alpha=1.0, beta=0.0)
    ref = A @ B
    sa = np.ldexp(1.0, np.frexp(np.abs(A).max(axis=1))[1])
    sb = np.ldexp(1.0, np.frexp(np.abs(B).max(axis=0))[1])
    assert np.all(np.abs(got - ref) <= k * 2.0 ** -40 * sa[:, None] * sb[None, :])
    assert np.abs(got - ref).max() > 0      # it is an emulation, not FP64


def test_oz1_deterministic(cuda):
    rng = np.random.default_rng(14)
    A = rng.uniform(-1, 1, (777, 1000))
    B = rng.uniform(-1, 1, (1000, 555))
    C = rng.uniform(-1, 1, (777, 555))
    assert _same(_oz1(A, B, C), _oz1(A, B, C))


def test_oz1_degenerate_and_limits(cuda):
    L = _lib.load()
    rng = np.random.default_rng(15)
    C = rng.uniform(-1, 1, (40, 30))
    # k = 0: C = beta C
    got = _oz1(np.zeros((40, 0)), np.zeros((0, 30)), C, alpha=-1.0, beta=0.5)
    assert np.array_equal(got, 0.5 * C)
    # the int32 accumulation bound: 6 k 127^2 < 2^31
    w = ctypes.c_size_t()
    assert L.chpl_oz1_worksize(64, 64, 21845, ctypes.byref(w)) == _lib.CHPL_OK
    assert L.chpl_oz1_worksize(64, 64, 21846, ctypes.byref(w)) == _lib.CHPL_ERR_UNSUPPORTED
    A = rng.uniform(-1, 1, (70, 21845))
    B = rng.uniform(-1, 1, (21845, 9))
    C = rng.uniform(-1, 1, (70, 9))
    assert _same(_oz1(A, B, C), oracle.oz1_gemm(A, B, C))
    a = torch.zeros(8, dtype=torch.float64, device="cuda")
    assert L.chpl_oz1_gemm(None, 4, 4, 21846, -1.0, a.data_ptr(), 4, a.data_ptr(), 21846, 1.0, a.data_ptr(), 4,
                           a.data_ptr()) == _lib.CHPL_ERR_UNSUPPORTED
    assert L.chpl_oz1_gemm(None, 4, 4, 4, -1.0, a.data_ptr(), 4, a.data_ptr(), 4, 1.0, a.data_ptr(), 4,
                           None) == _lib.CHPL_ERR_WORKSPACE


def test_oz1_golden_fixture(cuda):
    """The committed fixture (tests/golden/oz1_m48_n40_k200.npz), bit for bit."""
    import os
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "oz1_m48_n40_k200.npz"))
    assert _same(_oz1(g["A"], g["B"], g["C"]), g["update"])
    assert _same(_oz1(g["A"], g["B"], g["C"], alpha=1.0, beta=0.0), g["product"])
