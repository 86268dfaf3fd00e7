"""GPU tests of the library's FP64 kernels (DGEMM on the FP64 tensor path,
TRSM, TRSV, GEMV) through the C ABI, against FP64 references on the host
(numpy / scipy).  Tolerances are rigorous forward-error bounds of the
operations: |C - C_ref| <= 2 k u |alpha| (|A| |B|) + 2 u |beta C| elementwise
(u = 2^-53) for the products; the triangular solves are held to a
normwise backward error of a few ulps times the order."""
import ctypes

import numpy as np
import pytest
import scipy.linalg
import torch

from chpl_b200 import _lib
from gpu_util import from_dev, to_dev

pytestmark = pytest.mark.gpu
U = 2.0 ** -53


def _buf(a, ld=None, offset=0):
    """CUDA column-major copy of a (m x n) with leading dimension ld, starting
    `offset` doubles into the allocation (unaligned bases when odd)."""
    a = np.asarray(a, np.float64)
    m, n = a.shape
    ld = m if ld is None else ld
    host = np.full(offset + ld * n + 1, np.nan)
    host[offset:offset + ld * n].reshape(n, ld)[:, :m] = a.T
    t = torch.from_numpy(host).cuda()
    return t, t.data_ptr() + 8 * offset, ld


def _read(t, m, n, ld, offset=0):
    return t.cpu().numpy()[offset:offset + ld * n].reshape(n, ld)[:, :m].T.copy()


def _dgemm(m, n, k, alpha, A, B, beta, C, lds=(None, None, None), offs=(0, 0, 0)):
    L = _lib.load()
    tA, pA, lda = _buf(A if m and k else np.zeros((max(m, 1), max(k, 1))), lds[0], offs[0])
    tB, pB, ldb = _buf(B if k and n else np.zeros((max(k, 1), max(n, 1))), lds[1], offs[1])
    tC, pC, ldc = _buf(C, lds[2], offs[2])
    _lib.check(L.chpl_dgemm(None, m, n, k, alpha, pA, lda, pB, ldb, beta, pC, ldc), "chpl_dgemm")
    torch.cuda.synchronize()
    return _read(tC, m, n, ldc, offs[2])


def _bound(alpha, A, B, beta, C, k):
    return 2 * max(k, 1) * U * abs(alpha) * (np.abs(A) @ np.abs(B)) + 2 * U * np.abs(beta * C) + 1e-300


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 5, 3), (64, 128, 16), (65, 33, 17), (300, 40, 512),
                                   (129, 257, 130), (1000, 1000, 1000), (2049, 64, 256), (100, 3000, 31)])
def test_dgemm_matches_numpy(cuda, m, n, k):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    A = rng.uniform(-1, 1, (m, k))
    B = rng.uniform(-1, 1, (k, n))
    C = rng.uniform(-1, 1, (m, n))
    for alpha, beta in ((-1.0, 1.0), (0.5, -2.0), (1.0, 0.0)):
        got = _dgemm(m, n, k, alpha, A, B, beta, C)
        ref = alpha * (A @ B) + (beta * C if beta != 0 else 0.0)
        assert np.all(np.abs(got - ref) <= _bound(alpha, A, B, beta, C, k) + 4 * U * np.abs(ref)), (alpha, beta)


def test_dgemm_leading_dimensions_offsets_and_nan_c(cuda):
    """Padded and odd leading dimensions, unaligned base pointers (the 8-byte
    copy path), and beta = 0 with C full of NaN (C must not be read)."""
    rng = np.random.default_rng(1)
    m, n, k = 201, 77, 99
    A = rng.uniform(-1, 1, (m, k))
    B = rng.uniform(-1, 1, (k, n))
    C = np.full((m, n), np.nan)
    for lds, offs in (((m + 3, k + 1, m + 5), (1, 3, 5)), ((m + 8, k + 8, m + 8), (0, 0, 0)),
                      ((m, k, m), (1, 0, 1))):
        got = _dgemm(m, n, k, 2.0, A, B, 0.0, C, lds, offs)
        ref = 2.0 * (A @ B)
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - ref) <= _bound(2.0, A, B, 0.0, np.zeros_like(ref), k) + 4 * U * np.abs(ref))


def test_dgemm_k_zero_scales_c(cuda):
    C = np.arange(12.0).reshape(3, 4)
    assert np.array_equal(_dgemm(3, 4, 0, 1.0, None, None, 3.0, C), 3.0 * C)
    assert np.array_equal(_dgemm(3, 4, 0, 1.0, None, None, 0.0, np.full((3, 4), np.nan)), np.zeros((3, 4)))


def _unit_lower(n, rng):
    L = np.tril(rng.uniform(-1, 1, (n, n)) / np.sqrt(n), -1) + np.eye(n)
    L[np.triu_indices(n, 1)] = 1e300          # the upper part must not be read
    return L


@pytest.mark.parametrize("n,nrhs", [(1, 1), (63, 5), (64, 130), (65, 64), (200, 513), (1000, 1000), (4096, 300),
                                    (100, 40000)])
def test_dtrsm_matches_scipy(cuda, n, nrhs):
    rng = np.random.default_rng(n + nrhs)
    L = _unit_lower(n, rng)
    B = rng.uniform(-1, 1, (n, nrhs))
    tL, pL, ldl = _buf(L)
    tB, pB, ldb = _buf(B, n + 2)
    _lib.check(_lib.load().chpl_dtrsm_llnu(None, n, nrhs, pL, ldl, pB, ldb), "chpl_dtrsm_llnu")
    torch.cuda.synchronize()
    X = _read(tB, n, nrhs, ldb)
    Lt = np.tril(L, -1) + np.eye(n)
    ref = scipy.linalg.solve_triangular(Lt, B, lower=True, unit_diagonal=True)
    # backward error ||B - L X|| / (||L|| ||X||) of a few ulps times n
    be = np.linalg.norm(B - Lt @ X, np.inf) / (np.linalg.norm(Lt, np.inf) * np.linalg.norm(X, np.inf))
    assert be < 4 * n * U, be
    assert np.allclose(X, ref, rtol=1e-9, atol=1e-12)


def test_dtrsm_inverse_against_identity(cuda):
    """inv(L) as the solvers form it: the identity solved in place."""
    n = 1024
    L = _unit_lower(n, np.random.default_rng(2))
    tL, pL, ldl = _buf(L)
    tI, pI, ldi = _buf(np.eye(n))
    _lib.check(_lib.load().chpl_dtrsm_llnu(None, n, n, pL, ldl, pI, ldi), "chpl_dtrsm_llnu")
    torch.cuda.synchronize()
    Li = _read(tI, n, n, ldi)
    Lt = np.tril(L, -1) + np.eye(n)
    assert np.abs(Lt @ Li - np.eye(n)).max() < 1e-11
    assert np.array_equal(np.triu(Li, 1), np.zeros((n, n)))


@pytest.mark.parametrize("n", [1, 64, 65, 200, 1024, 2112, 3000, 4096, 6144])
def test_dtrtri_inverse(cuda, n):
    """inv(L) level by level (64 * 2^q orders: every pair of a level in one
    batched launch) and recursively for other orders: L X = I to a few ulps
    times n, the upper part exactly zero and the diagonal exactly one (X's
    prior contents are overwritten)."""
    L = _unit_lower(n, np.random.default_rng(n))
    tL, pL, ldl = _buf(L)
    tX, pX, ldx = _buf(np.full((n, n), np.nan), n + 3)
    _lib.check(_lib.load().chpl_dtrtri_llnu(None, n, pL, ldl, pX, ldx), "chpl_dtrtri_llnu")
    torch.cuda.synchronize()
    X = _read(tX, n, n, ldx)
    Lt = np.tril(L, -1) + np.eye(n)
    assert np.array_equal(np.triu(X, 1), np.zeros((n, n))) and np.array_equal(np.diag(X), np.ones(n))
    assert np.abs(Lt @ X - np.eye(n)).max() < 4 * n * U * np.abs(Lt).sum(axis=1).max() * np.abs(X).max()
    assert np.allclose(X, np.linalg.inv(Lt), rtol=1e-9, atol=1e-12)


@pytest.mark.parametrize("n", [1, 2, 63, 64, 65, 300, 2000, 9000])
def test_dtrsv_matches_scipy(cuda, n):
    rng = np.random.default_rng(n)
    Uu = np.triu(rng.uniform(-1, 1, (n, n)) / np.sqrt(n)) + np.diag(rng.uniform(1, 2, n) * np.sign(rng.uniform(-1, 1, n)))
    Uu[np.tril_indices(n, -1)] = np.nan        # the lower part must not be read
    b = rng.uniform(-1, 1, n)
    tU, pU, ldu = _buf(Uu, n + 1)
    tx, px, _ = _buf(b.reshape(-1, 1))
    work = torch.empty(n, dtype=torch.float64, device="cuda")
    _lib.check(_lib.load().chpl_dtrsv_unn(None, n, pU, ldu, px, work.data_ptr()), "chpl_dtrsv_unn")
    torch.cuda.synchronize()
    x = _read(tx, n, 1, n)[:, 0]
    Ut = np.triu(np.nan_to_num(Uu))
    ref = scipy.linalg.solve_triangular(Ut, b, lower=False)
    be = np.linalg.norm(b - Ut @ x, np.inf) / (np.linalg.norm(Ut, np.inf) * np.linalg.norm(x, np.inf))
    assert be < 4 * n * U, be
    assert np.allclose(x, ref, rtol=1e-9, atol=1e-12)


@pytest.mark.parametrize("m,n", [(1, 1), (31, 7), (33, 64), (4096, 4096), (200000, 9)])
def test_dgemv_matches_numpy(cuda, m, n):
    rng = np.random.default_rng(m + n)
    A = rng.uniform(-1, 1, (m, n))
    x = rng.uniform(-1, 1, n)
    y = rng.uniform(-1, 1, m)
    tA, pA, lda = _buf(A, m + 1)
    tx, px, _ = _buf(x.reshape(-1, 1))
    for alpha, beta in ((1.0, 1.0), (-0.5, 0.0)):
        ty, py, _ = _buf(y.reshape(-1, 1))
        _lib.check(_lib.load().chpl_dgemv(None, m, n, alpha, pA, lda, px, beta, py), "chpl_dgemv")
        torch.cuda.synchronize()
        got = _read(ty, m, 1, m)[:, 0]
        ref = alpha * (A @ x) + beta * y
        bound = 2 * n * U * abs(alpha) * (np.abs(A) @ np.abs(x)) + 2 * U * np.abs(beta * y) + 4 * U * np.abs(ref)
        assert np.all(np.abs(got - ref) <= bound + 1e-300)


def test_fp64_kernels_are_deterministic(cuda):
    rng = np.random.default_rng(3)
    m, n, k = 700, 300, 900
    A = rng.uniform(-1, 1, (m, k))
    B = rng.uniform(-1, 1, (k, n))
    C = rng.uniform(-1, 1, (m, n))
    a = _dgemm(m, n, k, -1.0, A, B, 1.0, C)
    b = _dgemm(m, n, k, -1.0, A, B, 1.0, C)
    assert np.array_equal(a, b)


def test_fp64_entry_points_reject_bad_sizes(cuda):
    L = _lib.load()
    d = torch.zeros(16, dtype=torch.float64, device="cuda")
    p = d.data_ptr()
    assert L.chpl_dgemm(None, 4, 4, 4, 1.0, p, 3, p, 4, 0.0, p, 4) == _lib.CHPL_ERR_INVALID
    assert L.chpl_dtrsm_llnu(None, 4, 1, p, 3, p, 4) == _lib.CHPL_ERR_INVALID
    assert L.chpl_dtrsv_unn(None, 4, p, 4, p, None) == _lib.CHPL_ERR_WORKSPACE
    assert L.chpl_dgemv(None, 4, 4, 1.0, p, 2, p, 0.0, p) == _lib.CHPL_ERR_INVALID
