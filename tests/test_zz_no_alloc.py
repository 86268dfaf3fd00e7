"""GPU test of chpl_oz2_gemm_noalloc, the entry point for callers that cannot
allocate device memory when they need the update (a host framework that owns
the whole memory pool, or a caller that cannot take cudaMalloc's
synchronization).  It is called through the C ABI and must give the same
result as chpl_oz2_gemm (bit-identical: both run the same kernels, and the
emulated GEMM's tests hold it to exact equality), on two calls in a row, since
every call reuses the library's fixed device scratch.

Collected last on purpose (file name): a run that stops at its first failure
has already run every other test by the time it gets here.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from chpl_b200 import _lib, oz2
from gpu_util import empty_bytes, from_dev, to_dev

pytestmark = pytest.mark.gpu


def _noalloc(m, n, k, L, A, B, C, alpha=-1.0, beta=1.0, opA=0, opB=0):
    lib = _lib.load()
    dA, lda = to_dev(A)
    dB, ldb = to_dev(B)
    dC, ldc = to_dev(C)
    a, b = ctypes.c_double(alpha), ctypes.c_double(beta)
    rc = lib.chpl_oz2_gemm_noalloc(0, opA, opB, m, n, k, ctypes.byref(a), dA.data_ptr(), lda, dB.data_ptr(), ldb,
                                   ctypes.byref(b), dC.data_ptr(), ldc, L)
    _lib.check(rc, "chpl_oz2_gemm_noalloc")
    torch.cuda.synchronize()
    return from_dev(dC, m, n)


def _with_work(m, n, k, L, A, B, C, alpha=-1.0, beta=1.0, opA=0, opB=0):
    dA, lda = to_dev(A)
    dB, ldb = to_dev(B)
    dC, ldc = to_dev(C)
    tot, _, _ = oz2.workSize(m, n, k, L)
    work = empty_bytes(tot)
    oz2.gemm(opA, opB, m, n, k, alpha, dA, lda, dB, ldb, beta, dC, ldc, L, True, work)
    torch.cuda.synchronize()
    return from_dev(dC, m, n)


def test_noalloc_matches_allocating_entry_point_twice(cuda):
    rng = np.random.default_rng(123)
    # call 1: larger problem; call 2: smaller and transposed, so stale scratch
    # from call 1 would show up if anything were not rewritten or cleared
    cases = [(1000, 900, 1024, 12, 0, 0), (300, 260, 200, 11, 1, 1)]
    for m, n, k, L, opA, opB in cases:
        A = rng.uniform(-0.5, 0.5, (k, m) if opA else (m, k))
        A *= np.exp2(rng.integers(-20, 21, size=A.shape[0]))[:, None]
        B = rng.uniform(-0.5, 0.5, (n, k) if opB else (k, n))
        C = rng.uniform(-0.5, 0.5, (m, n))
        got = _noalloc(m, n, k, L, A, B, C, opA=opA, opB=opB)
        ref = _with_work(m, n, k, L, A, B, C, opA=opA, opB=opB)
        assert np.array_equal(got, ref), (m, n, k, L)


def test_noalloc_persistent_tiles_match(cuda):
    """More output tiles (16 x 8 of 128 x 256) than the 64 CTAs the fixed
    scratch allows: each CTA reuses its CRT scratch slice for several tiles."""
    rng = np.random.default_rng(7)
    m = n = 2048
    k, L = 256, 12
    A = rng.uniform(-0.5, 0.5, (m, k))
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    for _ in range(2):
        got = _noalloc(m, n, k, L, A, B, C)
        ref = _with_work(m, n, k, L, A, B, C)
        assert np.array_equal(got, ref)


def test_noalloc_at_documented_limit_matches_oracle(cuda):
    """m = n = k = 1024 at 12 moduli, the size the header names as fitting,
    checked bit for bit against the CPU oracle's emulated GEMM."""
    rng = np.random.default_rng(11)
    m = n = k = 1024
    L = 12
    A = rng.uniform(-0.5, 0.5, (m, k))
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    got = _noalloc(m, n, k, L, A, B, C)
    ref = oracle.oz2_gemm(A, B, C, L, mode=1)
    assert np.array_equal(got, ref)


def test_noalloc_validates_before_early_return(cuda):
    """A bad moduli count is an error even when k == 0 (nothing to multiply)."""
    lib = _lib.load()
    a, b = ctypes.c_double(1.0), ctypes.c_double(1.0)
    d = torch.zeros(16, dtype=torch.float64, device="cuda")
    rc = lib.chpl_oz2_gemm_noalloc(0, 0, 0, 4, 4, 0, ctypes.byref(a), d.data_ptr(), 4, d.data_ptr(), 1,
                                   ctypes.byref(b), d.data_ptr(), 4, 1)
    assert rc == _lib.CHPL_ERR_INVALID


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    lib = _lib.load()
    a, b = ctypes.c_double(1.0), ctypes.c_double(0.0)
    m = n = 8192
    k = 4096
    dA = torch.zeros(1, dtype=torch.float64, device="cuda")
    rc = lib.chpl_oz2_gemm_noalloc(0, 0, 0, m, n, k, ctypes.byref(a), dA.data_ptr(), m, dA.data_ptr(), k,
                                   ctypes.byref(b), dA.data_ptr(), m, 11)
    assert rc == _lib.CHPL_ERR_WORKSPACE
    assert b"64 MiB" in lib.chpl_last_error_string()
