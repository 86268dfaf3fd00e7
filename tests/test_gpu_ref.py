"""GPU parity against the reference's own generator kernel.

chpl_single generates its matrix with cuRAND's Philox (hs_rand +
matgen_kernel, src/chpl_single.cu:73-94).  oracle/ref_build.py compiles those
lines, cut verbatim from the reference checkout, into
oracle/_ref/libref_single_matgen.so (sm_100a; it travels with the repository).
This library's Philox generator must write the same matrix bit for bit, and a
solve of that matrix must agree with the host LAPACK solution of it.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from chpl_b200 import _lib, hpl

pytestmark = pytest.mark.gpu

_REF_SO = oracle.ref_single_matgen_path()
needs_ref = pytest.mark.skipif(_REF_SO is None, reason="oracle/_ref not built (no reference checkout)")


def _ref_lib():
    L = ctypes.CDLL(_REF_SO)
    L.ref_single_matgen.restype = ctypes.c_int
    L.ref_single_matgen.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p]
    return L


def _philox(m, n, lda, row0, col0, ncg, seed):
    d = torch.full((n * lda,), float("nan"), dtype=torch.float64, device="cuda")
    _lib.check(_lib.load().chpl_matgen_philox(None, d.data_ptr(), lda, m, n, row0, col0, ncg, seed),
               "chpl_matgen_philox")
    torch.cuda.synchronize()
    return d


@needs_ref
def test_philox_matrix_equals_reference_kernel(cuda):
    ref = _ref_lib()
    for N, seed in ((1000, 42), (777, 7)):
        d = _philox(N, N + 1, N, 0, 0, N + 1, seed)
        r = torch.full_like(d, float("nan"))
        assert ref.ref_single_matgen(r.data_ptr(), N, 0, N + 1, N, seed, N, None) == 0
        torch.cuda.synchronize()
        assert torch.equal(d.view(torch.int64), r.view(torch.int64)), (N, seed)


@needs_ref
def test_philox_column_block_equals_reference_kernel(cuda):
    """A block of columns [c0, c0+nc) written at its own origin (row0 = 0,
    col0 = c0) equals the reference kernel's columns c0.. of the full matrix."""
    ref = _ref_lib()
    N, c0, nc = 512, 300, 100
    full = torch.zeros((N + 1) * N, dtype=torch.float64, device="cuda")
    assert ref.ref_single_matgen(full.data_ptr(), N, 0, N + 1, N, 42, N, None) == 0
    blk = _philox(N, nc, N, 0, c0, N + 1, 42)
    torch.cuda.synchronize()
    assert torch.equal(blk.view(torch.int64), full[c0 * N:(c0 + nc) * N].view(torch.int64))


def test_philox_solve_agrees_with_lapack(cuda):
    """chpl_single's matrix solved by the library (FP64 update and the
    Ozaki-II update) against scipy's LAPACK solve of the same matrix."""
    N, NB = 2048, 256
    d = _philox(N, N + 1, N, 0, 0, N + 1, 42)
    Ab = d.cpu().numpy().reshape(N + 1, N).T.copy()
    x_ref = oracle.lapack_hpl_solve(np.asfortranarray(Ab.copy()))
    for emulate, tol in ((False, 1e-9), (True, 1e-7)):
        r = hpl.run(hpl.Config(N=N, NB=NB, moduli=12, emulate=emulate, generator=_lib.CHPL_GEN_PHILOX), want_x=True)
        assert r.passed, r.resid
        x = r.x
        assert np.linalg.norm(x - x_ref) / np.linalg.norm(x_ref) < tol, emulate
        assert abs(r.resid - oracle.hpl_residual_from(Ab, x)) <= 1e-6 * max(1.0, r.resid) + 1e-3


# ---------------------------------------------------------------- chpl_single's Ozaki-I kernels
_OZ1_SO = oracle.ref_oz1_path()


@pytest.mark.skipif(_OZ1_SO is None, reason="oracle/_ref not built (no reference checkout)")
@pytest.mark.parametrize("m,n,k", [(300, 200, 257), (1000, 64, 1024), (129, 777, 96)])
def test_oz1_engine_equals_reference_kernels(cuda, m, n, k):
    """C -= A B through the reference's own Ozaki-I kernels (row / column
    scales, digit slices and reconstruction of src/chpl_single.cu:147-236,
    compiled from the reference checkout into oracle/_ref/libref_oz1.so) with
    the six diagonal products of their digits formed exactly on the host (the
    reference forms them with cuBLASLt int8 GEMMs: exact integers either way)
    equals this library's chpl_oz1_gemm bit for bit."""
    S = 6
    R = ctypes.CDLL(_OZ1_SO)
    vp, sz, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    R.ref_oz1_prepare.argtypes = [vp, sz, i32, i32, vp, sz, i32, i32, vp, vp, vp, vp, vp, vp]
    R.ref_oz1_recon.argtypes = [vp, sz, i32, i32, vp, vp, vp, vp, vp, vp, i32, vp, vp]
    rng = np.random.default_rng(m + n + k)
    A = rng.uniform(-1, 1, (m, k)) * np.exp2(rng.integers(-30, 30, m))[:, None]
    B = rng.uniform(-1, 1, (k, n))
    C = rng.uniform(-1, 1, (m, n))
    dA = torch.from_numpy(np.ascontiguousarray(A.T)).cuda()      # column-major, ld = m
    dB = torch.from_numpy(np.ascontiguousarray(B.T)).cuda()      # ld = k
    f64 = dict(dtype=torch.float64, device="cuda")
    rinv, rsc, cinv, csc = (torch.empty(x, **f64) for x in (m, m, n, n))
    SA = torch.empty(m * S * k, dtype=torch.int8, device="cuda")
    SB = torch.empty(n * S * k, dtype=torch.int8, device="cuda")
    assert R.ref_oz1_prepare(dA.data_ptr(), m, m, k, dB.data_ptr(), k, n, S, rinv.data_ptr(), rsc.data_ptr(),
                             cinv.data_ptr(), csc.data_ptr(), SA.data_ptr(), SB.data_ptr()) == 0
    sa = SA.cpu().numpy().reshape(m, S, k).astype(np.float64)          # [i][p][h]
    sb = SB.cpu().numpy().reshape(n, S, k)[:, ::-1, :].astype(np.float64)   # [j][q][h], q ascending
    D = []
    for d in range(S):   # integers below 2^53 in every partial sum: exact in float64
        P = sum(sa[:, p, :] @ sb[:, d - p, :].T for p in range(d + 1))
        D.append(torch.from_numpy(np.ascontiguousarray(P.T).astype(np.int32)).cuda())   # column-major m x n
    dC = torch.from_numpy(np.ascontiguousarray(C.T)).cuda()
    assert R.ref_oz1_recon(dC.data_ptr(), m, m, n, *[x.data_ptr() for x in D], S, rsc.data_ptr(),
                           csc.data_ptr()) == 0
    ref = dC.cpu().numpy().T
    # this library's engine on the same inputs
    L = _lib.load()
    w = ctypes.c_size_t()
    _lib.check(L.chpl_oz1_worksize(m, n, k, ctypes.byref(w)), "chpl_oz1_worksize")
    work = torch.empty(w.value, dtype=torch.uint8, device="cuda")
    dC2 = torch.from_numpy(np.ascontiguousarray(C.T)).cuda()
    _lib.check(L.chpl_oz1_gemm(None, m, n, k, -1.0, dA.data_ptr(), m, dB.data_ptr(), k, 1.0, dC2.data_ptr(), m,
                               work.data_ptr()), "chpl_oz1_gemm")
    torch.cuda.synchronize()
    got = dC2.cpu().numpy().T
    assert np.array_equal(got.view(np.uint64), ref.view(np.uint64))
    assert np.array_equal(got.view(np.uint64), oracle.oz1_gemm(A, B, C).view(np.uint64))
