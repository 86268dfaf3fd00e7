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
