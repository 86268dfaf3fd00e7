"""GPU parity of the Ozaki-II path against the CPU oracle, through the C ABI.

Bit-exact: shifts, int8 residues, per-modulus int32 products, and the full
emulated GEMM against the oracle's fixed-point mirror (same FP64 operations).
Within tolerance: against exact CRT and FP64 DGEMM (rigorous error bound, and
max|dC| / (||A||_oo ||B||_oo) <= 1e-15 at 11 moduli, the standalone update's tolerance).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from chpl_b200 import oz2
from gpu_util import empty_bytes, from_dev, round_up, to_dev

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(params=["pair", "single"])
def form(request, monkeypatch):
    """Both forms of the GEMM kernel: single CTAs (128 x 256 tiles, the
    default) and CTA pairs (256 x 256 tiles, above 128 rows)."""
    monkeypatch.setenv("CHPL_OZ2_FORM", request.param)
    return request.param


def _split_rows_gpu(A, L, opA=0):
    m, k = (A.shape[1], A.shape[0]) if opA else A.shape
    ldv, ldk = round_up(m, 128), round_up(k, 128)
    dA, lda = to_dev(A)
    res = torch.full((L * ldv * ldk,), 77, dtype=torch.int8, device="cuda")
    sh = torch.zeros(ldv, dtype=torch.int32, device="cuda")
    tmp = empty_bytes(oz2.split_tmp_bytes(ldv))
    oz2.split_rows(opA, m, k, dA, lda, L, res, ldv, ldk, sh, tmp)
    torch.cuda.synchronize()
    return res.cpu().numpy().reshape(L, ldv, ldk), sh.cpu().numpy(), m, k


def _split_cols_gpu(B, L, opB=0):
    k, n = (B.shape[1], B.shape[0]) if opB else B.shape
    ldv, ldk = round_up(n, 256), round_up(k, 128)
    dB, ldb = to_dev(B)
    res = torch.full((L * ldv * ldk,), 77, dtype=torch.int8, device="cuda")
    sh = torch.zeros(ldv, dtype=torch.int32, device="cuda")
    tmp = empty_bytes(oz2.split_tmp_bytes(ldv))
    oz2.split_cols(opB, k, n, dB, ldb, L, res, ldv, ldk, sh, tmp)
    torch.cuda.synchronize()
    return res.cpu().numpy().reshape(L, ldv, ldk), sh.cpu().numpy(), n, k


@pytest.mark.parametrize("L", [11, 12, 14])
@pytest.mark.parametrize("op", [0, 1])
@pytest.mark.parametrize("shape", [(37, 61), (300, 257), (129, 1024)])
def test_split_rows_bitexact(cuda, L, op, shape):
    rng = np.random.default_rng(hash((L, op, shape)) & 0xFFFF)
    m, k = shape
    A = rng.uniform(-0.5, 0.5, (m, k)) * np.exp2(rng.integers(-20, 21, size=m))[:, None]
    A[min(3, m - 1), :] = 0.0                      # a zero row
    Aop = np.ascontiguousarray(A.T) if op else A
    res, sh, m, k = _split_rows_gpu(Aop, L, op)
    a_bits, _ = oracle.oz2_shift_bits(L, k)
    sh_ref = oracle.oz2_row_shift(Aop, a_bits, opA=op)
    ra_ref = oracle.oz2_split_rows(Aop, sh_ref, L, opA=op)
    assert np.array_equal(sh[:m], sh_ref)
    assert np.array_equal(res[:, :m, :k], ra_ref)
    assert not res[:, :m, k:].any() and not res[:, m:, :].any()   # zero padding


@pytest.mark.parametrize("L", [11, 12])
@pytest.mark.parametrize("op", [0, 1])
@pytest.mark.parametrize("shape", [(61, 37), (257, 300), (1000, 33)])
def test_split_cols_bitexact(cuda, L, op, shape):
    rng = np.random.default_rng(hash((L, op, shape, 1)) & 0xFFFF)
    k, n = shape
    B = rng.uniform(-0.5, 0.5, (k, n))
    B[:, min(2, n - 1)] = 0.0
    Bop = np.ascontiguousarray(B.T) if op else B
    res, sh, n, k = _split_cols_gpu(Bop, L, op)
    _, b_bits = oracle.oz2_shift_bits(L, k)
    sh_ref = oracle.oz2_col_shift(Bop, b_bits, opB=op)
    rb_ref = oracle.oz2_split_cols(Bop, sh_ref, L, opB=op)
    assert np.array_equal(sh[:n], sh_ref)
    assert np.array_equal(res[:, :n, :k], rb_ref)


def test_split_golden(cuda):
    fx = np.load(os.path.join(GOLDEN, "oz2_m40_n36_k160.npz"))
    for L in (11, 12):
        ra, sa, m, k = _split_rows_gpu(fx["A"], L)
        rb, sb, n, _ = _split_cols_gpu(fx["B"], L)
        assert np.array_equal(sa[:m], fx[f"sa{L}"]) and np.array_equal(sb[:n], fx[f"sb{L}"])
        assert np.array_equal(ra[:, :m, :k], fx[f"ra{L}"]) and np.array_equal(rb[:, :n, :k], fx[f"rb{L}"])


def _products_gpu(ra, rb, m, n, k, L):
    """ra: [L, ldva, ldk] int8, rb: [L, ldvb, ldk]."""
    ldva, ldk = ra.shape[1], ra.shape[2]
    ldvb = rb.shape[1]
    dra = torch.from_numpy(np.ascontiguousarray(ra)).cuda()
    drb = torch.from_numpy(np.ascontiguousarray(rb)).cuda()
    P = torch.zeros(L * m * n, dtype=torch.int32, device="cuda")
    oz2.products(m, n, k, L, dra, ldva, drb, ldvb, ldk, P, m)
    torch.cuda.synchronize()
    return P.cpu().numpy().reshape(L, n, m).transpose(0, 2, 1)


@pytest.mark.parametrize("L", [11, 12])
@pytest.mark.parametrize("mnk", [(128, 256, 128), (300, 520, 384), (77, 33, 1000), (1000, 700, 256)])
def test_products_bitexact(cuda, form, L, mnk):
    m, n, k = mnk
    rng = np.random.default_rng(m * 7 + n + L)
    ldva, ldvb, ldk = round_up(m, 128), round_up(n, 256), round_up(k, 128)
    mods = oracle.oz2_moduli(L)
    ra = np.zeros((L, ldva, ldk), dtype=np.int8)
    rb = np.zeros((L, ldvb, ldk), dtype=np.int8)
    for l, md in enumerate(mods):
        hi = (md - 1) // 2
        ra[l, :m, :k] = rng.integers(hi - md + 1, hi + 1, size=(m, k))
        rb[l, :n, :k] = rng.integers(hi - md + 1, hi + 1, size=(n, k))
    P = _products_gpu(ra, rb, m, n, k, L)
    for l in range(L):
        ref = ra[l, :m, :k].astype(np.int64) @ rb[l, :n, :k].astype(np.int64).T
        assert np.array_equal(P[l], ref), f"modulus {l}"


def test_products_persistent_tiles(cuda, form):
    """More tiles than resident CTAs (each CTA or pair loops over tiles), and a
    last 256-row tile whose second half lies past m."""
    L, m, n, k = 2, 2600, 2304, 128
    rng = np.random.default_rng(5)
    ra = np.zeros((L, round_up(m, 128), k), dtype=np.int8)
    rb = np.zeros((L, round_up(n, 256), k), dtype=np.int8)
    ra[:, :m] = rng.integers(-128, 128, size=(L, m, k))
    rb[:, :n] = rng.integers(-128, 128, size=(L, n, k))
    P = _products_gpu(ra, rb, m, n, k, L)
    for l in range(L):
        ref = ra[l, :m].astype(np.int64) @ rb[l, :n].astype(np.int64).T
        assert np.array_equal(P[l], ref), f"modulus {l}"


def test_gemm_persistent_tiles_bitexact(cuda, form):
    m, n, k, L = 2600, 1100, 256, 11
    rng = np.random.default_rng(17)
    A = rng.uniform(-0.5, 0.5, (m, k)) * np.exp2(rng.integers(-20, 21, size=m))[:, None]
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    got = _gemm_gpu(A, B, C, L)
    ref = oracle.oz2_gemm(A, B, C, L, mode=1)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("m", [128, 256])
def test_products_extreme_magnitude(cuda, m):
    """All residues at -128: the largest int32 accumulation at k = 8192."""
    L, n, k = 2, 256, 8192
    ra = np.full((L, m, k), -128, dtype=np.int8)
    rb = np.full((L, 256, k), -128, dtype=np.int8)
    P = _products_gpu(ra, rb, m, n, k, L)
    assert np.all(P == 128 * 128 * k)


def _gemm_gpu(A, B, C, L, alpha=-1.0, beta=1.0, opA=0, opB=0, ldc_pad=0):
    m = A.shape[1] if opA else A.shape[0]
    k = A.shape[0] if opA else A.shape[1]
    n = B.shape[0] if opB else B.shape[1]
    dA, lda = to_dev(A)
    dB, ldb = to_dev(B)
    dC, ldc = to_dev(C, ld=C.shape[0] + ldc_pad)
    tot, _, _ = oz2.workSize(m, n, k, L)
    work = empty_bytes(tot)
    oz2.gemm(opA, opB, m, n, k, alpha, dA, lda, dB, ldb, beta, dC, ldc, L, True, work)
    torch.cuda.synchronize()
    return from_dev(dC, m, n)


@pytest.mark.parametrize("L", [11, 12])
@pytest.mark.parametrize("ops", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("mnk", [(130, 257, 200), (512, 300, 1000), (33, 17, 5)])
def test_gemm_bitexact_vs_oracle_mirror(cuda, form, L, ops, mnk):
    m, n, k = mnk
    opA, opB = ops
    rng = np.random.default_rng(m + n + k + 10 * opA + 20 * opB + L)
    A = rng.uniform(-0.5, 0.5, (m, k)) * np.exp2(rng.integers(-20, 21, size=m))[:, None]
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    Aop = np.ascontiguousarray(A.T) if opA else A
    Bop = np.ascontiguousarray(B.T) if opB else B
    got = _gemm_gpu(Aop, Bop, C, L, opA=opA, opB=opB, ldc_pad=3)
    ref = oracle.oz2_gemm(Aop, Bop, C, L, opA=opA, opB=opB, mode=1)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("ab", [(1.0, 0.0), (2.5, -0.75), (-1.0, 1.0)])
def test_gemm_alpha_beta(cuda, ab):
    alpha, beta = ab
    rng = np.random.default_rng(5)
    A = rng.uniform(-0.5, 0.5, (200, 96))
    B = rng.uniform(-0.5, 0.5, (96, 260))
    C = rng.uniform(-0.5, 0.5, (200, 260))
    got = _gemm_gpu(A, B, C, 12, alpha=alpha, beta=beta)
    ref = oracle.oz2_gemm(A, B, C, 12, alpha=alpha, beta=beta, mode=1)
    assert np.array_equal(got, ref)


def test_gemm_golden(cuda):
    fx = np.load(os.path.join(GOLDEN, "oz2_m40_n36_k160.npz"))
    for L in (11, 12):
        got = _gemm_gpu(fx["A"], fx["B"], fx["C"], L)
        assert np.array_equal(got, fx[f"C{L}"])


@pytest.mark.parametrize("L", [11, 12])
@pytest.mark.parametrize("scaled", [False, True])
def test_gemm_vs_fp64_dgemm(cuda, L, scaled):
    """Config-2 style check at a size the CPU DGEMM finishes quickly."""
    m, n, k = 2048, 1536, 1024
    rng = np.random.default_rng(42 + L)
    A = rng.uniform(-0.5, 0.5, (m, k))
    if scaled:
        A *= np.exp2(rng.integers(-20, 21, size=m))[:, None]
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    got = _gemm_gpu(A, B, C, L)
    ref = C - A @ B
    err = np.abs(got - ref)
    a_bits, b_bits = oracle.oz2_shift_bits(L, k)
    sa = oracle.oz2_row_shift(A, a_bits).astype(np.float64)
    sb = oracle.oz2_col_shift(B, b_bits).astype(np.float64)
    M = float(oracle.oz2_constants(L)["M"])
    bound = ((0.5 * np.exp2(-sa)[:, None] * np.abs(B).sum(0)[None, :]
              + 0.5 * np.abs(A).sum(1)[:, None] * np.exp2(-sb)[None, :]) * 1.01
             + 2.0 ** -52 * M * np.exp2(-(sa[:, None] + sb[None, :]))       # fixed-point CRT rounding
             + 8 * np.spacing(np.abs(ref)))
    assert np.all(err <= bound)
    normwise = err.max() / (np.abs(A).sum(1).max() * np.abs(B).sum(1).max())
    assert normwise <= (1e-15 if L == 11 else 1e-16)


def test_skip_scalA_reuse(cuda):
    """Column chunks with the residues of A reused (src/chpl_p2.cu:1642-1643,1684)."""
    rng = np.random.default_rng(9)
    m, k, n1, n2 = 700, 512, 600, 300
    A = rng.uniform(-0.5, 0.5, (m, k))
    B = rng.uniform(-0.5, 0.5, (k, n1 + n2))
    C = rng.uniform(-0.5, 0.5, (m, n1 + n2))
    dA, lda = to_dev(A)
    dB, ldb = to_dev(B)
    dC, ldc = to_dev(C)
    L = 11
    tot, _, _ = oz2.workSize(m, max(n1, n2), k, L, True, False)
    work = empty_bytes(tot)
    oz2.gemm(0, 0, m, n1, k, -1.0, dA, lda, dB, ldb, 1.0, dC, ldc, L, True, work, enable_skip_scalA=True)
    oz2.gemm(0, 0, m, n2, k, -1.0, dA, lda, dB.data_ptr() + n1 * ldb * 8, ldb, 1.0,
             dC.data_ptr() + n1 * ldc * 8, ldc, L, True, work, enable_skip_scalA=True, skip_scalA=True)
    torch.cuda.synchronize()
    got = from_dev(dC, m, n1 + n2)
    ref = oracle.oz2_gemm(A, B, C, L, mode=1)
    assert np.array_equal(got, ref)


def test_external_work_slots(cuda):
    rng = np.random.default_rng(11)
    m, n, k, L = 300, 400, 256, 12
    A = rng.uniform(-0.5, 0.5, (m, k))
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    dA, lda = to_dev(A)
    dB, ldb = to_dev(B)
    dC, ldc = to_dev(C)
    tot, wa, wb = oz2.workSize(m, n, k, L, True, True)
    work = empty_bytes(tot - wa - wb)
    workA = empty_bytes(wa)
    workB = empty_bytes(wb)
    oz2.gemm(0, 0, m, n, k, -1.0, dA, lda, dB, ldb, 1.0, dC, ldc, L, True, work, workA, workB)
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(dC, m, n), oracle.oz2_gemm(A, B, C, L, mode=1))


def test_invalid_arguments(cuda):
    from chpl_b200 import ChplError
    work = empty_bytes(1 << 20)
    with pytest.raises(ChplError):
        oz2.gemm(0, 0, 10, 10, 10, 1.0, 0, 10, 0, 10, 0.0, 0, 5, 11, True, work)   # ldc < m
    with pytest.raises(ChplError):
        oz2.workSize(10, 10, 10, 1)                                                 # too few moduli
    with pytest.raises(ChplError):
        oz2.workSize(10, 10, 200000, 11)                                            # k beyond int32 bound
