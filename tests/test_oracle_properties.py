"""Property tests of the CPU oracle's Ozaki-II pieces and interchanges on
random inputs (hypothesis).  These are the facts the GPU path's exactness
rests on, checked in exact integer arithmetic:

* the power-of-two scale of every row / column keeps the 2-norm of its integer
  image below 2^alpha (2^beta), so by Cauchy-Schwarz every dot product of
  images lies inside the symmetric CRT range (-M/2, M/2);
* every residue lies in its modulus' symmetric range and is congruent to the
  integer image;
* the emulated product recovers the exact integer dot product (exact CRT);
* a dlaswp sequence applied as one net permutation equals the swaps applied
  one by one.
"""
import math

import numpy as np
import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import oracle

SETTINGS = settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])


@st.composite
def scaled_matrix(draw, max_rows=6, max_k=48):
    """Rows of uniform values times 2^u, u drawn per row from a wide range,
    with some exact zeros and an occasional all-zero row."""
    m = draw(st.integers(1, max_rows))
    k = draw(st.integers(1, max_k))
    seed = draw(st.integers(0, 2**31 - 1))
    rng = np.random.default_rng(seed)
    A = rng.uniform(-0.5, 0.5, (m, k))
    A *= np.exp2(rng.integers(-300, 300, size=m))[:, None]
    A[rng.random((m, k)) < 0.1] = 0.0
    if draw(st.booleans()):
        A[rng.integers(0, m)] = 0.0
    return A


def _images(A, shift):
    return [[int(np.rint(np.ldexp(A[i, h], int(shift[i])))) for h in range(A.shape[1])] for i in range(A.shape[0])]


@SETTINGS
@given(A=scaled_matrix(), L=st.sampled_from([8, 11, 12, 14, 16]))
def test_row_images_stay_under_the_norm_bound(A, L):
    a_bits, _ = oracle.oz2_shift_bits(L, A.shape[1])
    sa = oracle.oz2_row_shift(A, a_bits)
    for row in _images(A, sa):
        assert sum(x * x for x in row) < 4 ** a_bits
        assert all(abs(x) <= 2**52 for x in row)


@SETTINGS
@given(A=scaled_matrix(), L=st.sampled_from([11, 12, 16]))
def test_column_images_stay_under_the_norm_bound(A, L):
    B = A.T.copy()                      # k x n: columns are the drawn rows
    _, b_bits = oracle.oz2_shift_bits(L, B.shape[0])
    sb = oracle.oz2_col_shift(B, b_bits)
    for col in _images(B.T, sb):
        assert sum(x * x for x in col) < 4 ** b_bits


@SETTINGS
@given(A=scaled_matrix(max_rows=4, max_k=24), L=st.sampled_from([2, 5, 11, 12, 16]))
def test_residues_symmetric_and_congruent(A, L):
    a_bits, _ = oracle.oz2_shift_bits(L, A.shape[1])
    sa = oracle.oz2_row_shift(A, a_bits)
    r = oracle.oz2_split_rows(A, sa, L)
    img = _images(A, sa)
    for l, md in enumerate(oracle.oz2_moduli(L)):
        hi = (md - 1) // 2
        for i, row in enumerate(img):
            for h, x in enumerate(row):
                v = int(r[l, i, h])
                assert hi - md + 1 <= v <= hi
                assert (v - x) % md == 0


@SETTINGS
@given(A=scaled_matrix(max_rows=3, max_k=16), seed=st.integers(0, 2**31 - 1), L=st.sampled_from([11, 12]))
def test_exact_crt_recovers_exact_dot_products(A, seed, L):
    rng = np.random.default_rng(seed)
    m, k = A.shape
    B = rng.uniform(-0.5, 0.5, (k, 3)) * np.exp2(rng.integers(-40, 40, size=3))[None, :]
    a_bits, b_bits = oracle.oz2_shift_bits(L, k)
    sa = oracle.oz2_row_shift(A, a_bits)
    sb = oracle.oz2_col_shift(B, b_bits)
    ai = _images(A, sa)
    bi = _images(B.T, sb)
    out = oracle.oz2_gemm(A, B, np.zeros((m, 3)), L, alpha=1.0, beta=0.0, mode=0)
    M = oracle.oz2_constants(L)["M"]
    for i in range(m):
        for j in range(3):
            exact = sum(x * y for x, y in zip(ai[i], bi[j]))
            assert abs(exact) < M // 2
            assert out[i, j] == math.ldexp(float(exact), -(int(sa[i]) + int(sb[j])))


@SETTINGS
@given(nrows=st.integers(2, 60), k1=st.integers(0, 10), ns=st.integers(1, 30), seed=st.integers(0, 2**31 - 1))
def test_laswp_equals_sequential_swaps(nrows, k1, ns, seed):
    k1 = min(k1, nrows - 1)
    ns = min(ns, nrows - k1)
    rng = np.random.default_rng(seed)
    ipiv = np.arange(nrows, dtype=np.int64)
    for i in range(k1, k1 + ns):
        ipiv[i] = rng.integers(i, nrows)         # partial pivoting: pivot at or below row i
    A = rng.standard_normal((nrows, 5))
    ref = A.copy()
    for i in range(k1, k1 + ns):
        ref[[i, ipiv[i]]] = ref[[ipiv[i], i]]
    got = oracle.laswp(np.asfortranarray(A), ipiv, k1, k1 + ns)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("L", list(range(2, 17)))
def test_shift_bits_fit_the_crt_range(L):
    """alpha + beta < log2(M) - 1: the Cauchy-Schwarz bound 2^(alpha+beta) < M/2."""
    a, b = oracle.oz2_shift_bits(L, 4096)
    assert 2 ** (a + b) < oracle.oz2_constants(L)["M"] // 2


# ---------------------------------------------------------------- Ozaki scheme I (oracle.oz1_gemm)
@SETTINGS
@given(scaled_matrix(max_rows=5, max_k=40), st.integers(1, 5), st.integers(0, 2**31 - 1))
def test_oz1_digits_and_products_are_exact(A, n, seed):
    """The Ozaki-I restatement's facts, in exact rational arithmetic: a scaled
    entry x in (-1, 1) is sum_p t_p 128^-(p+1) + r 128^-6 with integer digits
    t_p in [-128, 127] and |r| <= 1; the diagonal sums of digit products the
    float64 BLAS forms are the exact integers; and the emulated product keeps
    every entry within k 2^-40 of its row x column scale."""
    from fractions import Fraction
    m, k = A.shape
    B = np.random.default_rng(seed).uniform(-0.5, 0.5, (k, n))
    ea = np.frexp(np.max(np.abs(A), axis=1))[1]
    xa = np.ldexp(A, -ea[:, None])
    assert np.all(np.abs(xa) < 1.0)
    da = oracle._oz1_digits(xa)
    for p in range(oracle.OZ1_SLICES):
        assert np.all(da[p] == np.rint(da[p])) and np.all((da[p] >= -128) & (da[p] <= 127))
    # the remainder after six digits, recomputed exactly
    for i in range(m):
        for h in range(k):
            x = Fraction(float(xa[i, h]))
            head = sum(Fraction(int(da[p][i, h])) / 128 ** (p + 1) for p in range(oracle.OZ1_SLICES))
            assert abs(x - head) * 128 ** oracle.OZ1_SLICES <= 1
    eb = np.frexp(np.max(np.abs(B), axis=0))[1]
    db = oracle._oz1_digits(np.ldexp(B, -eb[None, :]))
    for d in range(oracle.OZ1_SLICES):
        P = np.hstack(da[:d + 1]) @ np.vstack(db[d::-1])
        Q = sum(da[p].astype(np.int64) @ db[d - p].astype(np.int64) for p in range(d + 1))
        assert np.array_equal(P.astype(np.int64), Q)
    got = oracle.oz1_gemm(A, B, np.zeros((m, n)), alpha=1.0, beta=0.0)
    bound = k * 2.0 ** -40 * np.ldexp(1.0, ea)[:, None] * np.ldexp(1.0, eb)[None, :]
    assert np.all(np.abs(got - A @ B) <= bound + 1e-300)
