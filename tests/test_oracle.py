"""CPU tests of the oracle itself: pins against published known answers, exact
integer arithmetic (Python big integers) and LAPACK, before the oracle is
trusted to check the GPU."""
import math
import os

import numpy as np
import pytest
import scipy.linalg

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_splitmix64_known_answers():
    # published SplitMix64 outputs for seed 0 (Steele et al. 2014 reference code)
    assert oracle.splitmix64(0, 0) == 0xE220A8397B1DCDAF
    assert oracle.splitmix64(0, 1) == 0x6E789E6AA1B965F4
    assert oracle.splitmix64(0, 2) == 0x06C45D188009454F


def _splitmix_py(seed: int, idx: int) -> int:
    M = (1 << 64) - 1
    z = (seed + (idx + 1) * 0x9E3779B97F4A7C15) & M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    return z ^ (z >> 31)


def test_generator_matches_reference_formula():
    # chpl_elem (src/chpl_p2.cu:66-73): top 53 bits / 2^53 - 0.5 at index i*(N+1)+j
    N = 37
    A = oracle.hpl_system(N, seed=42)
    for (i, j) in [(0, 0), (3, 5), (36, 37), (17, 0), (0, 37)]:
        z = _splitmix_py(42, i * (N + 1) + j)
        assert A[i, j] == (z >> 11) * 2.0 ** -53 - 0.5
    assert A.min() >= -0.5 and A.max() < 0.5


def test_generator_golden_fixture():
    fx = np.load(os.path.join(GOLDEN, "matgen_N64_seed42.npz"))
    A = oracle.hpl_system(64, seed=42)
    assert np.array_equal(A, fx["A"])


def test_moduli_pairwise_coprime():
    mods = oracle.oz2_moduli(16)
    assert mods[:11] == [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223]
    for a in range(16):
        for b in range(a + 1, 16):
            assert math.gcd(mods[a], mods[b]) == 1
    assert all(m <= 256 for m in mods)


@pytest.mark.parametrize("L", [2, 8, 11, 12, 14, 16])
def test_crt_constants_exact(L):
    c = oracle.oz2_constants(L)
    M = math.prod(c["moduli"])
    assert c["M"] == M
    for l, m in enumerate(c["moduli"]):
        assert (c["y"][l] * (M // m)) % m == 1
        # v_l = round(2^64 y_l / m_l)
        assert c["v"][l] == ((c["y"][l] << 64) + m // 2) // m
    assert abs(c["Mf"] - M / 2.0 ** 64) <= 2.0 ** -52 * (M / 2.0 ** 64)


def _sym(x: int, m: int) -> int:
    hi = (m - 1) // 2
    r = x % m
    return r - m if r > hi else r


@pytest.mark.parametrize("L", [11, 12])
def test_exact_crt_against_bigints(L):
    """mode 0 reconstruction == Python big-integer CRT of the same products."""
    rng = np.random.default_rng(L)
    m, n, k = 6, 5, 40
    a_bits, b_bits = oracle.oz2_shift_bits(L, k)
    A = rng.uniform(-0.5, 0.5, (m, k))
    B = rng.uniform(-0.5, 0.5, (k, n))
    sa = oracle.oz2_row_shift(A, a_bits)
    sb = oracle.oz2_col_shift(B, b_bits)
    ra = oracle.oz2_split_rows(A, sa, L)
    rb = oracle.oz2_split_cols(B, sb, L)
    mods = oracle.oz2_moduli(L)
    M = math.prod(mods)
    # exact integer images
    ai = [[int(np.rint(np.ldexp(A[i, h], int(sa[i])))) for h in range(k)] for i in range(m)]
    bi = [[int(np.rint(np.ldexp(B[h, j], int(sb[j])))) for j in range(n)] for h in range(k)]
    for l, md in enumerate(mods):
        for i in range(m):
            for h in range(k):
                assert ra[l, i, h] == _sym(ai[i][h], md)
    C0 = np.zeros((m, n))
    out = oracle.oz2_gemm(A, B, C0, L, alpha=1.0, beta=0.0, mode=0)
    for i in range(m):
        for j in range(n):
            exact = sum(ai[i][h] * bi[h][j] for h in range(k))
            assert abs(exact) < M // 2
            # residue recombination by big-int CRT reproduces the exact product
            res = [sum(int(ra[l, i, h]) * int(rb[l, j, h]) for h in range(k)) for l in range(L)]
            x = 0
            for l, md in enumerate(mods):
                Ml = M // md
                x = (x + res[l] * Ml * pow(Ml, -1, md)) % M
            if x > M // 2:
                x -= M
            assert x == exact
            assert out[i, j] == math.ldexp(float(exact), -(int(sa[i]) + int(sb[j])))


@pytest.mark.parametrize("L", [11, 12])
def test_fixed_point_crt_close_to_exact(L):
    rng = np.random.default_rng(100 + L)
    A = rng.uniform(-0.5, 0.5, (40, 96))
    B = rng.uniform(-0.5, 0.5, (96, 33))
    C = rng.uniform(-0.5, 0.5, (40, 33))
    e = oracle.oz2_gemm(A, B, C, L, mode=0)
    f = oracle.oz2_gemm(A, B, C, L, mode=1)
    a_bits, b_bits = oracle.oz2_shift_bits(L, 96)
    sa = oracle.oz2_row_shift(A, a_bits)
    sb = oracle.oz2_col_shift(B, b_bits)
    c = oracle.oz2_constants(L)
    # |fixed - exact| <= 2^-53 (M / 2^(sa+sb)) * 1.1 + one ulp of C
    scale = c["M"] * np.ldexp(1.0, -(sa[:, None] + sb[None, :]).astype(np.int64))
    assert np.all(np.abs(f - e) <= 2.0 ** -53 * scale * 1.1 + np.spacing(np.abs(e)) * 2)


def _rigorous_bound(A, B, L):
    """|C_emu - AB| <= sum_h |da||b| + |a||db| + |da||db| with |da| <= 2^-sa/2."""
    k = A.shape[1]
    a_bits, b_bits = oracle.oz2_shift_bits(L, k)
    sa = oracle.oz2_row_shift(A, a_bits).astype(np.float64)
    sb = oracle.oz2_col_shift(B, b_bits).astype(np.float64)
    da = 0.5 * np.exp2(-sa)[:, None] * np.ones_like(A)
    db = 0.5 * np.exp2(-sb)[None, :] * np.ones_like(B)
    return da @ np.abs(B) + np.abs(A) @ db + da @ db


@pytest.mark.parametrize("L", [11, 12])
def test_emulated_gemm_error_bound(L):
    rng = np.random.default_rng(7)
    A = rng.uniform(-0.5, 0.5, (64, 200))
    A *= np.exp2(rng.integers(-20, 21, size=64))[:, None]   # config 2 variant: rows scaled by 2^u
    B = rng.uniform(-0.5, 0.5, (200, 48))
    C = rng.uniform(-0.5, 0.5, (64, 48))
    out = oracle.oz2_gemm(A, B, C, L, mode=0)
    ref = C - A @ B
    bound = _rigorous_bound(A, B, L) + 4 * np.spacing(np.abs(ref)) + 1e-300
    assert np.all(np.abs(out - ref) <= bound)


def test_laswp_semantics():
    rng = np.random.default_rng(3)
    A = rng.standard_normal((20, 7))
    ipiv = np.array([4, 1, 9, 3, 19, 8, 6, 7, 8, 9], dtype=np.int64)
    ref = A.copy()
    for i in range(10):
        ref[[i, ipiv[i]]] = ref[[ipiv[i], i]]
    got = oracle.laswp(np.asfortranarray(A), ipiv, 0, 10)
    assert np.array_equal(got, ref)


def test_lu_matches_lapack():
    N = 96
    x, ipiv, F = oracle.hpl_solve(N, 16, L=0)
    S = oracle.hpl_system(N)
    lu, piv = scipy.linalg.lu_factor(S[:, :N])
    assert np.array_equal(ipiv, piv)
    # U matches; L of earlier panels is left unpermuted (as in the reference, only U and b are used)
    assert np.allclose(np.triu(F[:, :N]), np.triu(lu), rtol=1e-12, atol=1e-12)
    xs = scipy.linalg.lu_solve((lu, piv), S[:, N])
    assert np.allclose(x, xs, rtol=1e-11, atol=1e-11)


def test_residual_formula():
    N = 80
    S = oracle.hpl_system(N)
    x = np.linalg.solve(S[:, :N], S[:, N])
    r1 = oracle.hpl_residual(x, N)
    r2 = oracle.hpl_residual_from(S, x)
    # both evaluations sit at rounding level (their ratio is noise), far below 16
    assert r1 < 1.0 and r2 < 1.0
    # the formula itself: a known residual vector gives the known value
    xp = x + 1e-10
    rp = np.max(np.abs(S[:, :N] @ xp - S[:, N])) / (2.0 ** -53 * (np.max(np.abs(S[:, :N]).sum(1)) * np.max(np.abs(xp)) + np.max(np.abs(S[:, N]))) * N)
    assert oracle.hpl_residual(xp, N) == pytest.approx(rp, rel=1e-4)
    # a perturbed solution fails
    assert oracle.hpl_residual(x * (1 + 1e-9), N) > 16.0


def test_emulated_lu_residual_passes():
    """End-to-end restatement: the reference's own check (residual < 16,
    src/chpl_single.cu:931-948) holds for the restated method at 12 moduli."""
    x, _, _ = oracle.hpl_solve(512, 64, L=12)
    assert oracle.hpl_residual(x, 512) < 16.0


def test_oz1_golden_fixture():
    """The Ozaki-I restatement reproduces its committed fixture bit for bit."""
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "oz1_m48_n40_k200.npz"))
    upd = oracle.oz1_gemm(g["A"], g["B"], g["C"])
    prod = oracle.oz1_gemm(g["A"], g["B"], None, alpha=1.0, beta=0.0)
    assert np.array_equal(upd.view(np.uint64), g["update"].view(np.uint64))
    assert np.array_equal(prod.view(np.uint64), g["product"].view(np.uint64))
