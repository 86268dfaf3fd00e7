/*
 * CPU oracle for the chpl_b200 hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C on the host, the arithmetic that the
 * B200 kernels of chpl_b200 perform, so that tests/, __graft_entry__.smoke()
 * and the cpu_baseline leg of bench.py can check the GPU results.  Nothing in
 * the shipped library links, loads or calls this code.
 *
 * What is restated, and where it comes from (paths inside Koyingtw/CHPL):
 *   - matrix generator: chpl_elem() of src/chpl_p2.cu:66-73, element (i,j)
 *     of the N x (N+1) system at index i*(N+1)+j (src/chpl_p2.cu:84-86,
 *     ncg = ntot = N+1 at src/chpl_p2.cu:585); b is column N.
 *     chpl_elem() is the SplitMix64 output function applied to the counter
 *     (idx+1)*golden + seed, i.e. the idx-th SplitMix64 output for `seed`
 *     (Steele, Lea, Flood, "Fast splittable pseudorandom number generators",
 *     OOPSLA 2014).  Pinned against published SplitMix64 known answers.
 *   - Ozaki scheme II emulated DGEMM (C = alpha*A*B + beta*C), the call made
 *     at src/chpl_single.cu:641-649 and src/chpl_p2.cu:1674-1683 into
 *     GEMMul8 v3.2.0 (RIKEN-RCCS/GEMMul8, MIT; submodule absent from the
 *     reference checkout).  The method is restated from Ozaki, Uchino and
 *     Imamura, "Ozaki Scheme II: A GEMM-oriented emulation of floating-point
 *     matrix multiplication using an integer modular technique" (2025):
 *     power-of-two row/column scaling, rounding to integers, symmetric
 *     residues modulo pairwise-coprime moduli <= 256 (int8), one exact
 *     int8 x int8 -> int32 product per modulus, Chinese-remainder
 *     reconstruction, unscaling.  The moduli table, the fast-mode scaling
 *     rule and the fixed-point CRT are this project's own (GEMMul8's exact
 *     tables are not available); GEMMul8 kernel-level parity is unpinned.
 *     The exact CRT here uses 128-bit integers and is pinned against Python
 *     big integers in the tests.
 *   - row interchanges: LAPACK dlaswp semantics as used by apply_swaps()
 *     (src/chpl_single.cu:489-518): for i = k1..k2-1 swap row i with ipiv[i].
 *   - LU with partial pivoting + back substitution of the N x (N+1) system
 *     (src/chpl_single.cu:658-727), optional Ozaki-II trailing update.
 *   - HPL scaled residual ||Ax-b||_oo / (eps*(||A||_oo*||x||_oo+||b||_oo)*N),
 *     eps = 2^-53 (src/chpl_single.cu:785-802, src/chpl_p2.cu:1925-1932).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_MAX_MODULI 16

/* ------------------------------------------------------------------ */
/* Generator                                                           */
/* ------------------------------------------------------------------ */
uint64_t orc_splitmix64(uint64_t seed, uint64_t idx)
{
    uint64_t z = seed + (idx + 1u) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* top 53 bits scaled to [0,1), shifted to [-0.5, 0.5) (src/chpl_p2.cu:72) */
double orc_elem(uint64_t seed, uint64_t idx)
{
    return (double)(orc_splitmix64(seed, idx) >> 11) * (1.0 / 9007199254740992.0) - 0.5;
}

/* A[i + j*lda] = elem(seed, (row0+i)*ncg + col0+j) for an m x n block */
void orc_matgen(double *A, int64_t lda, int64_t m, int64_t n, int64_t row0,
                int64_t col0, int64_t ncg, uint64_t seed)
{
    for (int64_t j = 0; j < n; ++j)
        for (int64_t i = 0; i < m; ++i)
            A[i + j * lda] = orc_elem(seed, (uint64_t)(row0 + i) * (uint64_t)ncg +
                                                (uint64_t)(col0 + j));
}

/* ------------------------------------------------------------------ */
/* Ozaki scheme II                                                     */
/* ------------------------------------------------------------------ */
static int64_t gcd64(int64_t a, int64_t b)
{
    while (b) { int64_t t = a % b; a = b; b = t; }
    return a < 0 ? -a : a;
}

/* Greedy pairwise-coprime moduli, scanning down from 256. */
int orc_oz2_moduli(int L, int32_t *mod)
{
    if (L < 2 || L > ORC_MAX_MODULI) return -1;
    int n = 0;
    for (int c = 256; c > 1 && n < L; --c) {
        int ok = 1;
        for (int i = 0; i < n; ++i)
            if (gcd64(c, mod[i]) != 1) { ok = 0; break; }
        if (ok) mod[n++] = c;
    }
    return n == L ? 0 : -1;
}

/* symmetric range of residues modulo m: [lo, hi] with hi-lo+1 = m */
static void sym_range(int32_t m, int32_t *lo, int32_t *hi)
{
    *hi = (m - 1) / 2;
    *lo = *hi - m + 1;
}

static int32_t sym_mod64(int64_t x, int32_t m)
{
    int32_t lo, hi;
    sym_range(m, &lo, &hi);
    int64_t r = x % m;
    if (r > hi) r -= m;
    if (r < lo) r += m;
    return (int32_t)r;
}

static int64_t inv_mod(int64_t a, int64_t m)
{
    int64_t t = 0, nt = 1, r = m, nr = ((a % m) + m) % m;
    while (nr) {
        int64_t q = r / nr, tmp;
        tmp = t - q * nt; t = nt; nt = tmp;
        tmp = r - q * nr; r = nr; nr = tmp;
    }
    if (r != 1) return -1;
    return t < 0 ? t + m : t;
}

/*
 * CRT constants for L moduli:
 *   y[l]  = (M/m_l)^-1 mod m_l
 *   v[l]  = round(2^64 * y[l] / m_l)  (64-bit fixed-point fraction)
 *   Mf    = M / 2^64 (one rounding), log2M = log2(M)
 *   Mhi/Mlo = M as two 64-bit halves.
 */
int orc_oz2_constants(int L, int32_t *mod, int64_t *y, uint64_t *v, double *Mf,
                      double *log2M, uint64_t *Mhi, uint64_t *Mlo)
{
    if (orc_oz2_moduli(L, mod)) return -1;
    unsigned __int128 M = 1;
    double lg = 0.0;
    for (int l = 0; l < L; ++l) { M *= (unsigned __int128)mod[l]; lg += log2((double)mod[l]); }
    for (int l = 0; l < L; ++l) {
        int64_t ml = mod[l], p = 1;
        for (int i = 0; i < L; ++i)
            if (i != l) p = (p * (mod[i] % ml)) % ml;
        y[l] = inv_mod(p, ml);
        if (y[l] < 0) return -1;
        unsigned __int128 num = ((unsigned __int128)(uint64_t)y[l] << 64) + (unsigned __int128)(ml / 2);
        v[l] = (uint64_t)(num / (unsigned __int128)ml);
    }
    *Mf = (double)M * 0x1p-64;
    *log2M = lg;
    *Mhi = (uint64_t)(M >> 64);
    *Mlo = (uint64_t)M;
    return 0;
}

/*
 * Scaling budget (Cauchy-Schwarz form of the published fast mode): with
 * ||a'_i||_2 < 2^alpha and ||b'_j||_2 < 2^beta every exact dot product obeys
 * |sum_h a'_ih b'_hj| <= ||a'_i|| ||b'_j|| < 2^(alpha+beta) < M/2, so the
 * symmetric CRT range recovers it.  alpha+beta = floor(log2 M - 1.02) leaves
 * a 1.4 % margin for the rounding of a', b' (<= 0.5 sqrt(k) in norm).
 * alpha, beta <= 52 keeps every a', b' exact in FP64.  k is limited so that
 * the int8 x int8 -> int32 products cannot overflow: k * 128 * 128 < 2^31.
 */
#define ORC_MAX_K 131071

int orc_oz2_shift_bits(int L, int64_t k, int *alpha, int *beta)
{
    int32_t mod[ORC_MAX_MODULI];
    if (orc_oz2_moduli(L, mod) || k < 1 || k > ORC_MAX_K) return -1;
    double lg = 0.0;
    for (int l = 0; l < L; ++l) lg += log2((double)mod[l]);
    int T = (int)floor(lg - 1.02);
    int a = (T + 1) / 2, b = T / 2;
    if (a > 52) a = 52;
    if (b > 52) b = 52;
    *alpha = a; *beta = b;
    return 0;
}

static double opel(const double *A, int64_t ld, int op, int64_t r, int64_t c)
{
    return op ? A[c + r * ld] : A[r + c * ld];
}

/*
 * Deterministic upper bound of the 2-norm of a vector x[0..k), as the
 * exponent e with ||x||_2 < 2^e.  With E = ilogb(max|x|) + 1 (max|x| < 2^E),
 * q_h = ceil(|x_h| 2^(20-E)) in [0, 2^20] and Q = sum q_h^2 (exact in 64-bit
 * integers, independent of summation order): ||x|| <= 2^(E-20) sqrt(Q), and
 * sqrt(Q) < 2^p for p = ceil(bitlen(Q)/2).  Returns INT32_MIN for x = 0.
 */
int32_t orc_oz2_norm_exponent(const double *x, int64_t stride, int64_t k)
{
    double mx = 0.0;
    for (int64_t h = 0; h < k; ++h) {
        double a = fabs(x[h * stride]);
        if (a > mx) mx = a;
    }
    if (mx == 0.0) return INT32_MIN;
    const int E = ilogb(mx) + 1;
    uint64_t Q = 0;
    for (int64_t h = 0; h < k; ++h) {
        double q = ceil(ldexp(fabs(x[h * stride]), 20 - E));
        uint64_t qi = (uint64_t)q;
        Q += qi * qi;
    }
    int bl = 64 - __builtin_clzll(Q);
    return E - 20 + (bl + 1) / 2;
}

/* shift[i] = alpha - e_i where ||op(A)[i,:]||_2 < 2^e_i; 0 for a zero row */
void orc_oz2_row_shift(const double *A, int64_t lda, int opA, int64_t m, int64_t k,
                       int alpha, int32_t *shift)
{
    for (int64_t i = 0; i < m; ++i) {
        int32_t e = opA ? orc_oz2_norm_exponent(A + i * lda, 1, k)
                        : orc_oz2_norm_exponent(A + i, lda, k);
        shift[i] = e == INT32_MIN ? 0 : alpha - e;
    }
}

/* shift[j] = beta - e_j where ||op(B)[:,j]||_2 < 2^e_j; 0 for a zero column */
void orc_oz2_col_shift(const double *B, int64_t ldb, int opB, int64_t k, int64_t n,
                       int beta, int32_t *shift)
{
    for (int64_t j = 0; j < n; ++j) {
        int32_t e = opB ? orc_oz2_norm_exponent(B + j, ldb, k)
                        : orc_oz2_norm_exponent(B + j * ldb, 1, k);
        shift[j] = e == INT32_MIN ? 0 : beta - e;
    }
}

/* integer image a' = rint(a * 2^shift), exact in FP64 */
static int64_t int_image(double a, int32_t shift)
{
    return (int64_t)rint(ldexp(a, shift));
}

/* residues of op(A): res[(l*m + i)*k + h] = sym(a'_ih mod m_l), K-major */
void orc_oz2_split_rows(const double *A, int64_t lda, int opA, int64_t m, int64_t k,
                        const int32_t *shift, int L, int8_t *res)
{
    int32_t mod[ORC_MAX_MODULI];
    orc_oz2_moduli(L, mod);
    for (int64_t i = 0; i < m; ++i)
        for (int64_t h = 0; h < k; ++h) {
            int64_t a = int_image(opel(A, lda, opA, i, h), shift[i]);
            for (int l = 0; l < L; ++l)
                res[((int64_t)l * m + i) * k + h] = (int8_t)sym_mod64(a, mod[l]);
        }
}

/* residues of op(B) (k x n): res[(l*n + j)*k + h], K-major */
void orc_oz2_split_cols(const double *B, int64_t ldb, int opB, int64_t k, int64_t n,
                        const int32_t *shift, int L, int8_t *res)
{
    int32_t mod[ORC_MAX_MODULI];
    orc_oz2_moduli(L, mod);
    for (int64_t j = 0; j < n; ++j)
        for (int64_t h = 0; h < k; ++h) {
            int64_t b = int_image(opel(B, ldb, opB, h, j), shift[j]);
            for (int l = 0; l < L; ++l)
                res[((int64_t)l * n + j) * k + h] = (int8_t)sym_mod64(b, mod[l]);
        }
}

/* exact int8 GEMM: C[i + j*m] = sum_h A[i*k+h] * B[j*k+h] (both K-major) */
void orc_int8_gemm(const int8_t *A, const int8_t *B, int64_t m, int64_t n, int64_t k,
                   int32_t *C)
{
    for (int64_t j = 0; j < n; ++j)
        for (int64_t i = 0; i < m; ++i) {
            int64_t s = 0;
            const int8_t *a = A + i * k, *b = B + j * k;
            for (int64_t h = 0; h < k; ++h) s += (int32_t)a[h] * (int32_t)b[h];
            C[i + j * m] = (int32_t)s;
        }
}

/*
 * Reconstruction from per-modulus int32 products P[l][i + j*m].
 * mode 0 (exact): C' = CRT(residues) as a signed 128-bit integer,
 *   out = fma(alpha, ldexp((double)C', -(sa_i+sb_j)), beta*c).
 * mode 1 (fixed-point, the GPU's formula): S = sum_l sym(P mod m_l) * v_l
 *   (mod 2^64, two's complement), out = fma(alpha,
 *   scalbn((double)S * Mf, -(sa_i+sb_j)), beta*c).
 */
int orc_oz2_reconstruct(const int32_t *P, int64_t m, int64_t n, int L,
                        const int32_t *sa, const int32_t *sb, double alpha,
                        double beta, double *C, int64_t ldc, int mode)
{
    int32_t mod[ORC_MAX_MODULI];
    int64_t y[ORC_MAX_MODULI];
    uint64_t v[ORC_MAX_MODULI], Mhi, Mlo;
    double Mf, lg;
    if (orc_oz2_constants(L, mod, y, v, &Mf, &lg, &Mhi, &Mlo)) return -1;
    unsigned __int128 M = ((unsigned __int128)Mhi << 64) | Mlo;
    const int64_t mn = m * n;
    for (int64_t j = 0; j < n; ++j)
        for (int64_t i = 0; i < m; ++i) {
            const int64_t e = i + j * m;
            double prod;
            if (mode == 0) {
                unsigned __int128 acc = 0;
                for (int l = 0; l < L; ++l) {
                    int64_t r = sym_mod64(P[(int64_t)l * mn + e], mod[l]);
                    int64_t t = ((r % mod[l]) * y[l]) % mod[l];
                    if (t < 0) t += mod[l];
                    unsigned __int128 w = M / (unsigned __int128)mod[l];
                    acc = (acc + w * (unsigned __int128)t) % M;
                }
                double cd;
                if (acc > M / 2) cd = -(double)(M - acc);
                else cd = (double)acc;
                prod = ldexp(cd, -(sa[i] + sb[j]));
            } else {
                uint64_t S = 0;
                for (int l = 0; l < L; ++l) {
                    int64_t r = sym_mod64(P[(int64_t)l * mn + e], mod[l]);
                    S += (uint64_t)r * v[l];
                }
                prod = scalbn((double)(int64_t)S * Mf, -(sa[i] + sb[j]));
            }
            double *c = C + i + j * ldc;
            *c = fma(alpha, prod, beta * *c);
        }
    return 0;
}

/* whole emulated GEMM, C (m x n, ldc) = alpha * op(A) op(B) + beta * C */
int orc_oz2_gemm(int opA, int opB, int64_t m, int64_t n, int64_t k, double alpha,
                 const double *A, int64_t lda, const double *B, int64_t ldb,
                 double beta, double *C, int64_t ldc, int L, int mode)
{
    int al, be;
    if (orc_oz2_shift_bits(L, k, &al, &be)) return -1;
    int32_t *sa = malloc(sizeof(int32_t) * (size_t)m);
    int32_t *sb = malloc(sizeof(int32_t) * (size_t)n);
    int8_t *ra = malloc((size_t)L * m * k), *rb = malloc((size_t)L * n * k);
    int32_t *P = malloc(sizeof(int32_t) * (size_t)L * m * n);
    int rc = -2;
    if (sa && sb && ra && rb && P) {
        orc_oz2_row_shift(A, lda, opA, m, k, al, sa);
        orc_oz2_col_shift(B, ldb, opB, k, n, be, sb);
        orc_oz2_split_rows(A, lda, opA, m, k, sa, L, ra);
        orc_oz2_split_cols(B, ldb, opB, k, n, sb, L, rb);
        for (int l = 0; l < L; ++l)
            orc_int8_gemm(ra + (size_t)l * m * k, rb + (size_t)l * n * k, m, n, k,
                          P + (size_t)l * m * n);
        rc = orc_oz2_reconstruct(P, m, n, L, sa, sb, alpha, beta, C, ldc, mode);
    }
    free(sa); free(sb); free(ra); free(rb); free(P);
    return rc;
}

/* ------------------------------------------------------------------ */
/* LU / laswp / residual                                               */
/* ------------------------------------------------------------------ */
/* LAPACK dlaswp: for i = k1..k2-1: swap rows i and ipiv[i] in columns [c0,c1) */
void orc_laswp(double *A, int64_t lda, int64_t c0, int64_t c1, int64_t k1, int64_t k2,
               const int64_t *ipiv)
{
    for (int64_t i = k1; i < k2; ++i) {
        int64_t p = ipiv[i];
        if (p == i) continue;
        for (int64_t c = c0; c < c1; ++c) {
            double t = A[i + c * lda];
            A[i + c * lda] = A[p + c * lda];
            A[p + c * lda] = t;
        }
    }
}

/*
 * Right-looking LU with partial pivoting of the leading N x N part of an
 * N x (N+1) system (b in column N), blocked by NB; the trailing update of
 * each block column is exact FP64 (L=0) or the Ozaki-II emulation with L
 * moduli.  ipiv is 0-based and absolute.  Then U x = b' by back
 * substitution; x overwrites column N.  Returns 0 or the 1-based index of a
 * zero pivot.
 */
int orc_hpl_solve(double *A, int64_t lda, int64_t N, int64_t NB, int L, int64_t *ipiv)
{
    const int64_t nc = N + 1;
    for (int64_t J = 0; J < N; J += NB) {
        const int64_t jb = (NB < N - J) ? NB : N - J;
        for (int64_t j = J; j < J + jb; ++j) {
            int64_t p = j;
            double mx = fabs(A[j + j * lda]);
            for (int64_t i = j + 1; i < N; ++i)
                if (fabs(A[i + j * lda]) > mx) { mx = fabs(A[i + j * lda]); p = i; }
            ipiv[j] = p;
            if (A[p + j * lda] == 0.0) return (int)(j + 1);
            if (p != j)
                for (int64_t c = J; c < J + jb; ++c) {
                    double t = A[j + c * lda]; A[j + c * lda] = A[p + c * lda]; A[p + c * lda] = t;
                }
            const double inv = 1.0 / A[j + j * lda];
            for (int64_t i = j + 1; i < N; ++i) A[i + j * lda] *= inv;
            for (int64_t c = j + 1; c < J + jb; ++c) {
                const double u = A[j + c * lda];
                for (int64_t i = j + 1; i < N; ++i) A[i + c * lda] -= A[i + j * lda] * u;
            }
        }
        /* apply this block's interchanges to every column right of it */
        orc_laswp(A, lda, J + jb, nc, J, J + jb, ipiv);
        /* U12 = L11^-1 A12 */
        for (int64_t c = J + jb; c < nc; ++c)
            for (int64_t j = J; j < J + jb; ++j) {
                const double u = A[j + c * lda];
                for (int64_t i = j + 1; i < J + jb; ++i) A[i + c * lda] -= A[i + j * lda] * u;
            }
        const int64_t mt = N - (J + jb), nt = nc - (J + jb);
        if (mt > 0 && nt > 0) {
            double *L21 = A + (J + jb) + J * lda, *U12 = A + J + (J + jb) * lda;
            double *A22 = A + (J + jb) + (J + jb) * lda;
            if (L > 0) {
                if (orc_oz2_gemm(0, 0, mt, nt, jb, -1.0, L21, lda, U12, lda, 1.0, A22, lda, L, 1))
                    return -1;
            } else {
                for (int64_t c = 0; c < nt; ++c)
                    for (int64_t h = 0; h < jb; ++h) {
                        const double u = U12[h + c * lda];
                        for (int64_t i = 0; i < mt; ++i) A22[i + c * lda] -= L21[i + h * lda] * u;
                    }
            }
        }
    }
    for (int64_t i = N - 1; i >= 0; --i) {
        double s = A[i + N * lda];
        for (int64_t c = i + 1; c < N; ++c) s -= A[i + c * lda] * A[c + N * lda];
        A[i + N * lda] = s / A[i + i * lda];
    }
    return 0;
}

/* The scaled residual from per-row data, the reduction and formula of
 * src/chpl_single.cu:790-801 (also src/chpl_p2.cu:1925-1932): y = A x,
 * rs = row sums of |A|, b, x (all N long); eps = 2^-53. */
double orc_hpl_residual_parts(const double *y, const double *rs, const double *b, const double *x, int64_t N)
{
    double rmax = 0.0, anorm = 0.0, xnorm = 0.0, bnorm = 0.0;
    for (int64_t i = 0; i < N; ++i) {
        const double r = fabs(y[i] - b[i]);
        if (r > rmax) rmax = r;
        if (rs[i] > anorm) anorm = rs[i];
        if (fabs(x[i]) > xnorm) xnorm = fabs(x[i]);
        if (fabs(b[i]) > bnorm) bnorm = fabs(b[i]);
    }
    const double eps = ldexp(1.0, -53);
    return rmax / (eps * (anorm * xnorm + bnorm) * (double)N);
}

/* scaled residual of x against the regenerated system (A N x (N+1), b = col N) */
double orc_hpl_residual(const double *A, int64_t lda, int64_t N, const double *x)
{
    double *y = (double *)malloc((size_t)N * sizeof(double));
    double *rs = (double *)malloc((size_t)N * sizeof(double));
    if (!y || !rs) { free(y); free(rs); return NAN; }
    for (int64_t i = 0; i < N; ++i) {
        double ax = 0.0, s = 0.0;
        for (int64_t c = 0; c < N; ++c) { ax += A[i + c * lda] * x[c]; s += fabs(A[i + c * lda]); }
        y[i] = ax;
        rs[i] = s;
    }
    const double r = orc_hpl_residual_parts(y, rs, A + N * lda, x, N);
    free(y);
    free(rs);
    return r;
}
