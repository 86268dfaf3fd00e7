// Harness around host-computable fragments of the reference -- TEST
// INFRASTRUCTURE ONLY.  oracle/ref_build.py extracts the fragments verbatim
// from the reference checkout into oracle/_ref/ (never committed) and
// compiles this file against them into oracle/_ref/libref_host.so, so that
// the tests can check the CPU oracle and this project's host code against the
// reference's own code:
//   chpl_elem    (src/chpl_p2.cu)      generator element of chpl_p2 / chpl_p4
//   resolve_seq  (src/chpl_p2.cu)      net permutation of a pivot sequence
//   residual     (src/chpl_single.cu)  scaled-residual reduction of run_case
#include <cmath>
#include <cstdint>
#include <cstring>
#include <utility>
#include <vector>

// the generator is a __device__ function in the reference; on the host the
// qualifiers are dropped
#define __device__
#define __forceinline__ inline
typedef unsigned long long u64;

#include "chpl_elem.inc"
#include "resolve_seq.inc"

extern "C" {

double ref_chpl_elem(u64 seed, u64 idx) { return chpl_elem(seed, idx); }

// A[i + j*lda] = chpl_elem(seed, (row0+i)*ncg + col0+j): the element indexing
// of matgen2d_kernel (src/chpl_p2.cu) for a contiguous block of rows
void ref_matgen(double* A, int64_t lda, int64_t m, int64_t n, int64_t row0, int64_t col0, int64_t ncg, u64 seed)
{
    for (int64_t j = 0; j < n; ++j)
        for (int64_t i = 0; i < m; ++i)
            A[i + j * lda] = chpl_elem(seed, (u64)(row0 + i) * (u64)ncg + (u64)(col0 + j));
}

// resolve_seq(piv[0..n), base): top[i] = original row whose content ends at
// row base+i; below = (row >= base+n, original row) pairs, *nbelow of them
// (arrays of at least n entries).
void ref_resolve_seq(const long long* piv, long long base, int n, long long* top, long long* below_pos,
                     long long* below_src, int* nbelow)
{
    std::vector<long long> p(piv, piv + n), t;
    std::vector<std::pair<long long, long long>> b;
    resolve_seq(p, base, n, t, b);
    for (int i = 0; i < n; ++i) top[i] = t[i];
    *nbelow = (int)b.size();
    for (size_t i = 0; i < b.size(); ++i) {
        below_pos[i] = b[i].first;
        below_src[i] = b[i].second;
    }
}

// The reference's residual reduction on given per-row data: y = A x (its
// cuBLAS dgemv), rs = row sums of |A|, b, x (all N long); returns resid1.
double ref_residual(const double* y, const double* rs, const double* b, const double* x, int64_t N)
{
    std::vector<double> h_y(y, y + N), h_rs(rs, rs + N), h_b(b, b + N), h_x(x, x + N);
#include "residual.inc"
    return resid1;
}

}  // extern "C"
