// Harness around chpl_single's Ozaki-I kernels -- TEST INFRASTRUCTURE ONLY.
// oracle/ref_build.py extracts ozrowscale_kernel .. ozrecon_kernel verbatim
// from the reference (src/chpl_single.cu) into oracle/_ref/single_oz1.inc
// (never committed) and compiles this file into oracle/_ref/libref_oz1.so for
// sm_100a.  The GPU tests run the reference's scales, digit slices and
// reconstruction around exact host products of the digits and compare the
// result with this project's Ozaki-I engine, bit for bit.  Launch shapes are
// the reference driver's (src/chpl_single.cu:535-601).
#include <cstddef>
#include <cuda_runtime.h>

#include "single_oz1.inc"

// scales of A's rows and B's columns, then the digits: SA row i = [t_0 | .. | t_{s-1}]
// (k each), SB column j = [t_{s-1} | .. | t_0] (k each, ldS = s k)
extern "C" int ref_oz1_prepare(const double* A, size_t lda, int m, int k, const double* B, size_t ldb, int n, int s,
                               double* rinv, double* rsc, double* cinv, double* csc, signed char* SA, signed char* SB)
{
    ozrowscale_kernel<<<(unsigned)((m + 255) / 256), 256>>>(A, lda, m, k, rinv, rsc);
    dim3 blk(32, 8), grd((unsigned)((m + 31) / 32), (unsigned)((k + 31) / 32));
    ozsliceA_kernel<<<grd, blk>>>(A, lda, m, k, rinv, SA, s);
    ozcolscale_kernel<<<(unsigned)((n + 255) / 256), 256>>>(B, ldb, k, n, cinv, csc);
    dim3 gg(8, (unsigned)n);
    ozsliceB_kernel<<<gg, 256>>>(B, ldb, k, n, cinv, SB, s, (size_t)s * k);
    return (int)cudaDeviceSynchronize();
}

// C -= rsc csc sum_d D_d 128^-(d+2) with the diagonal products D_d (m x n, ld m)
extern "C" int ref_oz1_recon(double* C, size_t ldc, int m, int n, const int* D0, const int* D1, const int* D2,
                             const int* D3, const int* D4, const int* D5, int ndiag, const double* rsc,
                             const double* csc)
{
    dim3 blk(64, 4), grd((unsigned)((m + 63) / 64), (unsigned)((n + 3) / 4));
    ozrecon_kernel<<<grd, blk>>>(C, ldc, m, n, D0, D1, D2, D3, D4, D5, ndiag, rsc, csc);
    return (int)cudaDeviceSynchronize();
}
