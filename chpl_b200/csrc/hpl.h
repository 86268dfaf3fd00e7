// Internal interface of the HPL module (kernels in hpl_kernels.cu, panel in
// panel.cu, driver in hpl_single.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace chpl {

// rows (or columns) of an n-long dimension owned by process coordinate p of P
// under block-cyclic distribution with block nb (block i lives on i % P).
static inline int64_t local_extent(int64_t n, int64_t nb, int P, int p)
{
    const int64_t nblk = n / nb, rem = n % nb;
    int64_t ext = (nblk / P + (p < nblk % P ? 1 : 0)) * nb;
    if (rem && nblk % P == p) ext += rem;
    return ext;
}

// generator: CHPL_GEN_CHPL (SplitMix64 hash of chpl_p2) or CHPL_GEN_PHILOX (cuRAND Philox of chpl_single)
int matgen(cudaStream_t st, double* A, size_t lda, size_t m, size_t n, int64_t row0, int64_t col0, int64_t ncg,
           uint64_t seed, int generator = 0);
size_t laswp_work_bytes(int64_t nswaps);
// plan the swaps (i <-> ipiv[i] - pbase), i = k1..k2-1, into `work`
int laswp_plan(cudaStream_t st, const int64_t* ipiv, int64_t k1, int64_t k2, void* work, int64_t pbase = 0);
int laswp_apply(cudaStream_t st, double* A, size_t lda, int64_t c0, int64_t ncols, int64_t nswaps, const void* work);
int ipiv_to_abs(cudaStream_t st, const int64_t* rel, int64_t n, int64_t base, int64_t* out);
int identity(cudaStream_t st, double* X, int64_t n);
int residual(cudaStream_t st, int64_t N, uint64_t seed, const double* x, double* resid, int generator = 0);
// the same residual for [A | b] held in device memory (column N is b)
int residual_matrix(cudaStream_t st, int64_t N, const double* Ab, size_t ld, const double* x, double* resid);
int hpl_read_clear_status(int* st);
size_t panel_work_bytes(int64_t m, int64_t n);
// FP64 getrf of the m x n panel at A; ipiv[i] = base_row + pivot row within the panel.
// max_ctas > 0 bounds the base kernel's cooperative grid (the SMs a concurrent
// bulk update leaves free); 0 = one CTA per SM
int panel_getrf(cudaStream_t st, int64_t m, int64_t n, double* A, size_t lda, int64_t* ipiv, int64_t base_row, int* info,
                void* work, int max_ctas = 0);
// the fewest base-kernel CTAs that hold an m-row panel on chip (narrowest base block)
int panel_min_ctas(int64_t m);
int panel_status(void* work, int* err);

}  // namespace chpl
