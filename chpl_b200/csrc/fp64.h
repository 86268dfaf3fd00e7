// Internal interface of the FP64 kernels (fp64.cu): column-major, device
// pointers, asynchronous on the given stream, CHPL_* status codes.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace chpl {

// C (m x n) = alpha * A (m x k) * B (k x n) + beta * C; beta == 0 never reads C
int dgemm(cudaStream_t st, int64_t m, int64_t n, int64_t k, double alpha, const double* A, int64_t lda,
          const double* B, int64_t ldb, double beta, double* C, int64_t ldc);
// B (n x nrhs) = L^-1 B, L unit lower triangular (n x n; its upper part is not read)
int dtrsm_llnu(cudaStream_t st, int64_t n, int64_t nrhs, const double* L, int64_t ldl, double* B, int64_t ldb);
// X (n x n) = L^-1 for L unit lower triangular (X's upper part set to zero); it issues
// 1 + dtrtri_launches(n) kernels (X = I first)
int dtrtri_llnu(cudaStream_t st, int64_t n, const double* L, int64_t ldl, double* X, int64_t ldx);
int64_t dtrtri_launches(int64_t n);
// x = U^-1 x, U upper triangular with its diagonal (n x n); work: n doubles of device scratch
int dtrsv_unn(cudaStream_t st, int64_t n, const double* U, int64_t ldu, double* x, double* work);
// kernels dtrsv_unn launches for order n
int64_t dtrsv_launches(int64_t n);
// kernels dtrsm_llnu launches for order n (one leaf per 64 rows, one GEMM per split)
int64_t dtrsm_launches(int64_t n);
// y (m) = alpha * A (m x n) * x (n) + beta * y; beta == 0 never reads y
int dgemv_n(cudaStream_t st, int64_t m, int64_t n, double alpha, const double* A, int64_t lda, const double* x,
            double beta, double* y);

}  // namespace chpl
