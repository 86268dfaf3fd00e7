// Internal interface of the Ozaki scheme I module (oz1.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace chpl {
namespace oz1 {

constexpr int kOz1Slices = 6;   // base-128 digits per entry, anti-diagonals kept (src/chpl_single.cu OZ_S)

// workspace layout (byte offsets): A digits mPad x ldk, B planes kOz1Slices x nPad x ldk,
// exponents, the kOz1Slices int32 diagonal products (m x n each)
struct Layout {
    size_t mPad, nPad, ldk;
    size_t a_res, b_res, ea, eb, p, total;
};

Layout layout(size_t m, size_t n, size_t k);
// C = alpha A B + beta C (column-major, no transposes); C may alias B when beta == 0
int gemm(cudaStream_t st, size_t m, size_t n, size_t k, double alpha, const double* A, size_t lda, const double* B,
         size_t ldb, double beta, double* C, size_t ldc, void* work);
int launches();

}  // namespace oz1
}  // namespace chpl
