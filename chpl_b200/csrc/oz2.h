// Internal interface of the Ozaki-II module (oz2.cu), shared with the HPL driver.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace chpl {
namespace oz2 {

constexpr int kMaxModuli = 16;
constexpr int kMaxK = 131071;  // k * 128 * 128 < 2^31: int32 accumulation cannot overflow

// moduli table and CRT constants for one modulus count (passed to kernels by value)
struct Moduli {
    int L;
    int alpha, beta;                  // scaling exponents of op(A) rows / op(B) columns
    int mod[kMaxModuli];              // pairwise-coprime moduli, greedy from 256 down
    int hi[kMaxModuli];               // symmetric residue range [hi - m + 1, hi]
    float inv_f[kMaxModuli];
    double mod_d[kMaxModuli];
    double inv_d[kMaxModuli];
    unsigned long long v[kMaxModuli]; // round(2^64 y_l / m_l), y_l = (M/m_l)^-1 mod m_l
    double Mf;                        // M / 2^64
};

// workspace layout of chpl_oz2_gemm (byte offsets)
struct Layout {
    size_t mPad, nPad, kPad;
    size_t a_shift, a_res, a_bytes;   // inside the A part
    size_t b_shift, b_res, b_bytes;   // inside the B part
    size_t a_off, b_off;              // A / B part offsets inside `work` (when not external)
    size_t scratch_off, tmp_off, total;
    int grid_max;
};

const Moduli* moduli(int L);
int num_sms();
// grid_cap > 0 limits the persistent GEMM grid (and so the CRT scratch) to grid_cap CTAs
Layout layout(size_t m, size_t n, size_t k, int L, bool extA, bool extB, int grid_cap = 0);
size_t split_tmp_bytes(size_t nvec);
int split(cudaStream_t st, bool contiguous, const double* x, size_t ld, size_t nvec, size_t k, unsigned L, int bits,
          int8_t* res, size_t ldvec, size_t ldk, int32_t* shift, void* tmp);
int gemm_launch(cudaStream_t st, int mode, size_t m, size_t n, size_t kPad, unsigned L, const int8_t* ra, size_t rowsA,
                const int8_t* rb, size_t rowsB, const int32_t* shiftA, const int32_t* shiftB, double alpha,
                double beta, double* C, size_t ldc, int32_t* P, size_t ldp, int8_t* scratch, int grid_max,
                long long planeA = -1,    // A's plane stride in rows: -1 = rowsA; 0 = every plane reads the same rows
                long long kstep = 0);     // > 0: plane l multiplies only its first (l + 1) * kstep bytes of K
int scale(cudaStream_t st, double* C, size_t ldc, size_t m, size_t n, double beta);
int read_clear_status(int* st);

}  // namespace oz2
}  // namespace chpl
