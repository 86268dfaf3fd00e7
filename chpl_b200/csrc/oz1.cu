// Ozaki scheme I emulated DGEMM on B200 (the reference's alternative engine,
// HPLS_BACKEND=ozaki: src/chpl_single.cu:147-236 kernels, 532-612 driver):
//
//   1. power-of-two scales: row i of A by 2^-ea_i, column j of B by 2^-eb_j,
//      ea_i = ilogb(max_h |A(i,h)|) + 1, so every scaled entry lies in (-1, 1);
//   2. each scaled entry x is cut into kOz1Slices base-128 digits
//      t_p = rint(128 x_p) (clamped to 127), x_{p+1} = 128 x_p - t_p, so that
//      x = sum_p t_p 128^-(p+1) up to the last remainder;
//   3. anti-diagonal d of the digit products, sum_{p+q=d} A_p B_q, for
//      d < kOz1Slices, as one exact int8 x int8 -> int32 product per diagonal
//      on the tcgen05 kernel of oz2.cu (raw epilogue): A's digits are stored
//      once per row as [A_0 | A_1 | ... | A_5] along K, and B's plane d per
//      column as [B_d | B_(d-1) | ... | B_0 | 0 ...], so plane d of the
//      product pairs exactly the digits whose indices add up to d, and its
//      K loop stops after the (d + 1) k non-zero bytes;
//   4. C = alpha * 2^(ea_i + eb_j) * sum_d P_d 128^-(d+2) + beta * C, the sum
//      taken in order d = 0, 1, ... .
// The digits and the truncation are the reference's; the storage, the one
// GEMM launch for all diagonals and the kernels are this library's.  It is a
// comparison engine (slower than Ozaki-II, as in the reference): the launch
// runs 21 digit products' worth of K blocks (1 + 2 + ... + 6 of k each), the
// method's own count, against 11 modulus products of Ozaki-II.
#include <algorithm>

#include "common.cuh"
#include "oz1.h"
#include "oz2.h"

namespace chpl {
namespace oz1 {

namespace {

// exponent of one row of A (column-major m x k): thread per row, coalesced over rows
__global__ void row_exp_kernel(const double* __restrict__ A, long long lda, int m, int k, int* __restrict__ e)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    double mx = 0.0;
    for (int h = 0; h < k; ++h) mx = fmax(mx, fabs(A[i + (long long)h * lda]));
    e[i] = mx > 0.0 ? ilogb(mx) + 1 : 0;
}

// exponent of one column of B (column-major k x n): warp per column
__global__ void col_exp_kernel(const double* __restrict__ B, long long ldb, int k, int n, int* __restrict__ e)
{
    const int lane = threadIdx.x & 31;
    const int j = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (j >= n) return;
    double mx = 0.0;
    for (int h = lane; h < k; h += 32) mx = fmax(mx, fabs(B[h + (long long)j * ldb]));
    for (int o = 16; o; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) e[j] = mx > 0.0 ? ilogb(mx) + 1 : 0;
}

__device__ __forceinline__ void digits(double x, int8_t (&t)[kOz1Slices])
{
#pragma unroll
    for (int p = 0; p < kOz1Slices; ++p) {
        double a = rint(x * 128.0);
        if (a > 127.0) a = 127.0;
        x = x * 128.0 - a;
        t[p] = (int8_t)a;
    }
}

// digits of A: res[i * ldk + p*k + h] = digit p of A(i,h) 2^-e_i, rows i < mpad
// (zero beyond m), K positions up to ldk (zero beyond kOz1Slices * k).  Tiles
// of 32 rows x 32 columns through shared memory: loads walk down columns,
// stores along the K-major rows.
__global__ void __launch_bounds__(256) slice_a_kernel(const double* __restrict__ A, long long lda, int m, int k,
                                                      int mpad, int ldk, const int* __restrict__ e,
                                                      int8_t* __restrict__ res)
{
    __shared__ double t[32][33];
    const int i0 = blockIdx.x * 32, h0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 8 rows of 32 threads
    for (int hh = ty; hh < 32; hh += 8) {
        const int i = i0 + tx, h = h0 + hh;
        t[hh][tx] = (i < m && h < k) ? scalbn(A[i + (long long)h * lda], -e[i]) : 0.0;
    }
    __syncthreads();
    for (int ii = ty; ii < 32; ii += 8) {
        const int i = i0 + ii, h = h0 + tx;
        if (i >= mpad || h >= k) continue;
        int8_t d[kOz1Slices];
        digits(t[tx][ii], d);
        int8_t* row = res + (size_t)i * ldk;
#pragma unroll
        for (int p = 0; p < kOz1Slices; ++p) row[(size_t)p * k + h] = d[p];
    }
}

// zero tail of every row: K positions [kOz1Slices * k, ldk)
__global__ void zero_tail_kernel(int8_t* __restrict__ res, int rows, int ldk, int from)
{
    const int r = blockIdx.x;
    if (r >= rows) return;
    for (int h = from + threadIdx.x; h < ldk; h += blockDim.x) res[(size_t)r * ldk + h] = 0;
}

// B's planes: res[(d * npad + j) * ldk + s*k + h] = digit (d - s) of B(h,j) 2^-e_j
// for s <= d, zero for s > d; columns j < npad (zero beyond n)
__global__ void __launch_bounds__(256) slice_b_kernel(const double* __restrict__ B, long long ldb, int k, int n,
                                                      int npad, int ldk, const int* __restrict__ e,
                                                      int8_t* __restrict__ res)
{
    const int j = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= k) return;
    int8_t d[kOz1Slices];
    digits(j < n ? scalbn(B[h + (long long)j * ldb], -e[j]) : 0.0, d);
#pragma unroll
    for (int pl = 0; pl < kOz1Slices; ++pl) {
        int8_t* col = res + ((size_t)pl * npad + j) * ldk + h;
#pragma unroll
        for (int s = 0; s < kOz1Slices; ++s) col[(size_t)s * k] = s <= pl ? d[pl - s] : (int8_t)0;
    }
}

// C = alpha * 2^(ea_i + eb_j) * sum_d P_d 128^-(d+2) + beta * C (beta == 0 never reads C)
__global__ void recon_kernel(double* __restrict__ C, long long ldc, int m, int n, const int32_t* __restrict__ P,
                             long long ldp, const int* __restrict__ ea, const int* __restrict__ eb, double alpha,
                             double beta)
{
    const long long total = (long long)m * n;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e % m), j = (int)(e / m);
        double acc = 0.0, w = 0x1p-14;   // 128^-2
#pragma unroll
        for (int d = 0; d < kOz1Slices; ++d) {
            acc += (double)P[(size_t)d * ldp * n + i + (size_t)j * ldp] * w;
            w *= 0x1p-7;
        }
        const double v = scalbn(acc, ea[i] + eb[j]);
        double* c = C + i + (long long)j * ldc;
        *c = beta == 0.0 ? alpha * v : fma(alpha, v, beta * *c);
    }
}

}  // namespace

Layout layout(size_t m, size_t n, size_t k)
{
    Layout y;
    y.mPad = round_up(std::max<size_t>(m, 1), 128);
    y.nPad = round_up(std::max<size_t>(n, 1), 256);
    y.ldk = round_up((size_t)kOz1Slices * std::max<size_t>(k, 1), 128);
    size_t off = 0;
    y.a_res = off;
    off += round_up(y.mPad * y.ldk, 256);
    y.b_res = off;
    off += round_up((size_t)kOz1Slices * y.nPad * y.ldk, 256);
    y.ea = off;
    off += round_up(y.mPad * 4, 256);
    y.eb = off;
    off += round_up(y.nPad * 4, 256);
    y.p = off;
    off += round_up((size_t)kOz1Slices * m * n * 4, 256);
    y.total = off;
    return y;
}

int gemm(cudaStream_t st, size_t m, size_t n, size_t k, double alpha, const double* A, size_t lda, const double* B,
         size_t ldb, double beta, double* C, size_t ldc, void* work)
{
    if (m == 0 || n == 0) return CHPL_OK;
    if (k == 0 || alpha == 0.0) return oz2::scale(st, C, ldc, m, n, beta);
    if ((size_t)kOz1Slices * k > (size_t)oz2::kMaxK) {
        set_error("ozaki-I: k = %zu exceeds %d (int32 accumulation of %d digit products)", k,
                  oz2::kMaxK / kOz1Slices, kOz1Slices);
        return CHPL_ERR_UNSUPPORTED;
    }
    if (m > 0x7fffffffull || n > 0x7fffffffull) { set_error("ozaki-I: m, n must fit in int32"); return CHPL_ERR_UNSUPPORTED; }
    if (!work) { set_error("ozaki-I: work is NULL"); return CHPL_ERR_WORKSPACE; }
    const Layout y = layout(m, n, k);
    if (y.nPad > 65535) { set_error("ozaki-I: n = %zu exceeds 65280 columns per call", n); return CHPL_ERR_UNSUPPORTED; }
    uint8_t* w = static_cast<uint8_t*>(work);
    int8_t* ra = reinterpret_cast<int8_t*>(w + y.a_res);
    int8_t* rb = reinterpret_cast<int8_t*>(w + y.b_res);
    int* ea = reinterpret_cast<int*>(w + y.ea);
    int* eb = reinterpret_cast<int*>(w + y.eb);
    int32_t* P = reinterpret_cast<int32_t*>(w + y.p);
    const int mi = (int)m, ni = (int)n, ki = (int)k;
    row_exp_kernel<<<(unsigned)((m + 255) / 256), 256, 0, st>>>(A, (long long)lda, mi, ki, ea);
    col_exp_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(B, (long long)ldb, ki, ni, eb);
    slice_a_kernel<<<dim3((unsigned)(y.mPad / 32), (unsigned)((k + 31) / 32)), 256, 0, st>>>(
        A, (long long)lda, mi, ki, (int)y.mPad, (int)y.ldk, ea, ra);
    zero_tail_kernel<<<(unsigned)y.mPad, 128, 0, st>>>(ra, (int)y.mPad, (int)y.ldk, kOz1Slices * ki);
    slice_b_kernel<<<dim3((unsigned)((k + 255) / 256), (unsigned)y.nPad), 256, 0, st>>>(
        B, (long long)ldb, ki, ni, (int)y.nPad, (int)y.ldk, eb, rb);
    zero_tail_kernel<<<(unsigned)(kOz1Slices * y.nPad), 128, 0, st>>>(rb, (int)(kOz1Slices * y.nPad), (int)y.ldk,
                                                                      kOz1Slices * ki);
    CHPL_CUDA(cudaGetLastError());
    // one raw launch: plane d = diagonal d; A's plane stride 0 (every plane reads the same digit
    // rows), and plane d stops after its (d + 1) k non-zero bytes of K
    CHPL_TRY(oz2::gemm_launch(st, 1, m, n, y.ldk, (unsigned)kOz1Slices, ra, y.mPad, rb, y.nPad, nullptr, nullptr, 0.0,
                              0.0, nullptr, 0, P, m, nullptr, oz2::num_sms(), 0, (long long)k));
    const long long tot = (long long)m * n;
    const unsigned g = (unsigned)std::min<long long>((tot + 255) / 256, 148LL * 32);
    recon_kernel<<<g, 256, 0, st>>>(C, (long long)ldc, mi, ni, P, (long long)m, ea, eb, alpha, beta);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

int launches() { return 8; }

}  // namespace oz1
}  // namespace chpl

using namespace chpl;

extern "C" int chpl_oz1_worksize(size_t m, size_t n, size_t k, size_t* work_bytes)
{
    if (!work_bytes) { set_error("work_bytes is NULL"); return CHPL_ERR_INVALID; }
    if ((size_t)oz1::kOz1Slices * k > (size_t)oz2::kMaxK) { set_error("ozaki-I: k too large"); return CHPL_ERR_UNSUPPORTED; }
    *work_bytes = oz1::layout(m, n, k).total;
    return CHPL_OK;
}

extern "C" int chpl_oz1_gemm(void* stream, size_t m, size_t n, size_t k, double alpha, const double* A, size_t lda,
                             const double* B, size_t ldb, double beta, double* C, size_t ldc, void* work)
{
    if (ldc < m || lda < m || ldb < k) { set_error("ozaki-I: leading dimension too small"); return CHPL_ERR_INVALID; }
    if (m && n && (!C || (k && alpha != 0.0 && (!A || !B)))) { set_error("ozaki-I: NULL matrix"); return CHPL_ERR_INVALID; }
    return oz1::gemm((cudaStream_t)stream, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, work);
}
