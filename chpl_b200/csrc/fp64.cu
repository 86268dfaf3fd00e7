// FP64 BLAS kernels of this library (sm_100a): the matrix products,
// triangular solves and matrix-vector products of the FP64 side of the solve.
//
// They replace the cuBLAS / cuSOLVER calls of the reference's hot path:
//   dgemm      cublasDgemm  (src/chpl_single.cu:621-623 native update,
//              694-696 inner panel update; src/chpl_p2.cu:1377-1381,
//              1669-1673, 1697-1700)
//   dtrsm      cublasDtrsm  (src/chpl_single.cu:689-691, 708-710;
//              src/chpl_p2.cu:1211-1220 -- inv(L11) against the identity)
//   dtrsv      cublasDtrsv  (src/chpl_single.cu:724-725 back solve,
//              src/chpl_p2.cu:1851)
//   dgemv      cublasDgemv  (src/chpl_p2.cu:1870)
//
// DGEMM runs on B200's FP64 tensor path: mma.sync m16n8k8 .f64 (DMMA) tiles
// fed from a 4-stage cp.async ring in shared memory.  Operand tiles are padded
// so that every fragment load is two bank-conflict-free wavefronts: the A tile
// is stored k-major with a pitch of BM + 8 doubles (the four k rows a warp
// reads land on alternating 64-byte halves of the banks), the B tile n-major
// with a pitch of 20 doubles (eight n columns on four 32-byte bank groups).
// Out-of-range rows / columns / k are zero-filled by the copies, so any m, n,
// k and any leading dimension work; 16-byte copies are used where the
// operand's base and leading dimension allow them.
//
// Results are deterministic: every reduction runs in a fixed order.
#include <algorithm>

#include "common.cuh"
#include "fp64.h"

namespace chpl {

namespace {

constexpr int kBK = 16;          // k per shared-memory stage (two m16n8k8 steps)
constexpr int kPB = kBK + 4;     // pitch (doubles) of one n column of the B tile
constexpr int kStages = 4;

__device__ __forceinline__ void cp_async(void* smem, const void* gmem, int bytes, int src_bytes)
{
    const uint32_t s = smem_u32(smem);
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// D = A(16x8) B(8x8) + D, FP64 tensor path
__device__ __forceinline__ void dmma(double (&d)[4], const double (&a)[4], const double (&b)[2])
{
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
                 : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}

struct GemmArgs {
    long long m, n, k;
    double alpha, beta;
    const double* A;
    long long lda;
    const double* B;
    long long ldb;
    double* C;
    long long ldc;
    long long sA, sB, sC;   // batch strides (doubles) between the products of a batched launch
    int vecA, vecB;      // 16-byte copies allowed for A / B
};

template <int BM, int BN, int WM, int WN, int MINB>
struct GemmShape {
    static constexpr int kThreads = WM * WN * 32;
    static constexpr int kPA = BM + 8;                  // pitch (doubles) of one k row of the A tile
    static constexpr int kTM = BM / WM / 16;            // m16 tiles per warp
    static constexpr int kTN = BN / WN / 8;             // n8 tiles per warp
    static constexpr int kStageA = kBK * kPA;           // doubles
    static constexpr int kStageB = BN * kPB;
    static constexpr size_t kSmem = (size_t)kStages * (kStageA + kStageB) * sizeof(double);
    static_assert(BM % (WM * 16) == 0 && BN % (WN * 8) == 0, "warp tiling");
};

// C = alpha * A * B + beta * C (column-major; beta == 0 never reads C).
// MINB CTAs per SM: two CTAs of 128 x 64 (8 warps, 32 x 32 each) keep more
// independent barriers in flight than one of 128 x 128 and ran 11 % (square)
// to 31 % (tall, 512 wide) faster on B200.
template <int BM, int BN, int WM, int WN, int MINB>
__global__ void __launch_bounds__(WM * WN * 32, MINB) dgemm_kernel(GemmArgs p)
{
    using S = GemmShape<BM, BN, WM, WN, MINB>;
    extern __shared__ __align__(16) double smem[];
    double* As = smem;                                  // [stage][k][kPA]
    double* Bs = smem + kStages * S::kStageA;           // [stage][n][kPB]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int wm0 = (warp % WM) * (BM / WM), wn0 = (warp / WM) * (BN / WN);
    const long long m0 = (long long)blockIdx.x * BM, n0 = (long long)blockIdx.y * BN;
    const long long ktiles = (p.k + kBK - 1) / kBK;
    const double* Ag = p.A + blockIdx.z * p.sA;   // this CTA's product of a batch
    const double* Bg = p.B + blockIdx.z * p.sB;
    double* Cg = p.C + blockIdx.z * p.sC;

    auto load_tile = [&](int stage, long long kt) {
        const long long k0 = kt * kBK;
        double* as = As + stage * S::kStageA;
        double* bs = Bs + stage * S::kStageB;
        if (p.vecA) {
            for (int e = tid; e < kBK * BM / 2; e += S::kThreads) {
                const int kk = e / (BM / 2), r = (e % (BM / 2)) * 2;
                const long long gr = m0 + r, gk = k0 + kk;
                const long long left = (gk < p.k) ? p.m - gr : 0;
                const int nb = left >= 2 ? 16 : (left == 1 ? 8 : 0);
                cp_async(as + kk * S::kPA + r, nb ? Ag + gr + gk * p.lda : Ag, 16, nb);
            }
        } else {
            for (int e = tid; e < kBK * BM; e += S::kThreads) {
                const int kk = e / BM, r = e % BM;
                const long long gr = m0 + r, gk = k0 + kk;
                const bool ok = gk < p.k && gr < p.m;
                cp_async(as + kk * S::kPA + r, ok ? Ag + gr + gk * p.lda : Ag, 8, ok ? 8 : 0);
            }
        }
        if (p.vecB) {
            for (int e = tid; e < BN * kBK / 2; e += S::kThreads) {
                const int c = e / (kBK / 2), kk = (e % (kBK / 2)) * 2;
                const long long gc = n0 + c, gk = k0 + kk;
                const long long left = (gc < p.n) ? p.k - gk : 0;
                const int nb = left >= 2 ? 16 : (left == 1 ? 8 : 0);
                cp_async(bs + c * kPB + kk, nb ? Bg + gk + gc * p.ldb : Bg, 16, nb);
            }
        } else {
            for (int e = tid; e < BN * kBK; e += S::kThreads) {
                const int c = e / kBK, kk = e % kBK;
                const long long gc = n0 + c, gk = k0 + kk;
                const bool ok = gc < p.n && gk < p.k;
                cp_async(bs + c * kPB + kk, ok ? Bg + gk + gc * p.ldb : Bg, 8, ok ? 8 : 0);
            }
        }
    };

    double acc[S::kTM][S::kTN][4];
#pragma unroll
    for (int i = 0; i < S::kTM; ++i)
#pragma unroll
        for (int j = 0; j < S::kTN; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.0;

#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < ktiles) load_tile(s, s);
        cp_async_commit();
    }
    for (long long kt = 0; kt < ktiles; ++kt) {
        cp_async_wait<kStages - 2>();
        __syncthreads();   // tile kt landed for every thread; stage (kt-1) % kStages is free again
        if (kt + kStages - 1 < ktiles) load_tile((int)((kt + kStages - 1) % kStages), kt + kStages - 1);
        cp_async_commit();
        const double* as = As + (int)(kt % kStages) * S::kStageA;
        const double* bs = Bs + (int)(kt % kStages) * S::kStageB;
#pragma unroll
        for (int ks = 0; ks < kBK; ks += 8) {
            double a[S::kTM][4], b[S::kTN][2];
#pragma unroll
            for (int i = 0; i < S::kTM; ++i) {
                const int r = wm0 + i * 16 + gid;
                a[i][0] = as[(ks + tig) * S::kPA + r];
                a[i][1] = as[(ks + tig) * S::kPA + r + 8];
                a[i][2] = as[(ks + tig + 4) * S::kPA + r];
                a[i][3] = as[(ks + tig + 4) * S::kPA + r + 8];
            }
#pragma unroll
            for (int j = 0; j < S::kTN; ++j) {
                const int c = wn0 + j * 8 + gid;
                b[j][0] = bs[c * kPB + ks + tig];
                b[j][1] = bs[c * kPB + ks + tig + 4];
            }
#pragma unroll
            for (int i = 0; i < S::kTM; ++i)
#pragma unroll
                for (int j = 0; j < S::kTN; ++j) dmma(acc[i][j], a[i], b[j]);
        }
    }
    cp_async_wait<0>();

    // epilogue: each accumulator pair is two adjacent columns of one row
#pragma unroll
    for (int i = 0; i < S::kTM; ++i)
#pragma unroll
        for (int j = 0; j < S::kTN; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const long long r = m0 + wm0 + i * 16 + gid + (q >= 2 ? 8 : 0);
                const long long c = n0 + wn0 + j * 8 + tig * 2 + (q & 1);
                if (r < p.m && c < p.n) {
                    double* cp = Cg + r + c * p.ldc;
                    *cp = p.beta == 0.0 ? p.alpha * acc[i][j][q] : fma(p.alpha, acc[i][j][q], p.beta * *cp);
                }
            }
}

template <int BM, int BN, int WM, int WN, int MINB>
int launch_gemm(cudaStream_t st, const GemmArgs& a, int batch)
{
    using S = GemmShape<BM, BN, WM, WN, MINB>;
    static bool attr_done[64] = {};
    int dev = 0;
    CHPL_CUDA(cudaGetDevice(&dev));
    if (dev >= 64 || !attr_done[dev]) {
        CHPL_CUDA(cudaFuncSetAttribute(dgemm_kernel<BM, BN, WM, WN, MINB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)S::kSmem));
        if (dev < 64) attr_done[dev] = true;
    }
    const long long tm = (a.m + BM - 1) / BM, tn = (a.n + BN - 1) / BN;
    if (tm > 0x7fffffffLL || tn > 65535) { set_error("dgemm: %lld x %lld tiles exceed the grid", tm, tn); return CHPL_ERR_UNSUPPORTED; }
    dgemm_kernel<BM, BN, WM, WN, MINB><<<dim3((unsigned)tm, (unsigned)tn, (unsigned)batch), S::kThreads, S::kSmem, st>>>(a);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

// ---------------------------------------------------------------------------- scale C by beta (k == 0 or alpha == 0)
__global__ void scale_cols_kernel(double* __restrict__ C, long long ldc, long long m, long long n, double beta)
{
    const long long total = m * n;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const long long i = e % m, j = e / m;
        double* c = C + i + j * ldc;
        *c = beta == 0.0 ? 0.0 : beta * *c;
    }
}

// ---------------------------------------------------------------------------- TRSM leaf
// B(0:n, cols) = L^-1 B for a unit lower n x n L, n <= 64: one thread per
// right-hand side, its column in registers, L in shared memory; right-looking
// (x_j final, then every row below it updated), so each step's updates are
// independent of one another.
constexpr int kLeaf = 64;
constexpr int kLeafThreads = 128;

__global__ void __launch_bounds__(kLeafThreads) trsm_leaf_kernel(int n, const double* __restrict__ L, long long ldl,
                                                                  double* __restrict__ B, long long ldb, long long nrhs)
{
    __shared__ double Ls[kLeaf][kLeaf + 1];   // Ls[j][i] = L(i, j)
    for (int e = threadIdx.x; e < kLeaf * kLeaf; e += blockDim.x) {
        const int i = e % kLeaf, j = e / kLeaf;
        Ls[j][i] = (i < n && j < n && i > j) ? L[i + j * ldl] : 0.0;
    }
    __syncthreads();
    const long long c = (long long)blockIdx.x * kLeafThreads + threadIdx.x;
    if (c >= nrhs) return;
    double* col = B + c * ldb;
    double x[kLeaf];
#pragma unroll
    for (int i = 0; i < kLeaf; ++i) x[i] = i < n ? col[i] : 0.0;
#pragma unroll
    for (int j = 0; j < kLeaf; ++j)
#pragma unroll
        for (int i = j + 1; i < kLeaf; ++i) x[i] = fma(-Ls[j][i], x[j], x[i]);
#pragma unroll
    for (int i = 0; i < kLeaf; ++i)
        if (i < n) col[i] = x[i];
}

// The same solve with one warp per right-hand side (two rows per lane, x_j
// broadcast by shuffle), for few right-hand sides: the panel recursion's
// solves have 256-512 of them, which one thread each would spread over only
// 2-4 CTAs.
constexpr int kLeafWarps = 8;

__global__ void __launch_bounds__(kLeafWarps * 32) trsm_leaf_warp_kernel(int n, const double* __restrict__ L,
                                                                        long long ldl, double* __restrict__ B,
                                                                        long long ldb, long long nrhs, long long bsL,
                                                                        long long bsB)
{
    L += blockIdx.y * bsL;   // one independent solve per blockIdx.y (batch strides bsL, bsB)
    B += blockIdx.y * bsB;
    __shared__ double Ls[kLeaf][kLeaf + 1];   // Ls[j][i] = L(i, j)
    for (int e = threadIdx.x; e < kLeaf * kLeaf; e += blockDim.x) {
        const int i = e % kLeaf, j = e / kLeaf;
        Ls[j][i] = (i < n && j < n && i > j) ? L[i + j * ldl] : 0.0;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const long long c = (long long)blockIdx.x * kLeafWarps + (threadIdx.x >> 5);
    if (c >= nrhs) return;
    double* col = B + c * ldb;
    double r0 = lane < n ? col[lane] : 0.0;
    double r1 = lane + 32 < n ? col[lane + 32] : 0.0;
    for (int j = 0; j < n; ++j) {
        const double xj = __shfl_sync(0xffffffffu, j < 32 ? r0 : r1, j & 31);
        r0 = fma(-Ls[j][lane], xj, r0);          // Ls[j][i] = 0 for i <= j: rows at or above j keep their value
        r1 = fma(-Ls[j][lane + 32], xj, r1);
    }
    if (lane < n) col[lane] = r0;
    if (lane + 32 < n) col[lane + 32] = r1;
}

// ---------------------------------------------------------------------------- TRSV
// Upper triangular solve by blocks of kTrsvB rows from the bottom, one kernel
// per block j.  Every CTA first solves the diagonal block itself (one warp,
// in shared memory: the right-hand side rows j0..j0+b are final, since every
// block below has been subtracted by the kernels before), then subtracts
// U(rows, j0:j0+b) x_j from its own rows above j0.  Solved blocks go to a
// separate buffer (CTA 0 writes them), so no CTA overwrites rows another CTA
// of the same kernel still reads; the caller copies the buffer back.
constexpr int kTrsvB = 64;
constexpr int kTrsvRows = 64;       // rows per CTA of the update
constexpr int kTrsvGroups = 4;      // column groups per row: 16 independent loads per thread
constexpr int kTrsvThreads = kTrsvRows * kTrsvGroups;

__global__ void __launch_bounds__(kTrsvThreads) trsv_block_kernel(const double* __restrict__ U, long long ldu,
                                                                 double* __restrict__ x, double* __restrict__ xout,
                                                                 long long j0, int b)
{
    __shared__ double Us[kTrsvB][kTrsvB + 1];   // Us[c][r] = U(j0 + r, j0 + c)
    __shared__ double xs[kTrsvB];
    __shared__ double part[kTrsvGroups][kTrsvRows];
    const int tid = threadIdx.x, lane = tid & 31;
    for (int e = tid; e < b * b; e += blockDim.x) {
        const int i = e % b, j = e / b;
        Us[j][i] = U[(j0 + i) + (j0 + j) * ldu];
    }
    __syncthreads();
    if (tid < 32) {   // back substitution of the diagonal block, two rows per lane
        double r0 = lane < b ? x[j0 + lane] : 0.0;
        double r1 = lane + 32 < b ? x[j0 + lane + 32] : 0.0;
        for (int i = b - 1; i >= 0; --i) {
            double xi = __shfl_sync(0xffffffffu, i < 32 ? r0 : r1, i & 31);
            xi = xi / Us[i][i];
            if (lane == (i & 31)) {
                if (i < 32) r0 = xi;
                else r1 = xi;
            }
            if (lane < i) r0 = fma(-Us[i][lane], xi, r0);
            if (lane + 32 < i) r1 = fma(-Us[i][lane + 32], xi, r1);
        }
        xs[lane] = lane < b ? r0 : 0.0;
        xs[lane + 32] = lane + 32 < b ? r1 : 0.0;
    }
    __syncthreads();
    if (blockIdx.x == 0 && tid < b) xout[j0 + tid] = xs[tid];
    // rows [r0, r0 + 64) above the block: thread (row rl, group g) takes the 16 columns g*16 ..
    constexpr int kCols = kTrsvB / kTrsvGroups;
    const int rl = tid % kTrsvRows, g = tid / kTrsvRows;
    const long long r = (long long)blockIdx.x * kTrsvRows + rl;
    double s = 0.0;
    if (r < j0) {
        const double* u = U + r + (j0 + g * kCols) * ldu;
        double v[kCols];
#pragma unroll
        for (int c = 0; c < kCols; ++c) v[c] = (g * kCols + c < b) ? u[c * ldu] : 0.0;
#pragma unroll
        for (int c = 0; c < kCols; ++c) s = fma(v[c], xs[g * kCols + c], s);
    }
    part[g][rl] = s;
    __syncthreads();
    if (g == 0 && r < j0) x[r] -= ((part[0][rl] + part[1][rl]) + (part[2][rl] + part[3][rl]));
}

// ---------------------------------------------------------------------------- GEMV
constexpr int kGemvRows = 32;     // rows per CTA (one per lane)
constexpr int kGemvWarps = 8;     // the CTA's warps split the columns
// y = alpha A x + beta y: 32 rows per CTA (one per lane), the 8 warps split
// the columns in a fixed interleave and combine in a fixed order.
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(long long m, long long n, double alpha,
                                                              const double* __restrict__ A, long long lda,
                                                              const double* __restrict__ x, double beta,
                                                              double* __restrict__ y)
{
    __shared__ double part[kGemvWarps][kGemvRows];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long r = (long long)blockIdx.x * kGemvRows + lane;
    double s0 = 0.0, s1 = 0.0;
    if (r < m) {
        long long c = warp;
        for (; c + kGemvWarps < n; c += 2 * kGemvWarps) {
            s0 = fma(A[r + c * lda], x[c], s0);
            s1 = fma(A[r + (c + kGemvWarps) * lda], x[c + kGemvWarps], s1);
        }
        if (c < n) s0 = fma(A[r + c * lda], x[c], s0);
    }
    part[warp][lane] = s0 + s1;
    __syncthreads();
    if (warp == 0 && r < m) {
        double t = 0.0;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) t += part[w][lane];
        y[r] = beta == 0.0 ? alpha * t : fma(alpha, t, beta * y[r]);
    }
}

int trsm_rec(cudaStream_t st, int64_t n, int64_t nrhs, const double* L, int64_t ldl, double* B, int64_t ldb)
{
    if (n <= kLeaf) {
        if (nrhs < 32768) {   // few right-hand sides: a warp each
            const long long g = (nrhs + kLeafWarps - 1) / kLeafWarps;
            trsm_leaf_warp_kernel<<<(unsigned)g, kLeafWarps * 32, 0, st>>>((int)n, L, (long long)ldl, B, (long long)ldb,
                                                                           (long long)nrhs, 0LL, 0LL);
        } else {
            const long long g = (nrhs + kLeafThreads - 1) / kLeafThreads;
            if (g > 0x7fffffffLL) { set_error("dtrsm: too many right-hand sides"); return CHPL_ERR_UNSUPPORTED; }
            trsm_leaf_kernel<<<(unsigned)g, kLeafThreads, 0, st>>>((int)n, L, (long long)ldl, B, (long long)ldb,
                                                                   (long long)nrhs);
        }
        CHPL_CUDA(cudaGetLastError());
        return CHPL_OK;
    }
    // halves on a multiple of the leaf size: X1 = L11^-1 B1; B2 -= L21 X1; X2 = L22^-1 B2
    const int64_t n1 = std::max<int64_t>(kLeaf, (n / 2) / kLeaf * kLeaf);
    CHPL_TRY(trsm_rec(st, n1, nrhs, L, ldl, B, ldb));
    CHPL_TRY(dgemm(st, n - n1, nrhs, n1, -1.0, L + n1, ldl, B, ldb, 1.0, B + n1, ldb));
    return trsm_rec(st, n - n1, nrhs, L + n1 + n1 * ldl, ldl, B + n1, ldb);
}

// X (n x n, ld ldx) = I: the starting point of the triangular inverse
__global__ void set_identity_kernel(double* __restrict__ X, long long ldx, long long n)
{
    const long long total = n * n;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const long long i = e % n, j = e / n;
        X[i + j * ldx] = (i == j) ? 1.0 : 0.0;
    }
}

// C_z = alpha A_z B_z + beta C_z for z < batch, with A_z = A + z * sA (doubles) and
// likewise B_z, C_z: every product m x n x k, one launch (blockIdx.z = z)
int gemm_batched(cudaStream_t st, int64_t m, int64_t n, int64_t k, double alpha, const double* A, int64_t lda,
                 int64_t sA, const double* B, int64_t ldb, int64_t sB, double beta, double* C, int64_t ldc, int64_t sC,
                 int64_t batch)
{
    if (batch > 65535) { set_error("dgemm: batch of %lld exceeds the grid", (long long)batch); return CHPL_ERR_UNSUPPORTED; }
    GemmArgs a;
    a.m = m; a.n = n; a.k = k; a.alpha = alpha; a.beta = beta;
    a.A = A; a.lda = lda; a.B = B; a.ldb = ldb; a.C = C; a.ldc = ldc;
    a.sA = sA; a.sB = sB; a.sC = sC;
    a.vecA = ((reinterpret_cast<uintptr_t>(A) & 15) == 0 && (lda & 1) == 0 && (sA & 1) == 0) ? 1 : 0;
    a.vecB = ((reinterpret_cast<uintptr_t>(B) & 15) == 0 && (ldb & 1) == 0 && (sB & 1) == 0) ? 1 : 0;
    if (m <= 64) return launch_gemm<64, 128, 2, 4, 2>(st, a, (int)batch);
    if (n <= 32) return launch_gemm<128, 32, 4, 1, 2>(st, a, (int)batch);
    return launch_gemm<128, 64, 4, 2, 2>(st, a, (int)batch);
}

// zero the b x b blocks X + z * stride, z < nblk
__global__ void zero_blocks_kernel(double* __restrict__ X, long long ldx, long long b, long long stride, long long nblk)
{
    const long long per = b * b, total = per * nblk;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const long long z = e / per, r = e % per;
        X[z * stride + (r % b) + (r / b) * ldx] = 0.0;
    }
}

bool leaves_pow2(int64_t n)
{
    if (n < kLeaf || n % kLeaf) return false;
    const int64_t q = n / kLeaf;
    return (q & (q - 1)) == 0;
}

// X = inv(L) for n = kLeaf * 2^q and X = I on entry, level by level with every
// pair of a level in one launch: the diagonal leaves (L_b X_b = I, batched),
// then for b = kLeaf, 2 kLeaf, .. < n and all pairs of b-blocks at once
//   U = L21 X11       (into the pair's block above the diagonal, which is zero)
//   X21 = -X22 U      (= -inv(L22) L21 inv(L11))
//   U = 0
// 1 + 3 log2(n / kLeaf) launches.
int trtri_pow2(cudaStream_t st, int64_t n, const double* L, int64_t ldl, double* X, int64_t ldx)
{
    const int64_t nl = n / kLeaf;
    if (nl > 65535) { set_error("dtrtri: %lld leaves exceed the grid", (long long)nl); return CHPL_ERR_UNSUPPORTED; }
    trsm_leaf_warp_kernel<<<dim3(kLeaf / kLeafWarps, (unsigned)nl), kLeafWarps * 32, 0, st>>>(
        kLeaf, L, (long long)ldl, X, (long long)ldx, (long long)kLeaf, (long long)kLeaf * (1 + ldl),
        (long long)kLeaf * (1 + ldx));
    CHPL_CUDA(cudaGetLastError());
    for (int64_t b = kLeaf; b < n; b *= 2) {
        const int64_t np = n / (2 * b), sL = 2 * b * (1 + ldl), sX = 2 * b * (1 + ldx);
        CHPL_TRY(gemm_batched(st, b, b, b, 1.0, L + b, ldl, sL, X, ldx, sX, 0.0, X + b * ldx, ldx, sX, np));
        CHPL_TRY(gemm_batched(st, b, b, b, -1.0, X + b + b * ldx, ldx, sX, X + b * ldx, ldx, sX, 0.0, X + b, ldx, sX,
                              np));
        const unsigned g = (unsigned)std::min<long long>((np * b * b + 255) / 256, 148LL * 32);
        zero_blocks_kernel<<<g, 256, 0, st>>>(X + b * ldx, (long long)ldx, (long long)b, (long long)sX, (long long)np);
        CHPL_CUDA(cudaGetLastError());
    }
    return CHPL_OK;
}

// X = inv(L) for X = I on entry.  n = kLeaf * 2^q: level-batched (trtri_pow2);
// otherwise the largest such n1 < n first and X22 = inv(L22) recursively, then
// X21 = -X22 (L21 X11).  With n2 >= n1 / 4 that is products only, in column
// blocks of n2: T = L21 X11(:, blk) goes to X's zero upper block X(0:n2,
// n1:n1+n2), X21(:, blk) = -X22 T, and the block is zeroed again at the end;
// a thinner n2 uses X21 = -L21 X11 followed by the solve with L22.
int trtri_rec(cudaStream_t st, int64_t n, const double* L, int64_t ldl, double* X, int64_t ldx)
{
    if (n <= kLeaf) return trsm_rec(st, n, n, L, ldl, X, ldx);
    if (leaves_pow2(n)) return trtri_pow2(st, n, L, ldl, X, ldx);
    int64_t n1 = kLeaf;
    while (2 * n1 < n) n1 *= 2;
    const int64_t n2 = n - n1;
    CHPL_TRY(trtri_pow2(st, n1, L, ldl, X, ldx));
    CHPL_TRY(trtri_rec(st, n2, L + n1 + n1 * ldl, ldl, X + n1 + n1 * ldx, ldx));
    if (4 * n2 < n1) {
        CHPL_TRY(dgemm(st, n2, n1, n1, -1.0, L + n1, ldl, X, ldx, 0.0, X + n1, ldx));
        return trsm_rec(st, n2, n1, L + n1 + n1 * ldl, ldl, X + n1, ldx);
    }
    double* T = X + n1 * ldx;   // rows 0..n2-1 of the zero block right of X11 (n2 <= n1)
    for (int64_t j0 = 0; j0 < n1; j0 += n2) {
        const int64_t w = std::min(n2, n1 - j0);
        CHPL_TRY(dgemm(st, n2, w, n1 - j0, 1.0, L + n1 + j0 * ldl, ldl, X + j0 + j0 * ldx, ldx, 0.0, T, ldx));
        CHPL_TRY(dgemm(st, n2, w, n2, -1.0, X + n1 + n1 * ldx, ldx, T, ldx, 0.0, X + n1 + j0 * ldx, ldx));
    }
    const unsigned g = (unsigned)std::min<long long>((n2 * n2 + 255) / 256, 148LL * 32);
    zero_blocks_kernel<<<g, 256, 0, st>>>(T, (long long)ldx, (long long)n2, 0LL, 1LL);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

int64_t trsm_count(int64_t n)
{
    if (n <= kLeaf) return 1;
    const int64_t n1 = std::max<int64_t>(kLeaf, (n / 2) / kLeaf * kLeaf);
    return trsm_count(n1) + 1 + trsm_count(n - n1);
}

}  // namespace

int dgemm(cudaStream_t st, int64_t m, int64_t n, int64_t k, double alpha, const double* A, int64_t lda,
          const double* B, int64_t ldb, double beta, double* C, int64_t ldc)
{
    if (m < 0 || n < 0 || k < 0 || ldc < std::max<int64_t>(m, 1)) { set_error("dgemm: bad sizes"); return CHPL_ERR_INVALID; }
    if (m == 0 || n == 0) return CHPL_OK;
    if (k == 0 || alpha == 0.0) {
        if (beta == 1.0) return CHPL_OK;
        const long long tot = m * n;
        const unsigned g = (unsigned)std::min<long long>((tot + 255) / 256, 148LL * 32);
        scale_cols_kernel<<<g, 256, 0, st>>>(C, (long long)ldc, (long long)m, (long long)n, beta);
        CHPL_CUDA(cudaGetLastError());
        return CHPL_OK;
    }
    if (lda < std::max<int64_t>(m, 1) || ldb < std::max<int64_t>(k, 1)) { set_error("dgemm: bad leading dimension"); return CHPL_ERR_INVALID; }
    return gemm_batched(st, m, n, k, alpha, A, lda, 0, B, ldb, 0, beta, C, ldc, 0, 1);
}

int dtrsm_llnu(cudaStream_t st, int64_t n, int64_t nrhs, const double* L, int64_t ldl, double* B, int64_t ldb)
{
    if (n < 0 || nrhs < 0 || ldl < std::max<int64_t>(n, 1) || ldb < std::max<int64_t>(n, 1)) {
        set_error("dtrsm: bad sizes");
        return CHPL_ERR_INVALID;
    }
    if (n == 0 || nrhs == 0) return CHPL_OK;
    return trsm_rec(st, n, nrhs, L, ldl, B, ldb);
}

int64_t dtrsm_launches(int64_t n) { return n <= 0 ? 0 : trsm_count(n); }

int dtrtri_llnu(cudaStream_t st, int64_t n, const double* L, int64_t ldl, double* X, int64_t ldx)
{
    if (n < 0 || ldl < std::max<int64_t>(n, 1) || ldx < std::max<int64_t>(n, 1)) {
        set_error("dtrtri: bad sizes");
        return CHPL_ERR_INVALID;
    }
    if (n == 0) return CHPL_OK;
    const unsigned g = (unsigned)std::min<long long>((n * n + 255) / 256, 148LL * 32);
    set_identity_kernel<<<g, 256, 0, st>>>(X, (long long)ldx, (long long)n);
    CHPL_CUDA(cudaGetLastError());
    return trtri_rec(st, n, L, ldl, X, ldx);
}

int64_t dtrtri_launches(int64_t n)
{
    if (n <= 0) return 0;
    if (n <= kLeaf) return 1;
    int64_t n1 = kLeaf, levels = 0;
    while (2 * n1 <= n) { n1 *= 2; ++levels; }   // n1 = kLeaf * 2^levels <= n
    if (n1 == n) return 1 + 3 * levels;
    const int64_t n2 = n - n1;
    const int64_t rest = 4 * n2 < n1 ? 1 + trsm_count(n2) : 2 * ((n1 + n2 - 1) / n2) + 1;
    return (1 + 3 * levels) + dtrtri_launches(n2) + rest;
}

int dtrsv_unn(cudaStream_t st, int64_t n, const double* U, int64_t ldu, double* x, double* work)
{
    if (n < 0 || ldu < std::max<int64_t>(n, 1)) { set_error("dtrsv: bad sizes"); return CHPL_ERR_INVALID; }
    if (n == 0) return CHPL_OK;
    if (!work) { set_error("dtrsv: work is NULL"); return CHPL_ERR_WORKSPACE; }
    const int64_t nb = (n + kTrsvB - 1) / kTrsvB;
    for (int64_t j = nb - 1; j >= 0; --j) {
        const long long j0 = j * kTrsvB;
        const int b = (int)std::min<int64_t>(kTrsvB, n - j0);
        const unsigned g = (unsigned)std::max<long long>(1, (j0 + kTrsvRows - 1) / kTrsvRows);
        trsv_block_kernel<<<g, kTrsvThreads, 0, st>>>(U, (long long)ldu, x, work, j0, b);
        CHPL_CUDA(cudaGetLastError());
    }
    CHPL_CUDA(cudaMemcpyAsync(x, work, (size_t)n * sizeof(double), cudaMemcpyDeviceToDevice, st));
    return CHPL_OK;
}

int64_t dtrsv_launches(int64_t n) { return n <= 0 ? 0 : (n + kTrsvB - 1) / kTrsvB; }

int dgemv_n(cudaStream_t st, int64_t m, int64_t n, double alpha, const double* A, int64_t lda, const double* x,
            double beta, double* y)
{
    if (m < 0 || n < 0 || lda < std::max<int64_t>(m, 1)) { set_error("dgemv: bad sizes"); return CHPL_ERR_INVALID; }
    if (m == 0) return CHPL_OK;
    const long long g = (m + kGemvRows - 1) / kGemvRows;
    if (g > 0x7fffffffLL) { set_error("dgemv: too many rows"); return CHPL_ERR_UNSUPPORTED; }
    gemv_kernel<<<(unsigned)g, kGemvWarps * 32, 0, st>>>((long long)m, (long long)n, alpha, A, (long long)lda, x, beta, y);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

}  // namespace chpl

using namespace chpl;

extern "C" int chpl_dgemm(void* stream, int64_t m, int64_t n, int64_t k, double alpha, const double* A, size_t lda,
                          const double* B, size_t ldb, double beta, double* C, size_t ldc)
{
    return dgemm((cudaStream_t)stream, m, n, k, alpha, A, (int64_t)lda, B, (int64_t)ldb, beta, C, (int64_t)ldc);
}

extern "C" int chpl_dtrsm_llnu(void* stream, int64_t n, int64_t nrhs, const double* L, size_t ldl, double* B, size_t ldb)
{
    return dtrsm_llnu((cudaStream_t)stream, n, nrhs, L, (int64_t)ldl, B, (int64_t)ldb);
}

extern "C" int chpl_dtrtri_llnu(void* stream, int64_t n, const double* L, size_t ldl, double* X, size_t ldx)
{
    return dtrtri_llnu((cudaStream_t)stream, n, L, (int64_t)ldl, X, (int64_t)ldx);
}

extern "C" int chpl_dtrsv_unn(void* stream, int64_t n, const double* U, size_t ldu, double* x, double* work)
{
    return dtrsv_unn((cudaStream_t)stream, n, U, (int64_t)ldu, x, work);
}

extern "C" int chpl_dgemv(void* stream, int64_t m, int64_t n, double alpha, const double* A, size_t lda,
                          const double* x, double beta, double* y)
{
    return dgemv_n((cudaStream_t)stream, m, n, alpha, A, (int64_t)lda, x, beta, y);
}
