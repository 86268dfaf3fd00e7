// HPL building blocks on B200: matrix generation, row interchanges, residual.
#include <curand_kernel.h>

#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "hpl.h"

namespace chpl {

__device__ int g_hpl_status;

// ----------------------------------------------------------------------------
// generator: chpl_elem of src/chpl_p2.cu:66-73 (SplitMix64 output of counter
// idx, top 53 bits scaled to [0,1), minus 0.5)
// ----------------------------------------------------------------------------
__device__ __forceinline__ double hpl_elem(uint64_t seed, uint64_t idx)
{
    uint64_t z = (idx + 1ull) * 0x9E3779B97F4A7C15ull + seed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z = z ^ (z >> 31);
    return (double)(z >> 11) * (1.0 / 9007199254740992.0) - 0.5;
}

// generator of chpl_single (src/chpl_single.cu:73-80): cuRAND's
// Philox4_32_10 with one subsequence per element (subsequence = the element's
// index, offset 0), first uniform double in (0, 1] minus 0.5.  Computed by
// cuRAND's own device API, so the matrix is the reference chpl_single's.
__device__ __forceinline__ double philox_elem(uint64_t seed, uint64_t idx)
{
    curandStatePhilox4_32_10_t s;
    curand_init((unsigned long long)seed, (unsigned long long)idx, 0ull, &s);
    return curand_uniform_double(&s) - 0.5;
}

template <int G>
__device__ __forceinline__ double gen_elem(uint64_t seed, uint64_t idx)
{
    if constexpr (G == CHPL_GEN_PHILOX) return philox_elem(seed, idx);
    else return hpl_elem(seed, idx);
}

// A[i + j*lda] = elem(seed, (row0+i)*ncg + col0+j); one thread per element,
// consecutive threads walk down a column (coalesced 8-byte stores).
template <int G>
__global__ void matgen_kernel(double* __restrict__ A, long long lda, long long m, long long n, long long row0,
                              long long col0, long long ncg, uint64_t seed)
{
    const long long total = m * n;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long i = e % m, j = e / m;
        A[i + j * lda] = gen_elem<G>(seed, (uint64_t)(row0 + i) * (uint64_t)ncg + (uint64_t)(col0 + j));
    }
}

// block-cyclic local piece: local row r -> global (r/NB*P + pr)*NB + r%NB
__device__ __forceinline__ long long cyc_global(long long l, long long NB, int P, int p)
{
    return (l / NB * P + p) * NB + l % NB;
}

__global__ void matgen_cyclic_kernel(double* __restrict__ A, long long lda, long long mloc, long long nloc,
                                     long long NB, int P, int Q, int pr, int qc, long long ncg, uint64_t seed)
{
    const long long total = mloc * nloc;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long i = e % mloc, j = e / mloc;
        const long long gi = cyc_global(i, NB, P, pr), gj = cyc_global(j, NB, Q, qc);
        A[i + j * lda] = hpl_elem(seed, (uint64_t)gi * (uint64_t)ncg + (uint64_t)gj);
    }
}

static inline int grid_for(long long work, int block)
{
    long long g = (work + block - 1) / block;
    if (g > 148LL * 64) g = 148LL * 64;
    return (int)(g < 1 ? 1 : g);
}

int matgen(cudaStream_t st, double* A, size_t lda, size_t m, size_t n, int64_t row0, int64_t col0, int64_t ncg,
           uint64_t seed, int generator)
{
    if (generator != CHPL_GEN_CHPL && generator != CHPL_GEN_PHILOX) {
        set_error("unknown generator %d", generator);
        return CHPL_ERR_INVALID;
    }
    if (m == 0 || n == 0) return CHPL_OK;
    const int g = grid_for((long long)(m * n), 256);
    if (generator == CHPL_GEN_PHILOX)
        matgen_kernel<CHPL_GEN_PHILOX><<<g, 256, 0, st>>>(A, (long long)lda, (long long)m, (long long)n, row0, col0, ncg,
                                                          seed);
    else
        matgen_kernel<CHPL_GEN_CHPL><<<g, 256, 0, st>>>(A, (long long)lda, (long long)m, (long long)n, row0, col0, ncg,
                                                        seed);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

// ----------------------------------------------------------------------------
// row interchanges (dlaswp semantics) as one net permutation
// ----------------------------------------------------------------------------
// Build the net permutation of the swap sequence (i <-> ipiv[i], i = k1..k2-1,
// ipiv[i] >= i as produced by partial pivoting).  Touched positions are
// [k1, k2) plus the distinct ipiv[i] >= k2; the latter get compact slots
// through an open-addressing table in shared memory, then one thread replays
// the swaps on slot contents.  Output: cnt[0] pairs (dst[t], src[t]) with
// "row dst receives the old contents of row src".
constexpr int kLaswpMaxSwaps = 2048;
constexpr int kHash = 4096;  // power of two >= 2 * kLaswpMaxSwaps / 1 (load factor <= 0.5)
constexpr size_t kPlanSmem = (size_t)kHash * 4 * 2 + (size_t)2 * kLaswpMaxSwaps * 4 * 2 + (size_t)kLaswpMaxSwaps * 4 + 16;

__global__ void __launch_bounds__(1024) laswp_plan_kernel(const int64_t* __restrict__ ipiv, long long k1, int ns,
                                                          long long pbase, int* __restrict__ dst,
                                                          int* __restrict__ src, int* __restrict__ cnt)
{
    extern __shared__ int psm[];
    int* key = psm;                              // [kHash] row ids >= k2, -1 = empty
    int* slotof = key + kHash;                   // [kHash]
    int* occ = slotof + kHash;                   // [2*max] slot whose original row is now here
    int* pos = occ + 2 * kLaswpMaxSwaps;         // [2*max] row id of each slot
    int* pslot = pos + 2 * kLaswpMaxSwaps;       // [max] slot of ipiv[k1+i]
    int* counters = pslot + kLaswpMaxSwaps;      // [0] extra slots, [1] output pairs
    const long long k2 = k1 + ns;
    for (int h = threadIdx.x; h < kHash; h += blockDim.x) key[h] = -1;
    if (threadIdx.x == 0) { counters[0] = 0; counters[1] = 0; }
    __syncthreads();
    for (int i = threadIdx.x; i < ns; i += blockDim.x) {
        const int p = (int)(ipiv[k1 + i] - pbase);
        if (p < k2) { pslot[i] = (int)(p - k1); continue; }
        unsigned h = ((unsigned)p * 2654435761u) & (kHash - 1);
        while (true) {
            const int prev = atomicCAS(&key[h], -1, p);
            if (prev == -1) {
                const int s = ns + atomicAdd(&counters[0], 1);
                slotof[h] = s;
                pos[s] = p;
                break;
            }
            if (prev == p) break;
            h = (h + 1) & (kHash - 1);
        }
        pslot[i] = -1 - (int)h;  // resolved after the barrier
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ns; i += blockDim.x)
        if (pslot[i] < 0) pslot[i] = slotof[-1 - pslot[i]];
    const int nslots = ns + counters[0];
    for (int s = threadIdx.x; s < nslots; s += blockDim.x) {
        if (s < ns) pos[s] = (int)(k1 + s);
        occ[s] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 0; i < ns; ++i) {
            const int q = pslot[i];
            const int t = occ[i];
            occ[i] = occ[q];
            occ[q] = t;
        }
    }
    __syncthreads();
    for (int s = threadIdx.x; s < nslots; s += blockDim.x)
        if (occ[s] != s) {
            const int o = atomicAdd(&counters[1], 1);
            dst[o] = pos[s];
            src[o] = pos[occ[s]];
        }
    __syncthreads();
    if (threadIdx.x == 0) cnt[0] = counters[1];
}

// Apply the planned permutation to columns [c0, c0+ncols) of A.  Each CTA owns
// a few whole columns: it reads every source row of its columns, then (after a
// barrier) writes every destination row, so in-place is safe.  The moved rows
// of a column are scattered over ~N rows of a column-major matrix, so each
// access is its own DRAM sector; what bounds the kernel is how many of them
// are in flight.  The register form gives each thread PPT pairs x COLS columns
// of independent loads (up to 32) before the barrier.
template <int PPT, int COLS>
__global__ void __launch_bounds__(256) laswp_apply_reg_kernel(double* __restrict__ A, long long lda, long long ncols,
                                                              const int* __restrict__ dst, const int* __restrict__ src,
                                                              const int* __restrict__ cnt)
{
    const int np = cnt[0];
    const long long c0 = (long long)blockIdx.x * COLS;
    if (np == 0 || c0 >= ncols) return;
    const int nc = (int)min((long long)COLS, ncols - c0);
    int s[PPT], d[PPT];
#pragma unroll
    for (int j = 0; j < PPT; ++j) {
        const int t = threadIdx.x + j * 256;
        s[j] = t < np ? src[t] : -1;
        d[j] = t < np ? dst[t] : -1;
    }
    double v[COLS][PPT];
#pragma unroll
    for (int c = 0; c < COLS; ++c) {
        const double* col = A + (c0 + c) * lda;
#pragma unroll
        for (int j = 0; j < PPT; ++j) v[c][j] = (c < nc && s[j] >= 0) ? col[s[j]] : 0.0;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < COLS; ++c) {
        double* col = A + (c0 + c) * lda;
#pragma unroll
        for (int j = 0; j < PPT; ++j)
            if (c < nc && d[j] >= 0) col[d[j]] = v[c][j];
    }
}

size_t laswp_work_bytes(int64_t nswaps) { return round_up((size_t)(2 * nswaps) * 8 + 64, 256); }

int laswp_plan(cudaStream_t st, const int64_t* ipiv, int64_t k1, int64_t k2, void* work, int64_t pbase)
{
    const int ns = (int)(k2 - k1);
    if (ns <= 0) return CHPL_OK;
    if (ns > kLaswpMaxSwaps) { set_error("laswp: at most %d interchanges per call", kLaswpMaxSwaps); return CHPL_ERR_UNSUPPORTED; }
    int* cnt = static_cast<int*>(work);
    int* dst = cnt + 16;
    int* src = dst + 2 * ns;
    CHPL_CUDA(cudaFuncSetAttribute(laswp_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPlanSmem));
    laswp_plan_kernel<<<1, 1024, kPlanSmem, st>>>(ipiv, (long long)k1, ns, (long long)pbase, dst, src, cnt);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

template <int PPT, int COLS>
static int launch_apply_reg(cudaStream_t st, double* A, size_t lda, int64_t ncols, const int* dst, const int* src,
                            const int* cnt)
{
    const long long nb = (ncols + COLS - 1) / COLS;
    if (nb > 0x7fffffffLL) { set_error("laswp: too many columns"); return CHPL_ERR_UNSUPPORTED; }
    laswp_apply_reg_kernel<PPT, COLS><<<(unsigned)nb, 256, 0, st>>>(A, (long long)lda, (long long)ncols, dst, src, cnt);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

int laswp_apply(cudaStream_t st, double* A, size_t lda, int64_t c0, int64_t ncols, int64_t nswaps, const void* work)
{
    if (ncols <= 0 || nswaps <= 0) return CHPL_OK;
    const int* cnt = static_cast<const int*>(work);
    const int* dst = cnt + 16;
    const int* src = dst + 2 * nswaps;
    double* Ac = A + (size_t)c0 * lda;
    // the plan moves at most 2 * nswaps rows; pick the register form that holds them
    const int64_t maxpairs = 2 * nswaps;
    if (maxpairs <= 256) return launch_apply_reg<1, 8>(st, Ac, lda, ncols, dst, src, cnt);
    if (maxpairs <= 512) return launch_apply_reg<2, 8>(st, Ac, lda, ncols, dst, src, cnt);
    if (maxpairs <= 1024) return launch_apply_reg<4, 8>(st, Ac, lda, ncols, dst, src, cnt);
    if (maxpairs <= 2048) return launch_apply_reg<8, 4>(st, Ac, lda, ncols, dst, src, cnt);
    static_assert(2 * kLaswpMaxSwaps <= 16 * 256, "a plan's pairs must fit the widest register form");
    if (maxpairs <= 4096) return launch_apply_reg<16, 2>(st, Ac, lda, ncols, dst, src, cnt);
    set_error("laswp: at most %d interchanges per plan", kLaswpMaxSwaps);
    return CHPL_ERR_UNSUPPORTED;
}

// ipiv_abs[base + i] = base + rel[i] - 1 (1-based relative -> 0-based absolute)
__global__ void ipiv_abs_kernel(const int64_t* __restrict__ rel, int n, long long base, int64_t* __restrict__ out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = base + rel[i] - 1;
}

int ipiv_to_abs(cudaStream_t st, const int64_t* rel, int64_t n, int64_t base, int64_t* out)
{
    if (n <= 0) return CHPL_OK;
    ipiv_abs_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rel, (int)n, (long long)base, out);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

__global__ void identity_kernel(double* __restrict__ X, long long n)
{
    const long long total = n * n;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x)
        X[e] = (e % n == e / n) ? 1.0 : 0.0;
}

int identity(cudaStream_t st, double* X, int64_t n)
{
    if (n <= 0) return CHPL_OK;
    identity_kernel<<<grid_for(n * n, 256), 256, 0, st>>>(X, (long long)n);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

// ----------------------------------------------------------------------------
// residual: A and b regenerated on the fly (the generated system) or read from
// a device copy of [A | b]; deterministic two-stage reduction
// ----------------------------------------------------------------------------
constexpr int kResChunks = 64;

// element (i, j) of the generated N x (N+1) system; column N is b
template <int G>
struct GenSystem {
    long long N;
    uint64_t seed;
    __device__ __forceinline__ double at(long long i, long long j) const
    {
        return gen_elem<G>(seed, (uint64_t)i * (uint64_t)(N + 1) + (uint64_t)j);
    }
};

// element (i, j) of [A | b] held column-major in device memory
struct DeviceSystem {
    const double* Ab;
    long long ld;
    __device__ __forceinline__ double at(long long i, long long j) const { return Ab[i + j * ld]; }
};

// part[(chunk*2 + 0)*N + i] = sum_j a_ij x_j, part[(chunk*2+1)*N + i] = sum |a_ij|
// over the chunk's columns; one thread per row, columns walked in order
// (consecutive threads read consecutive rows of a column).
template <class Sys>
__global__ void __launch_bounds__(256) resid_partial_kernel(long long N, Sys sys, const double* __restrict__ x,
                                                            double* __restrict__ part)
{
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const int ch = blockIdx.y;
    if (i >= N) return;
    const long long per = (N + kResChunks - 1) / kResChunks;
    const long long j0 = ch * per, j1 = min(N, j0 + per);
    double ax = 0.0, rs = 0.0;
    for (long long j = j0; j < j1; ++j) {
        const double a = sys.at(i, j);
        ax = fma(a, x[j], ax);
        rs += fabs(a);
    }
    part[(ch * 2 + 0) * N + i] = ax;
    part[(ch * 2 + 1) * N + i] = rs;
}

// per row: r_i = |sum_chunks ax - b_i|, rs_i = sum_chunks |a|; block maxima of
// r, rs, |x|, |b| into out[blockIdx*4 + {0..3}]
template <class Sys>
__global__ void __launch_bounds__(256) resid_rows_kernel(long long N, Sys sys, const double* __restrict__ x,
                                                         const double* __restrict__ part, double* __restrict__ out)
{
    __shared__ double sm[4][256];
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    double r = 0.0, rs = 0.0, xa = 0.0, ba = 0.0;
    if (i < N) {
        double ax = 0.0, s = 0.0;
        for (int c = 0; c < kResChunks; ++c) {
            ax += part[(c * 2 + 0) * N + i];
            s += part[(c * 2 + 1) * N + i];
        }
        const double b = sys.at(i, N);
        r = fabs(ax - b);
        rs = s;
        xa = fabs(x[i]);
        ba = fabs(b);
    }
    sm[0][threadIdx.x] = r; sm[1][threadIdx.x] = rs; sm[2][threadIdx.x] = xa; sm[3][threadIdx.x] = ba;
    __syncthreads();
    for (int o = 128; o; o >>= 1) {
        if (threadIdx.x < o)
            for (int q = 0; q < 4; ++q) sm[q][threadIdx.x] = fmax(sm[q][threadIdx.x], sm[q][threadIdx.x + o]);
        __syncthreads();
    }
    if (threadIdx.x < 4) out[blockIdx.x * 4 + threadIdx.x] = sm[threadIdx.x][0];
}

template <class Sys>
static int residual_of(cudaStream_t st, int64_t N, Sys sys, const double* x, double* resid)
{
    if (N <= 0) { set_error("residual: N <= 0"); return CHPL_ERR_INVALID; }
    const long long nb = (N + 255) / 256;
    double* part = nullptr;
    double* out = nullptr;
    CHPL_CUDA(cudaMallocAsync((void**)&part, (size_t)kResChunks * 2 * N * sizeof(double), st));
    CHPL_CUDA(cudaMallocAsync((void**)&out, (size_t)nb * 4 * sizeof(double), st));
    dim3 g((unsigned)nb, kResChunks);
    resid_partial_kernel<Sys><<<g, 256, 0, st>>>((long long)N, sys, x, part);
    resid_rows_kernel<Sys><<<(unsigned)nb, 256, 0, st>>>((long long)N, sys, x, part, out);
    CHPL_CUDA(cudaGetLastError());
    double* h = (double*)malloc((size_t)nb * 4 * sizeof(double));
    if (!h) { set_error("out of host memory"); return CHPL_ERR_WORKSPACE; }
    cudaError_t e = cudaMemcpyAsync(h, out, (size_t)nb * 4 * sizeof(double), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFreeAsync(part, st);
    cudaFreeAsync(out, st);
    if (e != cudaSuccess) { free(h); return cuda_fail(e, "residual readback", __FILE__, __LINE__); }
    double rmax = 0.0, anorm = 0.0, xnorm = 0.0, bnorm = 0.0;
    for (long long b = 0; b < nb; ++b) {
        rmax = fmax(rmax, h[b * 4 + 0]);
        anorm = fmax(anorm, h[b * 4 + 1]);
        xnorm = fmax(xnorm, h[b * 4 + 2]);
        bnorm = fmax(bnorm, h[b * 4 + 3]);
    }
    free(h);
    const double eps = ldexp(1.0, -53);
    *resid = rmax / (eps * (anorm * xnorm + bnorm) * (double)N);
    return CHPL_OK;
}

int residual(cudaStream_t st, int64_t N, uint64_t seed, const double* x, double* resid, int generator)
{
    if (generator == CHPL_GEN_PHILOX) return residual_of(st, N, GenSystem<CHPL_GEN_PHILOX>{(long long)N, seed}, x, resid);
    if (generator != CHPL_GEN_CHPL) { set_error("unknown generator %d", generator); return CHPL_ERR_INVALID; }
    return residual_of(st, N, GenSystem<CHPL_GEN_CHPL>{(long long)N, seed}, x, resid);
}

int residual_matrix(cudaStream_t st, int64_t N, const double* Ab, size_t ld, const double* x, double* resid)
{
    if (!Ab || !x || (int64_t)ld < N) { set_error("residual: bad matrix arguments"); return CHPL_ERR_INVALID; }
    return residual_of(st, N, DeviceSystem{Ab, (long long)ld}, x, resid);
}

int hpl_read_clear_status(int* st)
{
    int v = 0, z = 0;
    CHPL_CUDA(cudaMemcpyFromSymbol(&v, g_hpl_status, sizeof(int)));
    CHPL_CUDA(cudaMemcpyToSymbol(g_hpl_status, &z, sizeof(int)));
    *st = v;
    return CHPL_OK;
}

}  // namespace chpl

using namespace chpl;

extern "C" int chpl_matgen(void* stream, double* A, size_t lda, size_t m, size_t n, int64_t row0, int64_t col0,
                           int64_t ncg, uint64_t seed)
{
    if (lda < m) { set_error("lda < m"); return CHPL_ERR_INVALID; }
    return matgen((cudaStream_t)stream, A, lda, m, n, row0, col0, ncg, seed);
}

extern "C" int chpl_matgen_philox(void* stream, double* A, size_t lda, size_t m, size_t n, int64_t row0, int64_t col0,
                                  int64_t ncg, uint64_t seed)
{
    if (lda < m) { set_error("lda < m"); return CHPL_ERR_INVALID; }
    return matgen((cudaStream_t)stream, A, lda, m, n, row0, col0, ncg, seed, CHPL_GEN_PHILOX);
}

extern "C" int chpl_matgen_host(int64_t N, uint64_t seed, double* Ab, size_t ldab)
{
    if (N <= 0 || !Ab || (int64_t)ldab < N) { set_error("matgen_host: bad arguments"); return CHPL_ERR_INVALID; }
    // column blocks of <= 256 MiB generated on the device and copied out
    const int64_t ncols = N + 1;
    const int64_t per = std::max<int64_t>(1, std::min<int64_t>(ncols, ((int64_t)256 << 20) / (N * 8)));
    double* d = nullptr;
    cudaStream_t st = nullptr;
    CHPL_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    cudaError_t e = cudaMalloc((void**)&d, (size_t)N * (size_t)per * sizeof(double));
    int rc = e == cudaSuccess ? CHPL_OK : cuda_fail(e, "matgen_host staging", __FILE__, __LINE__);
    for (int64_t c0 = 0; c0 < ncols && rc == CHPL_OK; c0 += per) {
        const int64_t nc = std::min(per, ncols - c0);
        rc = matgen(st, d, (size_t)N, (size_t)N, (size_t)nc, 0, c0, ncols, seed);
        if (rc != CHPL_OK) break;
        e = cudaMemcpy2DAsync(Ab + (size_t)c0 * ldab, ldab * sizeof(double), d, (size_t)N * sizeof(double),
                              (size_t)N * sizeof(double), (size_t)nc, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_fail(e, "matgen_host copy", __FILE__, __LINE__);
    }
    if (d) cudaFree(d);
    cudaStreamDestroy(st);
    return rc;
}

extern "C" int chpl_matgen_cyclic(void* stream, double* A, size_t lda, int64_t N, int64_t NB, int P, int Q, int pr,
                                  int qc, uint64_t seed)
{
    if (N <= 0 || NB <= 0 || P <= 0 || Q <= 0 || pr < 0 || pr >= P || qc < 0 || qc >= Q) {
        set_error("matgen_cyclic: bad grid arguments");
        return CHPL_ERR_INVALID;
    }
    const int64_t mloc = local_extent(N, NB, P, pr), nloc = local_extent(N + 1, NB, Q, qc);
    if ((int64_t)lda < mloc) { set_error("lda < local rows"); return CHPL_ERR_INVALID; }
    if (mloc == 0 || nloc == 0) return CHPL_OK;
    matgen_cyclic_kernel<<<grid_for(mloc * nloc, 256), 256, 0, (cudaStream_t)stream>>>(
        A, (long long)lda, mloc, nloc, NB, P, Q, pr, qc, N + 1, seed);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

extern "C" size_t chpl_laswp_work_bytes(int64_t nrows, int64_t nswaps)
{
    (void)nrows;
    return laswp_work_bytes(nswaps);
}

extern "C" int chpl_laswp(void* stream, double* A, size_t lda, int64_t ncols, int64_t k1, int64_t k2,
                          const int64_t* ipiv, int64_t nrows, void* work)
{
    (void)nrows;
    if (k2 <= k1 || ncols <= 0) return CHPL_OK;
    if (!work) { set_error("laswp: work is NULL"); return CHPL_ERR_WORKSPACE; }
    CHPL_TRY(laswp_plan((cudaStream_t)stream, ipiv, k1, k2, work));
    return laswp_apply((cudaStream_t)stream, A, lda, 0, ncols, k2 - k1, work);
}

extern "C" int chpl_residual(void* stream, int64_t N, uint64_t seed, const double* x, double* resid)
{
    if (!resid) { set_error("resid is NULL"); return CHPL_ERR_INVALID; }
    return residual((cudaStream_t)stream, N, seed, x, resid);
}

extern "C" int chpl_residual_matrix(void* stream, int64_t N, const double* Ab, size_t ldab, const double* x,
                                    double* resid)
{
    if (!resid) { set_error("resid is NULL"); return CHPL_ERR_INVALID; }
    return residual_matrix((cudaStream_t)stream, N, Ab, ldab, x, resid);
}
