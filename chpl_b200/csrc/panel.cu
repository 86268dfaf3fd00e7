// FP64 panel factorization with partial pivoting (getrf) of an m x n panel.
//
// Replaces the cusolverDnXgetrf call of src/chpl_single.cu:668-679.
// Recursive (left half, interchanges + U12 + Schur update, right half), down to
// base blocks of kBaseW columns.  A base block is factored by one cooperative
// kernel over all SMs: every CTA keeps a contiguous range of the block's rows
// in shared memory; per column a warp-shuffle argmax gives each CTA's
// candidate, one bounded grid barrier publishes the candidates, every CTA
// picks the same pivot (largest |a|, smallest row on ties, as LAPACK's
// idamax), and all CTAs apply the interchange, the scaling and the rank-1
// update to their rows.  The pivot row and the old diagonal row travel through
// double-buffered global slots written before the barrier, so no CTA ever
// reads a row another CTA is rewriting.  The recursion's FP64 GEMM / TRSM
// steps are plain cuBLAS calls; interchanges use the device-built net
// permutation of hpl_kernels.cu.
#include <cublas_v2.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "hpl.h"

namespace chpl {

constexpr int kBaseW = 32;          // widest base block (16 when the rows do not fit on chip at 32)
constexpr int kPanelThreads = 256;
constexpr int kSmemBytes = 217600;  // shared memory of one base-kernel CTA (rows x width x 8 B)

struct PanelSync {
    int err;       // a wait ran out of time
    int pad[63];
};

struct Cand {
    double val;
    long long row;
};

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p)
{
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release(unsigned int* p, unsigned int v)
{
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until every CTA's flag reaches `stamp` (flags are monotonic within one
// panel call).  Thread b polls CTA b's flag, so the whole exchange costs one
// L2 round trip after the last writer, with no atomics.  Bounded: on timeout
// it raises sync->err and returns false.
__device__ bool wait_flags(PanelSync* sync, const unsigned int* flags, unsigned int G, unsigned int stamp)
{
    int good = 1;
    if (threadIdx.x < G) {
        const uint64_t t0 = globaltimer();
        uint32_t it = 0;
        while ((int)(ld_acquire(&flags[threadIdx.x]) - stamp) < 0) {
            if ((++it & 255u) == 0 && (*(volatile int*)&sync->err || globaltimer() - t0 > 1000000000ull)) {  // 1 s
                atomicExch(&sync->err, 1);
                good = 0;
                break;
            }
        }
    }
    return __syncthreads_and(good) != 0;
}

__device__ __forceinline__ bool better(double v, long long r, double bv, long long br)
{
    return v > bv || (v == bv && r < br);
}

// Factor the m x w block at A (ld) in place.  ipiv[j] = base_row + pivot row
// (0-based, relative to the block top + base_row).  info: 1-based column of
// the first exact zero pivot (+ info_off), left unchanged otherwise.
__global__ void __launch_bounds__(kPanelThreads) panel_base_kernel(double* __restrict__ A, long long ld, long long m,
                                                                    int w, long long rows_per, int64_t* __restrict__ ipiv,
                                                                    long long base_row, int* __restrict__ info,
                                                                    int info_off, PanelSync* sync, unsigned int* flags,
                                                                    unsigned int sbase, Cand* cand, double* candrow,
                                                                    double* toprow)
{
    extern __shared__ double S[];  // column-major [kBaseW][rows_per]: conflict-free row-parallel access
    __shared__ double pv[kBaseW], tv[kBaseW];
    __shared__ Cand wbest[kPanelThreads / 32];
    __shared__ long long pivrow;
    __shared__ double pivval;
    const unsigned int G = gridDim.x;
    const long long r0 = (long long)blockIdx.x * rows_per;
    const long long r1 = min(m, r0 + rows_per);
    const int nr = (int)max(0LL, r1 - r0);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;

    // load own rows
    for (int e = tid; e < nr * w; e += blockDim.x) {
        const int i = e % nr, c = e / nr;
        S[c * rows_per + i] = A[(r0 + i) + (long long)c * ld];
    }
    __syncthreads();

    // candidate of column j among own rows >= jmin, published to slot (j & 1)
    auto publish = [&](int j, long long jmin) {
        double bv = -1.0;
        long long br = 0x7fffffffffffffffLL;
        for (int i = tid; i < nr; i += blockDim.x) {
            const long long gr = r0 + i;
            if (gr < jmin) continue;
            const double v = fabs(S[j * rows_per + i]);
            if (better(v, gr, bv, br)) { bv = v; br = gr; }
        }
        for (int o = 16; o; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const long long orr = __shfl_xor_sync(0xffffffffu, br, o);
            if (better(ov, orr, bv, br)) { bv = ov; br = orr; }
        }
        if (lane == 0) wbest[wid] = Cand{bv, br};
        __syncthreads();
        if (tid == 0) {
            Cand b = wbest[0];
            for (int q = 1; q < (int)(blockDim.x / 32); ++q)
                if (better(wbest[q].val, wbest[q].row, b.val, b.row)) b = wbest[q];
            cand[(j & 1) * G + blockIdx.x] = b;
            pivrow = b.row;
        }
        __syncthreads();
        const long long br2 = pivrow;
        if (br2 >= r0 && br2 < r1 && tid < w)
            candrow[((size_t)(j & 1) * G + blockIdx.x) * kBaseW + tid] = S[tid * rows_per + (br2 - r0)];
        // the owner of row j publishes it: it moves to the pivot's old place
        if (j < w && j >= r0 && j < r1 && tid < w) toprow[(j & 1) * kBaseW + tid] = S[tid * rows_per + (j - r0)];
        __syncthreads();  // the barrier orders every thread's slot writes before thread 0's release
        if (tid == 0) {
            __threadfence();
            st_release(&flags[blockIdx.x], sbase + (unsigned int)j + 1u);
        }
    };

    publish(0, 0);
    for (int j = 0; j < w; ++j) {
        if (!wait_flags(sync, flags, G, sbase + (unsigned int)j + 1u)) return;
        // every CTA reduces the same candidates to the same pivot; each lane
        // loads its candidates together with their rows (one round trip)
        if (wid == 0) {
            double bv = -1.0;
            long long br = 0x7fffffffffffffffLL;
            int bb = -1;
            for (int b = lane; b < (int)G; b += 32) {
                const Cand c = cand[(j & 1) * G + b];
                if (better(c.val, c.row, bv, br)) { bv = c.val; br = c.row; bb = b; }
            }
            double myrow[kBaseW];
            if (bb >= 0) {
                const double* src = candrow + ((size_t)(j & 1) * G + bb) * kBaseW;
#pragma unroll
                for (int c = 0; c < kBaseW; ++c) myrow[c] = c < w ? src[c] : 0.0;
            }
            double bv0 = bv;
            long long br0 = br;
            for (int o = 16; o; o >>= 1) {
                const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const long long orr = __shfl_xor_sync(0xffffffffu, br, o);
                if (better(ov, orr, bv, br)) { bv = ov; br = orr; }
            }
            // the lane holding the winner publishes its row
            if (bv0 == bv && br0 == br && bb >= 0) {
#pragma unroll
                for (int c = 0; c < kBaseW; ++c) if (c < w) pv[c] = myrow[c];
                pivrow = br;
                pivval = bv;
            }
            if (lane < w) tv[lane] = toprow[(j & 1) * kBaseW + lane];
        }
        __syncthreads();
        const long long p = pivrow;
        const double piv = pv[j];
        if (blockIdx.x == 0 && tid == 0) {
            ipiv[j] = base_row + p;
            if (pivval == 0.0 && *info == 0) *info = info_off + j + 1;
        }
        const double rp = (piv != 0.0) ? 1.0 / piv : 0.0;
        for (int i = tid; i < nr; i += blockDim.x) {
            const long long gr = r0 + i;
            double* x = &S[i];  // element c at x[c * rows_per]
            if (gr == j) {
                for (int c = 0; c < w; ++c) x[c * rows_per] = pv[c];
                continue;
            }
            if (gr == p)
                for (int c = 0; c < w; ++c) x[c * rows_per] = tv[c];
            if (gr > j && piv != 0.0) {
                const double l = x[j * rows_per] * rp;
                x[j * rows_per] = l;
                for (int c = j + 1; c < w; ++c) x[c * rows_per] = fma(-l, pv[c], x[c * rows_per]);
            }
        }
        __syncthreads();
        if (j + 1 < w) publish(j + 1, j + 1);
    }
    __syncthreads();
    for (int e = tid; e < nr * w; e += blockDim.x) {
        const int i = e % nr, c = e / nr;
        A[(r0 + i) + (long long)c * ld] = S[c * rows_per + i];
    }
}

// ---------------------------------------------------------------------------- host
struct PanelHandles {
    int dev = -1;
    cublasHandle_t hb = nullptr;
    int grid = 0;
};

static thread_local PanelHandles g_ph;

static int handles(cudaStream_t st, PanelHandles** out)
{
    int dev = 0;
    CHPL_CUDA(cudaGetDevice(&dev));
    if (g_ph.dev != dev) {
        if (g_ph.hb) cublasDestroy(g_ph.hb);
        g_ph = PanelHandles();
        if (cublasCreate(&g_ph.hb) != CUBLAS_STATUS_SUCCESS) { set_error("cublasCreate failed"); return CHPL_ERR_CUDA; }
        int nsm = 0, per = 0;
        CHPL_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
        CHPL_CUDA(cudaFuncSetAttribute(panel_base_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        CHPL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, panel_base_kernel, kPanelThreads, kSmemBytes));
        if (per < 1) { set_error("panel kernel does not fit on an SM"); return CHPL_ERR_UNSUPPORTED; }
        g_ph.grid = nsm;  // one CTA per SM: co-resident by construction
        g_ph.dev = dev;
    }
    if (cublasSetStream(g_ph.hb, st) != CUBLAS_STATUS_SUCCESS) { set_error("cublasSetStream failed"); return CHPL_ERR_CUDA; }
    *out = &g_ph;
    return CHPL_OK;
}

size_t panel_work_bytes(int64_t m, int64_t n)
{
    (void)m;
    const size_t G = 1024;  // upper bound on the grid
    return round_up(sizeof(PanelSync), 256) + round_up(G * sizeof(unsigned int), 256) + round_up(2 * G * sizeof(Cand), 256) +
           round_up(2 * G * kBaseW * sizeof(double), 256) + round_up(2 * kBaseW * sizeof(double), 256) +
           laswp_work_bytes(std::max<int64_t>(n, 1)) + 256;
}

namespace {

struct PanelCtx {
    cudaStream_t st;
    PanelHandles* h;
    PanelSync* sync;
    unsigned int* flags;
    Cand* cand;
    double* candrow;
    double* toprow;
    void* plan;
    unsigned int sbase;  // barrier arrivals so far in this call
    int* info;
    int* status;
};

int base_block(PanelCtx& c, double* A, int64_t lda, int64_t m, int w, int64_t* ipiv, int64_t base_row, int info_off)
{
    // the fewest CTAs whose shared memory holds the block (fewer flags to
    // exchange per column), at most one per SM, at least 4 rows per thread-pass
    const int64_t rows_fit = kSmemBytes / ((int64_t)w * (int64_t)sizeof(double));
    const int G = (int)std::max<int64_t>(1, std::min<int64_t>(c.h->grid, (m + rows_fit - 1) / rows_fit));
    const int64_t rows_per = (m + G - 1) / G;
    const size_t smem = (size_t)rows_per * w * sizeof(double);
    if (smem > (size_t)kSmemBytes) {
        set_error("panel of %lld rows x %d columns exceeds the on-chip capacity", (long long)m, w);
        return CHPL_ERR_UNSUPPORTED;
    }
    long long ldl = (long long)lda, ml = (long long)m, rp = (long long)rows_per, br = (long long)base_row;
    void* args[] = {&A, &ldl, &ml, &w, &rp, &ipiv, &br, &c.info, &info_off, &c.sync, &c.flags, &c.sbase, &c.cand,
                    &c.candrow, &c.toprow};
    CHPL_CUDA(cudaLaunchCooperativeKernel((const void*)panel_base_kernel, dim3(G), dim3(kPanelThreads), args, smem,
                                          c.st));
    c.sbase += (unsigned int)w;
    return CHPL_OK;
}

// ipiv entries of this node are relative to the node's top row + base_row
int rec(PanelCtx& c, double* A, int64_t lda, int64_t m, int64_t n, int64_t* ipiv, int64_t base_row, int info_off)
{
    // base width: the widest of 32 / 16 / 8 columns whose rows fit on chip
    const int64_t rows_sm = (m + c.h->grid - 1) / c.h->grid;
    const int bw = rows_sm * 32 * 8 <= kSmemBytes ? 32 : rows_sm * 16 * 8 <= kSmemBytes ? 16 : 8;
    if (n <= bw) return base_block(c, A, lda, m, (int)n, ipiv, base_row, info_off);
    int64_t n1 = ((n / 2) + bw - 1) / bw * bw;
    const int64_t n2 = n - n1;
    // left half
    CHPL_TRY(rec(c, A, lda, m, n1, ipiv, base_row, info_off));
    // its interchanges on the right half (pivots are relative to base_row)
    CHPL_TRY(laswp_plan(c.st, ipiv, 0, n1, c.plan, base_row));
    CHPL_TRY(laswp_apply(c.st, A, (size_t)lda, n1, n2, n1, c.plan));
    const double one = 1.0, mone = -1.0;
    if (cublasDtrsm_64(c.h->hb, CUBLAS_SIDE_LEFT, CUBLAS_FILL_MODE_LOWER, CUBLAS_OP_N, CUBLAS_DIAG_UNIT, n1, n2, &one, A,
                       lda, A + n1 * lda, lda) != CUBLAS_STATUS_SUCCESS) {
        set_error("panel: dtrsm failed");
        return CHPL_ERR_CUDA;
    }
    if (m > n1 &&
        cublasDgemm_64(c.h->hb, CUBLAS_OP_N, CUBLAS_OP_N, m - n1, n2, n1, &mone, A + n1, lda, A + n1 * lda, lda, &one,
                       A + n1 + n1 * lda, lda) != CUBLAS_STATUS_SUCCESS) {
        set_error("panel: dgemm failed");
        return CHPL_ERR_CUDA;
    }
    // right half (rows n1..m), pivots written relative to base_row + n1 -> shift to base_row
    CHPL_TRY(rec(c, A + n1 + n1 * lda, lda, m - n1, n2, ipiv + n1, base_row + n1, info_off + (int)n1));
    // its interchanges on the left half
    CHPL_TRY(laswp_plan(c.st, ipiv + n1, 0, n2, c.plan, base_row + n1));
    CHPL_TRY(laswp_apply(c.st, A + n1, (size_t)lda, 0, n1, n2, c.plan));
    return CHPL_OK;
}

}  // namespace

// Factor the m x n panel at A; ipiv[i] = base_row + (0-based pivot row within the panel).
int panel_getrf(cudaStream_t st, int64_t m, int64_t n, double* A, size_t lda, int64_t* ipiv, int64_t base_row, int* info,
                void* work)
{
    if (m < n || n <= 0 || (int64_t)lda < m) { set_error("panel_getrf: need m >= n > 0, lda >= m"); return CHPL_ERR_INVALID; }
    PanelHandles* h = nullptr;
    CHPL_TRY(handles(st, &h));
    uint8_t* w = static_cast<uint8_t*>(work);
    PanelCtx c;
    c.st = st;
    c.h = h;
    c.sync = reinterpret_cast<PanelSync*>(w);
    w += round_up(sizeof(PanelSync), 256);
    c.flags = reinterpret_cast<unsigned int*>(w);
    w += round_up(1024 * sizeof(unsigned int), 256);
    c.cand = reinterpret_cast<Cand*>(w);
    w += round_up(2 * 1024 * sizeof(Cand), 256);
    c.candrow = reinterpret_cast<double*>(w);
    w += round_up(2 * 1024 * kBaseW * sizeof(double), 256);
    c.toprow = reinterpret_cast<double*>(w);
    w += round_up(2 * kBaseW * sizeof(double), 256);
    c.plan = w;
    c.sbase = 0;
    c.info = info;
    CHPL_CUDA(cudaMemsetAsync(c.sync, 0, round_up(sizeof(PanelSync), 256) + 1024 * sizeof(unsigned int), st));
    return rec(c, A, (int64_t)lda, m, n, ipiv, base_row, 0);
}

int panel_status(void* work, int* err)
{
    PanelSync s;
    CHPL_CUDA(cudaMemcpy(&s, work, sizeof(s), cudaMemcpyDeviceToHost));
    *err = s.err;
    return CHPL_OK;
}

}  // namespace chpl

using namespace chpl;

extern "C" size_t chpl_panel_getrf_work_bytes(int64_t m, int64_t n) { return panel_work_bytes(m, n); }

extern "C" int chpl_panel_getrf_f64(void* stream, int64_t m, int64_t n, double* A, size_t lda, int64_t* ipiv, int* info,
                                    void* work)
{
    if (!work || !ipiv || !info) { set_error("panel_getrf: NULL argument"); return CHPL_ERR_INVALID; }
    CHPL_CUDA(cudaMemsetAsync(info, 0, sizeof(int), (cudaStream_t)stream));
    return panel_getrf((cudaStream_t)stream, m, n, A, lda, ipiv, 0, info, work);
}
