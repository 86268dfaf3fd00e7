// FP64 panel factorization with partial pivoting (getrf) of an m x n panel.
//
// Replaces the cusolverDnXgetrf call of src/chpl_single.cu:668-679.
// Recursive (left half, interchanges + U12 + Schur update, right half), down to
// base blocks of at most 32 columns.  A base block is factored by one
// cooperative kernel over up to all SMs (or the SMs a concurrent update leaves
// free: the base block then narrows to 16 / 8 / 4 columns until its rows fit
// those CTAs): every CTA keeps a contiguous range of the block's rows in
// shared memory, and the pivot of every column is found with one exchange
// between the CTAs:
//   * each CTA's candidate (largest |a| among its rows, smallest row on ties,
//     as LAPACK's idamax) is published as one record: value, row, the
//     candidate's whole row, and (CTA 0) the current diagonal row; then a
//     per-CTA flag is released;
//   * every CTA polls the flags, loads all records in the same round trip and
//     reduces them to the same pivot, so the pivot row and the row it
//     displaces arrive with the decision;
//   * after the interchange only column j+1 is updated before the next
//     candidates are published (the candidate row's other columns are updated
//     on the fly for its record); the update of columns j+2.. runs while the
//     exchange is in flight.
// Every element still receives exactly the operations of the unblocked
// right-looking algorithm (x = fma(-l, u, x), l = a * (1 / pivot)), in the
// same order.  Records and flags are double-buffered by column parity.
// The recursion's FP64 TRSM / GEMM steps run on this library's DMMA kernels
// (fp64.cu); interchanges use the device-built net permutation of
// hpl_kernels.cu.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "fp64.h"
#include "hpl.h"

namespace chpl {

constexpr int kBaseW = 32;          // widest base block (16 / 8 / 4 when the rows do not fit on chip)
constexpr int kMinBaseW = 4;
constexpr int kSmemBytes = 217600;  // shared memory of one base-kernel CTA (rows x width x 8 B)
constexpr int kMaxPanelCTAs = 1024;

struct PanelSync {
    int err;       // a wait ran out of time
    int pad[63];
};

// one CTA's candidate for one column
struct __align__(16) PanelRec {
    double val;            // |candidate|, -1 when the CTA has no row at or below the column
    long long row;         // its row (block-relative)
    double cand[kBaseW];   // the candidate's row, updated through the previous pivot
    double top[kBaseW];    // CTA 0: the diagonal row, updated through the previous pivot
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

__device__ __forceinline__ bool better(double v, long long r, double bv, long long br)
{
    return v > bv || (v == bv && r < br);
}

// Factor the m x w block at A (ld) in place, w <= W.  ipiv[j] = base_row +
// pivot row (block-relative).  info: 1-based column of the first exact zero
// pivot (+ info_off), left unchanged otherwise.
template <int W, int T>
__global__ void __launch_bounds__(T) panel_base_kernel(double* __restrict__ A, long long ld, long long m,
                                                                    int w, long long rows_per, int64_t* __restrict__ ipiv,
                                                                    long long base_row, int* __restrict__ info,
                                                                    int info_off, PanelSync* sync, unsigned int* flags,
                                                                    unsigned int sbase, PanelRec* recs)
{
    extern __shared__ double S[];  // column-major [W][rows_per]: conflict-free row-parallel access
    __shared__ double pv[W], tv[W];
    constexpr int kPanelWarps = T / 32;
    __shared__ double stage[kPanelWarps][W], stage_top[W];
    __shared__ double wv[kPanelWarps];
    __shared__ long long wr[kPanelWarps];
    __shared__ int wt[kPanelWarps];
    __shared__ long long pivrow;
    __shared__ double pivval;
    const int G = (int)gridDim.x;
    const long long r0 = (long long)blockIdx.x * rows_per;
    const long long r1 = min(m, r0 + rows_per);
    const int nr = (int)max(0LL, r1 - r0);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const long long kNone = 0x7fffffffffffffffLL;

    for (int e = tid; e < nr * w; e += blockDim.x) {
        const int i = e % nr, c = e / nr;
        S[c * rows_per + i] = A[(r0 + i) + (long long)c * ld];
    }
    __syncthreads();

    // Publish this CTA's candidate (bv, br: this thread's best) for column jc.
    // With upd, columns > jc of the published rows get pivot jc-1's update
    // (multiplier stored in column jc-1, pivot row in pv), which the rows in
    // shared memory receive only afterwards.
    auto publish = [&](int jc, double bv, long long br, bool upd) {
        for (int o = 16; o; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const long long orr = __shfl_xor_sync(0xffffffffu, br, o);
            if (better(ov, orr, bv, br)) { bv = ov; br = orr; }
        }
        __syncwarp();  // the lane that owns the warp's best row has written it
        if (bv >= 0.0 && lane < w) {
            const int i = (int)(br - r0);
            double x = S[lane * rows_per + i];
            if (upd && lane > jc) x = fma(-S[(jc - 1) * rows_per + i], pv[lane], x);
            stage[wid][lane] = x;
        }
        if (lane == 0) { wv[wid] = bv; wr[wid] = br; }
        if (blockIdx.x == 0 && wid == 0 && lane < w) {  // row jc lives in CTA 0, thread jc (warp 0)
            double x = S[lane * rows_per + jc];
            if (upd && lane > jc) x = fma(-S[(jc - 1) * rows_per + jc], pv[lane], x);
            stage_top[lane] = x;
        }
        __syncthreads();
        if (wid == 0) {
            double v = lane < kPanelWarps ? wv[lane] : -1.0;
            long long r = lane < kPanelWarps ? wr[lane] : kNone;
            int q = lane;
            for (int o = 16; o; o >>= 1) {  // full butterfly: every lane ends with the CTA's best
                const double ov = __shfl_xor_sync(0xffffffffu, v, o);
                const long long orr = __shfl_xor_sync(0xffffffffu, r, o);
                const int oq = __shfl_xor_sync(0xffffffffu, q, o);
                if (better(ov, orr, v, r)) { v = ov; r = orr; q = oq; }
            }
            // one writer: the record in program order, then the flag with release semantics
            // (no separate fence: a release store orders its own thread's earlier stores)
            if (lane == 0) {
                PanelRec* rec = recs + (size_t)(jc & 1) * G + blockIdx.x;
                if (v >= 0.0)
                    for (int c = 0; c < w; c += 2)
                        *reinterpret_cast<double2*>(&rec->cand[c]) = make_double2(stage[q][c], stage[q][c + 1]);
                if (blockIdx.x == 0)
                    for (int c = 0; c < w; c += 2)
                        *reinterpret_cast<double2*>(&rec->top[c]) = make_double2(stage_top[c], stage_top[c + 1]);
                *reinterpret_cast<double2*>(rec) = make_double2(v, __longlong_as_double(r));
                st_release(&flags[blockIdx.x], sbase + (unsigned int)jc + 1u);
            }
        }
    };

    {   // candidates of column 0
        double bv = -1.0;
        long long br = kNone;
        for (int i = tid; i < nr; i += blockDim.x) {
            const double v = fabs(S[i]);
            if (better(v, r0 + i, bv, br)) { bv = v; br = r0 + i; }
        }
        publish(0, bv, br, false);
    }

    for (int j = 0; j < w; ++j) {
        // ---- exchange: every CTA's record for column j ----
        double cr[W];
        double v = -1.0;
        long long r = kNone;
        int good = 1;
        const unsigned int want = sbase + (unsigned int)j + 1u;
        // bounded acquire-poll of CTA b's flag for column j
        auto poll = [&](int b) {
            const uint64_t t0 = globaltimer();
            uint32_t it = 0;
            while ((int)(ld_acquire(&flags[b]) - want) < 0) {
                if ((++it & 255u) == 0 && (*(volatile int*)&sync->err || globaltimer() - t0 > 1000000000ull)) {  // 1 s
                    atomicExch(&sync->err, 1);
                    return false;
                }
            }
            return true;
        };
        // threads [0, G) fetch the CTAs' records, threads [kTopT, kTopT + w) the diagonal
        // row from CTA 0's record, both at once
        constexpr int kTopT = T - W;
        if (tid < G) {
            good = poll(tid) ? 1 : 0;
            if (good) {  // the whole record in one round trip
                const PanelRec* rec = recs + (size_t)(j & 1) * G + tid;
                const double2 vr = __ldcg(reinterpret_cast<const double2*>(rec));
                v = vr.x;
                r = __double_as_longlong(vr.y);
                const double2* cp = reinterpret_cast<const double2*>(rec->cand);
#pragma unroll
                for (int c = 0; c < W / 2; ++c) {
                    const double2 x = 2 * c < w ? __ldcg(cp + c) : make_double2(0.0, 0.0);
                    cr[2 * c] = x.x;
                    cr[2 * c + 1] = x.y;
                }
            }
        }
        if (tid >= kTopT && tid - kTopT < w) {  // the diagonal row, one element per thread
            if (poll(0)) tv[tid - kTopT] = __ldcg(&(recs + (size_t)(j & 1) * G)->top[tid - kTopT]);
            else good = 0;
        }
        int t = tid;
        for (int o = 16; o; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, v, o);
            const long long orr = __shfl_xor_sync(0xffffffffu, r, o);
            const int ot = __shfl_xor_sync(0xffffffffu, t, o);
            if (better(ov, orr, v, r)) { v = ov; r = orr; t = ot; }
        }
        if (lane == 0) { wv[wid] = v; wr[wid] = r; wt[wid] = t; }
        if (!__syncthreads_and(good)) return;
        {
            double bv = wv[0];
            long long br = wr[0];
            int bt = wt[0];
            for (int q = 1; q < kPanelWarps; ++q)
                if (better(wv[q], wr[q], bv, br)) { bv = wv[q]; br = wr[q]; bt = wt[q]; }
            if (tid == bt) {
#pragma unroll
                for (int c = 0; c < W; ++c)
                    if (c < w) pv[c] = cr[c];
                pivrow = br;
                pivval = bv;
            }
        }
        __syncthreads();
        const long long p = pivrow;
        const double piv = pv[j];
        if (blockIdx.x == 0 && tid == 0) {
            ipiv[j] = base_row + p;
            if (pivval == 0.0 && *info == 0) *info = info_off + j + 1;
        }
        const double rp = (piv != 0.0) ? 1.0 / piv : 0.0;
        const bool next = j + 1 < w;
        // ---- interchange, scale column j, update column j+1 and find its candidates ----
        double bv = -1.0;
        long long br = kNone;
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
                if (next) x[(j + 1) * rows_per] = fma(-l, pv[j + 1], x[(j + 1) * rows_per]);
            }
            if (next && gr > j) {
                const double a = fabs(x[(j + 1) * rows_per]);
                if (better(a, gr, bv, br)) { bv = a; br = gr; }
            }
        }
        if (!next) break;
        publish(j + 1, bv, br, piv != 0.0);
        // ---- the rest of pivot j's update, while the exchange is in flight ----
        if (piv != 0.0 && j + 2 < w) {
            for (int i = tid; i < nr; i += blockDim.x) {
                if (r0 + i <= j) continue;
                double* x = &S[i];
                const double l = x[j * rows_per];
                for (int c = j + 2; c < w; ++c) x[c * rows_per] = fma(-l, pv[c], x[c * rows_per]);
            }
        }
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
    int grid = 0;
    int threads = 256;
    int min_rows = 0;
};

// the base kernel for block width w (<= 4, 8, 16, 32) and t threads (256 or 512)
static const void* base_kernel(int w, int t)
{
    if (t == 512)
        return w <= 4    ? (const void*)panel_base_kernel<4, 512>
               : w <= 8  ? (const void*)panel_base_kernel<8, 512>
               : w <= 16 ? (const void*)panel_base_kernel<16, 512>
                         : (const void*)panel_base_kernel<32, 512>;
    return w <= 4    ? (const void*)panel_base_kernel<4, 256>
           : w <= 8  ? (const void*)panel_base_kernel<8, 256>
           : w <= 16 ? (const void*)panel_base_kernel<16, 256>
                     : (const void*)panel_base_kernel<32, 256>;
}

static thread_local PanelHandles g_ph;

static int handles(cudaStream_t st, PanelHandles** out)
{
    int dev = 0;
    CHPL_CUDA(cudaGetDevice(&dev));
    if (g_ph.dev != dev) {
        g_ph = PanelHandles();
        int nsm = 0, per = 0;
        CHPL_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
        for (int t = 0; t < 2; ++t)
            for (int wi = 0; wi < 4; ++wi) {
                CHPL_CUDA(cudaFuncSetAttribute(base_kernel(4 << wi, 256 << t), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kSmemBytes));
                CHPL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, base_kernel(4 << wi, 256 << t), 256 << t,
                                                                        kSmemBytes));
                if (per < 1) { set_error("panel kernel does not fit on an SM"); return CHPL_ERR_UNSUPPORTED; }
            }
        g_ph.grid = nsm;  // one CTA per SM: co-resident by construction
        g_ph.dev = dev;
    }
    // tuning, read at every call: CTA size (CHPL_PANEL_THREADS 256 | 512) and the rows
    // a CTA is given at least (CHPL_PANEL_ROWS; 0: the fewest CTAs that hold the block).
    // Every element receives the same operations in the same order either way.
    const char* e = std::getenv("CHPL_PANEL_THREADS");
    g_ph.threads = (e && std::atoi(e) == 512) ? 512 : 256;
    e = std::getenv("CHPL_PANEL_ROWS");
    g_ph.min_rows = e ? std::max(0, std::atoi(e)) : 0;
    if (g_ph.min_rows > 0) g_ph.min_rows = std::max(g_ph.min_rows, 64);
    (void)st;
    *out = &g_ph;
    return CHPL_OK;
}

size_t panel_work_bytes(int64_t m, int64_t n)
{
    (void)m;
    const size_t G = kMaxPanelCTAs;  // upper bound on the grid
    return round_up(sizeof(PanelSync), 256) + round_up(G * sizeof(unsigned int), 256) +
           round_up(2 * G * sizeof(PanelRec), 256) + laswp_work_bytes(std::max<int64_t>(n, 1)) + 256;
}

namespace {

struct PanelCtx {
    cudaStream_t st;
    PanelHandles* h;
    PanelSync* sync;
    unsigned int* flags;
    PanelRec* recs;
    void* plan;
    unsigned int sbase;  // barrier arrivals so far in this call
    int cap;             // CTAs of a base kernel at most
    int* info;
    int* status;
};

int base_block(PanelCtx& c, double* A, int64_t lda, int64_t m, int w, int64_t* ipiv, int64_t base_row, int info_off)
{
    // the fewest CTAs whose shared memory holds the block (fewer flags to
    // exchange per column), or more when min_rows asks for smaller row ranges,
    // at most one per SM
    const int64_t rows_fit = kSmemBytes / ((int64_t)w * (int64_t)sizeof(double));
    int64_t want = (m + rows_fit - 1) / rows_fit;
    if (c.h->min_rows > 0) want = std::max<int64_t>(want, m / c.h->min_rows);
    // CTA 0 holds the block's top w rows (the diagonal rows the kernel reads from it)
    want = std::min<int64_t>(want, std::max<int64_t>(1, m / w));
    const int G = (int)std::max<int64_t>(1, std::min<int64_t>(c.cap, want));
    const int64_t rows_per = (m + G - 1) / G;
    const size_t smem = (size_t)rows_per * w * sizeof(double);
    const int T = c.h->threads;
    if (G > T - kBaseW) {   // the record fetchers and the diagonal-row fetchers must not overlap
        set_error("panel: %d CTAs exceed the exchange's %d record threads", G, T - kBaseW);
        return CHPL_ERR_UNSUPPORTED;
    }
    if (smem > (size_t)kSmemBytes) {
        set_error("panel of %lld rows x %d columns exceeds the on-chip capacity", (long long)m, w);
        return CHPL_ERR_UNSUPPORTED;
    }
    long long ldl = (long long)lda, ml = (long long)m, rp = (long long)rows_per, br = (long long)base_row;
    void* args[] = {&A, &ldl, &ml, &w, &rp, &ipiv, &br, &c.info, &info_off, &c.sync, &c.flags, &c.sbase, &c.recs};
    CHPL_CUDA(cudaLaunchCooperativeKernel(base_kernel(w, T), dim3(G), dim3(T), args, smem, c.st));
    c.sbase += (unsigned int)w;
    return CHPL_OK;
}

// ipiv entries of this node are relative to the node's top row + base_row
int rec(PanelCtx& c, double* A, int64_t lda, int64_t m, int64_t n, int64_t* ipiv, int64_t base_row, int info_off)
{
    // base width: the widest of 32 / 16 / 8 / 4 columns whose rows fit in the CTAs allowed
    const int64_t rows_sm = (m + c.cap - 1) / c.cap;
    int bw = kBaseW;
    while (bw > kMinBaseW && rows_sm * bw * (int64_t)sizeof(double) > kSmemBytes) bw /= 2;
    if (rows_sm * bw * (int64_t)sizeof(double) > kSmemBytes) {
        set_error("panel of %lld rows does not fit in the shared memory of %d CTAs", (long long)m, c.cap);
        return CHPL_ERR_UNSUPPORTED;
    }
    if (n <= bw) return base_block(c, A, lda, m, (int)n, ipiv, base_row, info_off);
    int64_t n1 = ((n / 2) + bw - 1) / bw * bw;
    const int64_t n2 = n - n1;
    // left half
    CHPL_TRY(rec(c, A, lda, m, n1, ipiv, base_row, info_off));
    // its interchanges on the right half (pivots are relative to base_row)
    CHPL_TRY(laswp_plan(c.st, ipiv, 0, n1, c.plan, base_row));
    CHPL_TRY(laswp_apply(c.st, A, (size_t)lda, n1, n2, n1, c.plan));
    // U12 = L11^-1 A12, then the Schur update A22 -= L21 U12
    CHPL_TRY(dtrsm_llnu(c.st, n1, n2, A, lda, A + n1 * lda, lda));
    if (m > n1) CHPL_TRY(dgemm(c.st, m - n1, n2, n1, -1.0, A + n1, lda, A + n1 * lda, lda, 1.0, A + n1 + n1 * lda, lda));
    // right half (rows n1..m), pivots written relative to base_row + n1 -> shift to base_row
    CHPL_TRY(rec(c, A + n1 + n1 * lda, lda, m - n1, n2, ipiv + n1, base_row + n1, info_off + (int)n1));
    // its interchanges on the left half
    CHPL_TRY(laswp_plan(c.st, ipiv + n1, 0, n2, c.plan, base_row + n1));
    CHPL_TRY(laswp_apply(c.st, A + n1, (size_t)lda, 0, n1, n2, c.plan));
    return CHPL_OK;
}

}  // namespace

// Factor the m x n panel at A; ipiv[i] = base_row + (0-based pivot row within the panel).
int panel_min_ctas(int64_t m)
{
    const int64_t rows_fit = kSmemBytes / (kMinBaseW * (int64_t)sizeof(double));
    return (int)std::max<int64_t>(1, (m + rows_fit - 1) / rows_fit);
}

int panel_getrf(cudaStream_t st, int64_t m, int64_t n, double* A, size_t lda, int64_t* ipiv, int64_t base_row, int* info,
                void* work, int max_ctas)
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
    w += round_up(kMaxPanelCTAs * sizeof(unsigned int), 256);
    c.recs = reinterpret_cast<PanelRec*>(w);
    w += round_up(2 * kMaxPanelCTAs * sizeof(PanelRec), 256);
    c.plan = w;
    c.sbase = 0;
    c.cap = max_ctas > 0 ? std::min(max_ctas, h->grid) : h->grid;
    c.info = info;
    CHPL_CUDA(cudaMemsetAsync(c.sync, 0, round_up(sizeof(PanelSync), 256) + kMaxPanelCTAs * sizeof(unsigned int), st));
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
