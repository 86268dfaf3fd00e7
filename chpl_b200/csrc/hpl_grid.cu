// Multi-GPU HPL on a P x Q process grid, one process per GPU (the chpl_p2
// path of the reference, src/chpl_p2.cu, rebuilt for B200 + NCCL).
//
// Layout: 2D block-cyclic with block NB; rank r has pr = r % P, qc = r / P
// (rank = P*qc + pr, src/chpl_p2.cu:528); global row block i lives on process
// row i % P, column block j on process column j % Q.  Each rank holds one
// column-major local array (lda = local rows rounded to 32).
//
// Per block column s (global columns [J, J+NB), J = s*NB; owner column
// qs = s % Q, diagonal owner row ps = s % P):
//   1. factor: the active rows of the block column are gathered onto
//      (ps, qs) (for P = 2 the other process row sends its rows over NVLink),
//      factored with exact partial pivoting (internal panels of width <= 1024,
//      this library's FP64 panel kernel, inner updates through the emulated
//      GEMM), then the factored rows are scattered back to their owners.
//   2. pivots go to every rank (ncclBroadcast on the world communicator);
//      inv(L11) and W = L21 go along process rows (row communicator).
//   3. interchanges of the trailing columns: moves inside a rank are a local
//      gather/scatter, moves across process rows an ncclSend/Recv pair on the
//      column communicator.
//   4. U12 = inv(L11) * A12 on process row ps (emulated GEMM, in place), then
//      broadcast down the process columns (column communicator).
//   5. A22 -= W * U12 locally (emulated GEMM).
// Back substitution is distributed (per block: ncclReduce of partial sums on
// the owning process row, trsv by the diagonal owner, ncclBroadcast of x_j on
// the owning process column); the residual regenerates A locally and reduces
// over process rows.  Communicators come from one unique id and
// ncclCommSplit; a host watchdog aborts them (ncclCommAbort) if a step does
// not finish within the configured timeout.
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cinttypes>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <thread>
#include <vector>

#include "common.cuh"
#include "fp64.h"
#include "hpl.h"
#include "oz2.h"

namespace chpl {

#define CHPL_NCCL(call)                                                                                   \
    do {                                                                                                  \
        ncclResult_t r_ = (call);                                                                         \
        if (r_ != ncclSuccess) {                                                                          \
            set_error("NCCL error %d (%s) in %s at %s:%d", (int)r_, ncclGetErrorString(r_), #call, __FILE__, \
                      __LINE__);                                                                          \
            return CHPL_ERR_NCCL;                                                                         \
        }                                                                                                 \
    } while (0)

// ---------------------------------------------------------------------------- kernels
__global__ void rows_gather_kernel(double* __restrict__ dst, long long ldd, const double* __restrict__ A, long long lda,
                                   const int* __restrict__ rows, int nrows, long long ncols)
{
    const long long total = (long long)nrows * ncols;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(e % nrows);
        const long long c = e / nrows;
        dst[t + c * ldd] = A[rows[t] + c * lda];
    }
}

__global__ void rows_scatter_kernel(double* __restrict__ A, long long lda, const double* __restrict__ src, long long lds,
                                    const int* __restrict__ rows, int nrows, long long ncols)
{
    const long long total = (long long)nrows * ncols;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(e % nrows);
        const long long c = e / nrows;
        A[rows[t] + c * lda] = src[t + c * lds];
    }
}

// Gathered panel row r (global J + r) <-> its owner's local row.  dir = 0:
// G <- (own A | partner's packed rows R); dir = 1: (own A | S for the
// partner) <- G.  Owner of global row g: (g / NB) % P; its local row
// (g / NB / P) * NB + g % NB; its first active local row lrb[p].
__global__ void panel_shuffle_kernel(double* __restrict__ G, long long ldg, long long mg, long long ncols, long long J,
                                     long long NB, int P, int me, double* __restrict__ Aown, long long lda,
                                     long long lrb_me, double* __restrict__ R, long long ldr, long long lrb_other, int dir)
{
    const long long total = mg * ncols;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const long long r = e % mg, c = e / mg;
        const long long g = J + r, b = g / NB;
        const int p = (int)(b % P);
        const long long l = (b / P) * NB + g % NB;
        double* src = (p == me) ? &Aown[(l - lrb_me) + c * lda] : &R[(l - lrb_other) + c * ldr];
        if (dir == 0) G[r + c * ldg] = *src;
        else *src = G[r + c * ldg];
    }
}

__global__ void axpby_rows_kernel(double* __restrict__ v, const double* __restrict__ b, const double* __restrict__ t,
                                  int n, int use_b)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = (use_b ? b[i] : 0.0) - t[i];
}

__device__ __forceinline__ double grid_elem(uint64_t seed, uint64_t idx)
{
    uint64_t z = (idx + 1ull) * 0x9E3779B97F4A7C15ull + seed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z = z ^ (z >> 31);
    return (double)(z >> 11) * (1.0 / 9007199254740992.0) - 0.5;
}

// partial A x and row |A| sums over this rank's local columns (global < N),
// chunked over columns for a deterministic two-stage sum
constexpr int kGridResChunks = 16;
__global__ void __launch_bounds__(256) grid_resid_partial_kernel(long long N, long long NB, int P, int Q, int pr, int qc,
                                                                 long long mloc, long long nloc, uint64_t seed,
                                                                 const double* __restrict__ x, double* __restrict__ part)
{
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const int ch = blockIdx.y;
    if (i >= mloc) return;
    const long long gi = (i / NB * P + pr) * NB + i % NB;
    const long long per = (nloc + kGridResChunks - 1) / kGridResChunks;
    const long long c0 = ch * per, c1 = min(nloc, c0 + per);
    double ax = 0.0, rs = 0.0;
    for (long long c = c0; c < c1; ++c) {
        const long long gc = (c / NB * Q + qc) * NB + c % NB;
        if (gc >= N) continue;
        const double a = grid_elem(seed, (uint64_t)gi * (uint64_t)(N + 1) + (uint64_t)gc);
        ax = fma(a, x[gc], ax);
        rs += fabs(a);
    }
    part[(ch * 2 + 0) * mloc + i] = ax;
    part[(ch * 2 + 1) * mloc + i] = rs;
}

__global__ void grid_resid_sum_kernel(long long mloc, const double* __restrict__ part, double* __restrict__ axrs)
{
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= mloc) return;
    double ax = 0.0, rs = 0.0;
    for (int c = 0; c < kGridResChunks; ++c) {
        ax += part[(c * 2 + 0) * mloc + i];
        rs += part[(c * 2 + 1) * mloc + i];
    }
    axrs[i] = ax;
    axrs[mloc + i] = rs;
}

// per local row: |ax - b|, rs, |b| maxima into out[blk*3 + {0,1,2}]
__global__ void __launch_bounds__(256) grid_resid_max_kernel(long long N, long long NB, int P, int pr, long long mloc,
                                                             uint64_t seed, const double* __restrict__ axrs,
                                                             double* __restrict__ out)
{
    __shared__ double sm[3][256];
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    double r = 0.0, rs = 0.0, ba = 0.0;
    if (i < mloc) {
        const long long gi = (i / NB * P + pr) * NB + i % NB;
        const double b = grid_elem(seed, (uint64_t)gi * (uint64_t)(N + 1) + (uint64_t)N);
        r = fabs(axrs[i] - b);
        rs = axrs[mloc + i];
        ba = fabs(b);
    }
    sm[0][threadIdx.x] = r; sm[1][threadIdx.x] = rs; sm[2][threadIdx.x] = ba;
    __syncthreads();
    for (int o = 128; o; o >>= 1) {
        if (threadIdx.x < o)
            for (int q = 0; q < 3; ++q) sm[q][threadIdx.x] = fmax(sm[q][threadIdx.x], sm[q][threadIdx.x + o]);
        __syncthreads();
    }
    if (threadIdx.x < 3) out[blockIdx.x * 3 + threadIdx.x] = sm[threadIdx.x][0];
}

static inline int grid1(long long work)
{
    long long g = (work + 255) / 256;
    return (int)std::max(1LL, std::min(g, 148LL * 32));
}

// ---------------------------------------------------------------------------- communicator handle
struct GridComm {
    int P = 1, Q = 1, rank = 0, pr = 0, qc = 0, dev = 0;
    ncclComm_t world = nullptr, row = nullptr, col = nullptr;
    ncclComm_t col2 = nullptr;   // second process-column communicator: the bulk exchanges of the lookahead
    double timeout_s = 300.0;
    bool aborted = false;
};

// abort every communicator of the grid (a rank stopped answering)
static void abort_comms(GridComm* g)
{
    if (g->aborted) return;
    for (ncclComm_t* c : {&g->row, &g->col, &g->col2, &g->world})
        if (*c) ncclCommAbort(*c);
    g->row = g->col = g->col2 = g->world = nullptr;
    g->aborted = true;
}

// Wait for `st` with a host-side limit; on expiry abort the communicators so
// that every rank's pending collectives end with an error instead of hanging.
static int watchdog_sync(GridComm* g, cudaStream_t st, const char* what)
{
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        cudaError_t e = cudaStreamQuery(st);
        if (e == cudaSuccess) return CHPL_OK;
        if (e != cudaErrorNotReady) return cuda_fail(e, what, __FILE__, __LINE__);
        ncclResult_t ae = ncclSuccess;
        if (g->world) ncclCommGetAsyncError(g->world, &ae);
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (ae != ncclSuccess || el > g->timeout_s) {
            abort_comms(g);
            set_error("%s: %s after %.1f s; communicators aborted", what,
                      ae != ncclSuccess ? "NCCL asynchronous error" : "timeout", el);
            return ae != ncclSuccess ? CHPL_ERR_NCCL : CHPL_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}


static bool getenv_flag(const char* name)
{
    const char* v = std::getenv(name);
    return v && *v && std::strcmp(v, "0") != 0;
}

// watchdog_sync for one event of a stream (the host may run ahead of it)
static int watchdog_event(GridComm* g, cudaEvent_t ev, const char* what)
{
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return CHPL_OK;
        if (e != cudaErrorNotReady) return cuda_fail(e, what, __FILE__, __LINE__);
        ncclResult_t ae = ncclSuccess;
        if (g->world) ncclCommGetAsyncError(g->world, &ae);
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (ae != ncclSuccess || el > g->timeout_s) {
            abort_comms(g);
            set_error("%s: %s after %.1f s; communicators aborted", what,
                      ae != ncclSuccess ? "NCCL asynchronous error" : "timeout", el);
            return ae != ncclSuccess ? CHPL_ERR_NCCL : CHPL_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// ---------------------------------------------------------------------------- interchange planning
// Net effect of the swaps (J+i <-> J+piv[i]), i = 0..K-1 in order, as row
// moves "dst receives the old contents of src", split for process row pr of P:
// moves inside this process row (local indices lsrc -> ldst), rows it sends
// (snd, local source rows) and rows it receives (rcv, local destination rows).
// Moves are listed in increasing destination order on every rank, so the
// partner's receive list pairs with this rank's send list element by element.
static void plan_exchange(int64_t J, int64_t K, const int64_t* piv, int64_t NB, int P, int pr, std::vector<int>& lsrc,
                          std::vector<int>& ldst, std::vector<int>& snd, std::vector<int>& rcv)
{
    std::map<int64_t, int64_t> occ;  // position -> original row now there
    auto get = [&](int64_t p) { auto it = occ.find(p); return it == occ.end() ? p : it->second; };
    for (int64_t i = 0; i < K; ++i) {
        const int64_t a = J + i, b = J + piv[i];
        if (a == b) continue;
        const int64_t va = get(a), vb = get(b);
        occ[a] = vb;
        occ[b] = va;
    }
    auto owner = [&](int64_t gr) { return (int)((gr / NB) % P); };
    auto local = [&](int64_t gr) { return (int)((gr / NB / P) * NB + gr % NB); };
    lsrc.clear(); ldst.clear(); snd.clear(); rcv.clear();
    for (auto& kv : occ) {
        const int64_t dst = kv.first, src = kv.second;
        if (dst == src) continue;
        const int od = owner(dst), os = owner(src);
        if (od == pr && os == pr) { ldst.push_back(local(dst)); lsrc.push_back(local(src)); }
        else if (os == pr) snd.push_back(local(src));
        else if (od == pr) rcv.push_back(local(dst));
    }
}

// ---------------------------------------------------------------------------- emulated GEMM helper
struct Emu {
    int L = 11;
    const oz2::Moduli* M = nullptr;
    void* work = nullptr;   // B part + scratch + split temporaries
    int64_t chunk = 32768;
    int grid_cap = 0;       // > 0: persistent GEMM grid limit (SMs left to concurrent communication)
    bool fp64 = false;      // CHPL2D_G8=0: the update runs as an FP64 DGEMM (src/chpl_p2.cu:1697-1700)
    int64_t launches = 0, gemm_n = 0;
    double ops = 0.0, flops = 0.0, kernel_s = 0.0;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;

    // C (m x n) = alpha * A (m x k) * B (k x n) + beta * C; residues of A in wa
    // (computed here when split_a).  C may alias B when beta == 0.
    int run(cudaStream_t st, void* wa, bool split_a, int64_t m, int64_t n, int64_t k, const double* A, int64_t lda,
            const double* B, int64_t ldb, double* C, int64_t ldc, double alpha, double beta)
    {
        if (m <= 0 || n <= 0 || k <= 0) return CHPL_OK;
        if (fp64) {   // C must not alias B here: the FP64 U12 step goes through u12_fp64
            CHPL_TRY(dgemm(st, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc));
            ++launches;
            flops += 2.0 * (double)m * (double)n * (double)k;
            return CHPL_OK;
        }
        for (int64_t c = 0; c < n;) {
            int64_t w = std::min(chunk, n - c);
            if (n - c - w > 0 && n - c - w < 1024) w = n - c;
            const oz2::Layout y = oz2::layout((size_t)m, (size_t)w, (size_t)k, L, true, false, grid_cap);
            uint8_t* pa = static_cast<uint8_t*>(wa);
            uint8_t* pb = static_cast<uint8_t*>(work) + y.b_off;
            int32_t* shA = reinterpret_cast<int32_t*>(pa + y.a_shift);
            int8_t* resA = reinterpret_cast<int8_t*>(pa + y.a_res);
            int32_t* shB = reinterpret_cast<int32_t*>(pb + y.b_shift);
            int8_t* resB = reinterpret_cast<int8_t*>(pb + y.b_res);
            void* tmp = static_cast<uint8_t*>(work) + y.tmp_off;
            if (split_a && c == 0) {
                CHPL_TRY(oz2::split(st, false, A, (size_t)lda, (size_t)m, (size_t)k, L, M->alpha, resA, y.mPad, y.kPad, shA, tmp));
                launches += 4;
            }
            CHPL_TRY(oz2::split(st, true, B + c * ldb, (size_t)ldb, (size_t)w, (size_t)k, L, M->beta, resB, y.nPad, y.kPad,
                                shB, tmp));
            cudaEvent_t e0, e1;
            cudaEventCreate(&e0);
            cudaEventCreate(&e1);
            cudaEventRecord(e0, st);
            CHPL_TRY(oz2::gemm_launch(st, 0, (size_t)m, (size_t)w, y.kPad, L, resA, y.mPad, resB, y.nPad, shA, shB, alpha,
                                      beta, C + c * ldc, (size_t)ldc, nullptr, 0,
                                      reinterpret_cast<int8_t*>(static_cast<uint8_t*>(work) + y.scratch_off), y.grid_max));
            cudaEventRecord(e1, st);
            ev.push_back({e0, e1});
            launches += 2;
            ++gemm_n;
            ops += 2.0 * (double)m * (double)w * (double)y.kPad * L;
            flops += 2.0 * (double)m * (double)w * (double)k;
            c += w;
        }
        return CHPL_OK;
    }

    // residues of A (m x k) into wa, the layout run() reads with split_a = false
    int split_only(cudaStream_t st, void* wa, int64_t m, int64_t k, const double* A, int64_t lda)
    {
        if (m <= 0 || k <= 0 || fp64) return CHPL_OK;
        const oz2::Layout y = oz2::layout((size_t)m, 256, (size_t)k, L, true, false, grid_cap);
        uint8_t* pa = static_cast<uint8_t*>(wa);
        CHPL_TRY(oz2::split(st, false, A, (size_t)lda, (size_t)m, (size_t)k, L, M->alpha,
                            reinterpret_cast<int8_t*>(pa + y.a_res), y.mPad, y.kPad, reinterpret_cast<int32_t*>(pa + y.a_shift),
                            static_cast<uint8_t*>(work) + y.tmp_off));
        launches += 4;
        return CHPL_OK;
    }

    void collect()
    {
        for (auto& p : ev) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, p.first, p.second) == cudaSuccess) kernel_s += ms * 1e-3;
            cudaEventDestroy(p.first);
            cudaEventDestroy(p.second);
        }
        ev.clear();
    }
};

// ---------------------------------------------------------------------------- per-phase stream time
// Busy time of one stream between two events, summed per phase (the indices
// of chpl_hpl_result.phase_s: 0 panel, 1 interchanges, 2 U12, 3 split of W,
// 4 update, 6 back substitution, 7 broadcasts).  Streams overlap, so the
// phases of a lookahead step add up to more than its wall time.
struct PhaseEvents {
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> recs;
    cudaEvent_t begin(cudaStream_t s)
    {
        cudaEvent_t e = nullptr;
        if (cudaEventCreate(&e) == cudaSuccess) cudaEventRecord(e, s);
        return e;
    }
    void end(cudaStream_t s, int ph, cudaEvent_t e0)
    {
        cudaEvent_t e1 = nullptr;
        if (!e0 || cudaEventCreate(&e1) != cudaSuccess) return;
        cudaEventRecord(e1, s);
        recs.push_back({ph, {e0, e1}});
    }
    void collect(double* out)
    {
        for (auto& r : recs) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, r.second.first, r.second.second) == cudaSuccess) out[r.first] += ms * 1e-3;
            cudaEventDestroy(r.second.first);
            cudaEventDestroy(r.second.second);
        }
        recs.clear();
    }
    ~PhaseEvents() { collect(sink); }
    double sink[8] = {0, 0, 0, 0, 0, 0, 0, 0};
};

// ---------------------------------------------------------------------------- grid solver
struct GridSolver {
    GridComm* g = nullptr;
    chpl_hpl_config cfg{};
    int64_t N = 0, NB = 0, NBp = 0, mloc = 0, nloc = 0, lda = 0, nblk = 0;
    cudaStream_t st = nullptr;
    double* A = nullptr;
    double* arena = nullptr;       // factor phase: gathered panel, pack buffer, inner residues; update phase: W, U12, W residues
    size_t arena_elems = 0;
    void* wres = nullptr;          // residues of W (A part), inside the arena
    void* win = nullptr;           // residues of inner-update L21 (A part), inside the arena
    double* linv = nullptr;        // inv(L11)
    double* linv2 = nullptr;       // second inv(L11) slot (lookahead)
    int64_t* piv2 = nullptr;       // second pivot slot (lookahead)
    void* plan2 = nullptr;         // interchange plans of the trailing columns (lookahead), kPlanSwaps swaps each
    static constexpr int64_t kPlanSwaps = 2048;    // swaps one device plan holds
    static constexpr int64_t kPlanChunks = 8;      // NB <= 16384
    cudaStream_t sm = nullptr;     // communication stream (lookahead)
    bool la = false;               // P = 1 depth-1 lookahead schedule
    bool la2 = false;              // P = 2 depth-1 lookahead schedule
    cudaStream_t sb = nullptr;     // bulk communication stream (P = 2 lookahead)
    double* Wd = nullptr;          // two W slots of mloc x NB; together the gathered panel (P = 2 lookahead)
    double* pk = nullptr;          // pack buffer of the gather / scatter, kPackCols columns
    double* Ub = nullptr;          // U12 of the bulk columns (K x nloc)
    double* Uu = nullptr;          // two slots of U12 of the urgent block (K x NB each)
    int64_t* hpiv = nullptr;       // pinned host copies of the two pivot slots
    int* hlist = nullptr;          // pinned staging of the two exchange-list slots
    cudaEvent_t evPk = nullptr;    // the chain partner's unpack has read the pack buffer
    static constexpr int64_t kPackCols = 512;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> panel_ev;
    void* wlinv = nullptr;         // its residues
    double* xch = nullptr;         // exchange buffers (3 x 2 NB x kXchCols)
    int* dlist = nullptr;          // device copies of exchange row lists
    int* dlist2 = nullptr;         // second list slot (P = 2 lookahead)
    int64_t* piv = nullptr;        // pivots of the current block column (relative to J)
    int* info = nullptr;
    void* pwork = nullptr;
    void* plan = nullptr;
    double* x = nullptr;           // solution (N)
    double* tsum = nullptr;        // back-substitution partial sums (mloc)
    double* vbuf = nullptr;        // NB
    Emu emu;
    int64_t n_launch = 0;
    double phase[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    PhaseEvents pev;               // stream-busy phases of the lookahead schedules and the back substitution
    static constexpr int64_t kXchCols = 4096;

    // the two W slots (mloc x NB each) and the gathered panel ((N - J) x NB at most) share Wd
    size_t wd_elems() const { return (size_t)std::max<int64_t>(2 * mloc, N) * (size_t)NB; }

    int owner_row(int64_t gr) const { return (int)((gr / NB) % g->P); }
    int64_t local_row(int64_t gr) const { return (gr / NB / g->P) * NB + gr % NB; }
    int root_of(int p, int q) const { return g->P * q + p; }

    int init(GridComm* gc, const chpl_hpl_config& c)
    {
        g = gc;
        cfg = c;
        N = c.N;
        NB = std::min<int64_t>(c.NB, N);
        // internal panel width of the block factorization: 1024, or 512 on two process rows (the
        // gathered panel's inner-update residues then take half the memory)
        NBp = std::min<int64_t>(NB, c.agg > 0 ? std::max<int64_t>(1, NB / c.agg) : (gc->P > 1 ? 512 : 1024));
        nblk = (N + NB - 1) / NB;
        mloc = local_extent(N, NB, g->P, g->pr);
        nloc = local_extent(N + 1, NB, g->Q, g->qc);
        lda = (int64_t)round_up((size_t)std::max<int64_t>(mloc, 1), 32);
        int lo = 0, hi = 0;
        CHPL_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
        CHPL_CUDA(cudaStreamCreateWithPriority(&st, cudaStreamNonBlocking, hi));
        const unsigned L = (unsigned)cfg.moduli;
        emu.L = (int)L;
        emu.M = oz2::moduli(cfg.moduli);
        if (!emu.M) { set_error("moduli must be in [2, 16]"); return CHPL_ERR_INVALID; }
        emu.chunk = cfg.chunk > 0 ? cfg.chunk : 32768;
        // sizes
        const size_t bytesA = (size_t)lda * (size_t)nloc * 8;
        const size_t g_elems = (g->P > 1) ? (size_t)N * NB + (size_t)(mloc + NB) * NB : 0;  // gathered panel + pack
        const size_t wu_elems = (size_t)mloc * NB + (size_t)NB * nloc;                       // W + U12
        size_t tot = 0, wa = 0, wb = 0, tin = 0, ain = 0, bin = 0, tl = 0, al = 0, bl = 0;
        const int64_t mmax = std::max<int64_t>(std::max(mloc, (g->P > 1) ? N : mloc), NB);
        CHPL_TRY(chpl_oz2_worksize((size_t)mloc, (size_t)std::min<int64_t>(emu.chunk + 1024, std::max<int64_t>(nloc, 1)),
                                   (size_t)NB, L, 1, 0, &tot, &wa, &wb));
        CHPL_TRY(chpl_oz2_worksize((size_t)mmax, (size_t)NB, (size_t)NBp, L, 1, 0, &tin, &ain, &bin));
        CHPL_TRY(chpl_oz2_worksize((size_t)NB, 256, (size_t)NB, L, 1, 0, &tl, &al, &bl));
        const size_t work_bytes = std::max(tot - wa, tin - ain);
        const size_t xch_bytes = (size_t)3 * 2 * NB * kXchCols * 8;
        size_t freeB = 0, totB = 0;
        CHPL_CUDA(cudaMemGetInfo(&freeB, &totB));
        // one arena, two phases that never overlap: factor = [gathered panel | pack | inner-update residues],
        // update = [W | U12 | residues of W]
        const size_t g_bytes = round_up(g_elems * 8, 256), wu_bytes = round_up(wu_elems * 8, 256);
        // the FP64 update (CHPL2D_G8=0) runs the serial block steps: the lookahead schedules release
        // W's FP64 copy as soon as its int8 residues exist
        emu.fp64 = !cfg.emulate;
        la = cfg.emulate && g->P == 1 && g->Q > 1 && !getenv_flag("CHPL_GRID_SERIAL");
        if (cfg.emulate && g->P == 2 && !getenv_flag("CHPL_GRID_SERIAL")) {
            // P = 2 lookahead: W slots (also the gathered panel), W residues, inner-update residues,
            // bulk and urgent U12, pack buffer; used instead of the arena
            const size_t wd = round_up(wd_elems() * 8, 256);
            const size_t need2 = bytesA + wd + wa + ain + round_up((size_t)NB * nloc * 8, 256) +
                                 (size_t)2 * NB * NB * 8 + (size_t)(mloc + NB) * kPackCols * 8 + (size_t)2 * NB * NB * 8 +
                                 al + xch_bytes + work_bytes + panel_work_bytes(mmax, NBp) + (size_t)N * 8 * 2 +
                                 (size_t)mloc * 8 + ((size_t)1024 << 20);
            // every rank must take the same schedule: the lookahead only if it fits on all of them
            int fits = need2 <= freeB ? 1 : 0;
            int* dfit = nullptr;
            CHPL_CUDA(cudaMalloc((void**)&dfit, sizeof(int)));
            CHPL_CUDA(cudaMemcpyAsync(dfit, &fits, sizeof(int), cudaMemcpyHostToDevice, st));
            if (ncclAllReduce(dfit, dfit, 1, ncclInt, ncclMin, g->world, st) != ncclSuccess) {
                cudaFree(dfit);
                set_error("schedule agreement failed");
                return CHPL_ERR_NCCL;
            }
            CHPL_CUDA(cudaMemcpyAsync(&fits, dfit, sizeof(int), cudaMemcpyDeviceToHost, st));
            const int wrc = watchdog_sync(g, st, "schedule agreement");
            cudaFree(dfit);
            if (wrc != CHPL_OK) return wrc;
            la2 = fits == 1;
            if (cfg.verbose && g->rank == 0)
                std::printf("GRID LOOKAHEAD PLAN (rank 0): %.2f GiB of %.2f GiB free -> %s\n", need2 / 1073741824.0,
                            freeB / 1073741824.0, la2 ? "lookahead" : "serial steps");
        }
        // lookahead: the factor of block s+1 (inner residues) runs while W_s's residues are live
        const size_t arena_bytes = la ? wu_bytes + wa + ain : std::max(g_bytes + ain, wu_bytes + wa);
        arena_elems = arena_bytes / 8;
        const size_t need = bytesA + arena_bytes + (size_t)NB * NB * 8 + al + xch_bytes + work_bytes +
                            panel_work_bytes(mmax, NBp) + (size_t)N * 8 * 2 + (size_t)mloc * 8 + ((size_t)768 << 20);
        if (cfg.verbose && g->rank == 0)
            std::printf("GRID MEM PLAN (rank 0): local %lld x %lld, matrix %.2f GiB, total %.2f GiB of %.2f GiB free\n",
                        (long long)mloc, (long long)nloc, bytesA / 1073741824.0, need / 1073741824.0, freeB / 1073741824.0);
        if (!la2 && need > freeB) {
            set_error("grid memory plan: need %.2f GiB, %.2f GiB free (reduce N)", need / 1073741824.0, freeB / 1073741824.0);
            return CHPL_ERR_WORKSPACE;
        }
        CHPL_CUDA(cudaMalloc((void**)&A, std::max<size_t>(bytesA, 8)));
        if (la2) {
            CHPL_CUDA(cudaMalloc((void**)&Wd, wd_elems() * 8));
            CHPL_CUDA(cudaMalloc(&wres, wa));
            CHPL_CUDA(cudaMalloc(&win, ain));
            CHPL_CUDA(cudaMalloc((void**)&Ub, std::max<size_t>((size_t)NB * nloc * 8, 256)));
            CHPL_CUDA(cudaMalloc((void**)&Uu, (size_t)2 * NB * NB * 8));
            CHPL_CUDA(cudaMalloc((void**)&pk, (size_t)(mloc + NB) * kPackCols * 8));
            CHPL_CUDA(cudaMallocHost((void**)&hpiv, (size_t)2 * NB * sizeof(int64_t)));
            CHPL_CUDA(cudaMallocHost((void**)&hlist, (size_t)2 * 8 * NB * sizeof(int)));
            CHPL_CUDA(cudaEventCreateWithFlags(&evPk, cudaEventDisableTiming));
            CHPL_CUDA(cudaStreamCreateWithPriority(&sm, cudaStreamNonBlocking, hi));
            CHPL_CUDA(cudaStreamCreateWithPriority(&sb, cudaStreamNonBlocking, hi));
            CHPL_CUDA(cudaMalloc((void**)&linv2, (size_t)NB * NB * 8));
            CHPL_CUDA(cudaMalloc((void**)&piv2, (size_t)NB * sizeof(int64_t)));
            CHPL_CUDA(cudaMalloc((void**)&dlist2, (size_t)4 * 2 * NB * sizeof(int)));
            const char* rs = std::getenv("CHPL_GRID_RESERVE_SMS");
            const int reserve = (rs && *rs) ? std::atoi(rs) : (cfg.reserve_sms >= 0 ? cfg.reserve_sms : 16);
            if (reserve > 0) emu.grid_cap = std::max(1, oz2::num_sms() - reserve);
        }
        CHPL_CUDA(cudaMalloc((void**)&arena, la2 ? 256 : std::max<size_t>(arena_bytes, 256)));
        if (!la2) {
            win = reinterpret_cast<uint8_t*>(arena) + (la ? wu_bytes + wa : g_bytes);
            wres = reinterpret_cast<uint8_t*>(arena) + wu_bytes;
        }
        if (la) {
            CHPL_CUDA(cudaStreamCreateWithPriority(&sm, cudaStreamNonBlocking, hi));
            CHPL_CUDA(cudaMalloc((void**)&linv2, (size_t)NB * NB * 8));
            CHPL_CUDA(cudaMalloc((void**)&piv2, (size_t)NB * sizeof(int64_t)));
            CHPL_CUDA(cudaMalloc(&plan2, kPlanChunks * round_up(laswp_work_bytes(kPlanSwaps), 256)));
            // SMs the persistent GEMM leaves to the communication stream's kernels
            const char* rs = std::getenv("CHPL_GRID_RESERVE_SMS");
            const int reserve = (rs && *rs) ? std::atoi(rs) : (cfg.reserve_sms >= 0 ? cfg.reserve_sms : 8);
            if (reserve > 0) emu.grid_cap = std::max(1, oz2::num_sms() - reserve);
        }
        CHPL_CUDA(cudaMalloc((void**)&linv, (size_t)NB * NB * 8));
        CHPL_CUDA(cudaMalloc(&wlinv, al));
        CHPL_CUDA(cudaMalloc((void**)&xch, xch_bytes));
        CHPL_CUDA(cudaMalloc((void**)&dlist, (size_t)4 * 2 * NB * sizeof(int)));
        CHPL_CUDA(cudaMalloc((void**)&piv, (size_t)NB * sizeof(int64_t)));
        CHPL_CUDA(cudaMalloc((void**)&info, 16 * sizeof(int)));
        CHPL_CUDA(cudaMemset(info, 0, 16 * sizeof(int)));
        CHPL_CUDA(cudaMalloc(&pwork, panel_work_bytes(mmax, NBp)));
        CHPL_CUDA(cudaMalloc(&plan, laswp_work_bytes(NBp)));
        CHPL_CUDA(cudaMalloc(&emu.work, work_bytes));
        CHPL_CUDA(cudaMalloc((void**)&x, (size_t)N * 8));
        CHPL_CUDA(cudaMalloc((void**)&tsum, (size_t)std::max<int64_t>(mloc, 1) * 8));
        CHPL_CUDA(cudaMalloc((void**)&vbuf, (size_t)NB * 8 * 2));
        return CHPL_OK;
    }

    // streams drained within a few seconds (false: work is stuck behind an aborted peer)
    bool streams_idle(double limit_s)
    {
        const auto t0 = std::chrono::steady_clock::now();
        for (cudaStream_t x : {st, sm, sb}) {
            if (!x) continue;
            while (cudaStreamQuery(x) == cudaErrorNotReady) {
                if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit_s) return false;
                std::this_thread::sleep_for(std::chrono::milliseconds(1));
            }
        }
        return true;
    }

    void destroy()
    {
        if (g && g->aborted && !streams_idle(10.0)) return;   // leave the memory to process exit rather than hang
        emu.collect();
        void* ps[] = {A, arena, linv, wlinv, xch, dlist, piv, info, pwork, plan, emu.work, x, tsum, vbuf, linv2, piv2, plan2,
                      Wd, Ub, Uu, pk, dlist2};
        for (void* p : ps)
            if (p) cudaFree(p);
        if (la2) {
            if (wres) cudaFree(wres);
            if (win) cudaFree(win);
        }
        if (hpiv) cudaFreeHost(hpiv);
        if (hlist) cudaFreeHost(hlist);
        if (evPk) cudaEventDestroy(evPk);
        if (sb) cudaStreamDestroy(sb);
        for (auto& e : panel_ev) {
            cudaEventDestroy(e.first);
            cudaEventDestroy(e.second);
        }
        panel_ev.clear();
        if (sm) cudaStreamDestroy(sm);
        if (st) cudaStreamDestroy(st);
    }

    // A12 (K x n, ld lda) = inv(L11) A12 in FP64: the product goes to T (K x n,
    // ld K) and is copied back, since a DGEMM must not write its own input
    int u12_fp64(int64_t K, int64_t n, double* A12, double* T)
    {
        CHPL_TRY(dgemm(st, K, n, K, 1.0, linv, K, A12, lda, 0.0, T, K));
        CHPL_CUDA(cudaMemcpy2DAsync(A12, (size_t)lda * 8, T, (size_t)K * 8, (size_t)K * 8, (size_t)n,
                                    cudaMemcpyDeviceToDevice, st));
        ++n_launch;
        return CHPL_OK;
    }

    // exact partial pivoting LU of an m x K panel (ld) in place, internal
    // panels of width NBp; piv[i] relative to the panel top
    int factor_panel(double* Pm, int64_t ldp, int64_t m, int64_t K) { return factor_panel_p(Pm, ldp, m, K, piv); }

    int factor_panel_p(double* Pm, int64_t ldp, int64_t m, int64_t K, int64_t* piv)
    {
        for (int64_t jp = 0; jp < K; jp += NBp) {
            const int64_t nb = std::min(NBp, K - jp);
            CHPL_TRY(panel_getrf(st, m - jp, nb, Pm + jp + jp * ldp, (size_t)ldp, piv + jp, jp, info, pwork));
            CHPL_TRY(laswp_plan(st, piv, jp, jp + nb, plan));
            CHPL_TRY(laswp_apply(st, Pm, (size_t)ldp, 0, jp, nb, plan));
            CHPL_TRY(laswp_apply(st, Pm, (size_t)ldp, jp + nb, K - jp - nb, nb, plan));
            n_launch += 4 + 2 * ((nb + 15) / 16) * 2;
            const int64_t nr = K - jp - nb;
            if (nr > 0) {
                CHPL_TRY(dtrsm_llnu(st, nb, nr, Pm + jp + jp * ldp, ldp, Pm + jp + (jp + nb) * ldp, ldp));
                n_launch += dtrsm_launches(nb);
                CHPL_TRY(emu.run(st, win, true, m - jp - nb, nr, nb, Pm + (jp + nb) + jp * ldp, ldp, Pm + jp + (jp + nb) * ldp,
                                 ldp, Pm + (jp + nb) + (jp + nb) * ldp, ldp, -1.0, 1.0));
            }
        }
        return CHPL_OK;
    }

    int rows_gather(double* dst, int64_t ldd, const double* Ab, const int* rows, int n, int64_t ncols)
    {
        if (n <= 0 || ncols <= 0) return CHPL_OK;
        rows_gather_kernel<<<grid1((long long)n * ncols), 256, 0, st>>>(dst, ldd, Ab, lda, rows, n, ncols);
        ++n_launch;
        CHPL_CUDA(cudaGetLastError());
        return CHPL_OK;
    }

    int rows_scatter(double* Ab, const double* src, int64_t lds, const int* rows, int n, int64_t ncols)
    {
        if (n <= 0 || ncols <= 0) return CHPL_OK;
        rows_scatter_kernel<<<grid1((long long)n * ncols), 256, 0, st>>>(Ab, lda, src, lds, rows, n, ncols);
        ++n_launch;
        CHPL_CUDA(cudaGetLastError());
        return CHPL_OK;
    }

    int block_step(int64_t s)
    {
        const int P = g->P, pr = g->pr, qc = g->qc;
        const int64_t J = s * NB, K = std::min(NB, N - J);
        const int ps = (int)(s % P), qs = (int)(s % g->Q);
        const int64_t lrb = local_extent(J, NB, P, pr);            // my first active local row
        const int64_t mact = mloc - lrb;
        const int64_t lc = local_extent(J, NB, g->Q, qc);          // local column of global J (on qs)
        const int64_t tc0 = local_extent(J + K, NB, g->Q, qc);     // first trailing local column
        const int64_t ntr = nloc - tc0;
        const int64_t lrw = local_extent(J + K, NB, P, pr);        // first local row below the diagonal block
        const int64_t mW = mloc - lrw;
        auto t0 = std::chrono::steady_clock::now();

        // ---- 1. factor the block column on its diagonal owner ----
        if (qc == qs) {
            if (P == 1) {
                CHPL_TRY(factor_panel(A + lrb + lc * lda, lda, N - J, K));
            } else {
                const int partner = 1 - pr;
                const int64_t lrb_o = local_extent(J, NB, P, partner), mact_o = local_extent(N, NB, P, partner) - lrb_o;
                double* G = arena;                          // (N - J) x K, ld N - J
                double* Sb = arena + (size_t)N * NB;        // pack buffer, ld = rows of the packing rank
                const int64_t mg = N - J;
                if (pr == ps) {
                    CHPL_NCCL(ncclRecv(Sb, (size_t)mact_o * K, ncclDouble, partner, g->col, st));
                    panel_shuffle_kernel<<<grid1(mg * K), 256, 0, st>>>(G, mg, mg, K, J, NB, P, pr, A + lrb + lc * lda, lda,
                                                                       lrb, Sb, mact_o, lrb_o, 0);
                    CHPL_TRY(factor_panel(G, mg, mg, K));
                    panel_shuffle_kernel<<<grid1(mg * K), 256, 0, st>>>(G, mg, mg, K, J, NB, P, pr, A + lrb + lc * lda, lda,
                                                                       lrb, Sb, mact_o, lrb_o, 1);
                    n_launch += 2;
                    CHPL_NCCL(ncclSend(Sb, (size_t)mact_o * K, ncclDouble, partner, g->col, st));
                } else {
                    CHPL_CUDA(cudaMemcpy2DAsync(Sb, (size_t)mact * 8, A + lrb + lc * lda, (size_t)lda * 8, (size_t)mact * 8,
                                                (size_t)K, cudaMemcpyDeviceToDevice, st));
                    CHPL_NCCL(ncclSend(Sb, (size_t)mact * K, ncclDouble, ps, g->col, st));
                    CHPL_NCCL(ncclRecv(Sb, (size_t)mact * K, ncclDouble, ps, g->col, st));
                    CHPL_CUDA(cudaMemcpy2DAsync(A + lrb + lc * lda, (size_t)lda * 8, Sb, (size_t)mact * 8, (size_t)mact * 8,
                                                (size_t)K, cudaMemcpyDeviceToDevice, st));
                }
            }
        }
        // ---- 2. pivots to everyone; inv(L11) along the diagonal process row ----
        CHPL_NCCL(ncclBroadcast(piv, piv, (size_t)K, ncclInt64, root_of(ps, qs), g->world, st));
        if (pr == ps) {
            if (qc == qs) {
                CHPL_TRY(dtrtri_llnu(st, K, A + lrb + lc * lda, lda, linv, K));
                n_launch += 1 + dtrtri_launches(K);
            }
            if (g->Q > 1) CHPL_NCCL(ncclBroadcast(linv, linv, (size_t)K * K, ncclDouble, qs, g->row, st));
        }
        // W = rows below the diagonal block of the block column, along process rows
        double* W = arena;
        double* U = arena + (size_t)mloc * NB;
        if (qc == qs && mW > 0)
            CHPL_CUDA(cudaMemcpy2DAsync(W, (size_t)mW * 8, A + lrw + lc * lda, (size_t)lda * 8, (size_t)mW * 8, (size_t)K,
                                        cudaMemcpyDeviceToDevice, st));
        if (g->Q > 1 && mW > 0) CHPL_NCCL(ncclBroadcast(W, W, (size_t)mW * K, ncclDouble, qs, g->row, st));
        // host copy of the pivots to plan the interchanges
        std::vector<int64_t> hp((size_t)K);
        CHPL_CUDA(cudaMemcpyAsync(hp.data(), piv, (size_t)K * 8, cudaMemcpyDeviceToHost, st));
        CHPL_TRY(watchdog_sync(g, st, "factor/broadcast"));
        phase[0] += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        t0 = std::chrono::steady_clock::now();

        // ---- 3. interchanges of the trailing columns ----
        std::vector<int> lsrc, ldst, snd, rcv;
        plan_exchange(J, K, hp.data(), NB, P, pr, lsrc, ldst, snd, rcv);
        if (ntr > 0 && (!ldst.empty() || !snd.empty() || !rcv.empty())) {
            int* dl = dlist;
            std::vector<int> all;
            all.insert(all.end(), lsrc.begin(), lsrc.end());
            all.insert(all.end(), ldst.begin(), ldst.end());
            all.insert(all.end(), snd.begin(), snd.end());
            all.insert(all.end(), rcv.begin(), rcv.end());
            CHPL_CUDA(cudaMemcpyAsync(dl, all.data(), all.size() * sizeof(int), cudaMemcpyHostToDevice, st));
            const int nl = (int)lsrc.size(), ns = (int)snd.size(), nr = (int)rcv.size();
            const int* d_lsrc = dl;
            const int* d_ldst = dl + nl;
            const int* d_snd = dl + 2 * nl;
            const int* d_rcv = dl + 2 * nl + ns;
            double* Tb = xch;
            double* Sb2 = xch + (size_t)2 * NB * kXchCols;
            double* Rb = xch + (size_t)4 * NB * kXchCols;
            for (int64_t c0 = tc0; c0 < nloc; c0 += kXchCols) {
                const int64_t nc = std::min(kXchCols, nloc - c0);
                double* Ab = A + c0 * lda;
                CHPL_TRY(rows_gather(Sb2, std::max(ns, 1), Ab, d_snd, ns, nc));
                CHPL_TRY(rows_gather(Tb, std::max(nl, 1), Ab, d_lsrc, nl, nc));
                if (ns > 0 || nr > 0) {
                    CHPL_NCCL(ncclGroupStart());
                    if (ns > 0) CHPL_NCCL(ncclSend(Sb2, (size_t)ns * nc, ncclDouble, 1 - pr, g->col, st));
                    if (nr > 0) CHPL_NCCL(ncclRecv(Rb, (size_t)nr * nc, ncclDouble, 1 - pr, g->col, st));
                    CHPL_NCCL(ncclGroupEnd());
                }
                CHPL_TRY(rows_scatter(Ab, Tb, std::max(nl, 1), d_ldst, nl, nc));
                CHPL_TRY(rows_scatter(Ab, Rb, std::max(nr, 1), d_rcv, nr, nc));
            }
        }
        CHPL_TRY(watchdog_sync(g, st, "interchanges"));
        phase[1] += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        t0 = std::chrono::steady_clock::now();
        // ---- 4. U12 on the diagonal process row, down the process columns ----
        if (ntr > 0) {
            if (pr == ps) {
                if (emu.fp64)
                    CHPL_TRY(u12_fp64(K, ntr, A + lrb + tc0 * lda, U));
                else
                    CHPL_TRY(emu.run(st, wlinv, true, K, ntr, K, linv, K, A + lrb + tc0 * lda, lda, A + lrb + tc0 * lda, lda,
                                     1.0, 0.0));
                if (P > 1)
                    CHPL_CUDA(cudaMemcpy2DAsync(U, (size_t)K * 8, A + lrb + tc0 * lda, (size_t)lda * 8, (size_t)K * 8,
                                                (size_t)ntr, cudaMemcpyDeviceToDevice, st));
            }
            if (P > 1) CHPL_NCCL(ncclBroadcast(U, U, (size_t)K * ntr, ncclDouble, ps, g->col, st));
            CHPL_TRY(watchdog_sync(g, st, "U12"));
            phase[2] += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            t0 = std::chrono::steady_clock::now();
            // ---- 5. trailing update ----
            if (mW > 0) {
                const double* Bp = (P > 1) ? U : A + lrb + tc0 * lda;
                const int64_t ldb = (P > 1) ? K : lda;
                CHPL_TRY(emu.run(st, wres, true, mW, ntr, K, W, mW, Bp, ldb, A + lrw + tc0 * lda, lda, -1.0, 1.0));
            }
        }
        CHPL_TRY(watchdog_sync(g, st, "update"));
        phase[3] += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        return CHPL_OK;
    }

    // ---------------------------------------------------------------- 1 x Q lookahead
    // With one process row every rank holds all rows: interchanges and U12
    // are local, and the only exchange per block is the broadcast of its
    // pivots, inv(L11) and W = L21 from the owner of the block column along
    // the row.  Two streams per rank: `st` computes, `sm` communicates.  The
    // owner of block s+1 first brings that block up to date with block s
    // (interchanges, U12, W*U12 on its columns only), factors it and hands it
    // to `sm`; only then does it update the rest of its columns, while the
    // other ranks, which have no panel to factor, update all of theirs.  So
    // no rank waits for a panel another rank is factoring unless its own
    // update of the step is shorter (depth-1 lookahead, src/chpl_p2.cu:1620-1741).
    // Slots: pivots and inv(L11) alternate by block parity; W (FP64) has one
    // buffer, released as soon as its residues are split; the panel's inner
    // update residues have their own region.
    int64_t Kof(int64_t s) const { return std::min(NB, N - s * NB); }

    // owner of block column s: factor it (rows J.., local columns from lc),
    // inv(L11) into its slot, W = L21 into the W buffer
    int factor_owned(int64_t s, int64_t lc, int64_t* pv, double* lv)
    {
        const int64_t J = s * NB, K = Kof(s);
        cudaEvent_t e0, e1;
        CHPL_CUDA(cudaEventCreate(&e0));
        CHPL_CUDA(cudaEventCreate(&e1));
        panel_ev.push_back({e0, e1});
        CHPL_CUDA(cudaEventRecord(e0, st));
        CHPL_TRY(factor_panel_p(A + J + lc * lda, lda, N - J, K, pv));
        CHPL_CUDA(cudaEventRecord(e1, st));
        CHPL_TRY(dtrtri_llnu(st, K, A + J + lc * lda, lda, lv, K));
        n_launch += 1 + dtrtri_launches(K);
        const int64_t mW = N - J - K;
        if (mW > 0)
            CHPL_CUDA(cudaMemcpy2DAsync(arena, (size_t)mW * 8, A + J + K + lc * lda, (size_t)lda * 8, (size_t)mW * 8,
                                        (size_t)K, cudaMemcpyDeviceToDevice, st));
        n_launch += 2;
        return CHPL_OK;
    }

    // local columns [c0, c0 + nc) through block s: interchanges, U12 = inv(L11) A12, A22 -= W U12
    int update_cols(int64_t s, int64_t c0, int64_t nc, const double* lv)
    {
        if (nc <= 0) return CHPL_OK;
        const int64_t J = s * NB, K = Kof(s), mW = N - J - K;
        cudaEvent_t t = pev.begin(st);
        for (int64_t k0 = 0; k0 < K; k0 += kPlanSwaps) {   // the block's swaps in order, one plan per chunk
            const void* pl = static_cast<uint8_t*>(plan2) + (k0 / kPlanSwaps) * round_up(laswp_work_bytes(kPlanSwaps), 256);
            CHPL_TRY(laswp_apply(st, A + J, (size_t)lda, c0, nc, std::min(kPlanSwaps, K - k0), pl));
            ++n_launch;
        }
        pev.end(st, 1, t);
        t = pev.begin(st);
        CHPL_TRY(emu.run(st, wlinv, true, K, nc, K, lv, K, A + J + c0 * lda, lda, A + J + c0 * lda, lda, 1.0, 0.0));
        pev.end(st, 2, t);
        if (mW > 0) {
            t = pev.begin(st);
            CHPL_TRY(emu.run(st, wres, false, mW, nc, K, arena, mW, A + J + c0 * lda, lda, A + J + K + c0 * lda, lda, -1.0,
                             1.0));
            pev.end(st, 4, t);
        }
        return CHPL_OK;
    }

    int run_p1()
    {
        const int Q = g->Q, qc = g->qc;
        int64_t* Pv[2] = {piv, piv2};
        double* Lv[2] = {linv, linv2};
        std::vector<cudaEvent_t> evs;
        auto mk = [&](cudaEvent_t* e) -> int {
            CHPL_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
            evs.push_back(*e);
            return CHPL_OK;
        };
        auto cleanup = [&]() { for (auto e : evs) cudaEventDestroy(e); };
        cudaEvent_t start, evF = nullptr, evWfree = nullptr, evLfree[2] = {nullptr, nullptr}, prev_end = nullptr;
        int rc = mk(&start);
        if (rc == CHPL_OK) rc = (cudaEventRecord(start, st) == cudaSuccess) ? CHPL_OK : CHPL_ERR_CUDA;
        if (rc == CHPL_OK) rc = (cudaStreamWaitEvent(sm, start, 0) == cudaSuccess) ? CHPL_OK : CHPL_ERR_CUDA;
        if (rc == CHPL_OK && qc == 0) {   // prologue: block 0 on its owner
            rc = factor_owned(0, 0, Pv[0], Lv[0]);
            if (rc == CHPL_OK) rc = mk(&evF);
            if (rc == CHPL_OK) cudaEventRecord(evF, st);
        }
        for (int64_t s = 0; s < nblk && rc == CHPL_OK; ++s) {
            const int64_t J = s * NB, K = Kof(s), mW = N - J - K;
            const int qs = (int)(s % Q), slot = (int)(s & 1);
            // ---- communication: pivots, inv(L11), W of block s from its owner ----
            if (qc == qs) {
                cudaStreamWaitEvent(sm, evF, 0);
            } else {
                if (evWfree) cudaStreamWaitEvent(sm, evWfree, 0);
                if (evLfree[slot]) cudaStreamWaitEvent(sm, evLfree[slot], 0);
            }
            cudaEvent_t tb = pev.begin(sm);
            ncclGroupStart();
            ncclBroadcast(Pv[slot], Pv[slot], (size_t)K, ncclInt64, qs, g->row, sm);
            ncclBroadcast(Lv[slot], Lv[slot], (size_t)K * K, ncclDouble, qs, g->row, sm);
            if (mW > 0) ncclBroadcast(arena, arena, (size_t)mW * K, ncclDouble, qs, g->row, sm);
            if (ncclGroupEnd() != ncclSuccess) { set_error("NCCL broadcast of block %lld failed", (long long)s); rc = CHPL_ERR_NCCL; break; }
            pev.end(sm, 7, tb);
            cudaEvent_t evW;
            if ((rc = mk(&evW)) != CHPL_OK) break;
            cudaEventRecord(evW, sm);
            // ---- computation ----
            cudaStreamWaitEvent(st, evW, 0);
            cudaEvent_t ts = pev.begin(st);
            if ((rc = emu.split_only(st, wres, mW, K, arena, mW)) != CHPL_OK) break;
            pev.end(st, 3, ts);
            if ((rc = mk(&evWfree)) != CHPL_OK) break;
            cudaEventRecord(evWfree, st);
            const int64_t tc0 = local_extent(J + K, NB, Q, qc), ntr = nloc - tc0;
            for (int64_t k0 = 0; ntr > 0 && k0 < K && rc == CHPL_OK; k0 += kPlanSwaps)
                rc = laswp_plan(st, Pv[slot], k0, std::min(K, k0 + kPlanSwaps),
                                static_cast<uint8_t*>(plan2) + (k0 / kPlanSwaps) * round_up(laswp_work_bytes(kPlanSwaps), 256));
            if (rc != CHPL_OK) break;
            const bool own_next = s + 1 < nblk && (int)((s + 1) % Q) == qc;
            int64_t urgent = 0;
            if (own_next) {   // block s+1 first: bring it up to date, factor it, hand it to sm
                urgent = Kof(s + 1);
                if ((rc = update_cols(s, tc0, urgent, Lv[slot])) != CHPL_OK) break;
                if ((rc = factor_owned(s + 1, tc0, Pv[slot ^ 1], Lv[slot ^ 1])) != CHPL_OK) break;
                if ((rc = mk(&evF)) != CHPL_OK) break;
                cudaEventRecord(evF, st);
            }
            if ((rc = update_cols(s, tc0 + urgent, ntr - urgent, Lv[slot])) != CHPL_OK) break;
            if ((rc = mk(&evLfree[slot])) != CHPL_OK) break;
            cudaEventRecord(evLfree[slot], st);
            // keep the host at most one block ahead of the device
            if (prev_end && (rc = watchdog_event(g, prev_end, "lookahead step")) != CHPL_OK) break;
            prev_end = evLfree[slot];
        }
        if (rc == CHPL_OK) rc = watchdog_sync(g, sm, "lookahead communication");
        if (rc == CHPL_OK) rc = watchdog_sync(g, st, "lookahead update");
        for (auto& e : panel_ev) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, e.first, e.second) == cudaSuccess) phase[0] += ms * 1e-3;
        }
        cleanup();
        return rc;
    }

    // ---------------------------------------------------------------- 2 x Q lookahead
    // Streams per rank: `st` computes; `sm` carries the chain of the next
    // block (pivot, inv(L11) and W broadcasts, the urgent interchanges and
    // U12 of the process column that owns the next block, the gather and
    // scatter of its panel) on the world / row / column communicators; `sb`
    // carries the bulk interchanges and U12 broadcasts on a second column
    // communicator, so a column pair's bulk exchange never queues behind the
    // panel the other column pair is factoring.  In block step s the process
    // column owning block s+1 updates that block first, gathers and factors
    // it on its diagonal owner and hands pivots, inv(L11) and W to `sm`; all
    // ranks then update the rest of their columns.  W alternates between two
    // slots (one step of slack between the ranks of a process row); the
    // gathered panel occupies both slots while it is factored, after the
    // diagonal owner has split the current W into int8 residues.
    struct Lists {
        std::vector<int> lsrc, ldst, snd, rcv;
    };

    // interchanges of block s on local columns [c0, c0 + nc): local moves,
    // rows across process rows on stream cs / communicator cm, in tiles
    int exchange2(int64_t c0, int64_t nc, const int* dl, const Lists& Ls, cudaStream_t cs, ncclComm_t cm, cudaEvent_t e1,
                  cudaEvent_t e2)
    {
        const int nl = (int)Ls.lsrc.size(), ns = (int)Ls.snd.size(), nr = (int)Ls.rcv.size();
        if (nc <= 0 || (nl == 0 && ns == 0 && nr == 0)) return CHPL_OK;
        const int *d_lsrc = dl, *d_ldst = dl + nl, *d_snd = dl + 2 * nl, *d_rcv = dl + 2 * nl + ns;
        double* Tb = xch;
        double* Sb2 = xch + (size_t)2 * NB * kXchCols;
        double* Rb = xch + (size_t)4 * NB * kXchCols;
        for (int64_t t0 = c0; t0 < c0 + nc; t0 += kXchCols) {
            const int64_t n = std::min(kXchCols, c0 + nc - t0);
            double* Ab = A + t0 * lda;
            CHPL_TRY(rows_gather(Sb2, std::max(ns, 1), Ab, d_snd, ns, n));
            CHPL_TRY(rows_gather(Tb, std::max(nl, 1), Ab, d_lsrc, nl, n));
            if (ns > 0 || nr > 0) {
                CHPL_CUDA(cudaEventRecord(e1, st));
                CHPL_CUDA(cudaStreamWaitEvent(cs, e1, 0));
                CHPL_NCCL(ncclGroupStart());
                if (ns > 0) CHPL_NCCL(ncclSend(Sb2, (size_t)ns * n, ncclDouble, 1 - g->pr, cm, cs));
                if (nr > 0) CHPL_NCCL(ncclRecv(Rb, (size_t)nr * n, ncclDouble, 1 - g->pr, cm, cs));
                CHPL_NCCL(ncclGroupEnd());
                CHPL_CUDA(cudaEventRecord(e2, cs));
                CHPL_CUDA(cudaStreamWaitEvent(st, e2, 0));
            }
            CHPL_TRY(rows_scatter(Ab, Tb, std::max(nl, 1), d_ldst, nl, n));
            CHPL_TRY(rows_scatter(Ab, Rb, std::max(nr, 1), d_rcv, nr, n));
        }
        return CHPL_OK;
    }

    // U12 of block s on local columns [c0, c0 + nc) (process row ps computes
    // it in place and copies it to Ud, ld K), broadcast down the process
    // column on cs / cm; every rank then reads U12 from Ud
    int u12(int64_t s, int64_t c0, int64_t nc, const double* lv, double* Ud, cudaStream_t cs, ncclComm_t cm,
            cudaEvent_t e1, cudaEvent_t e2)
    {
        if (nc <= 0) return CHPL_OK;
        const int64_t J = s * NB, K = Kof(s);
        const int ps = (int)(s % 2);
        const int64_t lrb = local_extent(J, NB, 2, g->pr);
        if (g->pr == ps) {
            CHPL_TRY(emu.run(st, wlinv, true, K, nc, K, lv, K, A + lrb + c0 * lda, lda, A + lrb + c0 * lda, lda, 1.0, 0.0));
            CHPL_CUDA(cudaMemcpy2DAsync(Ud, (size_t)K * 8, A + lrb + c0 * lda, (size_t)lda * 8, (size_t)K * 8, (size_t)nc,
                                        cudaMemcpyDeviceToDevice, st));
            CHPL_CUDA(cudaEventRecord(e1, st));
            CHPL_CUDA(cudaStreamWaitEvent(cs, e1, 0));
        }
        CHPL_NCCL(ncclBroadcast(Ud, Ud, (size_t)K * nc, ncclDouble, ps, cm, cs));
        CHPL_CUDA(cudaEventRecord(e2, cs));
        CHPL_CUDA(cudaStreamWaitEvent(st, e2, 0));
        return CHPL_OK;
    }

    // block s1 (global columns J1.., local columns from lc1) on its process
    // column: the other process row sends its rows to the diagonal owner in
    // chunks of kPackCols columns, the owner factors the gathered panel
    // (exact partial pivoting) in the W slots and sends the rows back; then
    // each rank of the column copies its W = L21 rows into W slot s1 & 1 and
    // the owner computes inv(L11).  Returns with evF recorded where A1(s1)
    // must wait (owner: st; partner: sm itself).
    int chain_factor(int64_t s1, int64_t lc1, int64_t* pv, double* lv, cudaEvent_t evF, cudaEvent_t evG,
                     cudaEvent_t e1, cudaEvent_t e2)
    {
        const int pr = g->pr, p1 = (int)(s1 % 2), partner = 1 - pr;
        const int64_t J1 = s1 * NB, K1 = Kof(s1), mg = N - J1;
        const int64_t lrb1 = local_extent(J1, NB, 2, pr), mact1 = mloc - lrb1;
        const int64_t lrb1_o = local_extent(J1, NB, 2, partner), mact1_o = local_extent(N, NB, 2, partner) - lrb1_o;
        const int64_t lrw1 = local_extent(J1 + K1, NB, 2, pr), mW1 = mloc - lrw1;
        double* Wslot = Wd + (size_t)(s1 & 1) * mloc * NB;
        if (pr == p1) {
            CHPL_CUDA(cudaStreamWaitEvent(st, evPk, 0));   // an earlier unpack (as partner) has read pk
            double* G = Wd;   // both W slots: (N - J1) x K1, ld mg
            for (int64_t c0 = 0; c0 < K1; c0 += kPackCols) {
                const int64_t nc = std::min(kPackCols, K1 - c0);
                CHPL_CUDA(cudaEventRecord(e1, st));   // the previous chunk's shuffle has read pk
                CHPL_CUDA(cudaStreamWaitEvent(sm, e1, 0));
                CHPL_NCCL(ncclRecv(pk, (size_t)mact1_o * nc, ncclDouble, partner, g->col, sm));
                CHPL_CUDA(cudaEventRecord(e2, sm));
                CHPL_CUDA(cudaStreamWaitEvent(st, e2, 0));
                panel_shuffle_kernel<<<grid1(mg * nc), 256, 0, st>>>(G + c0 * mg, mg, mg, nc, J1, NB, 2, pr,
                                                                      A + lrb1 + (lc1 + c0) * lda, lda, lrb1, pk,
                                                                      std::max<int64_t>(mact1_o, 1), lrb1_o, 0);
                ++n_launch;
            }
            cudaEvent_t p0, p1e;
            CHPL_CUDA(cudaEventCreate(&p0));
            CHPL_CUDA(cudaEventCreate(&p1e));
            panel_ev.push_back({p0, p1e});
            CHPL_CUDA(cudaEventRecord(p0, st));
            CHPL_TRY(factor_panel_p(G, mg, mg, K1, pv));
            CHPL_CUDA(cudaEventRecord(p1e, st));
            for (int64_t c0 = 0; c0 < K1; c0 += kPackCols) {
                const int64_t nc = std::min(kPackCols, K1 - c0);
                panel_shuffle_kernel<<<grid1(mg * nc), 256, 0, st>>>(G + c0 * mg, mg, mg, nc, J1, NB, 2, pr,
                                                                      A + lrb1 + (lc1 + c0) * lda, lda, lrb1, pk,
                                                                      std::max<int64_t>(mact1_o, 1), lrb1_o, 1);
                ++n_launch;
                CHPL_CUDA(cudaEventRecord(e1, st));
                CHPL_CUDA(cudaStreamWaitEvent(sm, e1, 0));
                CHPL_NCCL(ncclSend(pk, (size_t)mact1_o * nc, ncclDouble, partner, g->col, sm));
                CHPL_CUDA(cudaEventRecord(e2, sm));
                CHPL_CUDA(cudaStreamWaitEvent(st, e2, 0));   // pk is free again
            }
            CHPL_CUDA(cudaEventRecord(evG, st));   // the W slots hold no panel any more
            CHPL_TRY(dtrtri_llnu(st, K1, A + lrb1 + lc1 * lda, lda, lv, K1));
            n_launch += 1 + dtrtri_launches(K1);
            if (mW1 > 0)
                CHPL_CUDA(cudaMemcpy2DAsync(Wslot, (size_t)mW1 * 8, A + lrw1 + lc1 * lda, (size_t)lda * 8, (size_t)mW1 * 8,
                                            (size_t)K1, cudaMemcpyDeviceToDevice, st));
            CHPL_CUDA(cudaEventRecord(evF, st));
            n_launch += 2;
        } else {
            CHPL_CUDA(cudaStreamWaitEvent(st, evPk, 0));   // an earlier unpack has read pk
            for (int64_t c0 = 0; c0 < K1; c0 += kPackCols) {
                const int64_t nc = std::min(kPackCols, K1 - c0);
                if (mact1 > 0)
                    CHPL_CUDA(cudaMemcpy2DAsync(pk, (size_t)mact1 * 8, A + lrb1 + (lc1 + c0) * lda, (size_t)lda * 8,
                                                (size_t)mact1 * 8, (size_t)nc, cudaMemcpyDeviceToDevice, st));
                CHPL_CUDA(cudaEventRecord(e1, st));
                CHPL_CUDA(cudaStreamWaitEvent(sm, e1, 0));
                CHPL_NCCL(ncclSend(pk, (size_t)mact1 * nc, ncclDouble, p1, g->col, sm));
                CHPL_CUDA(cudaEventRecord(e2, sm));
                CHPL_CUDA(cudaStreamWaitEvent(st, e2, 0));   // pk is free again
            }
            // the factored rows come back on sm, which also unpacks them and copies W:
            // this rank's computation goes on with its bulk update meanwhile
            for (int64_t c0 = 0; c0 < K1; c0 += kPackCols) {
                const int64_t nc = std::min(kPackCols, K1 - c0);
                CHPL_NCCL(ncclRecv(pk, (size_t)mact1 * nc, ncclDouble, p1, g->col, sm));
                if (mact1 > 0)
                    CHPL_CUDA(cudaMemcpy2DAsync(A + lrb1 + (lc1 + c0) * lda, (size_t)lda * 8, pk, (size_t)mact1 * 8,
                                                (size_t)mact1 * 8, (size_t)nc, cudaMemcpyDeviceToDevice, sm));
            }
            if (mW1 > 0)
                CHPL_CUDA(cudaMemcpy2DAsync(Wslot, (size_t)mW1 * 8, A + lrw1 + lc1 * lda, (size_t)lda * 8, (size_t)mW1 * 8,
                                            (size_t)K1, cudaMemcpyDeviceToDevice, sm));
            CHPL_CUDA(cudaEventRecord(evF, sm));
            CHPL_CUDA(cudaEventRecord(evG, sm));
            CHPL_CUDA(cudaEventRecord(evPk, sm));   // st writes pk again only after this (next chain step)
        }
        return CHPL_OK;
    }

    int run_p2()
    {
        const int Q = g->Q, pr = g->pr, qc = g->qc;
        int64_t* Pv[2] = {piv, piv2};
        double* Lv[2] = {linv, linv2};
        int* DL[2] = {dlist, dlist2};
        std::vector<cudaEvent_t> evs;
        auto mk = [&]() {
            cudaEvent_t e = nullptr;
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess) evs.push_back(e);
            return e;
        };
        cudaEvent_t start = mk(), evF = mk(), evG = mk(), e1 = mk(), e2 = mk(), e3 = mk(), e4 = mk(), evA = mk(),
                    evPH = mk(), evWfree[2] = {mk(), mk()}, evLfree[2] = {mk(), mk()}, evEnd[2] = {mk(), mk()};
        bool wfree_rec[2] = {false, false}, lfree_rec[2] = {false, false}, g_rec = false;
        int rc = CHPL_OK;
        auto done = [&](int r) {
            for (auto e : evs) cudaEventDestroy(e);
            return r;
        };
        for (auto e : evs)
            if (!e) return done(cuda_fail(cudaErrorMemoryAllocation, "event", __FILE__, __LINE__));
        CHPL_CUDA(cudaEventRecord(start, st));
        CHPL_CUDA(cudaStreamWaitEvent(sm, start, 0));
        CHPL_CUDA(cudaStreamWaitEvent(sb, start, 0));
        // prologue: block 0 on process column 0
        if (qc == 0) {
            if ((rc = chain_factor(0, 0, Pv[0], Lv[0], evF, evG, e1, e2)) != CHPL_OK) return done(rc);
            g_rec = true;
        }
        Lists Ls;
        for (int64_t s = 0; s < nblk && rc == CHPL_OK; ++s) {
            const int64_t J = s * NB, K = Kof(s);
            const int ps = (int)(s % 2), qs = (int)(s % Q), slot = (int)(s & 1);
            const int64_t lrw = local_extent(J + K, NB, 2, pr), mW = mloc - lrw;
            double* Wslot = Wd + (size_t)slot * mloc * NB;
            // ---- A1: pivots (world), inv(L11) and W (process rows) of block s ----
            if (qc == qs && pr == ps) {
                cudaStreamWaitEvent(sm, evF, 0);   // this rank factored block s
            } else {
                if (wfree_rec[slot]) cudaStreamWaitEvent(sm, evWfree[slot], 0);
                if (lfree_rec[slot]) cudaStreamWaitEvent(sm, evLfree[slot], 0);
                if (g_rec) cudaStreamWaitEvent(sm, evG, 0);
            }
            cudaEvent_t tb = pev.begin(sm);
            ncclGroupStart();
            ncclBroadcast(Pv[slot], Pv[slot], (size_t)K, ncclInt64, 2 * qs + ps, g->world, sm);
            if (ncclGroupEnd() != ncclSuccess) { rc = CHPL_ERR_NCCL; set_error("pivot broadcast failed"); break; }
            ncclGroupStart();
            if (pr == ps) ncclBroadcast(Lv[slot], Lv[slot], (size_t)K * K, ncclDouble, qs, g->row, sm);
            if (mW > 0) ncclBroadcast(Wslot, Wslot, (size_t)mW * K, ncclDouble, qs, g->row, sm);
            if (ncclGroupEnd() != ncclSuccess) { rc = CHPL_ERR_NCCL; set_error("W broadcast failed"); break; }
            pev.end(sm, 7, tb);
            cudaEventRecord(evA, sm);
            cudaMemcpyAsync(hpiv + (size_t)slot * NB, Pv[slot], (size_t)K * sizeof(int64_t), cudaMemcpyDeviceToHost, sm);
            cudaEventRecord(evPH, sm);
            // ---- computation ----
            cudaStreamWaitEvent(st, evA, 0);
            cudaEvent_t ts = pev.begin(st);
            if ((rc = emu.split_only(st, wres, mW, K, Wslot, mW)) != CHPL_OK) break;
            pev.end(st, 3, ts);
            cudaEventRecord(evWfree[slot], st);
            wfree_rec[slot] = true;
            if ((rc = watchdog_event(g, evPH, "pivots")) != CHPL_OK) break;
            plan_exchange(J, K, hpiv + (size_t)slot * NB, NB, 2, pr, Ls.lsrc, Ls.ldst, Ls.snd, Ls.rcv);
            {   // lists to the device through this slot's pinned staging (its copy of two steps ago has run:
                // the host waited for the end of step s-1)
                int* hl = hlist + (size_t)slot * 8 * NB;
                size_t n = 0;
                for (const std::vector<int>* v : {&Ls.lsrc, &Ls.ldst, &Ls.snd, &Ls.rcv})
                    for (int x : *v) hl[n++] = x;
                if (n > (size_t)8 * NB) { rc = CHPL_ERR_INVALID; set_error("exchange lists overflow"); break; }
                if (n) cudaMemcpyAsync(DL[slot], hl, n * sizeof(int), cudaMemcpyHostToDevice, st);
            }
            const int64_t tc0 = local_extent(J + K, NB, Q, qc), ntr = nloc - tc0;
            const int q1 = (int)((s + 1) % Q);
            const bool chain = s + 1 < nblk && qc == q1;
            const int64_t urg = chain ? std::min<int64_t>(Kof(s + 1), ntr) : 0;
            if (chain) {   // block s+1 first: interchanges, U12, update, then its factorization
                cudaEvent_t t = pev.begin(st);
                if ((rc = exchange2(tc0, urg, DL[slot], Ls, sm, g->col, e1, e2)) != CHPL_OK) break;
                pev.end(st, 1, t);
                double* Us = Uu + (size_t)slot * NB * NB;
                t = pev.begin(st);
                if ((rc = u12(s, tc0, urg, Lv[slot], Us, sm, g->col, e1, e2)) != CHPL_OK) break;
                pev.end(st, 2, t);
                t = pev.begin(st);
                if (mW > 0 &&
                    (rc = emu.run(st, wres, false, mW, urg, K, Wslot, mW, Us, K, A + lrw + tc0 * lda, lda, -1.0, 1.0)) !=
                        CHPL_OK)
                    break;
                pev.end(st, 4, t);
                if ((rc = chain_factor(s + 1, tc0, Pv[slot ^ 1], Lv[slot ^ 1], evF, evG, e1, e2)) != CHPL_OK) break;
                g_rec = true;
            }
            // ---- the rest of the columns ----
            const int64_t c0 = tc0 + urg, nc = ntr - urg;
            cudaEvent_t tx = pev.begin(st);
            if ((rc = exchange2(c0, nc, DL[slot], Ls, sb, g->col2, e3, e4)) != CHPL_OK) break;
            pev.end(st, 1, tx);
            if (nc > 0) {
                if (s > 0) cudaStreamWaitEvent(sb, evEnd[slot ^ 1], 0);   // Ub is free (read by step s-1's update)
                cudaEvent_t t = pev.begin(st);
                if ((rc = u12(s, c0, nc, Lv[slot], Ub, sb, g->col2, e3, e4)) != CHPL_OK) break;
                pev.end(st, 2, t);
                t = pev.begin(st);
                if (mW > 0 &&
                    (rc = emu.run(st, wres, false, mW, nc, K, Wslot, mW, Ub, K, A + lrw + c0 * lda, lda, -1.0, 1.0)) !=
                        CHPL_OK)
                    break;
                pev.end(st, 4, t);
            }
            cudaEventRecord(evLfree[slot], st);
            lfree_rec[slot] = true;
            cudaEventRecord(evEnd[slot], st);
            // keep the host at most one block ahead of the device
            if (s > 0 && (rc = watchdog_event(g, evEnd[slot ^ 1], "lookahead step")) != CHPL_OK) break;
        }
        if (rc == CHPL_OK) rc = watchdog_sync(g, sm, "lookahead chain");
        if (rc == CHPL_OK) rc = watchdog_sync(g, sb, "lookahead bulk communication");
        if (rc == CHPL_OK) rc = watchdog_sync(g, st, "lookahead update");
        for (auto& e : panel_ev) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, e.first, e.second) == cudaSuccess) phase[0] += ms * 1e-3;
        }
        return done(rc);
    }

    // distributed back substitution U x = b' (b' in global column N)
    int back_solve()
    {
        const int P = g->P, Q = g->Q, pr = g->pr, qc = g->qc;
        const int qN = (int)((N / NB) % Q);
        const int64_t lcN = local_extent(N, NB, Q, qN);
        cudaEvent_t tbs = pev.begin(st);
        CHPL_CUDA(cudaMemsetAsync(tsum, 0, (size_t)std::max<int64_t>(mloc, 1) * 8, st));
        CHPL_CUDA(cudaMemsetAsync(x, 0, (size_t)N * 8, st));
        for (int64_t j = nblk - 1; j >= 0; --j) {
            const int64_t J = j * NB, jb = std::min(NB, N - J);
            const int pj = (int)(j % P), qj = (int)(j % Q);
            const int64_t lrj = local_extent(J, NB, P, pj);
            double* v = vbuf;
            if (pr == pj) {
                axpby_rows_kernel<<<(unsigned)((jb + 255) / 256), 256, 0, st>>>(v, A + lrj + lcN * lda, tsum + lrj, (int)jb,
                                                                              qc == qN ? 1 : 0);
                ++n_launch;
                if (Q > 1) CHPL_NCCL(ncclReduce(v, v, (size_t)jb, ncclDouble, ncclSum, qj, g->row, st));
                if (qc == qj) {
                    const int64_t lcj = local_extent(J, NB, Q, qj);
                    CHPL_TRY(dtrsv_unn(st, jb, A + lrj + lcj * lda, lda, v, vbuf + NB));
                    n_launch += dtrsv_launches(jb);
                }
            }
            if (qc == qj) {
                if (P > 1) CHPL_NCCL(ncclBroadcast(v, v, (size_t)jb, ncclDouble, pj, g->col, st));
                const int64_t lcj = local_extent(J, NB, Q, qj);
                const int64_t rows_above = local_extent(J, NB, P, pr);
                if (rows_above > 0)
                    CHPL_TRY(dgemv_n(st, rows_above, jb, 1.0, A + lcj * lda, lda, v, 1.0, tsum));
                    ++n_launch;
                if (pr == 0) CHPL_CUDA(cudaMemcpyAsync(x + J, v, (size_t)jb * 8, cudaMemcpyDeviceToDevice, st));
            }
        }
        if (g->P * g->Q > 1) CHPL_NCCL(ncclAllReduce(x, x, (size_t)N, ncclDouble, ncclSum, g->world, st));
        pev.end(st, 6, tbs);
        return watchdog_sync(g, st, "back substitution");
    }

    int residual(double* resid)
    {
        const long long nbk = (mloc + 255) / 256;
        double* part = nullptr;
        double* axrs = nullptr;
        double* out = nullptr;
        CHPL_CUDA(cudaMallocAsync((void**)&part, (size_t)kGridResChunks * 2 * std::max<int64_t>(mloc, 1) * 8, st));
        CHPL_CUDA(cudaMallocAsync((void**)&axrs, (size_t)2 * std::max<int64_t>(mloc, 1) * 8, st));
        CHPL_CUDA(cudaMallocAsync((void**)&out, (size_t)std::max(nbk, 1LL) * 3 * 8 + 64, st));
        if (mloc > 0) {
            grid_resid_partial_kernel<<<dim3((unsigned)nbk, kGridResChunks), 256, 0, st>>>(
                N, NB, g->P, g->Q, g->pr, g->qc, mloc, nloc, cfg.seed, x, part);
            grid_resid_sum_kernel<<<(unsigned)nbk, 256, 0, st>>>(mloc, part, axrs);
        }
        if (g->Q > 1 && mloc > 0) CHPL_NCCL(ncclAllReduce(axrs, axrs, (size_t)2 * mloc, ncclDouble, ncclSum, g->row, st));
        if (mloc > 0) grid_resid_max_kernel<<<(unsigned)nbk, 256, 0, st>>>(N, NB, g->P, g->pr, mloc, cfg.seed, axrs, out);
        std::vector<double> h((size_t)std::max(nbk, 1LL) * 3, 0.0);
        if (mloc > 0) CHPL_CUDA(cudaMemcpyAsync(h.data(), out, (size_t)nbk * 3 * 8, cudaMemcpyDeviceToHost, st));
        CHPL_TRY(watchdog_sync(g, st, "residual"));
        double loc[4] = {0, 0, 0, 0};
        for (long long b = 0; b < nbk; ++b)
            for (int q = 0; q < 3; ++q) loc[q] = std::max(loc[q], h[(size_t)b * 3 + q]);
        // ||x||_oo (x is complete on every rank)
        std::vector<double> hx((size_t)N);
        CHPL_CUDA(cudaMemcpy(hx.data(), x, (size_t)N * 8, cudaMemcpyDeviceToHost));
        for (double v : hx) loc[3] = std::max(loc[3], std::fabs(v));
        double* dm = out;
        CHPL_CUDA(cudaMemcpyAsync(dm, loc, 4 * 8, cudaMemcpyHostToDevice, st));
        if (g->P * g->Q > 1) CHPL_NCCL(ncclAllReduce(dm, dm, 4, ncclDouble, ncclMax, g->world, st));
        double gl[4];
        CHPL_CUDA(cudaMemcpyAsync(gl, dm, 4 * 8, cudaMemcpyDeviceToHost, st));
        CHPL_TRY(watchdog_sync(g, st, "residual reduce"));
        cudaFreeAsync(part, st);
        cudaFreeAsync(axrs, st);
        cudaFreeAsync(out, st);
        const double eps = std::ldexp(1.0, -53);
        *resid = gl[0] / (eps * (gl[1] * gl[3] + gl[2]) * (double)N);
        return CHPL_OK;
    }
};

static int grid_run(GridComm* g, const chpl_hpl_config* cfg, chpl_hpl_result* res, double* x_out)
{
    if (!g || !cfg || !res) { set_error("grid_run: NULL argument"); return CHPL_ERR_INVALID; }
    std::memset(res, 0, sizeof(*res));
    if (g->aborted) { set_error("communicators were aborted"); return CHPL_ERR_NCCL; }
    if (cfg->P != g->P || cfg->Q != g->Q) { set_error("config grid %dx%d != communicator grid %dx%d", cfg->P, cfg->Q, g->P, g->Q); return CHPL_ERR_INVALID; }
    if (g->P > 2) { set_error("process grids with P > 2 are not supported (P = 1 or 2)"); return CHPL_ERR_UNSUPPORTED; }
    if (cfg->N <= 0 || cfg->NB <= 0 || cfg->NB > 16384) { set_error("bad N/NB"); return CHPL_ERR_INVALID; }
    if (cfg->emulate < 0 || cfg->emulate > 2) { set_error("emulate must be 0, 1 or 2"); return CHPL_ERR_INVALID; }
    if (cfg->emulate == 2) { set_error("the Ozaki-I update is the one-GPU engine's (chpl_hpl_run); the grid runs 0 or 1"); return CHPL_ERR_UNSUPPORTED; }
    GridSolver s;
    int rc = s.init(g, *cfg);
    auto finish = [&](int code) { s.destroy(); return code; };
    if (rc != CHPL_OK) return finish(rc);
    // generation (not timed)
    const int P = g->P, Q = g->Q;
    if (s.mloc > 0 && s.nloc > 0) CHPL_TRY(chpl_matgen_cyclic(s.st, s.A, (size_t)s.lda, s.N, s.NB, P, Q, g->pr, g->qc, cfg->seed));
    rc = watchdog_sync(g, s.st, "matgen");
    if (rc != CHPL_OK) return finish(rc);
    cudaEvent_t t0, t1;
    cudaEventCreate(&t0);
    cudaEventCreate(&t1);
    cudaEventRecord(t0, s.st);
    if (s.la) rc = s.run_p1();
    else if (s.la2) rc = s.run_p2();
    else
        for (int64_t b = 0; b < s.nblk && rc == CHPL_OK; ++b) rc = s.block_step(b);
    if (rc == CHPL_OK) rc = s.back_solve();
    if (rc != CHPL_OK) return finish(rc);
    cudaEventRecord(t1, s.st);
    cudaEventSynchronize(t1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, t0, t1);
    cudaEventDestroy(t0);
    cudaEventDestroy(t1);
    int hinfo = 0;
    cudaMemcpy(&hinfo, s.info, sizeof(int), cudaMemcpyDeviceToHost);
    int perr = 0;
    panel_status(s.pwork, &perr);
    int dstat = 0;
    oz2::read_clear_status(&dstat);
    if (perr || dstat) { set_error("device-side timeout (panel %d, update %d)", perr, dstat); return finish(CHPL_ERR_TIMEOUT); }
    res->time_s = ms * 1e-3;
    const double dN = (double)s.N;
    res->tflops = ((2.0 / 3.0) * dN * dN * dN + 2.0 * dN * dN) / res->time_s / 1e12;
    rc = s.residual(&res->resid);
    if (rc != CHPL_OK) return finish(rc);
    res->passed = hinfo == 0 && std::isfinite(res->resid) && res->resid < cfg->threshold;
    s.emu.collect();
    res->schedule = s.la || s.la2 ? 1 : 0;
    // serial block steps: wall time of each step's phases (host clock); lookahead: stream-busy time of each
    // phase (device events), plus the panel factorizations (device events) in phase 0 either way
    double pe[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    s.pev.collect(pe);
    res->phase_s[0] = s.phase[0];
    res->phase_s[1] = s.la || s.la2 ? pe[1] : s.phase[1];
    res->phase_s[2] = s.la || s.la2 ? pe[2] : s.phase[2];
    res->phase_s[3] = pe[3];
    res->phase_s[4] = s.la || s.la2 ? pe[4] : s.phase[3];
    res->phase_s[6] = pe[6];
    res->phase_s[7] = pe[7];
    res->gemm_launches = s.emu.gemm_n;
    res->gemm_kernel_s = s.emu.kernel_s;
    res->gemm_int8_ops = s.emu.ops;
    res->gemm_fp64eq_flops = s.emu.flops;
    res->n_launches = s.n_launch + s.emu.launches;
    res->n_emulated = s.emu.gemm_n;
    if (x_out) {
        cudaError_t e = cudaMemcpy(x_out, s.x, (size_t)s.N * 8, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return finish(cuda_fail(e, "x readback", __FILE__, __LINE__));
    }
    if (hinfo != 0) { set_error("exact zero pivot (info %d)", hinfo); return finish(CHPL_ERR_SINGULAR); }
    return finish(CHPL_OK);
}

}  // namespace chpl

using namespace chpl;

extern "C" int chpl_grid_unique_id(unsigned char* id, size_t len)
{
    if (!id || len < sizeof(ncclUniqueId)) { set_error("unique id buffer must hold %zu bytes", sizeof(ncclUniqueId)); return CHPL_ERR_INVALID; }
    ncclUniqueId u;
    CHPL_NCCL(ncclGetUniqueId(&u));
    std::memcpy(id, &u, sizeof(u));
    return CHPL_OK;
}

extern "C" int chpl_grid_create(int P, int Q, int rank, const unsigned char* id, size_t len, double timeout_s,
                                void** grid)
{
    if (!grid || !id || len < sizeof(ncclUniqueId) || P < 1 || Q < 1 || rank < 0 || rank >= P * Q) {
        set_error("chpl_grid_create: bad arguments");
        return CHPL_ERR_INVALID;
    }
    GridComm* g = new GridComm();
    g->P = P;
    g->Q = Q;
    g->rank = rank;
    g->pr = rank % P;
    g->qc = rank / P;
    g->timeout_s = timeout_s > 0 ? timeout_s : 300.0;
    CHPL_CUDA(cudaGetDevice(&g->dev));
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    // The grid's collectives are broadcasts, point-to-point pairs and tiny
    // reductions: NVLink SHARP (NVLS) would only add multicast buffers to
    // every communicator, so it is off unless the caller set it explicitly.
    setenv("NCCL_NVLS_ENABLE", "0", 0);
    // NCCL kernels run beside the persistent GEMM (lookahead): cap their CTAs
    // (CHPL_NCCL_MAX_CTAS, default 8) so they fit in the SMs the GEMM leaves free
    ncclConfig_t conf = NCCL_CONFIG_INITIALIZER;
    const char* mc = std::getenv("CHPL_NCCL_MAX_CTAS");
    conf.maxCTAs = (mc && *mc) ? std::max(1, std::atoi(mc)) : 8;
    conf.minCTAs = std::min(conf.minCTAs > 0 ? conf.minCTAs : 1, conf.maxCTAs);
    ncclResult_t r = ncclCommInitRankConfig(&g->world, P * Q, u, rank, &conf);
    if (r == ncclSuccess) r = ncclCommSplit(g->world, g->pr, g->qc, &g->row, &conf);   // same process row
    if (r == ncclSuccess) r = ncclCommSplit(g->world, g->qc, g->pr, &g->col, &conf);   // same process column
    if (r == ncclSuccess && P > 1) r = ncclCommSplit(g->world, g->qc, g->pr, &g->col2, &conf);
    if (r != ncclSuccess) {
        set_error("NCCL communicator setup failed: %s", ncclGetErrorString(r));
        delete g;
        return CHPL_ERR_NCCL;
    }
    *grid = g;
    return CHPL_OK;
}

extern "C" int chpl_grid_run(void* grid, const chpl_hpl_config* cfg, chpl_hpl_result* res, double* x_out)
{
    return grid_run(static_cast<GridComm*>(grid), cfg, res, x_out);
}

extern "C" int chpl_grid_destroy(void* grid)
{
    GridComm* g = static_cast<GridComm*>(grid);
    if (!g) return CHPL_OK;
    if (!g->aborted) {
        if (g->row) ncclCommDestroy(g->row);
        if (g->col) ncclCommDestroy(g->col);
        if (g->col2) ncclCommDestroy(g->col2);
        if (g->world) ncclCommDestroy(g->world);
    }
    delete g;
    return CHPL_OK;
}

extern "C" int chpl_grid_plan_exchange(int64_t J, int64_t K, const int64_t* piv, int64_t NB, int P, int pr, int* lsrc,
                                       int* ldst, int* nl, int* snd, int* ns, int* rcv, int* nr)
{
    if (!piv || K < 0 || NB <= 0 || P < 1 || pr < 0 || pr >= P || !nl || !ns || !nr) {
        set_error("chpl_grid_plan_exchange: bad arguments");
        return CHPL_ERR_INVALID;
    }
    for (int64_t i = 0; i < K; ++i)
        if (piv[i] < i) { set_error("pivot %lld < position %lld", (long long)piv[i], (long long)i); return CHPL_ERR_INVALID; }
    std::vector<int> a, b, c, d;
    plan_exchange(J, K, piv, NB, P, pr, a, b, c, d);
    *nl = (int)a.size();
    *ns = (int)c.size();
    *nr = (int)d.size();
    if (lsrc) std::copy(a.begin(), a.end(), lsrc);
    if (ldst) std::copy(b.begin(), b.end(), ldst);
    if (snd) std::copy(c.begin(), c.end(), snd);
    if (rcv) std::copy(d.begin(), d.end(), rcv);
    return CHPL_OK;
}
