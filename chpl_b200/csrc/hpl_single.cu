// Single-GPU HPL solver (P = Q = 1): the chpl_single path of the reference
// (src/chpl_single.cu:658-727) rebuilt around the B200 kernels of this library.
//
// Right-looking blocked LU with partial pivoting of the N x (N+1) system
// [A | b] (b is column N and is carried through the elimination), then one
// upper-triangular solve.  Per NB-wide panel jp:
//   panel   FP64 getrf of the (N-jp) x nb panel (pivots on the device)
//   laswp   the panel's interchanges on all columns right of it (net
//           permutation, no host synchronization)
//   trsm    U12 = L11^-1 A12
//   update  A22 -= L21 U12 through the Ozaki-II emulated GEMM (chpl_oz2_gemm,
//           L21 split once per panel and reused across column chunks), or
//           FP64 DGEMM when emulation is off.
// Columns left of the panel are not interchanged: only U and the transformed
// b are read afterwards (as src/chpl_p2.cu does: its interchanges cover the
// trailing columns only).
//
// Depth-1 lookahead (cfg.lookahead): the columns of panel k+1 are updated
// first, on the high-priority stream sP, which then factors panel k+1 while
// the low-priority stream s0 updates the remaining columns of step k.
// Every FP64 step (triangular solves, the FP64 update, the back substitution)
// runs on this library's kernels (fp64.cu): no cuBLAS / cuSOLVER call.
#include <chrono>
#include <cinttypes>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "fp64.h"
#include "hpl.h"
#include "oz1.h"
#include "oz2.h"

namespace chpl {

// CUDA call whose failure returns fin(status) (fin releases the caller's resources)
#define CHPL_CUDA_OR(call, fin)                                                    \
    do {                                                                           \
        cudaError_t e_ = (call);                                                   \
        if (e_ != cudaSuccess) return fin(::chpl::cuda_fail(e_, #call, __FILE__, __LINE__)); \
    } while (0)

enum Phase { PH_PANEL = 0, PH_LASWP, PH_TRSM, PH_SPLIT, PH_GEMM, PH_UPD_FP64, PH_SOLVE, PH_COMM, PH_N };

namespace {

struct PhaseTimer {
    struct Rec { cudaEvent_t a, b; int ph; };
    std::vector<Rec> recs;
    int begin(cudaStream_t st, int ph, Rec& r)
    {
        r.ph = ph;
        CHPL_CUDA(cudaEventCreate(&r.a));
        CHPL_CUDA(cudaEventCreate(&r.b));
        CHPL_CUDA(cudaEventRecord(r.a, st));
        return CHPL_OK;
    }
    int end(cudaStream_t st, Rec& r)
    {
        CHPL_CUDA(cudaEventRecord(r.b, st));
        recs.push_back(r);
        return CHPL_OK;
    }
    void sums(double* out)
    {
        for (int p = 0; p < PH_N; ++p) out[p] = 0.0;
        for (auto& r : recs) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) out[r.ph] += ms * 1e-3;
        }
    }
    ~PhaseTimer()
    {
        for (auto& r : recs) { cudaEventDestroy(r.a); cudaEventDestroy(r.b); }
    }
};

// Panels per super-block when the caller leaves it to the library (agg = 0).
// Aggregating panels into updates of depth k = 4096 runs the GEMM at its best
// rate, but each emulated update carries an error that grows with sqrt(k), and
// the aggregated form also computes U12 as inv(L) * A12 through the emulated
// GEMM.  The HPL residual divides by eps * N * ||A|| ||x||, which outgrows that
// error only at large N: at 11 moduli the aggregated solve measured residuals
// 23.7 (N = 16384, a failure), 9.1 (32768), 4.8 (65536) and 2.3 (139264),
// while N = 16384 without aggregation (k = NB = 1024) gave 3.9 in the same
// time.  Below N = 65536 the panel dominates anyway, so nothing is aggregated.
// From N = 131072 on, k = 6144: fewer modulus-plane switches per MAC in the
// bulk GEMM outweigh the larger U12 product and inner updates (N = 139264,
// NB = 1024: k = 4096 / 6144 / 8192 ran 13.76 / 13.51 / 13.63 s, residuals
// 2.5 / 3.8 / 5.2).
constexpr int64_t kAggMinN = 65536;
constexpr int64_t kAggDeepN = 131072;
static int auto_agg(int64_t N, int64_t NB)
{
    if (N < kAggMinN) return 1;
    return (int)std::max<int64_t>(1, (N >= kAggDeepN ? 6144 : 4096) / NB);
}

struct Solver {
    chpl_hpl_config cfg{};
    int64_t N = 0, NB = 0, K = 0, ld = 0, ncols = 0;
    int agg = 1, nsm = 148, reserve = 0;
    cudaStream_t s0 = nullptr, sP = nullptr;  // bulk update (low priority), super-block chain (high priority)
    double* A = nullptr;
    int64_t* ipiv = nullptr;
    int* info = nullptr;
    double* xwork = nullptr;               // back substitution scratch (N)
    void* pwork = nullptr;                 // workspace of the FP64 panel kernel
    std::vector<void*> lw[2];              // laswp plans of the panels of a super-block, by super-block parity
    void* wA[2] = {nullptr, nullptr};      // residues of a super-block's L21 (k = K), by parity, shared by streams
    void* wAin = nullptr;                  // residues of a panel's L21 for the inner updates (k = NB), sP only
    double* Linv[2] = {nullptr, nullptr};  // inv(L) of a super-block's unit lower triangle (K x K), by parity
    void* wLinv[2] = {nullptr, nullptr};   // residues of inv(L) (A part, k = K), by parity
    bool emu_trsm = false;                 // U12 = inv(L) * A12 through the emulated GEMM
    // host ingest (a system in host memory, serial schedule): [A | b] arrives on its own copy
    // stream in column chunks while the factorization runs on the chunks already present
    bool ingest = false;
    cudaStream_t sC = nullptr;
    std::vector<int64_t> in_bound;         // chunk c = columns [in_bound[c], in_bound[c + 1])
    std::vector<cudaEvent_t> in_ev;        // chunk c has landed
    std::vector<cudaEvent_t> in_take;      // s0 reached an intake's waits (verbose runs: timed events)
    std::vector<int64_t> in_step;          // its step
    std::vector<size_t> in_first, in_last; // its chunks
    std::vector<void*> lw_old;             // laswp plans of an earlier super-block, rebuilt for a late chunk
    double* Linv_old = nullptr;            // inv(L) of an earlier super-block and its residues, the same
    void* wLinv_old = nullptr;
    void* w0 = nullptr;                    // oz2 B part + scratch for s0
    void* wP = nullptr;                    // oz2 B part + scratch for sP
    int64_t chunk = 0;
    int64_t n_emu = 0;
    int64_t n_launch = 0;                  // kernels of this library issued in factor + solve
    std::vector<PhaseTimer::Rec> gemm_recs;
    double gemm_ops = 0.0, gemm_flops = 0.0;
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_next = 0;
    PhaseTimer clk;

    double* at(int64_t i, int64_t j) { return A + i + j * ld; }

    cudaEvent_t event()
    {
        if (ev_next == ev_pool.size()) {
            cudaEvent_t e;
            cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
            ev_pool.push_back(e);
        }
        return ev_pool[ev_next++];
    }

    int init(const chpl_hpl_config& c)
    {
        cfg = c;
        N = c.N;
        NB = std::min<int64_t>(c.NB, N);
        agg = c.agg > 0 ? c.agg : auto_agg(N, NB);
        K = std::min<int64_t>(agg * NB, N);
        ld = (int64_t)round_up((size_t)N, 32);
        ncols = N + 1;
        nsm = oz2::num_sms();
        reserve = cfg.lookahead ? (c.reserve_sms >= 0 ? c.reserve_sms : 16) : 0;
        // the chain's panels must fit on the reserved SMs (4-column base blocks at the narrowest)
        if (cfg.lookahead) reserve = std::max(reserve, panel_min_ctas(N));
        reserve = std::min(reserve, nsm / 2);
        emu_trsm = cfg.emulate == 1 && (cfg.trsm_mode == 1 || (cfg.trsm_mode == 0 && K > NB));
        int lo = 0, hi = 0;
        CHPL_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
        CHPL_CUDA(cudaStreamCreateWithPriority(&s0, cudaStreamNonBlocking, lo));
        if (cfg.lookahead)
            CHPL_CUDA(cudaStreamCreateWithPriority(&sP, cudaStreamNonBlocking, hi));
        else
            sP = s0;

        const size_t bytesA = (size_t)ld * (size_t)ncols * sizeof(double);
        const int64_t mmax = std::max<int64_t>(N - NB, 0);
        const int64_t wide = std::max<int64_t>(ncols - K, 1);
        // Ozaki-I keeps kOz1Slices int32 products of m x chunk: 4096 columns by default
        chunk = std::min<int64_t>(cfg.chunk > 0 ? cfg.chunk : (cfg.emulate == 2 ? 4096 : 32768), wide);
        size_t tot = 0, a_big = 0, b_big = 0, tot_in = 0, a_in = 0, b_in = 0, oz1b = 0;
        if (cfg.emulate == 2 && mmax > 0) {
            if (chunk + 1024 > 65280) { set_error("ozaki-I: chunk must be <= 64256 columns"); return CHPL_ERR_INVALID; }
            // every call has n <= chunk + 1023 (a narrow tail joins the last chunk) and k <= K
            CHPL_TRY(chpl_oz1_worksize((size_t)mmax, (size_t)std::min<int64_t>(chunk + 1024, wide), (size_t)K, &oz1b));
        }
        if (cfg.emulate == 1 && mmax > 0) {
            const unsigned L = (unsigned)cfg.moduli;
            CHPL_TRY(chpl_oz2_worksize((size_t)mmax, (size_t)std::min<int64_t>(chunk + 1024, wide), (size_t)K, L, 1, 0,
                                       &tot, &a_big, &b_big));
            CHPL_TRY(chpl_oz2_worksize((size_t)mmax, (size_t)std::max<int64_t>(K, 256), (size_t)NB, L, 1, 0, &tot_in,
                                       &a_in, &b_in));
        }
        const size_t rest0 = tot - a_big;                         // B part + scratch for s0 (k = K)
        const size_t restP = std::max(rest0, tot_in - a_in);      // sP runs both k = K and k = NB updates
        size_t freeB = 0, totB = 0;
        CHPL_CUDA(cudaMemGetInfo(&freeB, &totB));
        const int npl = (int)((K + NB - 1) / NB);
        const size_t ozbytes = (cfg.lookahead ? 2 : 1) * a_big + a_in + rest0 + (cfg.lookahead ? restP : 0) +
                               oz1b * (cfg.lookahead ? 2 : 1);
        const size_t pbytes = panel_work_bytes(N, NB);
        size_t linv_res = 0, linv_tot = 0;   // residues of one inv(L) (A part, k = K)
        if (emu_trsm)
            CHPL_TRY(chpl_oz2_worksize((size_t)K, 256, (size_t)K, (unsigned)cfg.moduli, 1, 0, &linv_tot, &linv_res,
                                       nullptr));
        const size_t linv_bytes = emu_trsm ? (size_t)K * K * sizeof(double) + linv_res : 0;
        const size_t need = bytesA + ozbytes + pbytes + (ingest ? 3 : 2) * (npl * laswp_work_bytes(NB) + linv_bytes) +
                            (size_t)(3 * N + 64) * 8 + ((size_t)768 << 20);
        if (cfg.verbose)
            std::printf("MEM PLAN: matrix %.2f GiB | oz2 work %.2f GiB | getrf %.3f GiB | total %.2f GiB vs free %.2f GiB"
                        " | K=%" PRId64 " (agg %d) reserve %d SMs\n",
                        bytesA / 1073741824.0, ozbytes / 1073741824.0, pbytes / 1073741824.0, need / 1073741824.0,
                        freeB / 1073741824.0, K, agg, reserve);
        if (need > freeB) {
            set_error("memory plan: need %.2f GiB, %.2f GiB free (reduce N or HPLS_AGG)", need / 1073741824.0,
                      freeB / 1073741824.0);
            return CHPL_ERR_WORKSPACE;
        }
        CHPL_CUDA(cudaMalloc((void**)&A, bytesA));
        CHPL_CUDA(cudaMalloc((void**)&ipiv, (size_t)N * sizeof(int64_t)));
        CHPL_CUDA(cudaMalloc((void**)&info, 64 * sizeof(int)));
        CHPL_CUDA(cudaMemset(info, 0, 64 * sizeof(int)));
        CHPL_CUDA(cudaMalloc((void**)&xwork, (size_t)N * sizeof(double)));
        CHPL_CUDA(cudaMalloc(&pwork, pbytes));
        for (int b = 0; b < 2; ++b) {
            lw[b].assign(npl, nullptr);
            for (int p = 0; p < npl; ++p) CHPL_CUDA(cudaMalloc(&lw[b][p], laswp_work_bytes(NB)));
        }
        if (ingest) {
            lw_old.assign(npl, nullptr);
            for (int p = 0; p < npl; ++p) CHPL_CUDA(cudaMalloc(&lw_old[p], laswp_work_bytes(NB)));
        }
        if (a_big) {
            // the serial schedule orders every use of L21(s)'s residues before step s+1 splits
            // L21(s+1): one buffer serves both parities
            CHPL_CUDA(cudaMalloc(&wA[0], a_big));
            if (cfg.lookahead) CHPL_CUDA(cudaMalloc(&wA[1], a_big));
            else wA[1] = wA[0];
            CHPL_CUDA(cudaMalloc(&wAin, a_in));
            if (emu_trsm) {
                for (int b = 0; b < 2; ++b) {
                    CHPL_CUDA(cudaMalloc((void**)&Linv[b], (size_t)K * K * sizeof(double)));
                    CHPL_CUDA(cudaMalloc(&wLinv[b], linv_res));
                }
                if (ingest) {
                    CHPL_CUDA(cudaMalloc((void**)&Linv_old, (size_t)K * K * sizeof(double)));
                    CHPL_CUDA(cudaMalloc(&wLinv_old, linv_res));
                }
            }
            CHPL_CUDA(cudaMalloc(&w0, cfg.lookahead ? rest0 : std::max(rest0, restP)));
            if (cfg.lookahead) CHPL_CUDA(cudaMalloc(&wP, restP));
            else wP = w0;
        }
        if (oz1b) {
            CHPL_CUDA(cudaMalloc(&w0, oz1b));
            if (cfg.lookahead) CHPL_CUDA(cudaMalloc(&wP, oz1b));
            else wP = w0;
        }
        return CHPL_OK;
    }

    void destroy()
    {
        if (sC) cudaStreamSynchronize(sC);
        for (auto e : in_ev) cudaEventDestroy(e);
        for (auto e : in_take) cudaEventDestroy(e);
        if (sC) cudaStreamDestroy(sC);
        for (void* p : lw_old) if (p) cudaFree(p);
        if (Linv_old) cudaFree(Linv_old);
        if (wLinv_old) cudaFree(wLinv_old);
        for (auto e : ev_pool) cudaEventDestroy(e);
        if (wP && wP != w0) cudaFree(wP);
        if (w0) cudaFree(w0);
        if (wAin) cudaFree(wAin);
        for (int b = 0; b < 2; ++b) {
            if (Linv[b]) cudaFree(Linv[b]);
            if (wLinv[b]) cudaFree(wLinv[b]);
        }
        for (int b = 0; b < 2; ++b) {
            if (wA[b] && !(b == 1 && wA[1] == wA[0])) cudaFree(wA[b]);
            for (void* p : lw[b]) if (p) cudaFree(p);
        }
        if (pwork) cudaFree(pwork);
        if (xwork) cudaFree(xwork);
        if (info) cudaFree(info);
        if (ipiv) cudaFree(ipiv);
        if (A) cudaFree(A);
        if (sP && sP != s0) cudaStreamDestroy(sP);
        if (s0) cudaStreamDestroy(s0);
    }

    int wait(cudaStream_t waiter, cudaStream_t producer)
    {
        if (waiter == producer) return CHPL_OK;
        cudaEvent_t e = event();
        CHPL_CUDA(cudaEventRecord(e, producer));
        CHPL_CUDA(cudaStreamWaitEvent(waiter, e, 0));
        return CHPL_OK;
    }

    // C[:, c0:c0+nc] -= L21 * U12 with L21 = A(r0:N, a0:a0+k), U12 = A(a0:a0+k, c0:c0+nc),
    // C = A(r0:N, ...).  wa: A part of the residues (split here when split_a).
    int update(cudaStream_t st, void* work, void* wa, bool split_a, int64_t r0, int64_t a0, int64_t k, int64_t c0,
               int64_t nc, int grid_cap)
    {
        return emu(st, work, wa, split_a, N - r0, k, at(r0, a0), ld, a0, c0, nc, at(r0, c0), -1.0, 1.0, grid_cap);
    }

    // C(mt x nc) = alpha * Am(mt x k) * A(a0:a0+k, c0:c0+nc) + beta * C, C at Cp (ld).
    // B is split completely before the GEMM kernel writes C, so C may alias B
    // when beta == 0 (the kernel never reads B or, with beta == 0, C).
    int emu(cudaStream_t st, void* work, void* wa, bool split_a, int64_t mt, int64_t k, const double* Am,
            int64_t lda_m, int64_t a0, int64_t c0, int64_t nc, double* Cp, double alpha, double beta, int grid_cap)
    {
        if (nc <= 0 || mt <= 0 || k <= 0) return CHPL_OK;
        const double one = beta, mone = alpha;
        PhaseTimer::Rec r;
        if (!cfg.emulate) {
            CHPL_TRY(clk.begin(st, PH_UPD_FP64, r));
            CHPL_TRY(dgemm(st, mt, nc, k, mone, Am, lda_m, at(a0, c0), ld, one, Cp, ld));
            ++n_launch;
            CHPL_TRY(clk.end(st, r));
            return CHPL_OK;
        }
        if (cfg.emulate == 2) return emu_oz1(st, work, mt, k, Am, lda_m, a0, c0, nc, Cp, alpha, beta);
        const oz2::Moduli* M = oz2::moduli(cfg.moduli);
        for (int64_t c = 0; c < nc;) {
            int64_t w = std::min(chunk, nc - c);
            if (nc - c - w > 0 && nc - c - w < 1024) w = nc - c;  // absorb a narrow tail (src/chpl_single.cu:637-639)
            // the body of chpl_oz2_gemm, unrolled here to time split and GEMM separately
            const oz2::Layout y = oz2::layout((size_t)mt, (size_t)w, (size_t)k, cfg.moduli, true, false, grid_cap);
            uint8_t* pa = static_cast<uint8_t*>(wa);
            uint8_t* pb = static_cast<uint8_t*>(work) + y.b_off;
            int32_t* shA = reinterpret_cast<int32_t*>(pa + y.a_shift);
            int8_t* resA = reinterpret_cast<int8_t*>(pa + y.a_res);
            int32_t* shB = reinterpret_cast<int32_t*>(pb + y.b_shift);
            int8_t* resB = reinterpret_cast<int8_t*>(pb + y.b_res);
            void* tmp = static_cast<uint8_t*>(work) + y.tmp_off;
            CHPL_TRY(clk.begin(st, PH_SPLIT, r));
            if (split_a && c == 0) {
                CHPL_TRY(oz2::split(st, false, Am, (size_t)lda_m, (size_t)mt, (size_t)k, cfg.moduli, M->alpha, resA,
                                    y.mPad, y.kPad, shA, tmp));
                n_launch += 4;
            }
            CHPL_TRY(oz2::split(st, true, at(a0, c0 + c), (size_t)ld, (size_t)w, (size_t)k, cfg.moduli, M->beta, resB,
                                y.nPad, y.kPad, shB, tmp));
            ++n_launch;
            CHPL_TRY(clk.end(st, r));
            PhaseTimer::Rec g;
            CHPL_TRY(clk.begin(st, PH_GEMM, g));
            CHPL_TRY(oz2::gemm_launch(st, 0, (size_t)mt, (size_t)w, y.kPad, cfg.moduli, resA, y.mPad, resB, y.nPad, shA,
                                      shB, mone, one, Cp + (size_t)c * ld, (size_t)ld, nullptr, 0,
                                      reinterpret_cast<int8_t*>(static_cast<uint8_t*>(work) + y.scratch_off),
                                      y.grid_max));
            CHPL_TRY(clk.end(st, g));
            gemm_recs.push_back(g);
            ++n_launch;
            gemm_ops += 2.0 * (double)mt * (double)w * (double)y.kPad * cfg.moduli;
            gemm_flops += 2.0 * (double)mt * (double)w * (double)k;
            ++n_emu;
            c += w;
        }
        return CHPL_OK;
    }

    // the same product through Ozaki scheme I (src/chpl_single.cu:617-630): digits, diagonal
    // products and the reconstruction inside oz1::gemm, one call per column chunk
    int emu_oz1(cudaStream_t st, void* work, int64_t mt, int64_t k, const double* Am, int64_t lda_m, int64_t a0,
                int64_t c0, int64_t nc, double* Cp, double alpha, double beta)
    {
        for (int64_t c = 0; c < nc;) {
            int64_t w = std::min(chunk, nc - c);
            if (nc - c - w > 0 && nc - c - w < 1024) w = nc - c;
            PhaseTimer::Rec g;
            CHPL_TRY(clk.begin(st, PH_GEMM, g));
            CHPL_TRY(oz1::gemm(st, (size_t)mt, (size_t)w, (size_t)k, alpha, Am, (size_t)lda_m, at(a0, c0 + c),
                               (size_t)ld, beta, Cp + (size_t)c * ld, (size_t)ld, work));
            CHPL_TRY(clk.end(st, g));
            gemm_recs.push_back(g);
            n_launch += oz1::launches();
            const oz1::Layout y = oz1::layout((size_t)mt, (size_t)w, (size_t)k);
            double kk = 0.0;   // K bytes the launch multiplies: diagonal d stops after (d + 1) k
            for (int d = 0; d < oz1::kOz1Slices; ++d)
                kk += (double)std::min<size_t>(y.ldk, round_up((size_t)(d + 1) * (size_t)k, 128));
            gemm_ops += 2.0 * (double)mt * (double)w * kk;
            gemm_flops += 2.0 * (double)mt * (double)w * (double)k;
            ++n_emu;
            c += w;
        }
        return CHPL_OK;
    }

    int laswp_cols(cudaStream_t st, void* plan, int64_t nswaps, int64_t c0, int64_t nc)
    {
        if (nc <= 0) return CHPL_OK;
        PhaseTimer::Rec r;
        CHPL_TRY(clk.begin(st, PH_LASWP, r));
        CHPL_TRY(laswp_apply(st, A, (size_t)ld, c0, nc, nswaps, plan));
        ++n_launch;
        CHPL_TRY(clk.end(st, r));
        return CHPL_OK;
    }

    int trsm(cudaStream_t st, int64_t d0, int64_t kd, int64_t c0, int64_t nc)
    {
        if (nc <= 0 || kd <= 0) return CHPL_OK;
        PhaseTimer::Rec r;
        CHPL_TRY(clk.begin(st, PH_TRSM, r));
        CHPL_TRY(dtrsm_llnu(st, kd, nc, at(d0, d0), ld, at(d0, c0), ld));
        n_launch += dtrsm_launches(kd);
        CHPL_TRY(clk.end(st, r));
        return CHPL_OK;
    }

    int64_t sb_start(int64_t s) const { return s * K; }
    int64_t sb_width(int64_t s) const { return std::max<int64_t>(0, std::min(K, N - s * K)); }

    // Factor super-block s (columns [J, J+KJ), all rows below J) on sP: per
    // panel, FP64 getrf, its interchanges on the super-block's other columns
    // (left: L columns the bulk update reads; right: columns still to factor),
    // U12 of the panel row and the inner update of the super-block's
    // remaining columns.
    int factor_superblock(int64_t s, int cap)
    {
        const int64_t J = sb_start(s), KJ = sb_width(s);
        for (int64_t p = 0; J + p * NB < J + KJ; ++p) {
            const int64_t jp = J + p * NB, nb = std::min(NB, J + KJ - jp);
            void* plan = lw[s & 1][p];
            PhaseTimer::Rec r;
            CHPL_TRY(clk.begin(sP, PH_PANEL, r));
            CHPL_TRY(panel_getrf(sP, N - jp, nb, at(jp, jp), (size_t)ld, ipiv + jp, jp, info + 1, pwork, cap));
            n_launch += 2 * ((nb + 15) / 16) * 2;
            CHPL_TRY(laswp_plan(sP, ipiv, jp, jp + nb, plan));
            n_launch += 2;
            CHPL_TRY(clk.end(sP, r));
            CHPL_TRY(laswp_cols(sP, plan, nb, J, jp - J));
            const int64_t c0 = jp + nb, nc = J + KJ - c0;
            CHPL_TRY(laswp_cols(sP, plan, nb, c0, nc));
            CHPL_TRY(trsm(sP, jp, nb, c0, nc));
            CHPL_TRY(update(sP, wP, wAin, true, jp + nb, jp, nb, c0, nc, cap));
        }
        return invert_l(s);
    }

    // trailing work of super-block s on columns [c0, c0+nc): interchanges and U12
    int trailing_swap_trsm(cudaStream_t st, int64_t s, int64_t c0, int64_t nc)
    {
        const int64_t J = sb_start(s), KJ = sb_width(s);
        for (int64_t p = 0; J + p * NB < J + KJ; ++p)
            CHPL_TRY(laswp_cols(st, lw[s & 1][p], std::min(NB, J + KJ - (J + p * NB)), c0, nc));
        if (!emu_trsm) return trsm(st, J, KJ, c0, nc);
        // U12 = inv(L) * A12 in place (beta = 0: the kernel writes C from residues only)
        return emu(st, st == s0 ? w0 : wP, wLinv[s & 1], false, KJ, KJ, Linv[s & 1], KJ, J, c0, nc, at(J, c0), 1.0, 0.0,
                   st == s0 ? cap_bulk_cur : cap_chain_cur);
    }

    // inv(L) of super-block s (unit lower KJ x KJ at A(J, J)), then its residues
    int invert_l(int64_t s)
    {
        if (!emu_trsm) return CHPL_OK;
        return invert_l_into(sP, s, Linv[s & 1], wLinv[s & 1]);
    }

    // Li = inv(L11) of super-block s (unit lower), then its residues (A part, k = K) into wli
    int invert_l_into(cudaStream_t st, int64_t s, double* Li, void* wli)
    {
        const int64_t J = sb_start(s), KJ = sb_width(s);
        PhaseTimer::Rec r;
        CHPL_TRY(clk.begin(st, PH_TRSM, r));
        CHPL_TRY(dtrtri_llnu(st, KJ, at(J, J), ld, Li, KJ));
        n_launch += 1 + dtrtri_launches(KJ);
        CHPL_TRY(clk.end(st, r));
        const oz2::Moduli* M = oz2::moduli(cfg.moduli);
        const oz2::Layout y = oz2::layout((size_t)KJ, 256, (size_t)KJ, cfg.moduli, true, false);
        uint8_t* pa = static_cast<uint8_t*>(wli);
        CHPL_TRY(clk.begin(st, PH_SPLIT, r));
        CHPL_TRY(oz2::split(st, false, Li, (size_t)KJ, (size_t)KJ, (size_t)KJ, cfg.moduli, M->alpha,
                            reinterpret_cast<int8_t*>(pa + y.a_res), y.mPad, y.kPad, reinterpret_cast<int32_t*>(pa + y.a_shift),
                            static_cast<uint8_t*>(st == s0 ? w0 : wP) + y.tmp_off));
        n_launch += 5;
        CHPL_TRY(clk.end(st, r));
        return CHPL_OK;
    }
    int cap_bulk_cur = 0, cap_chain_cur = 0;

    // Super-block s.  sP: urgent update of super-block s+1's columns (splits
    // L21 once), then factor super-block s+1.  s0: interchanges + U12 of the
    // remaining columns, then the update of super-block s+2's columns ("head",
    // signalled to sP), then the rest.  Without lookahead sP == s0.
    // The bulk update of super-block s runs beside the chain only when it is
    // long enough to hide it: then the persistent GEMM of the bulk leaves
    // `reserve` SMs free and the chain's GEMMs use only those.
    bool overlapped(int64_t s) const
    {
        const int64_t c2 = std::min(N, sb_start(s) + sb_width(s) + sb_width(s + 1));
        return cfg.lookahead && reserve > 0 && (N - c2) >= 8 * K;
    }

    // x = U^-1 b': the back substitution on column N, on s0
    int back_solve()
    {
        PhaseTimer::Rec r;
        CHPL_TRY(clk.begin(s0, PH_SOLVE, r));
        CHPL_TRY(dtrsv_unn(s0, N, A, ld, at(0, N), xwork));
        n_launch += dtrsv_launches(N);
        CHPL_TRY(clk.end(s0, r));
        return CHPL_OK;
    }

    // Enqueue [A | b] from host memory (leading dimension ldab) on the copy stream in column
    // chunks of 2K columns (two super-blocks; the last chunk ends at column N), each followed
    // by its event.  The copies start once `start` has been reached on s0.
    int ingest_enqueue(const double* Ab, size_t ldab, cudaEvent_t start)
    {
        CHPL_CUDA(cudaStreamCreateWithFlags(&sC, cudaStreamNonBlocking));
        CHPL_CUDA(cudaStreamWaitEvent(sC, start, 0));
        in_bound.assign(1, 0);
        while (in_bound.back() < ncols) in_bound.push_back(std::min<int64_t>(ncols, in_bound.back() + 2 * K));
        for (size_t c = 0; c + 1 < in_bound.size(); ++c) {
            const int64_t a = in_bound[c], b = in_bound[c + 1];
            CHPL_CUDA(cudaMemcpy2DAsync(at(0, a), (size_t)ld * sizeof(double), Ab + (size_t)a * ldab,
                                        ldab * sizeof(double), (size_t)N * sizeof(double), (size_t)(b - a),
                                        cudaMemcpyHostToDevice, sC));
            cudaEvent_t e;
            CHPL_CUDA(cudaEventCreateWithFlags(&e, cfg.verbose ? cudaEventDefault : cudaEventDisableTiming));
            in_ev.push_back(e);
            CHPL_CUDA(cudaEventRecord(e, sC));
        }
        return CHPL_OK;
    }

    // Super-block t's interchanges, U12 and trailing update on the columns [c0, c0 + nc), on s0.
    // live: t is the super-block factored last (its plans and inv(L) residues are current);
    // otherwise they are rebuilt from ipiv and L11(t), which the matrix still holds, and give
    // the same values.
    int apply_step(int64_t t, bool live, int64_t c0, int64_t nc)
    {
        if (nc <= 0) return CHPL_OK;
        const int64_t J = sb_start(t), KJ = sb_width(t);
        std::vector<void*>& plans = live ? lw[t & 1] : lw_old;
        for (int64_t p = 0; J + p * NB < J + KJ; ++p) {
            const int64_t jp = J + p * NB, nb = std::min(NB, J + KJ - jp);
            if (!live) {
                CHPL_TRY(laswp_plan(s0, ipiv, jp, jp + nb, plans[p]));
                n_launch += 2;
            }
            CHPL_TRY(laswp_cols(s0, plans[p], nb, c0, nc));
        }
        if (!emu_trsm) CHPL_TRY(trsm(s0, J, KJ, c0, nc));
        else {
            double* Li = live ? Linv[t & 1] : Linv_old;
            void* wli = live ? wLinv[t & 1] : wLinv_old;
            if (!live) CHPL_TRY(invert_l_into(s0, t, Li, wli));
            CHPL_TRY(emu(s0, w0, wli, false, KJ, KJ, Li, KJ, J, c0, nc, at(J, c0), 1.0, 0.0, 0));
        }
        return update(s0, w0, wA[0], true, J + KJ, J, KJ, c0, nc, 0);
    }

    // The serial factorization over a matrix still arriving (ingest_enqueue).  Before
    // super-block s is factored, the chunks holding its columns are taken in, together with
    // every later chunk whose copy has already completed when the host gets there (one
    // intake: the columns catch up on steps 0..s-1 in one pass per step, with L21 split
    // again and inv(L11) rebuilt for each); then step s runs on all columns present.  Every
    // column gets the same operations in the same order as in factor_and_solve's serial
    // schedule whatever the intakes were, so the results are bit-identical to it.
    int factor_and_solve_ingest()
    {
        const int64_t nsb = (N + K - 1) / K;
        const size_t nch = in_ev.size();
        int64_t ready = 0;   // columns [0, ready) are present and up to date with the steps issued
        size_t c = 0;
        for (int64_t s = 0; s < nsb; ++s) {
            const int64_t J = sb_start(s), KJ = sb_width(s), c1 = J + KJ;
            size_t e = c;
            while (e < nch && (in_bound[e] < c1 || s == nsb - 1 || cudaEventQuery(in_ev[e]) == cudaSuccess)) ++e;
            if (e > c) {
                if (cfg.verbose) {
                    cudaEvent_t ev;
                    CHPL_CUDA(cudaEventCreate(&ev));
                    CHPL_CUDA(cudaEventRecord(ev, s0));
                    in_take.push_back(ev);
                    in_step.push_back(s);
                    in_first.push_back(c);
                    in_last.push_back(e - 1);
                }
                for (size_t q = c; q < e; ++q) CHPL_CUDA(cudaStreamWaitEvent(s0, in_ev[q], 0));
                const int64_t a = in_bound[c], b = in_bound[e];
                for (int64_t t = 0; t < s; ++t) CHPL_TRY(apply_step(t, false, a, b - a));
                ready = b;
                c = e;
            }
            CHPL_TRY(factor_superblock(s, 0));
            CHPL_TRY(apply_step(s, true, c1, ready - c1));
        }
        return back_solve();
    }

    int factor_and_solve()
    {
        const int64_t nsb = (N + K - 1) / K;
        CHPL_TRY(factor_superblock(0, 0));
        cudaEvent_t ev_head = nullptr;   // bulk(s-1) finished super-block s+1's columns
        for (int64_t s = 0; s < nsb; ++s) {
            const int64_t J = sb_start(s), KJ = sb_width(s);
            const int64_t c1 = J + KJ, K1 = sb_width(s + 1);
            const int64_t c2 = c1 + K1, K2 = std::max<int64_t>(0, std::min(K, N - c2));
            const int cap_prev = (s > 0 && overlapped(s - 1)) ? reserve : 0;   // urgent(s) runs beside bulk(s-1)
            const int cap_chain = overlapped(s) ? reserve : 0;                 // factor(s+1) runs beside bulk(s)
            const int cap_bulk = overlapped(s) ? nsm - reserve : 0;
            cap_bulk_cur = cap_bulk;
            cap_chain_cur = cap_prev;
            if (ev_head) CHPL_CUDA(cudaStreamWaitEvent(sP, ev_head, 0));
            CHPL_TRY(trailing_swap_trsm(sP, s, c1, K1));
            CHPL_TRY(update(sP, wP, wA[s & 1], true, c1, J, KJ, c1, K1, cap_prev));
            const bool a_split = K1 > 0 && N - c1 > 0;
            CHPL_TRY(wait(s0, sP));
            cap_chain_cur = cap_chain;
            if (K1 > 0) CHPL_TRY(factor_superblock(s + 1, cap_chain));
            CHPL_TRY(trailing_swap_trsm(s0, s, c2, ncols - c2));
            CHPL_TRY(update(s0, w0, wA[s & 1], !a_split, c1, J, KJ, c2, K2, cap_bulk));
            ev_head = event();
            CHPL_CUDA(cudaEventRecord(ev_head, s0));
            CHPL_TRY(update(s0, w0, wA[s & 1], !a_split && K2 == 0, c1, J, KJ, c2 + K2, ncols - c2 - K2, cap_bulk));
        }
        CHPL_TRY(wait(s0, sP));
        return back_solve();
    }

    void gemm_stats(chpl_hpl_result* res)
    {
        double t = 0.0;
        for (auto& g : gemm_recs) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, g.a, g.b) == cudaSuccess) t += ms * 1e-3;
        }
        res->gemm_launches = (int64_t)gemm_recs.size();
        res->gemm_kernel_s = t;
        res->gemm_int8_ops = gemm_ops;
        res->gemm_fp64eq_flops = gemm_flops;
        res->n_launches = n_launch;
    }
};

}  // namespace

namespace {

struct Events {
    cudaEvent_t e[4] = {nullptr, nullptr, nullptr, nullptr};
    int create()
    {
        for (auto& x : e) CHPL_CUDA(cudaEventCreate(&x));
        return CHPL_OK;
    }
    ~Events()
    {
        for (auto x : e)
            if (x) cudaEventDestroy(x);
    }
};

// One solve.  Ab == nullptr: the generated system (seed cfg->seed), verified
// against the generator.  Otherwise [A | b] is copied in from host memory Ab
// (leading dimension ldab) and, when verify, copied in again after the solve
// to compute the residual against it.
int run_impl(const chpl_hpl_config* cfg, const double* Ab, size_t ldab, int verify, chpl_hpl_result* res,
             double* x_out)
{
    if (!cfg || !res) { set_error("cfg/res NULL"); return CHPL_ERR_INVALID; }
    std::memset(res, 0, sizeof(*res));
    if (cfg->N <= 0 || cfg->NB <= 0 || cfg->NB > 2048) { set_error("bad N/NB (NB must be in [1, 2048])"); return CHPL_ERR_INVALID; }
    if (cfg->agg < 0 || (int64_t)cfg->agg * cfg->NB > 16384) { set_error("agg * NB must be <= 16384"); return CHPL_ERR_INVALID; }
    if (cfg->P != 1 || cfg->Q != 1) { set_error("chpl_hpl_run drives one GPU; use the grid driver for P x Q > 1"); return CHPL_ERR_INVALID; }
    if (cfg->panel_mode != 0) { set_error("panel_mode: only this library's FP64 panel kernel (0) is built"); return CHPL_ERR_UNSUPPORTED; }
    if (cfg->emulate < 0 || cfg->emulate > 2) { set_error("emulate must be 0 (FP64), 1 (Ozaki-II) or 2 (Ozaki-I)"); return CHPL_ERR_INVALID; }
    if (cfg->emulate == 1 && !oz2::moduli(cfg->moduli)) { set_error("moduli must be in [2, 16]"); return CHPL_ERR_INVALID; }
    if (Ab && (int64_t)ldab < cfg->N) { set_error("ldab < N"); return CHPL_ERR_INVALID; }
    if (cfg->generator != CHPL_GEN_CHPL && cfg->generator != CHPL_GEN_PHILOX) {
        set_error("generator must be CHPL_GEN_CHPL or CHPL_GEN_PHILOX");
        return CHPL_ERR_INVALID;
    }
    Solver s;
    // a system in host memory streams in while the serial schedule factors what has arrived
    s.ingest = Ab != nullptr && !cfg->lookahead;
    int rc = s.init(*cfg);
    if (rc != CHPL_OK) { s.destroy(); return rc; }
    double* xs = nullptr;   // x kept aside while [A | b] is copied in again for the residual
    auto finish = [&](int code) {
        if (xs) cudaFree(xs);
        s.destroy();
        return code;
    };
    Events ev;
    rc = ev.create();
    if (rc != CHPL_OK) return finish(rc);
    cudaEvent_t g0 = ev.e[0], g1 = ev.e[1], t0 = ev.e[2], t1 = ev.e[3];
    const size_t row_bytes = (size_t)s.N * sizeof(double);
    cudaEventRecord(g0, s.s0);
    if (Ab && !s.ingest) {
        cudaError_t e = cudaMemcpy2DAsync(s.A, (size_t)s.ld * sizeof(double), Ab, ldab * sizeof(double), row_bytes,
                                          (size_t)s.ncols, cudaMemcpyHostToDevice, s.s0);
        if (e != cudaSuccess) return finish(cuda_fail(e, "[A|b] host to device", __FILE__, __LINE__));
    } else if (!Ab) {
        rc = matgen(s.s0, s.A, (size_t)s.ld, (size_t)s.N, (size_t)s.ncols, 0, 0, s.ncols, cfg->seed, cfg->generator);
        if (rc != CHPL_OK) return finish(rc);
    }
    cudaEventRecord(g1, s.s0);
    cudaEventRecord(t0, s.s0);
    cudaStreamWaitEvent(s.sP, t0, 0);
    if (s.ingest) {   // the timed region then covers the host-to-device copy as well
        rc = s.ingest_enqueue(Ab, ldab, t0);
        if (rc == CHPL_OK) rc = s.factor_and_solve_ingest();
    } else {
        rc = s.factor_and_solve();
    }
    if (rc != CHPL_OK) { cudaDeviceSynchronize(); return finish(rc); }
    cudaEventRecord(t1, s.s0);
    cudaError_t e = cudaEventSynchronize(t1);
    if (e != cudaSuccess) return finish(cuda_fail(e, "solve", __FILE__, __LINE__));
    float ms_gen = 0.f, ms = 0.f;
    cudaEventElapsedTime(&ms_gen, g0, g1);
    cudaEventElapsedTime(&ms, t0, t1);
    if (s.ingest && cfg->verbose) {   // when each intake's last chunk landed and when the factorization reached it
        for (size_t i = 0; i < s.in_take.size(); ++i) {
            float landed = 0.f, reached = 0.f;
            cudaEventElapsedTime(&landed, t0, s.in_ev[s.in_last[i]]);
            cudaEventElapsedTime(&reached, t0, s.in_take[i]);
            std::printf("INGEST: step %" PRId64 " takes chunks %zu..%zu, columns [%" PRId64 ", %" PRId64
                        "): landed %.1f ms, reached %.1f ms\n",
                        s.in_step[i], s.in_first[i], s.in_last[i], s.in_bound[s.in_first[i]],
                        s.in_bound[s.in_last[i] + 1], landed, reached);
        }
        std::fflush(stdout);
    }
    int hinfo = 0;
    cudaMemcpy(&hinfo, s.info + 1, sizeof(int), cudaMemcpyDeviceToHost);
    int perr = 0;
    if (s.pwork) panel_status(s.pwork, &perr);
    if (perr) { set_error("device-side timeout in the panel factorization"); return finish(CHPL_ERR_TIMEOUT); }
    int dstat = 0;
    oz2::read_clear_status(&dstat);
    if (dstat) { set_error("device-side timeout in the emulated update"); return finish(CHPL_ERR_TIMEOUT); }
    res->time_s = ms * 1e-3;
    res->matgen_s = ms_gen * 1e-3;
    const double dN = (double)s.N;
    res->tflops = ((2.0 / 3.0) * dN * dN * dN + 2.0 * dN * dN) / res->time_s / 1e12;
    s.clk.sums(res->phase_s);
    res->n_emulated = s.n_emu;
    s.gemm_stats(res);
    // x = column N
    const double* dx = s.at(0, s.N);
    if (!Ab) {
        rc = residual(s.s0, s.N, cfg->seed, dx, &res->resid, cfg->generator);
        if (rc != CHPL_OK) return finish(rc);
    } else if (verify) {
        CHPL_CUDA_OR(cudaMalloc((void**)&xs, row_bytes), finish);
        CHPL_CUDA_OR(cudaMemcpyAsync(xs, dx, row_bytes, cudaMemcpyDeviceToDevice, s.s0), finish);
        CHPL_CUDA_OR(cudaMemcpy2DAsync(s.A, (size_t)s.ld * sizeof(double), Ab, ldab * sizeof(double), row_bytes,
                                       (size_t)s.ncols, cudaMemcpyHostToDevice, s.s0), finish);
        rc = residual_matrix(s.s0, s.N, s.A, (size_t)s.ld, xs, &res->resid);
        if (rc != CHPL_OK) return finish(rc);
        dx = xs;
    } else {
        res->resid = std::nan("");
    }
    res->passed = (hinfo == 0) && std::isfinite(res->resid) && res->resid < cfg->threshold;
    if (x_out) {
        e = cudaMemcpyAsync(x_out, dx, row_bytes, cudaMemcpyDeviceToHost, s.s0);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s.s0);
        if (e != cudaSuccess) return finish(cuda_fail(e, "x readback", __FILE__, __LINE__));
    }
    if (hinfo != 0) { set_error("exact zero pivot at column %d", hinfo); return finish(CHPL_ERR_SINGULAR); }
    return finish(CHPL_OK);
}

}  // namespace

int hpl_single_run(const chpl_hpl_config* cfg, chpl_hpl_result* res, double* x_out)
{
    return run_impl(cfg, nullptr, 0, 1, res, x_out);
}

int hpl_single_run_host(const chpl_hpl_config* cfg, const double* Ab, size_t ldab, int verify, chpl_hpl_result* res,
                        double* x_out)
{
    if (!Ab) { set_error("Ab is NULL"); return CHPL_ERR_INVALID; }
    return run_impl(cfg, Ab, ldab, verify, res, x_out);
}

}  // namespace chpl

extern "C" void chpl_hpl_default_config(chpl_hpl_config* cfg)
{
    if (!cfg) return;
    std::memset(cfg, 0, sizeof(*cfg));
    cfg->N = 16384;     // src/chpl_p2.cu:570 fallback
    cfg->NB = 1024;
    cfg->P = 1;
    cfg->Q = 1;
    cfg->moduli = 11;
    cfg->emulate = 1;
    cfg->fast = 1;
    cfg->chunk = 0;
    cfg->lookahead = 0;
    cfg->agg = 0;
    cfg->reserve_sms = -1;
    cfg->seed = 42;
    cfg->threshold = 16.0;
    cfg->verbose = 0;
    cfg->generator = CHPL_GEN_CHPL;
}

extern "C" int chpl_hpl_run(const chpl_hpl_config* cfg, chpl_hpl_result* res, double* x_out)
{
    return chpl::hpl_single_run(cfg, res, x_out);
}

extern "C" int chpl_hpl_run_host(const chpl_hpl_config* cfg, const double* Ab, size_t ldab, int verify,
                                 chpl_hpl_result* res, double* x_out)
{
    return chpl::hpl_single_run_host(cfg, Ab, ldab, verify, res, x_out);
}
