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
// b are read afterwards (as src/chpl_p2.cu does, docs/DESIGN.md section 6.2).
//
// Depth-1 lookahead (cfg.lookahead): the columns of panel k+1 are updated
// first, on the high-priority stream sP, which then factors panel k+1 while
// the low-priority stream s0 updates the remaining columns of step k.
#include <cublas_v2.h>
#include <cusolverDn.h>

#include <chrono>
#include <cinttypes>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "hpl.h"
#include "oz2.h"

namespace chpl {

#define CHPL_CUBLAS(call)                                                          \
    do {                                                                           \
        cublasStatus_t s_ = (call);                                                \
        if (s_ != CUBLAS_STATUS_SUCCESS) {                                         \
            set_error("cuBLAS error %d in %s at %s:%d", (int)s_, #call, __FILE__, __LINE__); \
            return CHPL_ERR_CUDA;                                                  \
        }                                                                          \
    } while (0)
#define CHPL_CUSOLVER(call)                                                        \
    do {                                                                           \
        cusolverStatus_t s_ = (call);                                              \
        if (s_ != CUSOLVER_STATUS_SUCCESS) {                                       \
            set_error("cuSOLVER error %d in %s at %s:%d", (int)s_, #call, __FILE__, __LINE__); \
            return CHPL_ERR_CUDA;                                                  \
        }                                                                          \
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

struct Solver {
    chpl_hpl_config cfg{};
    int64_t N = 0, NB = 0, ld = 0, ncols = 0;
    cudaStream_t s0 = nullptr, sP = nullptr;  // bulk update (low priority), panel chain (high priority)
    cublasHandle_t hb0 = nullptr, hbP = nullptr;
    cusolverDnHandle_t hs = nullptr;
    cusolverDnParams_t hp = nullptr;
    double* A = nullptr;
    int64_t* ipiv_rel = nullptr;
    int64_t* ipiv = nullptr;
    int* info = nullptr;
    void* fwork_d = nullptr;
    void* fwork_h = nullptr;
    size_t fwd = 0, fwh = 0;
    void* lwork[2] = {nullptr, nullptr};   // laswp plans, by panel parity
    void* wA[2] = {nullptr, nullptr};      // L21 residues, by panel parity (shared by both streams)
    void* w0 = nullptr;                    // oz2 B part + scratch for s0
    void* wP = nullptr;                    // oz2 B part + scratch for sP
    size_t wsA = 0, wsRest = 0;
    int64_t chunk = 0;
    int64_t n_emu = 0;
    int64_t n_launch = 0;          // kernels of this library issued in factor + solve
    std::vector<PhaseTimer::Rec> gemm_recs;   // one per tcgen05 GEMM launch
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
        NB = c.NB;
        ld = (int64_t)round_up((size_t)N, 32);
        ncols = N + 1;
        int lo = 0, hi = 0;
        CHPL_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
        CHPL_CUDA(cudaStreamCreateWithPriority(&s0, cudaStreamNonBlocking, lo));
        if (cfg.lookahead)
            CHPL_CUDA(cudaStreamCreateWithPriority(&sP, cudaStreamNonBlocking, hi));
        else
            sP = s0;
        CHPL_CUBLAS(cublasCreate(&hb0));
        CHPL_CUBLAS(cublasSetStream(hb0, s0));
        CHPL_CUBLAS(cublasCreate(&hbP));
        CHPL_CUBLAS(cublasSetStream(hbP, sP));
        CHPL_CUSOLVER(cusolverDnCreate(&hs));
        CHPL_CUSOLVER(cusolverDnSetStream(hs, sP));
        CHPL_CUSOLVER(cusolverDnCreateParams(&hp));

        const size_t bytesA = (size_t)ld * (size_t)ncols * sizeof(double);
        const int64_t mmax = N > NB ? N - NB : 0;
        const int64_t wide = ncols - NB;
        chunk = cfg.chunk > 0 ? std::min<int64_t>(cfg.chunk, wide) : wide;
        size_t total = 0, wsB = 0;
        if (cfg.emulate && mmax > 0 && wide > 0) {
            const int64_t nmax = std::min<int64_t>(chunk + 1024, wide);
            CHPL_TRY(chpl_oz2_worksize((size_t)mmax, (size_t)nmax, (size_t)NB, (unsigned)cfg.moduli, 1, 0, &total, &wsA,
                                       &wsB));
            wsRest = total - wsA;
        }
        size_t freeB = 0, totB = 0;
        CHPL_CUDA(cudaMemGetInfo(&freeB, &totB));
        CHPL_CUSOLVER(cusolverDnXgetrf_bufferSize(hs, hp, N, NB, CUDA_R_64F, nullptr, ld, CUDA_R_64F, &fwd, &fwh));
        const int nrest = cfg.lookahead ? 2 : 1;
        const size_t ozbytes = 2 * wsA + nrest * wsRest;
        const size_t need = bytesA + ozbytes + fwd + 2 * laswp_work_bytes(NB) + (size_t)(2 * N + 64) * 8 +
                            ((size_t)512 << 20);
        if (cfg.verbose)
            std::printf("MEM PLAN: matrix %.2f GiB | oz2 work %.2f GiB | getrf %.3f GiB | total %.2f GiB vs free %.2f GiB\n",
                        bytesA / 1073741824.0, ozbytes / 1073741824.0, fwd / 1073741824.0, need / 1073741824.0,
                        freeB / 1073741824.0);
        if (need > freeB) {
            set_error("memory plan: need %.2f GiB, %.2f GiB free (reduce N)", need / 1073741824.0, freeB / 1073741824.0);
            return CHPL_ERR_WORKSPACE;
        }
        CHPL_CUDA(cudaMalloc((void**)&A, bytesA));
        CHPL_CUDA(cudaMalloc((void**)&ipiv_rel, (size_t)NB * sizeof(int64_t)));
        CHPL_CUDA(cudaMalloc((void**)&ipiv, (size_t)N * sizeof(int64_t)));
        CHPL_CUDA(cudaMalloc((void**)&info, 64 * sizeof(int)));
        CHPL_CUDA(cudaMemset(info, 0, 64 * sizeof(int)));
        CHPL_CUDA(cudaMalloc(&fwork_d, fwd ? fwd : 8));
        fwork_h = std::malloc(fwh ? fwh : 8);
        for (int b = 0; b < 2; ++b) CHPL_CUDA(cudaMalloc(&lwork[b], laswp_work_bytes(NB)));
        if (wsA) {
            for (int b = 0; b < 2; ++b) CHPL_CUDA(cudaMalloc(&wA[b], wsA));
            CHPL_CUDA(cudaMalloc(&w0, wsRest));
            if (cfg.lookahead) CHPL_CUDA(cudaMalloc(&wP, wsRest));
            else wP = w0;
        }
        return CHPL_OK;
    }

    void destroy()
    {
        for (auto e : ev_pool) cudaEventDestroy(e);
        if (wP && wP != w0) cudaFree(wP);
        if (w0) cudaFree(w0);
        for (int b = 0; b < 2; ++b) {
            if (wA[b]) cudaFree(wA[b]);
            if (lwork[b]) cudaFree(lwork[b]);
        }
        if (fwork_d) cudaFree(fwork_d);
        std::free(fwork_h);
        if (info) cudaFree(info);
        if (ipiv) cudaFree(ipiv);
        if (ipiv_rel) cudaFree(ipiv_rel);
        if (A) cudaFree(A);
        if (hp) cusolverDnDestroyParams(hp);
        if (hs) cusolverDnDestroy(hs);
        if (hbP) cublasDestroy(hbP);
        if (hb0) cublasDestroy(hb0);
        if (sP && sP != s0) cudaStreamDestroy(sP);
        if (s0) cudaStreamDestroy(s0);
    }

    // factor panel k (rows jp..N-1, columns [jp, jp+nb)) on sP and plan its interchanges
    int panel(int64_t k)
    {
        const int64_t jp = k * NB, nb = std::min(NB, N - jp);
        PhaseTimer::Rec r;
        CHPL_TRY(clk.begin(sP, PH_PANEL, r));
        CHPL_CUSOLVER(cusolverDnXgetrf(hs, hp, N - jp, nb, CUDA_R_64F, at(jp, jp), ld, ipiv_rel, CUDA_R_64F, fwork_d,
                                       fwd, fwork_h, fwh, info + 1));
        CHPL_TRY(ipiv_to_abs(sP, ipiv_rel, nb, jp, ipiv + jp));
        CHPL_TRY(laswp_plan(sP, ipiv, jp, jp + nb, lwork[k & 1]));
        n_launch += 2;
        CHPL_TRY(clk.end(sP, r));
        return CHPL_OK;
    }

    // interchanges + U12 = L11^-1 A12 for columns [c0, c0+nc) of step k
    int swap_trsm(cudaStream_t st, cublasHandle_t hb, int64_t k, int64_t c0, int64_t nc)
    {
        if (nc <= 0) return CHPL_OK;
        const int64_t jp = k * NB, nb = std::min(NB, N - jp);
        const double one = 1.0;
        PhaseTimer::Rec r;
        CHPL_TRY(clk.begin(st, PH_LASWP, r));
        CHPL_TRY(laswp_apply(st, A, (size_t)ld, c0, nc, nb, lwork[k & 1]));
        ++n_launch;
        CHPL_TRY(clk.end(st, r));
        CHPL_TRY(clk.begin(st, PH_TRSM, r));
        CHPL_CUBLAS(cublasDtrsm_64(hb, CUBLAS_SIDE_LEFT, CUBLAS_FILL_MODE_LOWER, CUBLAS_OP_N, CUBLAS_DIAG_UNIT, nb, nc,
                                   &one, at(jp, jp), ld, at(jp, c0), ld));
        CHPL_TRY(clk.end(st, r));
        return CHPL_OK;
    }

    // A22[:, c0:c0+nc] -= L21 U12 for step k; split_a: quantize L21 here
    int gemm(cudaStream_t st, cublasHandle_t hb, void* work, int64_t k, int64_t c0, int64_t nc, bool split_a)
    {
        const int64_t jp = k * NB, nb = std::min(NB, N - jp), mt = N - (jp + nb);
        if (nc <= 0 || mt <= 0) return CHPL_OK;
        const double one = 1.0, mone = -1.0;
        PhaseTimer::Rec r;
        if (!cfg.emulate) {
            CHPL_TRY(clk.begin(st, PH_UPD_FP64, r));
            CHPL_CUBLAS(cublasDgemm_64(hb, CUBLAS_OP_N, CUBLAS_OP_N, mt, nc, nb, &mone, at(jp + nb, jp), ld, at(jp, c0),
                                       ld, &one, at(jp + nb, c0), ld));
            CHPL_TRY(clk.end(st, r));
            return CHPL_OK;
        }
        const oz2::Moduli* M = oz2::moduli(cfg.moduli);
        for (int64_t c = 0; c < nc;) {
            int64_t w = std::min(chunk, nc - c);
            if (nc - c - w > 0 && nc - c - w < 1024) w = nc - c;  // absorb a narrow tail (src/chpl_single.cu:637-639)
            // the body of chpl_oz2_gemm, unrolled here to time split and GEMM separately
            const oz2::Layout y = oz2::layout((size_t)mt, (size_t)w, (size_t)nb, cfg.moduli, true, false);
            uint8_t* pa = static_cast<uint8_t*>(wA[k & 1]);
            uint8_t* pb = static_cast<uint8_t*>(work) + y.b_off;
            int32_t* shA = reinterpret_cast<int32_t*>(pa + y.a_shift);
            int8_t* resA = reinterpret_cast<int8_t*>(pa + y.a_res);
            int32_t* shB = reinterpret_cast<int32_t*>(pb + y.b_shift);
            int8_t* resB = reinterpret_cast<int8_t*>(pb + y.b_res);
            void* tmp = static_cast<uint8_t*>(work) + y.tmp_off;
            CHPL_TRY(clk.begin(st, PH_SPLIT, r));
            if (split_a && c == 0) {
                CHPL_TRY(oz2::split(st, false, at(jp + nb, jp), (size_t)ld, (size_t)mt, (size_t)nb, cfg.moduli, M->alpha,
                                    resA, y.mPad, y.kPad, shA, tmp));
                n_launch += 4;
            }
            CHPL_TRY(oz2::split(st, true, at(jp, c0 + c), (size_t)ld, (size_t)w, (size_t)nb, cfg.moduli, M->beta, resB,
                                y.nPad, y.kPad, shB, tmp));
            ++n_launch;
            CHPL_TRY(clk.end(st, r));
            PhaseTimer::Rec g;
            CHPL_TRY(clk.begin(st, PH_GEMM, g));
            CHPL_TRY(oz2::gemm_launch(st, 0, (size_t)mt, (size_t)w, y.kPad, cfg.moduli, resA, y.mPad, resB, y.nPad, shA,
                                      shB, mone, one, at(jp + nb, c0 + c), (size_t)ld, nullptr, 0,
                                      reinterpret_cast<int8_t*>(static_cast<uint8_t*>(work) + y.scratch_off),
                                      y.grid_max));
            CHPL_TRY(clk.end(st, g));
            gemm_recs.push_back(g);
            ++n_launch;
            gemm_ops += 2.0 * (double)mt * (double)w * (double)y.kPad * cfg.moduli;
            gemm_flops += 2.0 * (double)mt * (double)w * (double)nb;
            ++n_emu;
            c += w;
        }
        return CHPL_OK;
    }

    int wait(cudaStream_t waiter, cudaStream_t producer)
    {
        if (waiter == producer) return CHPL_OK;
        cudaEvent_t e = event();
        CHPL_CUDA(cudaEventRecord(e, producer));
        CHPL_CUDA(cudaStreamWaitEvent(waiter, e, 0));
        return CHPL_OK;
    }

    // Step k.  sP: urgent update of panel k+1's columns (splits L21 once),
    // then factor panel k+1.  s0: interchanges + U12 of the remaining columns,
    // then the update of panel k+2's columns ("head", signalled to sP), then
    // the rest.  Without lookahead sP == s0 and the same order runs serially.
    int factor_and_solve()
    {
        const int64_t npan = (N + NB - 1) / NB;
        CHPL_TRY(panel(0));
        cudaEvent_t ev_head = nullptr;  // bulk(k-1) finished panel k+1's columns
        for (int64_t k = 0; k < npan; ++k) {
            const int64_t jp = k * NB, nb = std::min(NB, N - jp);
            const int64_t c1 = jp + nb;                                   // panel k+1's first column
            const int64_t nb1 = std::max<int64_t>(0, std::min(NB, N - c1));
            const int64_t c2 = c1 + nb1;                                  // panel k+2's first column
            const int64_t nb2 = std::max<int64_t>(0, std::min(NB, N - c2));
            // urgent (sP): columns of panel k+1 must have received step k-1 first
            if (ev_head) CHPL_CUDA(cudaStreamWaitEvent(sP, ev_head, 0));
            CHPL_TRY(swap_trsm(sP, hbP, k, c1, nb1));
            CHPL_TRY(gemm(sP, hbP, wP, k, c1, nb1, true));
            const bool a_split = nb1 > 0 && N - c1 > 0;
            // bulk (s0) needs panel k factored and L21 split by the urgent update
            CHPL_TRY(wait(s0, sP));
            if (nb1 > 0) CHPL_TRY(panel(k + 1));
            CHPL_TRY(swap_trsm(s0, hb0, k, c2, ncols - c2));
            CHPL_TRY(gemm(s0, hb0, w0, k, c2, nb2, !a_split));
            ev_head = event();
            CHPL_CUDA(cudaEventRecord(ev_head, s0));
            CHPL_TRY(gemm(s0, hb0, w0, k, c2 + nb2, ncols - c2 - nb2, !a_split && nb2 == 0));
        }
        CHPL_TRY(wait(s0, sP));
        PhaseTimer::Rec r;
        CHPL_TRY(clk.begin(s0, PH_SOLVE, r));
        CHPL_CUBLAS(cublasDtrsv_64(hb0, CUBLAS_FILL_MODE_UPPER, CUBLAS_OP_N, CUBLAS_DIAG_NON_UNIT, N, A, ld, at(0, N), 1));
        CHPL_TRY(clk.end(s0, r));
        return CHPL_OK;
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

int hpl_single_run(const chpl_hpl_config* cfg, chpl_hpl_result* res, double* x_out)
{
    if (!cfg || !res) { set_error("cfg/res NULL"); return CHPL_ERR_INVALID; }
    std::memset(res, 0, sizeof(*res));
    if (cfg->N <= 0 || cfg->NB <= 0 || cfg->NB > 2048) { set_error("bad N/NB (NB must be in [1, 2048])"); return CHPL_ERR_INVALID; }
    if (cfg->P != 1 || cfg->Q != 1) { set_error("chpl_hpl_run drives one GPU; use the grid driver for P x Q > 1"); return CHPL_ERR_INVALID; }
    if (cfg->emulate && !oz2::moduli(cfg->moduli)) { set_error("moduli must be in [2, 16]"); return CHPL_ERR_INVALID; }
    Solver s;
    int rc = s.init(*cfg);
    if (rc != CHPL_OK) { s.destroy(); return rc; }
    auto finish = [&](int code) { s.destroy(); return code; };

    cudaEvent_t g0, g1, t0, t1;
    cudaEventCreate(&g0); cudaEventCreate(&g1); cudaEventCreate(&t0); cudaEventCreate(&t1);
    cudaEventRecord(g0, s.s0);
    rc = matgen(s.s0, s.A, (size_t)s.ld, (size_t)s.N, (size_t)s.ncols, 0, 0, s.ncols, cfg->seed);
    if (rc != CHPL_OK) return finish(rc);
    cudaEventRecord(g1, s.s0);
    cudaEventRecord(t0, s.s0);
    cudaStreamWaitEvent(s.sP, t0, 0);
    rc = s.factor_and_solve();
    if (rc != CHPL_OK) { cudaDeviceSynchronize(); return finish(rc); }
    cudaEventRecord(t1, s.s0);
    cudaError_t e = cudaEventSynchronize(t1);
    if (e != cudaSuccess) return finish(cuda_fail(e, "solve", __FILE__, __LINE__));
    float ms_gen = 0.f, ms = 0.f;
    cudaEventElapsedTime(&ms_gen, g0, g1);
    cudaEventElapsedTime(&ms, t0, t1);
    int hinfo = 0;
    cudaMemcpy(&hinfo, s.info + 1, sizeof(int), cudaMemcpyDeviceToHost);
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
    double* dx = s.at(0, s.N);
    rc = residual(s.s0, s.N, cfg->seed, dx, &res->resid);
    if (rc != CHPL_OK) return finish(rc);
    res->passed = (hinfo == 0) && std::isfinite(res->resid) && res->resid < cfg->threshold;
    if (x_out) {
        e = cudaMemcpy(x_out, dx, (size_t)s.N * sizeof(double), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return finish(cuda_fail(e, "x readback", __FILE__, __LINE__));
    }
    cudaEventDestroy(g0); cudaEventDestroy(g1); cudaEventDestroy(t0); cudaEventDestroy(t1);
    if (hinfo != 0) { set_error("exact zero pivot at column %d", hinfo); return finish(CHPL_ERR_SINGULAR); }
    return finish(CHPL_OK);
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
    cfg->lookahead = 1;
    cfg->seed = 42;
    cfg->threshold = 16.0;
    cfg->verbose = 0;
}

extern "C" int chpl_hpl_run(const chpl_hpl_config* cfg, chpl_hpl_result* res, double* x_out)
{
    return chpl::hpl_single_run(cfg, res, x_out);
}
