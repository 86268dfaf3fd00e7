// chpl_single -- one-GPU HPL driver over libchpl's C ABI.
//
// Same command line, environment and report as the reference executable
// (src/chpl_single.cu:950-965):
//   chpl_single N                   one HPL solve of order N
//   chpl_single HPL.dat             the same, N / NB / threshold from HPL.dat
//                                   lines 6 / 8 / 13 (the translation the
//                                   reference's launcher does for one GPU,
//                                   scripts/mpirun_chpl:66-77)
//   chpl_single --selftest          small FP64 and emulated solves
//   chpl_single --gemmtest m k n [nt]  emulated update vs cuBLAS DGEMM
//                                   (Ozaki-I with HPLS_BACKEND=ozaki, else Ozaki-II)
// Environment (src/chpl_single.cu:842-869, same names and defaults):
//   HPLS_NB (2048) HPLS_AGG (6) HPLS_BACKEND (native | ozaki | gemmul8)
//   HPLS_SEED (42) HPLS_G8_MODULI (14) HPLS_G8_FAST (0) HPLS_G8_CHUNK (16384)
//   HPLS_OZ_NT (columns per Ozaki-I call; 4096 here, the reference tiles 1024)
// The matrix is the reference chpl_single's: cuRAND Philox4_32_10, one
// subsequence per element (src/chpl_single.cu:73-80).  HPLS_GEN=chpl (this
// build's switch) selects chpl_p2's SplitMix64 matrix instead.
// Exit status: 0 = passed, 1 = failed or bad arguments, 4 = the memory plan
// does not fit the device (src/chpl_single.cu:389-394).  CHPL_DRY_RUN=1
// prints the configuration and exits before any GPU work.
#include <cuda_runtime.h>
#include <cublas_v2.h>

#include <algorithm>
#include <cinttypes>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "chpl.h"

namespace {

const char* backend_name(int emulate) { return emulate == 2 ? "ozaki" : emulate == 1 ? "gemmul8" : "native"; }

const char* kPhase[8] = {"panel", "laswp", "trsm", "oz2_split", "oz2_gemm", "update_fp64", "back_solve", "comm"};

int64_t env_i64(const char* name, int64_t dflt)
{
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoll(v) : dflt;
}

int exit_code(int rc) { return rc == CHPL_ERR_WORKSPACE ? 4 : 1; }

// configuration of one solve from the HPLS_* environment; false on bad input
bool cfg_from_env(int64_t N, chpl_hpl_config* c)
{
    chpl_hpl_default_config(c);
    c->N = N;
    c->NB = env_i64("HPLS_NB", 2048);
    c->agg = (int)env_i64("HPLS_AGG", 6);
    c->moduli = (int)env_i64("HPLS_G8_MODULI", 14);
    c->fast = (int)env_i64("HPLS_G8_FAST", 0);
    c->chunk = env_i64("HPLS_G8_CHUNK", 16384);
    c->seed = (uint64_t)env_i64("HPLS_SEED", 42);
    c->verbose = 1;  // the MEM PLAN line, as src/chpl_single.cu:379-388 prints it
    c->emulate = 0;
    c->generator = CHPL_GEN_PHILOX;
    const char* gen = std::getenv("HPLS_GEN");
    if (gen && *gen) {
        if (std::strcmp(gen, "chpl") == 0) {
            c->generator = CHPL_GEN_CHPL;
        } else if (std::strcmp(gen, "philox") != 0) {
            std::fprintf(stderr, "[chpl_single] unknown HPLS_GEN '%s' (philox | chpl)\n", gen);
            return false;
        }
    }
    const char* b = std::getenv("HPLS_BACKEND");
    if (b && std::strcmp(b, "gemmul8") == 0) {
        c->emulate = 1;
    } else if (b && std::strcmp(b, "ozaki") == 0) {
        c->emulate = 2;
        c->chunk = env_i64("HPLS_OZ_NT", 4096);
    } else if (b && std::strcmp(b, "native") != 0) {
        std::fprintf(stderr, "[chpl_single] unknown HPLS_BACKEND '%s'\n", b);
        return false;
    }
    if (c->N <= 0 || c->NB <= 0 || c->agg <= 0 || c->NB > c->N) {
        std::fprintf(stderr, "[chpl_single] bad N/NB/AGG\n");
        return false;
    }
    return true;
}

void report(const chpl_hpl_config& c, const chpl_hpl_result& r)
{
    const double dN = (double)c.N;
    const double gflops = ((2.0 / 3.0) * dN * dN * dN + 2.0 * dN * dN) / r.time_s / 1e9;
    std::printf("==========================================================\n"
                "T/V                   N    NB   AGG      K           Time                 Gflops\n"
                "----------------------------------------------------------\n"
                "%-16s%8" PRId64 " %5" PRId64 " %5d %6" PRId64 " %14.2f     %18.4e\n"
                "----------------------------------------------------------\n"
                "||Ax-b||_oo/(eps*(||A||_oo*||x||_oo+||b||_oo)*N)= %13.7f ...... %s\n",
                c.emulate == 2 ? "HPLS_ozaki" : c.emulate ? "HPLS_gemmul8" : "HPLS_native", c.N, c.NB, c.agg, c.NB * (int64_t)c.agg, r.time_s, gflops,
                r.resid, r.passed ? "PASSED" : "FAILED");
    std::printf("----------------------------------------------------------\nPHASE              sec     %%wall\n");
    double sum = 0.0;
    for (int p = 0; p < 8; ++p) {
        std::printf("%-14s%9.3f   %6.2f%%\n", kPhase[p], r.phase_s[p], 100.0 * r.phase_s[p] / r.time_s);
        sum += r.phase_s[p];
    }
    std::printf("%-14s%9.3f   %6.2f%%   (stream-busy time; streams overlap)\n", "sum_phases", sum, 100.0 * sum / r.time_s);
    if (c.emulate == 2)
        std::printf("wide_gemm calls: ozaki=%" PRId64 " (slices=6 nt=%" PRId64 ") | digits+int8 GEMM+recon %.3f s, "
                    "%.0f int8 TOPS\n",
                    r.n_emulated, c.chunk, r.gemm_kernel_s,
                    r.gemm_kernel_s > 0 ? r.gemm_int8_ops / r.gemm_kernel_s / 1e12 : 0.0);
    else
        std::printf("wide_gemm calls: gemmul8=%" PRId64 " (moduli=%d fast=%d chunk=%" PRId64 ") | int8 GEMM %.3f s, "
                    "%.0f TOPS\n",
                    r.n_emulated, c.moduli, c.fast, c.chunk, r.gemm_kernel_s,
                    r.gemm_kernel_s > 0 ? r.gemm_int8_ops / r.gemm_kernel_s / 1e12 : 0.0);
    std::printf("==========================================================\n");
    std::fflush(stdout);
}

// N, NB, threshold from lines 6, 8 and 13 of an HPL.dat; false when the file
// cannot be read or is shorter than 13 lines
bool read_dat(const char* path, int64_t* N, int64_t* NB, double* thresh)
{
    FILE* f = std::fopen(path, "r");
    if (!f) return false;
    std::vector<std::string> L;
    char ln[4096];
    while (std::fgets(ln, sizeof(ln), f)) L.push_back(ln);
    std::fclose(f);
    if (L.size() < 13) return false;
    *N = std::atoll(L[5].c_str());
    *NB = std::atoll(L[7].c_str());
    *thresh = std::atof(L[12].c_str());
    return true;
}

bool is_integer(const char* s)
{
    if (!*s) return false;
    for (; *s; ++s)
        if (*s < '0' || *s > '9') return false;
    return true;
}

int run_case(const chpl_hpl_config& c)
{
    chpl_hpl_result r;
    std::printf("[chpl_single] %s N=%" PRId64 " NB=%" PRId64 " AGG=%d moduli=%d (%s)\n",
                backend_name(c.emulate), c.N, c.NB, c.agg, c.moduli, chpl_version());
    std::fflush(stdout);
    const int rc = chpl_hpl_run(&c, &r, nullptr);
    if (rc != CHPL_OK) {
        std::fprintf(stderr, "[chpl_single] %s\n", chpl_last_error_string());
        return exit_code(rc);
    }
    report(c, r);
    return r.passed ? 0 : 1;
}

// emulated C -= A B against cuBLAS DGEMM on generated data (src/chpl_single.cu:875-929):
// Ozaki-I (HPLS_BACKEND=ozaki, n in tiles of nt columns as the reference's oz_nt) or Ozaki-II
int gemmtest(int64_t m, int64_t k, int64_t n, int64_t nt)
{
    const char* be = std::getenv("HPLS_BACKEND");
    const bool ozaki = be && std::strcmp(be, "ozaki") == 0;
    if (nt <= 0) nt = n;
    std::printf("GEMMTEST: m=%" PRId64 " k=%" PRId64 " n=%" PRId64 " (%s)\n", m, k, n, ozaki ? "ozaki" : "gemmul8");
    const unsigned L = (unsigned)env_i64("HPLS_G8_MODULI", 14);
    // A, B, C are disjoint blocks of one generated system (ld = Ns)
    const int64_t Ns = k + std::max(m, n) + 8;
    double *S = nullptr, *Cref = nullptr;
    void* work = nullptr;
    size_t wbytes = 0;
    int rc = ozaki ? chpl_oz1_worksize((size_t)m, (size_t)std::min(nt, n), (size_t)k, &wbytes)
                   : chpl_oz2_worksize((size_t)m, (size_t)n, (size_t)k, L, 0, 0, &wbytes, nullptr, nullptr);
    if (rc != CHPL_OK) { std::fprintf(stderr, "[chpl_single] %s\n", chpl_last_error_string()); return 1; }
    if (cudaMalloc(&S, (size_t)Ns * (Ns + 1) * 8) != cudaSuccess || cudaMalloc(&Cref, (size_t)m * n * 8) != cudaSuccess ||
        cudaMalloc(&work, wbytes) != cudaSuccess) {
        std::fprintf(stderr, "[chpl_single] device allocation failed\n");
        return 4;
    }
    rc = chpl_matgen(nullptr, S, (size_t)Ns, (size_t)Ns, (size_t)Ns + 1, 0, 0, Ns + 1, 7);
    const double* A = S + k;               // rows k.., columns 0..k-1
    const double* B = S + (size_t)k * Ns;  // rows 0..k-1, columns k..
    double* C = S + k + (size_t)k * Ns;    // rows k.., columns k..
    cudaMemcpy2D(Cref, (size_t)m * 8, C, (size_t)Ns * 8, (size_t)m * 8, (size_t)n, cudaMemcpyDeviceToDevice);
    cublasHandle_t h;
    cublasCreate(&h);
    const double one = 1.0, mone = -1.0;
    cublasDgemm(h, CUBLAS_OP_N, CUBLAS_OP_N, (int)m, (int)n, (int)k, &mone, A, (int)Ns, B, (int)Ns, &one, Cref, (int)m);
    for (int64_t j = 0; ozaki && rc == CHPL_OK && j < n; j += nt)
        rc = chpl_oz1_gemm(nullptr, (size_t)m, (size_t)std::min(nt, n - j), (size_t)k, -1.0, A, (size_t)Ns,
                           B + (size_t)j * Ns, (size_t)Ns, 1.0, C + (size_t)j * Ns, (size_t)Ns, work);
    if (!ozaki && rc == CHPL_OK)
        rc = chpl_oz2_gemm(nullptr, CHPL_OP_N, CHPL_OP_N, (size_t)m, (size_t)n, (size_t)k, &mone, A, (size_t)Ns, B,
                           (size_t)Ns, &one, C, (size_t)Ns, L, 1, work, nullptr, nullptr, 0, 0, 0, 0, nullptr);
    if (rc != CHPL_OK) { std::fprintf(stderr, "[chpl_single] %s\n", chpl_last_error_string()); return 1; }
    std::vector<double> hr((size_t)m * n), ho((size_t)m * n);
    cudaMemcpy(hr.data(), Cref, (size_t)m * n * 8, cudaMemcpyDeviceToHost);
    cudaMemcpy2D(ho.data(), (size_t)m * 8, C, (size_t)Ns * 8, (size_t)m * 8, (size_t)n, cudaMemcpyDeviceToHost);
    double maxabs = 0.0, maxrel = 0.0, sumref = 0.0;
    for (size_t e = 0; e < hr.size(); ++e) {
        const double d = std::fabs(hr[e] - ho[e]);
        maxabs = std::max(maxabs, d);
        maxrel = std::max(maxrel, d / (std::fabs(hr[e]) + 1e-12));
        sumref += std::fabs(hr[e]);
    }
    std::printf("GEMMTEST: max_abs_err=%.6e max_rel_err=%.6e mean|ref|=%.3e (%s)\n", maxabs, maxrel,
                sumref / (double)hr.size(), ozaki ? "slices=6" : ("moduli=" + std::to_string(L)).c_str());
    const bool ok = maxrel < 1e-2;
    std::printf("GEMMTEST_%s\n", ok ? "PASS" : "FAIL");
    cublasDestroy(h);
    cudaFree(S);
    cudaFree(Cref);
    cudaFree(work);
    return ok ? 0 : 1;
}

// the reference's selftest sizes (src/chpl_single.cu:931-948): N=8192, NB=512, AGG=4
int selftest()
{
    chpl_hpl_config c1;
    chpl_hpl_default_config(&c1);
    c1.N = 8192;
    c1.NB = 512;
    c1.agg = 4;
    c1.emulate = 0;
    c1.seed = 42;
    c1.generator = CHPL_GEN_PHILOX;   // the reference selftest's matrix (src/chpl_single.cu:750)
    chpl_hpl_config c2 = c1;
    c2.emulate = 1;
    c2.moduli = 14;
    c2.chunk = 3072;  // several column chunks per update: the A residues are reused
    chpl_hpl_config c3 = c1;
    c3.emulate = 2;
    c3.chunk = 512;   // the reference selftest's oz_nt
    std::printf("SELFTEST run 1/3: native\n");
    const int r1 = run_case(c1);
    std::printf("SELFTEST run 2/3: ozaki (6 slices, nt=512)\n");
    const int r3 = run_case(c3);
    std::printf("SELFTEST run 3/3: gemmul8 (moduli=14, chunked)\n");
    const int r2 = run_case(c2);
    const bool ok = r1 == 0 && r2 == 0 && r3 == 0;
    std::printf("SELFTEST_%s (native=%s ozaki=%s gemmul8=%s)\n", ok ? "PASS" : "FAIL", r1 == 0 ? "PASS" : "FAIL",
                r3 == 0 ? "PASS" : "FAIL", r2 == 0 ? "PASS" : "FAIL");
    return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv)
{
    if (argc == 2 && std::strcmp(argv[1], "--selftest") == 0) return selftest();
    if ((argc == 5 || argc == 6) && std::strcmp(argv[1], "--gemmtest") == 0)
        return gemmtest(std::atoll(argv[2]), std::atoll(argv[3]), std::atoll(argv[4]), argc == 6 ? std::atoll(argv[5]) : 0);
    if (argc != 2) {
        std::fprintf(stderr, "usage: chpl_single N | chpl_single --selftest | chpl_single --gemmtest m k n [nt]\n"
                             "env: HPLS_NB HPLS_AGG HPLS_BACKEND(native|ozaki|gemmul8) HPLS_SEED HPLS_G8_MODULI "
                             "HPLS_G8_FAST HPLS_G8_CHUNK HPLS_OZ_NT HPLS_GEN(philox|chpl)\n");
        return 1;
    }
    chpl_hpl_config c;
    if (is_integer(argv[1])) {
        if (!cfg_from_env(std::atoll(argv[1]), &c)) return 1;
    } else {
        int64_t N = 0, NB = 0;
        double thresh = 16.0;
        if (!read_dat(argv[1], &N, &NB, &thresh)) {
            std::fprintf(stderr, "[chpl_single] cannot read N/NB/threshold from '%s' (13-line HPL.dat)\n", argv[1]);
            return 1;
        }
        if (!cfg_from_env(N, &c)) return 1;
        c.NB = NB;
        c.threshold = thresh;
        if (c.NB <= 0 || c.NB > c.N) {
            std::fprintf(stderr, "[chpl_single] bad N/NB/AGG\n");
            return 1;
        }
    }
    if (const char* d = std::getenv("CHPL_DRY_RUN"); d && std::atoi(d)) {
        std::printf("[chpl_single] N=%" PRId64 " NB=%" PRId64 " AGG=%d backend=%s moduli=%d fast=%d chunk=%" PRId64
                    " threshold=%g\n",
                    c.N, c.NB, c.agg, backend_name(c.emulate), c.moduli, c.fast, c.chunk, c.threshold);
        return 0;
    }
    return run_case(c);
}
