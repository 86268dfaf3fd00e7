// chpl_p2 -- P x Q grid HPL driver over libchpl's C ABI, one process per GPU.
//
//   chpl_p2 [HPL.dat]
//
// Same input and report as the reference executable (src/chpl_p2.cu:518-1953):
// HPL.dat lines 6 (N), 8 (NB) and 13 (threshold), with N=16384, NB=1024,
// 16.0 when the file is missing or shorter than 13 lines (570-584);
// CHPL2D_G8 (1: the Ozaki-II emulated update; 0: the FP64 update, serial
// block steps), CHPL2D_G8_MODULI (11),
// CHPL2D_G8_FAST, CHPL2D_G8_NT (column chunk of the update) (685-691).
// The grid is P x Q with rank = P*qc + pr (528): HPL.dat's P and Q (lines 11
// and 12) when they multiply to the rank count with P <= 2, otherwise P = 2
// for an even rank count (the reference's fixed P = 2); one rank runs 1 x 1.
// CHPL_DRY_RUN=1 prints the configuration and exits before any GPU or
// network work.
//
// There is no MPI: rank, rank count and local rank come from the launcher's
// environment (RANK / WORLD_SIZE / LOCAL_RANK as torchrun sets them, or
// OMPI_COMM_WORLD_* / PMI_RANK, PMI_SIZE), and rank 0 hands the NCCL unique
// id to the others over TCP at MASTER_ADDR (127.0.0.1) and port
// CHPL_BOOTSTRAP_PORT (MASTER_PORT + 17, 29517 without MASTER_PORT), which
// replaces the MPI_Bcast of src/chpl_p2.cu:552-568.  Every bootstrap wait is
// bounded (CHPL_BOOTSTRAP_TIMEOUT seconds, 120).
// Exit status 0 when the solve ran (PASSED or FAILED is printed, as in the
// reference), 1 on an error.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cinttypes>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <string>
#include <thread>
#include <vector>

#include "chpl.h"

namespace {

int env_int(const char* const* names, int dflt)
{
    for (int i = 0; names[i]; ++i) {
        const char* v = std::getenv(names[i]);
        if (v && *v) return std::atoi(v);
    }
    return dflt;
}

double now_s() { return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count(); }

bool send_all(int fd, const unsigned char* p, size_t n)
{
    while (n) {
        const ssize_t w = ::send(fd, p, n, MSG_NOSIGNAL);
        if (w <= 0) return false;
        p += w;
        n -= (size_t)w;
    }
    return true;
}

bool recv_all(int fd, unsigned char* p, size_t n, double deadline)
{
    while (n) {
        pollfd q{fd, POLLIN, 0};
        const int ms = (int)std::max(0.0, (deadline - now_s()) * 1e3);
        if (::poll(&q, 1, ms) <= 0) return false;
        const ssize_t r = ::recv(fd, p, n, 0);
        if (r <= 0) return false;
        p += r;
        n -= (size_t)r;
    }
    return true;
}

// rank 0: serve the id to world - 1 peers
bool serve_id(int port, int peers, const unsigned char* id, size_t len, double timeout)
{
    const int s = ::socket(AF_INET, SOCK_STREAM, 0);
    if (s < 0) return false;
    int one = 1;
    ::setsockopt(s, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_addr.s_addr = htonl(INADDR_ANY);
    a.sin_port = htons((uint16_t)port);
    if (::bind(s, (sockaddr*)&a, sizeof(a)) != 0 || ::listen(s, 64) != 0) {
        std::perror("[chpl_p2] bootstrap bind/listen");
        ::close(s);
        return false;
    }
    const double deadline = now_s() + timeout;
    int served = 0;
    while (served < peers) {
        pollfd q{s, POLLIN, 0};
        const int ms = (int)std::max(0.0, (deadline - now_s()) * 1e3);
        if (::poll(&q, 1, ms) <= 0) break;
        const int c = ::accept(s, nullptr, nullptr);
        if (c < 0) continue;
        if (send_all(c, id, len)) ++served;
        ::close(c);
    }
    ::close(s);
    return served == peers;
}

// other ranks: fetch the id from rank 0 (retrying until it listens)
bool fetch_id(const char* host, int port, unsigned char* id, size_t len, double timeout)
{
    const double deadline = now_s() + timeout;
    while (now_s() < deadline) {
        const int s = ::socket(AF_INET, SOCK_STREAM, 0);
        if (s < 0) return false;
        sockaddr_in a{};
        a.sin_family = AF_INET;
        a.sin_port = htons((uint16_t)port);
        if (::inet_pton(AF_INET, host, &a.sin_addr) != 1) { ::close(s); return false; }
        if (::connect(s, (sockaddr*)&a, sizeof(a)) == 0) {
            const bool ok = recv_all(s, id, len, deadline);
            ::close(s);
            return ok;
        }
        ::close(s);
        std::this_thread::sleep_for(std::chrono::milliseconds(100));
    }
    return false;
}

struct Dat {
    int64_t N = 16384, NB = 1024;
    double thresh = 16.0;
    int P = 0, Q = 0;  // lines 11 / 12, 0 when absent
};

Dat read_dat(const char* path)
{
    Dat d;
    if (!path) return d;
    FILE* f = std::fopen(path, "r");
    if (!f) return d;
    std::vector<std::string> L;
    char ln[4096];
    while (std::fgets(ln, sizeof(ln), f)) L.push_back(ln);
    std::fclose(f);
    if (L.size() > 12) {
        d.N = std::atoll(L[5].c_str());
        d.NB = std::atoll(L[7].c_str());
        d.thresh = std::atof(L[12].c_str());
        d.P = std::atoi(L[10].c_str());
        d.Q = std::atoi(L[11].c_str());
    }
    return d;
}

}  // namespace

int main(int argc, char** argv)
{
    static const char* kRank[] = {"RANK", "OMPI_COMM_WORLD_RANK", "PMI_RANK", nullptr};
    static const char* kSize[] = {"WORLD_SIZE", "OMPI_COMM_WORLD_SIZE", "PMI_SIZE", nullptr};
    static const char* kLocal[] = {"LOCAL_RANK", "OMPI_COMM_WORLD_LOCAL_RANK", nullptr};
    const int rank = env_int(kRank, 0), size = env_int(kSize, 1), local = env_int(kLocal, rank);
    if (size < 1 || rank < 0 || rank >= size || (size > 1 && size % 2)) {
        if (rank == 0) std::fprintf(stderr, "chpl_p2 runs on 1 rank or an even number of ranks (got %d)\n", size);
        return 1;
    }
    const Dat dat = read_dat(argc > 1 ? argv[1] : nullptr);
    const bool dat_grid = dat.P >= 1 && dat.P <= 2 && dat.Q >= 1 && dat.P * dat.Q == size;
    const int P = dat_grid ? dat.P : (size > 1 ? 2 : 1), Q = size / P;
    chpl_hpl_config cfg;
    chpl_hpl_default_config(&cfg);
    cfg.N = dat.N;
    cfg.NB = dat.NB;
    cfg.threshold = dat.thresh;
    cfg.P = P;
    cfg.Q = Q;
    static const char* kG8[] = {"CHPL2D_G8", nullptr};
    static const char* kMod[] = {"CHPL2D_G8_MODULI", nullptr};
    static const char* kFast[] = {"CHPL2D_G8_FAST", nullptr};
    static const char* kNT[] = {"CHPL2D_G8_NT", nullptr};
    cfg.emulate = env_int(kG8, 1);
    cfg.moduli = env_int(kMod, 11);
    cfg.fast = env_int(kFast, 1);
    cfg.chunk = env_int(kNT, 0);
    cfg.verbose = 1;  // rank 0's memory plan line
    static const char* kDry[] = {"CHPL_DRY_RUN", nullptr};
    if (env_int(kDry, 0)) {
        if (rank == 0)
            std::printf("[chpl_p2] grid %dx%d N=%" PRId64 " NB=%" PRId64 " threshold=%g moduli=%d ranks=%d\n", P, Q,
                        cfg.N, cfg.NB, cfg.threshold, cfg.moduli, size);
        return 0;
    }

    static const char* kTimeout[] = {"CHPL_BOOTSTRAP_TIMEOUT", nullptr};
    static const char* kMPort[] = {"MASTER_PORT", nullptr};
    static const char* kBPort[] = {"CHPL_BOOTSTRAP_PORT", nullptr};
    const double timeout = env_int(kTimeout, 120);
    const int port = env_int(kBPort, env_int(kMPort, 29500) + 17);
    const char* host = std::getenv("MASTER_ADDR") ? std::getenv("MASTER_ADDR") : "127.0.0.1";

    // the NCCL id first (host only): a rank that never shows up ends every
    // other rank's bootstrap with an error after `timeout` seconds
    unsigned char id[128] = {0};
    int rc = CHPL_OK;
    if (size > 1) {
        if (rank == 0) {
            rc = chpl_grid_unique_id(id, sizeof(id));
            if (rc == CHPL_OK && !serve_id(port, size - 1, id, sizeof(id), timeout)) {
                std::fprintf(stderr, "[chpl_p2] bootstrap: not every rank fetched the NCCL id within %.0f s\n", timeout);
                return 1;
            }
        } else if (!fetch_id(host, port, id, sizeof(id), timeout)) {
            std::fprintf(stderr, "[chpl_p2] rank %d: no NCCL id from %s:%d within %.0f s\n", rank, host, port, timeout);
            return 1;
        }
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev < 1) {
        std::fprintf(stderr, "[chpl_p2] rank %d: no CUDA device\n", rank);
        return 1;
    }
    cudaSetDevice(local % ndev);

    if (rank == 0 && cfg.emulate)   // the backend banner of src/chpl_p2.cu:764-767
        std::printf("[chpl_p2] G8 backend on: moduli=%d fast=%d nt=%lld (grid %dx%d)\n", cfg.moduli, cfg.fast,
                    (long long)cfg.chunk, P, Q);
    chpl_hpl_result res;
    const time_t ts0 = std::time(nullptr);
    if (size == 1) {
        rc = chpl_hpl_run(&cfg, &res, nullptr);
    } else {
        void* g = nullptr;
        if (rc == CHPL_OK) rc = chpl_grid_create(P, Q, rank, id, sizeof(id), 600.0, &g);
        if (rc == CHPL_OK) rc = chpl_grid_run(g, &cfg, &res, nullptr);
        if (g) chpl_grid_destroy(g);
    }
    if (rc != CHPL_OK) {
        std::fprintf(stderr, "[chpl_p2] rank %d: %s\n", rank, chpl_last_error_string());
        return 1;
    }
    const time_t ts1 = std::time(nullptr);
    if (rank == 0) {
        char b1[64], b2[64];
        tm tmv;
        localtime_r(&ts0, &tmv);
        std::strftime(b1, sizeof(b1), "%a %b %e %H:%M:%S %Y", &tmv);
        localtime_r(&ts1, &tmv);
        std::strftime(b2, sizeof(b2), "%a %b %e %H:%M:%S %Y", &tmv);
        const double dN = (double)cfg.N;
        const double gflops = ((2.0 / 3.0) * dN * dN * dN + 2.0 * dN * dN) / res.time_s / 1e9;
        std::printf("================================================================================\n");
        std::printf("T/V                N    NB     P     Q         Time          Gflops (   per GPU)\n");
        std::printf("--------------------------------------------------------------------------------\n");
        std::printf("%-4s%16" PRId64 " %5" PRId64 " %5d %5d %12.2f %15.3e (%10.3e)\n", "WC2", cfg.N, cfg.NB, P, Q,
                    res.time_s, gflops, gflops / (P * Q));
        std::printf("\nHPL_pdgesv() start time %s\nHPL_pdgesv() end time   %s\n\n", b1, b2);
        std::printf("--------------------------------------------------------------------------------\n");
        std::printf("||Ax-b||_oo/(eps*(||A||_oo*||x||_oo+||b||_oo)*N)= %16.12f ...... %s\n", res.resid,
                    res.resid < cfg.threshold ? "PASSED" : "FAILED");
        std::fflush(stdout);
    }
    return 0;
}
