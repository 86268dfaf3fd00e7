// FP64 panel factorization (getrf with partial pivoting) of an m x n panel.
#include <cusolverDn.h>

#include <vector>

#include "common.cuh"
#include "hpl.h"

namespace chpl {

struct PanelHandle {
    int dev = -1;
    cusolverDnHandle_t hs = nullptr;
    cusolverDnParams_t hp = nullptr;
};

static thread_local PanelHandle g_ph;

static int panel_handle(cudaStream_t st, PanelHandle** out)
{
    int dev = 0;
    CHPL_CUDA(cudaGetDevice(&dev));
    if (g_ph.dev != dev) {
        if (g_ph.hs) { cusolverDnDestroyParams(g_ph.hp); cusolverDnDestroy(g_ph.hs); }
        g_ph = PanelHandle();
        if (cusolverDnCreate(&g_ph.hs) != CUSOLVER_STATUS_SUCCESS || cusolverDnCreateParams(&g_ph.hp) != CUSOLVER_STATUS_SUCCESS) {
            set_error("cusolverDnCreate failed");
            return CHPL_ERR_CUDA;
        }
        g_ph.dev = dev;
    }
    if (cusolverDnSetStream(g_ph.hs, st) != CUSOLVER_STATUS_SUCCESS) { set_error("cusolverDnSetStream failed"); return CHPL_ERR_CUDA; }
    *out = &g_ph;
    return CHPL_OK;
}

__global__ void ipiv_rel0_kernel(int64_t* ipiv, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) ipiv[i] -= 1;
}

}  // namespace chpl

using namespace chpl;

extern "C" size_t chpl_panel_getrf_work_bytes(int64_t m, int64_t n)
{
    PanelHandle* h = nullptr;
    if (panel_handle(nullptr, &h) != CHPL_OK) return 0;
    size_t d = 0, hh = 0;
    if (cusolverDnXgetrf_bufferSize(h->hs, h->hp, m, n, CUDA_R_64F, nullptr, m, CUDA_R_64F, &d, &hh) != CUSOLVER_STATUS_SUCCESS)
        return 0;
    return round_up(d + 256, 256);
}

extern "C" int chpl_panel_getrf_f64(void* stream, int64_t m, int64_t n, double* A, size_t lda, int64_t* ipiv, int* info,
                                    void* work)
{
    if (m < n || n <= 0 || (int64_t)lda < m) { set_error("panel_getrf: need m >= n > 0, lda >= m"); return CHPL_ERR_INVALID; }
    PanelHandle* h = nullptr;
    CHPL_TRY(panel_handle((cudaStream_t)stream, &h));
    size_t d = 0, hh = 0;
    if (cusolverDnXgetrf_bufferSize(h->hs, h->hp, m, n, CUDA_R_64F, A, (int64_t)lda, CUDA_R_64F, &d, &hh) != CUSOLVER_STATUS_SUCCESS) {
        set_error("getrf buffer query failed");
        return CHPL_ERR_CUDA;
    }
    std::vector<char> hw(hh ? hh : 8);
    if (cusolverDnXgetrf(h->hs, h->hp, m, n, CUDA_R_64F, A, (int64_t)lda, ipiv, CUDA_R_64F, work, d, hw.data(), hh, info) !=
        CUSOLVER_STATUS_SUCCESS) {
        set_error("getrf failed");
        return CHPL_ERR_CUDA;
    }
    ipiv_rel0_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(ipiv, (int)n);
    CHPL_CUDA(cudaGetLastError());
    if (hh) CHPL_CUDA(cudaStreamSynchronize((cudaStream_t)stream));  // host workspace must outlive the call
    return CHPL_OK;
}
