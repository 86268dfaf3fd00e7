// Library-wide C ABI pieces: error strings, version, device status.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"
#include "oz2.h"

namespace chpl {

static thread_local char g_err[512] = "no error";

void set_error(const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char* what, const char* file, int line)
{
    set_error("CUDA error %d (%s) in %s at %s:%d", (int)e, cudaGetErrorString(e), what, file, line);
    return CHPL_ERR_CUDA;
}

int hpl_read_clear_status(int* st);

}  // namespace chpl

extern "C" const char* chpl_last_error_string(void) { return chpl::g_err; }

extern "C" const char* chpl_version(void) { return "chpl_b200 0.1 (sm_100a)"; }

extern "C" int chpl_device_status(int* status)
{
    CHPL_CUDA(cudaDeviceSynchronize());
    int a = 0, b = 0;
    CHPL_TRY(chpl::oz2::read_clear_status(&a));
    CHPL_TRY(chpl::hpl_read_clear_status(&b));
    if (status) *status = a ? a : b;
    return CHPL_OK;
}

extern "C" int chpl_host_alloc(size_t bytes, void** ptr)
{
    if (!ptr || bytes == 0) { chpl::set_error("host_alloc: bad arguments"); return CHPL_ERR_INVALID; }
    *ptr = nullptr;
    CHPL_CUDA(cudaHostAlloc(ptr, bytes, cudaHostAllocPortable));
    return CHPL_OK;
}

extern "C" int chpl_host_free(void* ptr)
{
    if (ptr) CHPL_CUDA(cudaFreeHost(ptr));
    return CHPL_OK;
}
