// Failure-detection self-test: one bounded device-side wait on something no
// one ever signals, through the same helpers every kernel of the library
// uses for its waits (mbarrier phase waits with an abort flag; acquire polls
// of a flag in global memory, as the panel's cross-CTA exchange).  The wait
// gives up after `limit_ns` of %globaltimer, the kernel records the error
// code and returns, and the context stays usable: this is how a missing
// partner (a TMA copy, an MMA commit, a CTA of the panel) surfaces as
// CHPL_ERR_TIMEOUT instead of a hung GPU.  Nothing faults, traps or spins
// without a bound.
#include "common.cuh"

namespace chpl {

__global__ void diag_wait_kernel(int kind, unsigned long long limit_ns, const unsigned int* never, int* out)
{
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x != 0) return;
    int status = CHPL_OK;
    if (kind == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
        // phase 0 completes only when one arrival comes: none does
        if (!mbar_wait(&bar, 0, &abort_flag, limit_ns)) status = CHPL_ERR_TIMEOUT;
    } else {
        const uint64_t t0 = globaltimer();
        uint32_t it = 0;
        unsigned int v = 0;
        while (true) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(never) : "memory");
            if (v != 0) break;
            if ((++it & 255u) == 0 && globaltimer() - t0 > limit_ns) {
                status = CHPL_ERR_TIMEOUT;
                break;
            }
        }
    }
    *out = status;
}

}  // namespace chpl

using namespace chpl;

extern "C" int chpl_diag_bounded_wait(void* stream, int kind, uint64_t limit_ns)
{
    if (kind != 0 && kind != 1) { set_error("kind must be 0 (mbarrier) or 1 (global flag)"); return CHPL_ERR_INVALID; }
    if (limit_ns == 0 || limit_ns > 2000000000ull) { set_error("limit_ns must be in (0, 2 s]"); return CHPL_ERR_INVALID; }
    cudaStream_t st = (cudaStream_t)stream;
    unsigned int* flag = nullptr;
    int* out = nullptr;
    CHPL_CUDA(cudaMallocAsync((void**)&flag, sizeof(unsigned int), st));
    CHPL_CUDA(cudaMallocAsync((void**)&out, sizeof(int), st));
    CHPL_CUDA(cudaMemsetAsync(flag, 0, sizeof(unsigned int), st));
    CHPL_CUDA(cudaMemsetAsync(out, 0xff, sizeof(int), st));
    diag_wait_kernel<<<1, 32, 0, st>>>(kind, (unsigned long long)limit_ns, flag, out);
    CHPL_CUDA(cudaGetLastError());
    int h = 0;
    CHPL_CUDA(cudaMemcpyAsync(&h, out, sizeof(int), cudaMemcpyDeviceToHost, st));
    CHPL_CUDA(cudaStreamSynchronize(st));
    cudaFreeAsync(flag, st);
    cudaFreeAsync(out, st);
    if (h == CHPL_ERR_TIMEOUT) set_error("bounded wait ran out after %llu ns (nothing signalled it)", (unsigned long long)limit_ns);
    return h;
}
