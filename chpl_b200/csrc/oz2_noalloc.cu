// Allocation-free variant of the emulated GEMM (chpl_oz2_gemm_noalloc).
//
// Some callers cannot allocate device memory at the point where they need the
// update: a host framework that reserves the whole device memory pool up front
// (so cudaMalloc fails or fragments its pool), or a latency-sensitive caller
// that cannot afford the device-wide synchronization cudaMalloc / cudaFree may
// imply.  They still own their inputs and outputs; this entry point needs
// nothing else from them.  Its scratch -- the int8 residue planes and shifts
// of op(A) and op(B), the split temporaries and the per-CTA CRT scratch of the
// GEMM kernel -- lives in one file-scope device array of kNoAllocBytes.  Every
// GPU that loads this module holds the array until the process exits.
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "oz2.h"

namespace chpl {
namespace oz2 {

constexpr size_t kNoAllocBytes = 64ull << 20;  // 64 MiB of scratch per device
constexpr int kNoAllocCtas = 64;                // GEMM grid cap: CRT scratch <= 64 * L * 32 KB

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch for the current device.  In host code
// the symbol is only a host-side handle, so the kernels must be given this
// address, never the symbol itself.  It is looked up (cudaGetSymbolAddress,
// with the device current) on the first call in each CUDA context and cached
// under the context's unique id: after cudaDeviceReset the device gets a new
// primary context with a new id, so a stale address is never reused.  The
// per-call check is two host-only driver queries (no stream work, no
// allocation).
using PfnCtxGetCurrent = int (*)(void**);
using PfnCtxGetId = int (*)(void*, unsigned long long*);

// *id: unique id of the calling thread's current CUDA context; *have = false
// when the thread has no current context yet (the runtime binds the device's
// primary context lazily, on the first call that needs it).
static int current_context_id(unsigned long long* id, bool* have)
{
    static PfnCtxGetCurrent get_current = nullptr;
    static PfnCtxGetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PfnCtxGetCurrent>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PfnCtxGetId>(p);
    });
    if (!get_current || !get_id) { set_error("cuCtxGetCurrent / cuCtxGetId unavailable"); return CHPL_ERR_CUDA; }
    void* ctx = nullptr;
    *have = false;
    if (get_current(&ctx) != 0) { set_error("cuCtxGetCurrent failed"); return CHPL_ERR_CUDA; }
    if (!ctx) return CHPL_OK;
    if (get_id(ctx, id) != 0) { set_error("cuCtxGetId failed"); return CHPL_ERR_CUDA; }
    *have = true;
    return CHPL_OK;
}

static int noalloc_scratch(uint8_t** out)
{
    static std::mutex mu;
    static void* addr[256] = {};
    static unsigned long long ctx_of[256] = {};
    int dev = 0;
    CHPL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 256) { set_error("device ordinal %d out of range", dev); return CHPL_ERR_INVALID; }
    unsigned long long ctx = 0;
    bool have = false;
    CHPL_TRY(current_context_id(&ctx, &have));
    std::lock_guard<std::mutex> lock(mu);
    if (!have || !addr[dev] || ctx_of[dev] != ctx) {
        void* p = nullptr;
        // also makes the device's primary context current when the thread had none
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)", __FILE__, __LINE__);
        if (!have) {
            CHPL_TRY(current_context_id(&ctx, &have));
            if (!have) { set_error("no CUDA context after cudaGetSymbolAddress"); return CHPL_ERR_CUDA; }
        }
        addr[dev] = p;
        ctx_of[dev] = ctx;
    }
    *out = static_cast<uint8_t*>(addr[dev]);
    return CHPL_OK;
}

}  // namespace oz2
}  // namespace chpl

using namespace chpl;
using namespace chpl::oz2;

// C = alpha * op(A) * op(B) + beta * C like chpl_oz2_gemm (fast-mode scaling),
// using only the module's fixed device scratch.  See include/chpl.h.
extern "C" int chpl_oz2_gemm_noalloc(void* stream, int opA, int opB, size_t m, size_t n, size_t k,
                                     const double* alpha, const double* A, size_t lda, const double* B, size_t ldb,
                                     const double* beta, double* C, size_t ldc, unsigned num_moduli)
{
    cudaStream_t st = (cudaStream_t)stream;
    if (!alpha || !beta) { set_error("alpha/beta must be host pointers"); return CHPL_ERR_INVALID; }
    if ((opA != CHPL_OP_N && opA != CHPL_OP_T) || (opB != CHPL_OP_N && opB != CHPL_OP_T)) {
        set_error("op must be CHPL_OP_N or CHPL_OP_T");
        return CHPL_ERR_INVALID;
    }
    // arguments are validated before any early return, so a bad call never reports success
    const Moduli* M = moduli((int)num_moduli);
    if (!M) { set_error("num_moduli must be in [2, %d] (got %u)", kMaxModuli, num_moduli); return CHPL_ERR_INVALID; }
    if (k > (size_t)kMaxK) { set_error("k = %zu exceeds %d (int32 accumulation bound)", k, kMaxK); return CHPL_ERR_UNSUPPORTED; }
    if (m > 0x7fffffffull || n > 0x7fffffffull) { set_error("m, n must fit in int32"); return CHPL_ERR_UNSUPPORTED; }
    if (m == 0 || n == 0) return CHPL_OK;
    if (ldc < m || lda < (opA == CHPL_OP_N ? m : k) || ldb < (opB == CHPL_OP_N ? k : n)) {
        set_error("leading dimension too small");
        return CHPL_ERR_INVALID;
    }
    if (k == 0 || *alpha == 0.0) return scale(st, C, ldc, m, n, *beta);
    const Layout y = layout(m, n, k, (int)num_moduli, false, false, kNoAllocCtas);
    if (y.total > kNoAllocBytes) {
        set_error("chpl_oz2_gemm_noalloc: m=%zu n=%zu k=%zu with %u moduli needs %zu bytes of scratch, the fixed "
                  "limit is %zu bytes (64 MiB); use chpl_oz2_gemm with a caller-provided workspace",
                  m, n, k, num_moduli, y.total, kNoAllocBytes);
        return CHPL_ERR_WORKSPACE;
    }
    uint8_t* w = nullptr;
    CHPL_TRY(noalloc_scratch(&w));
    int32_t* shA = reinterpret_cast<int32_t*>(w + y.a_off + y.a_shift);
    int8_t* resA = reinterpret_cast<int8_t*>(w + y.a_off + y.a_res);
    int32_t* shB = reinterpret_cast<int32_t*>(w + y.b_off + y.b_shift);
    int8_t* resB = reinterpret_cast<int8_t*>(w + y.b_off + y.b_res);
    int8_t* scratch = reinterpret_cast<int8_t*>(w + y.scratch_off);
    void* tmp = w + y.tmp_off;
    // The split kernels rewrite every residue (padding included) and clear the
    // split temporaries; the CRT scratch is fully written before it is read.
    CHPL_TRY(split(st, opA == CHPL_OP_T, A, lda, m, k, num_moduli, M->alpha, resA, y.mPad, y.kPad, shA, tmp));
    CHPL_TRY(split(st, opB == CHPL_OP_N, B, ldb, n, k, num_moduli, M->beta, resB, y.nPad, y.kPad, shB, tmp));
    return gemm_launch(st, 0, m, n, y.kPad, num_moduli, resA, y.mPad, resB, y.nPad, shA, shB, *alpha, *beta, C, ldc,
                       nullptr, 0, scratch, y.grid_max);
}
