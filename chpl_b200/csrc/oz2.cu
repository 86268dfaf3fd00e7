// Ozaki scheme II emulated DGEMM on B200: C = alpha*op(A)*op(B) + beta*C.
//
// Replaces gemmul8::gemm<double, Backend::INT8> (GEMMul8 v3.2.0), which the
// reference calls at src/chpl_single.cu:641-649 and src/chpl_p2.cu:1674-1683.
// The method follows Ozaki, Uchino, Imamura, "Ozaki Scheme II" (2025):
//
//   1. split (HBM bound): for every row i of op(A) a power-of-two scale
//      2^sa_i from a Cauchy-Schwarz bound (||a'_i||_2 < 2^alpha), integer image
//      a' = rint(a 2^sa), and its symmetric residue modulo each modulus m_l
//      (<= 256, pairwise coprime) as int8, K-major; the same for the columns
//      of op(B) with 2^sb_j, beta.  alpha + beta < log2(M/2), M = prod m_l,
//      so every exact dot product of integer images lies in (-M/2, M/2).
//   2. one exact int8 x int8 -> int32 GEMM per modulus on the 5th-generation
//      tensor cores (tcgen05.mma kind::i8, operands staged by TMA, int32
//      accumulators in TMEM);
//   3. fused epilogue: each accumulator tile is reduced modulo m_l as it
//      leaves TMEM (int8 residue, kept in a small per-CTA scratch that stays
//      in L2); after the last modulus the CRT is evaluated as a 64-bit
//      fixed-point fraction  S = sum_l r_l v_l mod 2^64,
//      v_l = round(2^64 y_l / m_l), y_l = (M/m_l)^-1 mod m_l, so that
//      S / 2^64 = C'/M (mod 1) with |error| < 2^-54; then
//      C = fma(alpha, scalbn((double)S * (M/2^64), -(sa_i+sb_j)), beta*C).
//
// Kernel structure (persistent, one CTA per SM, 320 threads):
//   warp 0      TMA producer (4-stage ring of 128x128 A + 256x128 B int8 tiles)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue: TMEM -> residues -> scratch; CRT -> C
// The TMEM accumulator (128 lanes x 256 int32 columns) is double buffered, so
// the tensor core computes modulus l+1 while the epilogue drains modulus l.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "oz2.h"

namespace chpl {
namespace oz2 {

__device__ int g_status;  // sticky device-side error of this module

// ----------------------------------------------------------------------------
// moduli and CRT constants
// ----------------------------------------------------------------------------
static long long gcdll(long long a, long long b)
{
    while (b) { long long t = a % b; a = b; b = t; }
    return a;
}

static long long inv_mod(long long a, long long m)
{
    long long t = 0, nt = 1, r = m, nr = ((a % m) + m) % m;
    while (nr) {
        long long q = r / nr, tmp;
        tmp = t - q * nt; t = nt; nt = tmp;
        tmp = r - q * nr; r = nr; nr = tmp;
    }
    return r == 1 ? (t < 0 ? t + m : t) : -1;
}

static bool build_moduli(int L, Moduli& M)
{
    if (L < 2 || L > kMaxModuli) return false;
    std::memset(&M, 0, sizeof(M));
    int n = 0;
    for (int c = 256; c > 1 && n < L; --c) {
        bool ok = true;
        for (int i = 0; i < n; ++i)
            if (gcdll(c, M.mod[i]) != 1) { ok = false; break; }
        if (ok) M.mod[n++] = c;
    }
    if (n != L) return false;
    M.L = L;
    unsigned __int128 prod = 1;
    double lg = 0.0;
    for (int l = 0; l < L; ++l) {
        prod *= (unsigned __int128)M.mod[l];
        lg += std::log2((double)M.mod[l]);
    }
    for (int l = 0; l < L; ++l) {
        const long long ml = M.mod[l];
        long long p = 1;
        for (int i = 0; i < L; ++i)
            if (i != l) p = (p * (M.mod[i] % ml)) % ml;
        const long long y = inv_mod(p, ml);
        if (y < 0) return false;
        const unsigned __int128 num = ((unsigned __int128)(unsigned long long)y << 64) + (unsigned __int128)(ml / 2);
        M.v[l] = (unsigned long long)(num / (unsigned __int128)ml);
        M.hi[l] = (int)((ml - 1) / 2);
        M.mod_d[l] = (double)ml;
        M.inv_d[l] = 1.0 / (double)ml;
        M.inv_f[l] = 1.0f / (float)ml;
    }
    M.Mf = (double)prod * 0x1p-64;
    const int T = (int)std::floor(lg - 1.02);
    M.alpha = std::min(52, (T + 1) / 2);
    M.beta = std::min(52, T / 2);
    return true;
}

const Moduli* moduli(int L)
{
    static Moduli table[kMaxModuli + 1];
    static bool ok[kMaxModuli + 1];
    static std::once_flag once;
    std::call_once(once, [] {
        for (int l = 2; l <= kMaxModuli; ++l) ok[l] = build_moduli(l, table[l]);
    });
    if (L < 2 || L > kMaxModuli || !ok[L]) return nullptr;
    return &table[L];
}

// ----------------------------------------------------------------------------
// split kernels
// ----------------------------------------------------------------------------
// Symmetric residue of an integer-valued double |a| <= 2^52 modulo m_l.
// q = rint(a / m) is exact to within one unit, r = a - q m is exact (fma), and
// one correction each way lands r in [hi - m + 1, hi].
__device__ __forceinline__ int residue_f64(double a, int l, const Moduli& M)
{
    const double m = M.mod_d[l];
    const double q = rint(a * M.inv_d[l]);
    double r = fma(-q, m, a);
    const double hi = (double)M.hi[l];
    r = (r > hi) ? r - m : r;
    r = (r < hi - m + 1.0) ? r + m : r;
    return (int)r;
}

// exponent e with ||x||_2 < 2^e from E = ilogb(max|x|) + 1 and the exact
// integer sum Q = sum ceil(|x_h| 2^(20-E))^2 (order independent).
__device__ __forceinline__ int norm_exponent(int E, unsigned long long Q)
{
    const int bl = 64 - __clzll((long long)Q);
    return E - 20 + (bl + 1) / 2;
}

__device__ __forceinline__ unsigned long long q_square(double x, int E)
{
    const unsigned long long q = (unsigned long long)ceil(scalbn(fabs(x), 20 - E));
    return q * q;
}

// One warp per vector whose K elements are contiguous (x + v*ld, stride 1):
// columns of op(B) = B, rows of op(A) = A^T.  Writes shift[v] and the
// residues res[(l*ldvec + v)*ldk + h] for h < ldk (zero padded), v < nvpad.
__global__ void __launch_bounds__(256) split_contig_kernel(const double* __restrict__ x, long long ld, int nvec,
                                                           int k, int nvpad, int ldvec, int ldk, int bits,
                                                           const __grid_constant__ Moduli M, int8_t* __restrict__ res,
                                                           int* __restrict__ shift)
{
    const int lane = threadIdx.x & 31;
    const int v = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (v >= nvpad) return;
    int s = 0;
    const double* xv = x + (long long)v * ld;
    if (v < nvec) {
        double mx = 0.0;
        for (int h = lane; h < k; h += 32) mx = fmax(mx, fabs(xv[h]));
        for (int o = 16; o; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (mx > 0.0) {
            const int E = ilogb(mx) + 1;
            unsigned long long Q = 0;
            for (int h = lane; h < k; h += 32) Q += q_square(xv[h], E);
            for (int o = 16; o; o >>= 1) Q += __shfl_xor_sync(0xffffffffu, Q, o);
            s = bits - norm_exponent(E, Q);
        }
    }
    if (lane == 0) shift[v] = s;
    for (int h0 = 0; h0 < ldk; h0 += 128) {
        const int h = h0 + 4 * lane;
        double a[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) a[t] = (v < nvec && h + t < k) ? rint(scalbn(xv[h + t], s)) : 0.0;
        for (int l = 0; l < M.L; ++l) {
            uint32_t w = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) w |= ((uint32_t)residue_f64(a[t], l, M) & 0xffu) << (8 * t);
            *reinterpret_cast<uint32_t*>(res + ((size_t)l * ldvec + v) * ldk + h) = w;
        }
    }
}

// Vectors whose K elements are strided (x[v + h*ld]): rows of op(A) = A,
// columns of op(B) = B^T.  Three passes with exact integer atomics.
constexpr int kStrideChunk = 64;

__global__ void __launch_bounds__(256) absmax_strided_kernel(const double* __restrict__ x, long long ld, int nvec,
                                                             int k, unsigned long long* __restrict__ maxbits)
{
    const int v = blockIdx.x * 256 + threadIdx.x;
    if (v >= nvec) return;
    const int h0 = blockIdx.y * kStrideChunk, h1 = min(k, h0 + kStrideChunk);
    double mx = 0.0;
    for (int h = h0; h < h1; ++h) mx = fmax(mx, fabs(x[v + (long long)h * ld]));
    if (mx > 0.0) atomicMax(&maxbits[v], (unsigned long long)__double_as_longlong(mx));
}

__global__ void __launch_bounds__(256) sumsq_strided_kernel(const double* __restrict__ x, long long ld, int nvec,
                                                            int k, const unsigned long long* __restrict__ maxbits,
                                                            unsigned long long* __restrict__ Q)
{
    const int v = blockIdx.x * 256 + threadIdx.x;
    if (v >= nvec) return;
    const double mx = __longlong_as_double((long long)maxbits[v]);
    if (mx == 0.0) return;
    const int E = ilogb(mx) + 1;
    const int h0 = blockIdx.y * kStrideChunk, h1 = min(k, h0 + kStrideChunk);
    unsigned long long q = 0;
    for (int h = h0; h < h1; ++h) q += q_square(x[v + (long long)h * ld], E);
    if (q) atomicAdd(&Q[v], q);
}

__global__ void shift_finalize_kernel(int nvec, int nvpad, int bits, const unsigned long long* __restrict__ maxbits,
                                      const unsigned long long* __restrict__ Q, int* __restrict__ shift)
{
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= nvpad) return;
    int s = 0;
    if (v < nvec) {
        const double mx = __longlong_as_double((long long)maxbits[v]);
        if (mx > 0.0) s = bits - norm_exponent(ilogb(mx) + 1, Q[v]);
    }
    shift[v] = s;
}

// 32 vectors x 128 K per CTA, transposed through shared memory so that both
// the FP64 reads (32 consecutive vectors of one K) and the int8 writes
// (K-contiguous residues) stay coalesced.
__global__ void __launch_bounds__(256) split_strided_kernel(const double* __restrict__ x, long long ld, int nvec,
                                                            int k, int ldvec, int ldk, const __grid_constant__ Moduli M,
                                                            const int* __restrict__ shift, int8_t* __restrict__ res)
{
    __shared__ double tile[32][129];
    const int v0 = blockIdx.x * 32, h0 = blockIdx.y * 128;
    const int t = threadIdx.x, vl = t & 31, g = t >> 5;
    const int v = v0 + vl;
    const int s = (v < ldvec) ? shift[v] : 0;
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
        const int hl = g + 8 * i, h = h0 + hl;
        double a = 0.0;
        if (v < nvec && h < k) a = rint(scalbn(x[v + (long long)h * ld], s));
        tile[vl][hl] = a;
    }
    __syncthreads();
    const int hs = g * 16;
    const double* row = &tile[vl][hs];
    int8_t* dst = res + (size_t)v * ldk + h0 + hs;
    if (v >= ldvec) return;
    for (int l = 0; l < M.L; ++l) {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int e = 0; e < 16; ++e) w[e >> 2] |= ((uint32_t)residue_f64(row[e], l, M) & 0xffu) << (8 * (e & 3));
        *reinterpret_cast<uint4*>(dst + (size_t)l * ldvec * ldk) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// ----------------------------------------------------------------------------
// tcgen05 int8 GEMM with fused modular reduction + CRT epilogue
// ----------------------------------------------------------------------------
constexpr int BM = 128;                 // rows per CTA (TMEM lanes)
constexpr int BN = 256;                 // tile columns (TMEM columns per accumulator)
constexpr int BK = 128;                 // K bytes per stage (one 128 B swizzle row)
constexpr int A_BYTES = BM * BK;        // 16 KB
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 2 * BN;       // double-buffered accumulator
constexpr int SCRATCH_TILE = BM * BN;   // bytes per modulus per CTA

// Two forms of the kernel share one body:
//   single: one CTA computes a 128 x 256 tile; it stages A 128 x 128 and
//           B 256 x 128 per K block (48 KB, 4 stages);
//   pair:   a cluster of two CTAs computes a 256 x 256 tile with
//           tcgen05.mma.cta_group::2 issued by the even CTA; each CTA stages
//           its own 128 rows of A and 128 of the 256 B rows (32 KB, 6 stages),
//           so one int8 MAC needs 2/3 of the shared-memory fill of the single
//           form; each CTA's TMEM holds the accumulator of its 128 rows.
template <bool PAIR>
struct Form {
    static constexpr int TBM = PAIR ? 2 * BM : BM;      // tile rows
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;   // B rows staged by one CTA
    static constexpr int B_BYTES = B_ROWS * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = PAIR ? 6 : 4;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
};

struct GemmParams {
    int m, n;
    int mtiles, ntiles, kblocks;
    int kstep;          // > 0: plane l stops after (l + 1) * kstep bytes of K (the rest of its B rows is zero)
    int magic[kMaxModuli];            // ceil(2^32 / m_l): the epilogue's residue estimate
    unsigned long long crt_bias;      // -128 * sum_l v_l mod 2^64: removes the residues' +128 bias
    int rowsA, rowsB;   // padded rows per modulus plane in the residue buffers
    int planeA;         // row offset between A's planes: rowsA, or 0 when every plane reads the same rows
    int mode;           // 0: CRT into C; 1: raw int32 products into P
    int group_m;
    double* C;
    long long ldc;
    int32_t* P;
    long long ldp;
    const int* shiftA;
    const int* shiftB;
    double alpha, beta;
    int8_t* scratch;
    Moduli M;
};

__device__ __forceinline__ void tile_coords(const GemmParams& p, int tile, int& mt, int& nt)
{
    const int per_group = p.group_m * p.ntiles;
    const int g = tile / per_group;
    const int first = g * p.group_m;
    const int gsz = min(p.group_m, p.mtiles - first);
    const int local = tile - g * per_group;
    mt = first + local % gsz;
    nt = local / gsz;
}

// Symmetric residue of an int32 accumulator modulo m (129 <= m <= 256): q =
// floor(x * magic / 2^32) with magic = ceil(2^32 / m) is floor(x / m) to within
// one either way (|x| < 2^31 keeps the estimate's error below 1/2), so x - q m
// lies in [-m, 2m) and three conditional steps give [hi - m + 1, hi].  Integer
// multiply-adds only: no int <-> float conversions.
__device__ __forceinline__ int residue_i32(int x, int mod, int hi, int magic)
{
    if (mod == 256) return (int)(int8_t)(x & 0xff);
    int r = x - __mulhi(x, magic) * mod;
    r += (r < 0) ? mod : 0;
    r -= (r >= mod) ? mod : 0;
    return (r > hi) ? r - mod : r;
}

__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns)
{
    int never = 0;
    return mbar_wait(bar, parity, &never, limit_ns);
}

// K blocks of plane l: all of them, or with p.kstep > 0 the ones that hold the
// plane's non-zero (l + 1) * kstep bytes (producer and MMA issuer agree on it)
__device__ __forceinline__ int plane_kblocks(const GemmParams& p, int l)
{
    return p.kstep > 0 ? min(p.kblocks, ((l + 1) * p.kstep + BK - 1) / BK) : p.kblocks;
}

__device__ __forceinline__ void spin_ns(uint64_t ns)
{
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < ns) {
    }
}

template <bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    oz2_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ GemmParams p)
{
    using F = Form<PAIR>;
    constexpr int STAGES = F::STAGES;
    constexpr int STAGE_BYTES = F::STAGE_BYTES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = warp_id(), lane = lane_id();
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;   // 0: the CTA that issues the MMAs
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int nunits = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], EPI_WARPS * (PAIR ? 2 : 1)); }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
    if (warp == 1) {
        if (PAIR) { tmem_alloc_pair(tmem_slot, TMEM_COLS); tmem_relinquish_pair(); }
        else { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
    }
    tc_fence_before();
    if (PAIR) cluster_sync(); else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = p.mtiles * p.ntiles;
    const int L = p.M.L;
    // barriers of the MMA-issuing CTA, as shared::cluster addresses
    const uint32_t lead_full = PAIR ? map_to_rank(smem_u32(full), 0) : 0u;
    const uint32_t lead_acc_empty = PAIR ? map_to_rank(smem_u32(acc_empty), 0) : 0u;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs of a pair) ----------------
        if (elect_one()) {
            int stage = 0;
            uint32_t ph = 0;
            int issued[STAGES];
            for (int s = 0; s < STAGES; ++s) issued[s] = -1;
            bool ok = true;
            for (int tile = unit; tile < total && ok; tile += nunits) {
                int mt, nt;
                tile_coords(p, tile, mt, nt);
                const int rowA = mt * F::TBM + (int)rank * BM;
                const int rowB = nt * BN + (int)rank * F::B_ROWS;
                for (int l = 0; l < L && ok; ++l)
                    for (int kb = 0; kb < plane_kblocks(p, l); ++kb) {
                        if (!mbar_wait(&empty[stage], ph ^ 1u, abort_flag)) { ok = false; break; }
                        uint8_t* sa = smem + stage * STAGE_BYTES;
                        if (PAIR) {
                            // the even CTA's full barrier counts both CTAs' bytes
                            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
                            const uint32_t fb = lead_full + stage * 8;
                            tma_load_2d_pair(sa, &tmA, fb, kb * BK, l * p.planeA + rowA);
                            tma_load_2d_pair(sa + A_BYTES, &tmB, fb, kb * BK, l * p.rowsB + rowB);
                        } else {
                            mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                            tma_load_2d(sa, &tmA, &full[stage], kb * BK, l * p.planeA + rowA);
                            tma_load_2d(sa + A_BYTES, &tmB, &full[stage], kb * BK, l * p.rowsB + rowB);
                        }
                        issued[stage] = (int)ph;
                        if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                    }
            }
            if (!ok) {  // let the copies already in flight land before the CTA exits
                if (PAIR) spin_ns(1000000ull);
                else
                    for (int s = 0; s < STAGES; ++s)
                        if (issued[s] >= 0) bounded_wait(&full[s], (uint32_t)issued[s], 20000000ull);
            } else if (PAIR) {
                // producer tail: every stage's last release (a commit from the
                // even CTA's MMA thread) has landed in this CTA's barriers
                for (int s = 0; s < STAGES; ++s) {
                    if (issued[stage] >= 0 && !mbar_wait(&empty[stage], ph ^ 1u, abort_flag)) break;
                    if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (the even CTA of a pair) ----------------
        if (rank == 0 && elect_one()) {
            const uint32_t idesc = idesc_i8(F::TBM, BN);
            const uint32_t peer_empty = PAIR ? map_to_rank(smem_u32(empty), 1) : 0u;
            const uint32_t peer_acc_full = PAIR ? map_to_rank(smem_u32(acc_full), 1) : 0u;
            int stage = 0;
            uint32_t ph = 0, acc = 0;
            bool ok = true;
            for (int tile = unit; tile < total && ok; tile += nunits) {
                for (int l = 0; l < L && ok; ++l) {
                    const uint32_t buf = acc & 1u, aph = (acc >> 1) & 1u;
                    if (!mbar_wait(&acc_empty[buf], aph ^ 1u, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d = tmem_base + buf * BN;
                    for (int kb = 0; kb < plane_kblocks(p, l); ++kb) {
                        if (!mbar_wait(&full[stage], ph, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(smem + stage * STAGE_BYTES), b0 = a0 + A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / 32; ++kk) {
                            const uint64_t ad = umma_desc_sw128(a0 + kk * 32), bd = umma_desc_sw128(b0 + kk * 32);
                            if (PAIR) mma_i8_pair(d, ad, bd, idesc, (kb | kk) ? 1u : 0u);
                            else mma_i8(d, ad, bd, idesc, (kb | kk) ? 1u : 0u);
                        }
                        if (PAIR) {
                            mma_commit_pair(smem_u32(&empty[stage]));
                            mma_commit_pair(peer_empty + stage * 8);
                        } else {
                            mma_commit(&empty[stage]);
                        }
                        if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                    }
                    if (!ok) break;
                    if (PAIR) {
                        mma_commit_pair(smem_u32(&acc_full[buf]));
                        mma_commit_pair(peer_acc_full + buf * 8);
                    } else {
                        mma_commit(&acc_full[buf]);
                    }
                    ++acc;
                }
            }
            if (!ok) {  // wait for the MMAs already issued before TMEM is released
                if (PAIR) mma_commit_pair(smem_u32(drain));
                else mma_commit(drain);
                bounded_wait(drain, 0, 20000000ull);
            } else if (PAIR) {
                // accumulator tail: both CTAs' epilogues have released both
                // buffers (their arrivals on this CTA's barriers have landed)
                for (int t = 0; t < 2; ++t) {
                    const uint32_t buf = acc & 1u, aph = (acc >> 1) & 1u;
                    if (!mbar_wait(&acc_empty[buf], aph ^ 1u, abort_flag)) break;
                    ++acc;
                }
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (both CTAs of a pair) ----------------
        const int ew = warp - 2;
        const int quarter = warp & 3;        // TMEM lane quarter this warp may access
        const int half = ew >> 2;            // column half of the 256-wide tile
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        int8_t* scr = p.scratch + (size_t)blockIdx.x * L * SCRATCH_TILE;
        uint32_t acc = 0;
        bool ok = true;
        for (int tile = unit; tile < total && ok; tile += nunits) {
            int mt, nt;
            tile_coords(p, tile, mt, nt);
            const int gi = mt * F::TBM + (int)rank * BM + row;
            for (int l = 0; l < L; ++l) {
                const uint32_t buf = acc & 1u, aph = (acc >> 1) & 1u;
                if (!mbar_wait(&acc_full[buf], aph, abort_flag)) { ok = false; break; }
                tc_fence_after();
                if (p.mode == 0 && l == (L >= 2 ? L - 2 : 0) && gi < p.m) {
                    // warm L2 with this thread's C row segment (128 columns) for the final pass
                    const int gj0 = nt * BN + half * 128;
                    const double* cp = p.C + gi + (size_t)gj0 * p.ldc;
                    for (int j = 0; j < 128 && gj0 + j < p.n; ++j)
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(cp + (size_t)j * p.ldc));
                }
                const int mod = p.M.mod[l], hi = p.M.hi[l];
                const int magic = p.magic[l];
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tmem_base + lane_addr + buf * BN + half * 128 + c * 32, v);
                    tmem_wait_ld();
                    if (c == 3) {  // every column of this warp is in registers: release the accumulator early
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            if (PAIR) mbar_arrive_cluster(lead_acc_empty + buf * 8);
                            else mbar_arrive(&acc_empty[buf]);
                        }
                    }
                    if (p.mode == 1) {
                        const int gj0 = nt * BN + half * 128 + c * 32;
                        if (gi < p.m) {
                            int32_t* dst = p.P + (size_t)l * p.ldp * p.n + gi;
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (gj0 + j < p.n) dst[(size_t)(gj0 + j) * p.ldp] = (int32_t)v[j];
                        }
                    } else {
                        // residues biased by +128 into bytes 0..255 (the CRT removes the bias)
                        uint32_t w[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            uint32_t x = 0;
#pragma unroll
                            for (int t = 0; t < 4; ++t)
                                x |= (uint32_t)(residue_i32((int)v[4 * q + t], mod, hi, magic) + 128) << (8 * t);
                            w[q] = x;
                        }
                        uint4* dst = reinterpret_cast<uint4*>(scr + (((size_t)l * 8 + half * 4 + c) * BM + row) * 32);
                        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    }
                }
                ++acc;
            }
            if (!ok || p.mode != 0) continue;
            // ---- CRT + unscale + C update for this warp's 32 rows x 128 columns ----
            // 16 columns per block.  Every load of a block (16 C values, L
            // residue words) is issued before any arithmetic, so the HBM and
            // L2 latencies of a block overlap instead of adding up.
            if (gi < p.m) {
                const int sa = p.shiftA[gi];
                const bool readc = p.beta != 0.0;
                const uint8_t* srow = reinterpret_cast<const uint8_t*>(scr) + ((size_t)(half * 4) * BM + row) * 32;
#pragma unroll 1
                for (int blk = 0; blk < 8; ++blk) {
                    const int c = blk >> 1, hh = blk & 1;
                    const int gj0 = nt * BN + half * 128 + c * 32 + hh * 16;
                    double* __restrict__ cbase = p.C + gi + (size_t)gj0 * p.ldc;
                    double cv[16];
#pragma unroll
                    for (int t = 0; t < 16; ++t)
                        cv[t] = (readc && gj0 + t < p.n) ? __ldcs(cbase + (size_t)t * p.ldc) : 0.0;
                    uint4 w[kMaxModuli];
                    const uint8_t* sp = srow + (size_t)c * BM * 32 + hh * 16;
#pragma unroll
                    for (int l = 0; l < kMaxModuli; ++l)
                        if (l < L) w[l] = __ldcg(reinterpret_cast<const uint4*>(sp + (size_t)l * 8 * BM * 32));
                    // S = sum_l r_l v_l mod 2^64 = sum_l (r_l + 128) v_l - 128 sum_l v_l: the
                    // biased bytes multiply unsigned (one wide multiply-add per term)
                    unsigned long long S[16];
#pragma unroll
                    for (int t = 0; t < 16; ++t) S[t] = p.crt_bias;
#pragma unroll
                    for (int l = 0; l < kMaxModuli; ++l) {
                        if (l < L) {
                            const unsigned long long vl = p.M.v[l];
                            const uint32_t ws[4] = {w[l].x, w[l].y, w[l].z, w[l].w};
#pragma unroll
                            for (int t = 0; t < 16; ++t) {
                                const uint32_t u = (ws[t >> 2] >> (8 * (t & 3))) & 0xffu;
                                S[t] += (unsigned long long)u * vl;
                            }
                        }
                    }
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        const int gj = gj0 + t;
                        if (gj < p.n) {
                            // prod * 2^-e: one exact power-of-two multiply (rounded once, as
                            // scalbn) while 2^-e is a normal double
                            const int e = sa + __ldg(&p.shiftB[gj]);
                            double prod = (double)(long long)S[t] * p.M.Mf;
                            prod = (e >= -1022 && e <= 1022) ? prod * __longlong_as_double((long long)(1023 - e) << 52)
                                                             : scalbn(prod, -e);
                            __stcs(cbase + (size_t)t * p.ldc, readc ? fma(p.alpha, prod, p.beta * cv[t]) : p.alpha * prod);
                        }
                    }
                }
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    if (PAIR) cluster_sync(); else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
        else tmem_dealloc(tmem_base, TMEM_COLS);
    }
    if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_status, CHPL_ERR_TIMEOUT);
}

__global__ void scale_kernel(double* C, long long ldc, int m, int n, double beta)
{
    const long long total = (long long)m * n;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const long long i = e % m, j = e / m;
        double* c = C + i + j * ldc;
        *c = (beta == 0.0) ? 0.0 : beta * *c;
    }
}

// ----------------------------------------------------------------------------
// host side
// ----------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

static int make_tmap_i8(CUtensorMap* tm, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_rows)
{
    auto fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled unavailable"); return CHPL_ERR_CUDA; }
    cuuint64_t dims[2] = {inner_bytes, rows};
    cuuint64_t strides[1] = {inner_bytes};
    cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return CHPL_ERR_CUDA; }
    return CHPL_OK;
}

int num_sms()
{
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

Layout layout(size_t m, size_t n, size_t k, int L, bool extA, bool extB, int grid_cap)
{
    Layout y;
    y.mPad = round_up(m, BM);
    y.nPad = round_up(n, BN);
    y.kPad = round_up(k, BK);
    y.a_shift = 0;
    y.a_res = round_up(y.mPad * 4, 256);
    y.a_bytes = round_up(y.a_res + (size_t)L * y.mPad * y.kPad, 256);
    y.b_shift = 0;
    y.b_res = round_up(y.nPad * 4, 256);
    y.b_bytes = round_up(y.b_res + (size_t)L * y.nPad * y.kPad, 256);
    size_t off = 0;
    y.a_off = off; if (!extA) off += y.a_bytes;
    y.b_off = off; if (!extB) off += y.b_bytes;
    y.grid_max = num_sms();
    if (grid_cap > 0 && grid_cap < y.grid_max) y.grid_max = grid_cap;
    y.scratch_off = off;
    off += round_up((size_t)y.grid_max * L * SCRATCH_TILE, 256);
    y.tmp_off = off;
    off += round_up(split_tmp_bytes(std::max(y.mPad, y.nPad)), 256);
    y.total = off;
    return y;
}

size_t split_tmp_bytes(size_t nvec) { return round_up(nvec, 256) * 16; }

static int check_common(unsigned L, size_t k)
{
    if (!moduli((int)L)) { set_error("num_moduli must be in [2, %d] (got %u)", kMaxModuli, L); return CHPL_ERR_INVALID; }
    if (k > (size_t)kMaxK) { set_error("k = %zu exceeds %d (int32 accumulation bound)", k, kMaxK); return CHPL_ERR_UNSUPPORTED; }
    return CHPL_OK;
}

// residues + shifts of nvec vectors of length k; contiguous (K stride 1, vector
// stride ld) or strided (vector stride 1, K stride ld).
int split(cudaStream_t st, bool contiguous, const double* x, size_t ld, size_t nvec, size_t k, unsigned L, int bits,
          int8_t* res, size_t ldvec, size_t ldk, int32_t* shift, void* tmp)
{
    const Moduli* M = moduli((int)L);
    if (!M) { set_error("bad num_moduli %u", L); return CHPL_ERR_INVALID; }
    if (ldk % BK || ldk < k || ldvec < nvec) { set_error("bad residue layout"); return CHPL_ERR_INVALID; }
    if (nvec > 0x7fffffff || k > (size_t)kMaxK) { set_error("split: size out of range"); return CHPL_ERR_UNSUPPORTED; }
    if (ldvec == 0) return CHPL_OK;
    if (contiguous) {
        const int nvpad = (int)ldvec;
        split_contig_kernel<<<(nvpad + 7) / 8, 256, 0, st>>>(x, (long long)ld, (int)nvec, (int)k, nvpad, (int)ldvec,
                                                            (int)ldk, bits, *M, res, shift);
        CHPL_CUDA(cudaGetLastError());
        return CHPL_OK;
    }
    const size_t nv4 = round_up(nvec, 256);
    unsigned long long* maxbits = reinterpret_cast<unsigned long long*>(tmp);
    unsigned long long* Q = maxbits + nv4;
    CHPL_CUDA(cudaMemsetAsync(tmp, 0, nv4 * 16, st));
    if (nvec > 0 && k > 0) {
        dim3 g((unsigned)((nvec + 255) / 256), (unsigned)((k + kStrideChunk - 1) / kStrideChunk));
        absmax_strided_kernel<<<g, 256, 0, st>>>(x, (long long)ld, (int)nvec, (int)k, maxbits);
        sumsq_strided_kernel<<<g, 256, 0, st>>>(x, (long long)ld, (int)nvec, (int)k, maxbits, Q);
    }
    shift_finalize_kernel<<<(unsigned)((ldvec + 255) / 256), 256, 0, st>>>((int)nvec, (int)ldvec, bits, maxbits, Q, shift);
    dim3 g2((unsigned)((ldvec + 31) / 32), (unsigned)(ldk / BK));
    split_strided_kernel<<<g2, 256, 0, st>>>(x, (long long)ld, (int)nvec, (int)k, (int)ldvec, (int)ldk, *M, shift, res);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

// The single form is the default: sustained under the 1 kW power cap it keeps
// the SM clock near 1.5 GHz where the pair form drops to ~1.1 GHz (m = n =
// 32768, k = 4096, 11 moduli: 163-166 vs 137-140 FP64-equivalent TFLOPS), although
// per clock the pair form is ~15 % faster (tensor pipe 62 % vs 54 % active).
// CHPL_OZ2_FORM=pair (read at every launch) selects the pair form for
// updates of more than 128 rows.
static bool use_pair(size_t m)
{
    const char* e = std::getenv("CHPL_OZ2_FORM");
    return e && std::strcmp(e, "pair") == 0 && m > (size_t)BM;
}

// clusters of two CTAs of the pair kernel that can be resident at once on this device
static int max_pair_clusters()
{
    static int dev_cached = -1, n_cached = 0;
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return num_sms() / 2;
    std::lock_guard<std::mutex> lk(mu);
    if (dev == dev_cached) return n_cached;
    int n = 0;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)num_sms());
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = Form<true>::SMEM;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaFuncSetAttribute(oz2_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Form<true>::SMEM) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, oz2_gemm_kernel<true>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = num_sms() / 2;
    }
    dev_cached = dev;
    n_cached = n;
    return n;
}

int gemm_launch(cudaStream_t st, int mode, size_t m, size_t n, size_t kPad, unsigned L, const int8_t* ra, size_t rowsA,
                const int8_t* rb, size_t rowsB, const int32_t* shiftA, const int32_t* shiftB, double alpha,
                double beta, double* C, size_t ldc, int32_t* P, size_t ldp, int8_t* scratch, int grid_max,
                long long planeA, long long kstep)
{
    const Moduli* M = moduli((int)L);
    if (!M) { set_error("bad num_moduli"); return CHPL_ERR_INVALID; }
    if (rowsA % BM || rowsB % BN || kPad % BK || rowsA < m || rowsB < n) {
        set_error("gemm_launch: bad padded layout");
        return CHPL_ERR_INVALID;
    }
    if ((size_t)L * std::max(rowsA, rowsB) > 0x7fffffffull) { set_error("residue planes too tall"); return CHPL_ERR_UNSUPPORTED; }
    const bool pair = use_pair(m);
    CUtensorMap tmA, tmB;
    if (planeA < 0) planeA = (long long)rowsA;
    if (planeA != 0 && planeA != (long long)rowsA) { set_error("gemm_launch: A plane stride must be 0 or rowsA"); return CHPL_ERR_INVALID; }
    CHPL_TRY(make_tmap_i8(&tmA, ra, kPad, (uint64_t)(L - 1) * (uint64_t)planeA + rowsA, BM));
    CHPL_TRY(make_tmap_i8(&tmB, rb, kPad, (uint64_t)L * rowsB, pair ? Form<true>::B_ROWS : BN));
    GemmParams p;
    std::memset(&p, 0, sizeof(p));
    const int tbm = pair ? Form<true>::TBM : BM;
    p.m = (int)m;
    p.n = (int)n;
    p.mtiles = (int)((m + tbm - 1) / tbm);
    p.ntiles = (int)((n + BN - 1) / BN);
    p.kblocks = (int)(kPad / BK);
    if (kstep < 0 || kstep > (long long)kPad) { set_error("gemm_launch: bad plane K step"); return CHPL_ERR_INVALID; }
    p.kstep = (int)kstep;
    p.rowsA = (int)rowsA;
    p.planeA = (int)planeA;
    p.rowsB = (int)rowsB;
    p.mode = mode;
    p.group_m = pair ? 8 : 16;
    if (const char* g = std::getenv("CHPL_OZ2_GROUP_M")) p.group_m = std::max(1, std::atoi(g));
    p.C = C;
    p.ldc = (long long)ldc;
    p.P = P;
    p.ldp = (long long)ldp;
    p.shiftA = shiftA;
    p.shiftB = shiftB;
    p.alpha = alpha;
    p.beta = beta;
    p.scratch = scratch;
    p.M = *M;
    p.crt_bias = 0;
    for (unsigned l = 0; l < L; ++l) {
        p.magic[l] = (int)((0x100000000ull + (unsigned long long)M->mod[l] - 1) / (unsigned long long)M->mod[l]);
        p.crt_bias -= 128ull * M->v[l];
    }
    const int tiles = p.mtiles * p.ntiles;
    if (!pair) {
        const int grid = std::min(tiles, grid_max);
        CHPL_CUDA(cudaFuncSetAttribute(oz2_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Form<false>::SMEM));
        oz2_gemm_kernel<false><<<grid, THREADS, Form<false>::SMEM, st>>>(tmA, tmB, p);
        CHPL_CUDA(cudaGetLastError());
        return CHPL_OK;
    }
    // pairs: as many clusters of two as can be resident at once (the grid is
    // persistent), at most grid_max CTAs (the CRT scratch holds grid_max tiles)
    CHPL_CUDA(cudaFuncSetAttribute(oz2_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Form<true>::SMEM));
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = Form<true>::SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int clusters = std::min(tiles, std::min(max_pair_clusters(), grid_max / 2));
    if (clusters < 1) { set_error("gemm_launch: no CTA pair fits"); return CHPL_ERR_UNSUPPORTED; }
    cfg.gridDim = dim3((unsigned)(2 * clusters));
    CHPL_CUDA(cudaLaunchKernelEx(&cfg, oz2_gemm_kernel<true>, tmA, tmB, p));
    return CHPL_OK;
}

int scale(cudaStream_t st, double* C, size_t ldc, size_t m, size_t n, double beta)
{
    if (beta == 1.0 || m == 0 || n == 0) return CHPL_OK;
    scale_kernel<<<1024, 256, 0, st>>>(C, (long long)ldc, (int)m, (int)n, beta);
    CHPL_CUDA(cudaGetLastError());
    return CHPL_OK;
}

int read_clear_status(int* st)
{
    int v = 0, z = 0;
    CHPL_CUDA(cudaMemcpyFromSymbol(&v, g_status, sizeof(int)));
    CHPL_CUDA(cudaMemcpyToSymbol(g_status, &z, sizeof(int)));
    *st = v;
    return CHPL_OK;
}

}  // namespace oz2
}  // namespace chpl

// ============================================================================
// C ABI
// ============================================================================
using namespace chpl;
using namespace chpl::oz2;

extern "C" int chpl_oz2_shift_bits(unsigned num_moduli, size_t k, int* alpha_bits, int* beta_bits)
{
    CHPL_TRY(check_common(num_moduli, k));
    const Moduli* M = moduli((int)num_moduli);
    if (alpha_bits) *alpha_bits = M->alpha;
    if (beta_bits) *beta_bits = M->beta;
    return CHPL_OK;
}

extern "C" int chpl_oz2_worksize(size_t m, size_t n, size_t k, unsigned num_moduli, int enable_skip_scalA,
                                 int enable_skip_scalB, size_t* work_bytes, size_t* wsA, size_t* wsB)
{
    (void)enable_skip_scalA;
    (void)enable_skip_scalB;
    CHPL_TRY(check_common(num_moduli, k));
    const Layout y = layout(m, n, k, (int)num_moduli, false, false);
    if (work_bytes) *work_bytes = y.total;
    if (wsA) *wsA = y.a_bytes;
    if (wsB) *wsB = y.b_bytes;
    return CHPL_OK;
}

extern "C" size_t chpl_oz2_split_tmp_bytes(size_t num_vectors) { return split_tmp_bytes(num_vectors); }

extern "C" int chpl_oz2_split_rows(void* stream, int opA, size_t m, size_t k, const double* A, size_t lda,
                                   unsigned num_moduli, int8_t* res, size_t ld_vec, size_t ld_k, int32_t* shift,
                                   void* tmp)
{
    CHPL_TRY(check_common(num_moduli, k));
    const Moduli* M = moduli((int)num_moduli);
    return split((cudaStream_t)stream, opA == CHPL_OP_T, A, lda, m, k, num_moduli, M->alpha, res, ld_vec, ld_k, shift,
                 tmp);
}

extern "C" int chpl_oz2_split_cols(void* stream, int opB, size_t k, size_t n, const double* B, size_t ldb,
                                   unsigned num_moduli, int8_t* res, size_t ld_vec, size_t ld_k, int32_t* shift,
                                   void* tmp)
{
    CHPL_TRY(check_common(num_moduli, k));
    const Moduli* M = moduli((int)num_moduli);
    return split((cudaStream_t)stream, opB == CHPL_OP_N, B, ldb, n, k, num_moduli, M->beta, res, ld_vec, ld_k, shift,
                 tmp);
}

extern "C" int chpl_oz2_products(void* stream, size_t m, size_t n, size_t k, unsigned num_moduli, const int8_t* ra,
                                 size_t lda_vec, const int8_t* rb, size_t ldb_vec, size_t ld_k, int32_t* P, size_t ldp)
{
    CHPL_TRY(check_common(num_moduli, k));
    if (m == 0 || n == 0) return CHPL_OK;
    if (ldp < m) { set_error("ldp < m"); return CHPL_ERR_INVALID; }
    return gemm_launch((cudaStream_t)stream, 1, m, n, ld_k, num_moduli, ra, lda_vec, rb, ldb_vec, nullptr, nullptr, 0.0,
                       0.0, nullptr, 0, P, ldp, nullptr, num_sms());
}

extern "C" int chpl_oz2_gemm(void* stream, int opA, int opB, size_t m, size_t n, size_t k, const double* alpha,
                             const double* A, size_t lda, const double* B, size_t ldb, const double* beta, double* C,
                             size_t ldc, unsigned num_moduli, int fastmode, void* work, void* workA, void* workB,
                             int enable_skip_scalA, int enable_skip_scalB, int skip_scalA, int skip_scalB,
                             double* phase_seconds)
{
    (void)fastmode;
    cudaStream_t st = (cudaStream_t)stream;
    if (phase_seconds)
        for (int i = 0; i < 4; ++i) phase_seconds[i] = 0.0;
    if (!alpha || !beta) { set_error("alpha/beta must be host pointers"); return CHPL_ERR_INVALID; }
    if ((opA != CHPL_OP_N && opA != CHPL_OP_T) || (opB != CHPL_OP_N && opB != CHPL_OP_T)) {
        set_error("op must be CHPL_OP_N or CHPL_OP_T");
        return CHPL_ERR_INVALID;
    }
    // arguments are validated before any early return, so a bad call never reports success
    CHPL_TRY(check_common(num_moduli, k));
    if (m > 0x7fffffffull || n > 0x7fffffffull) { set_error("m, n must fit in int32"); return CHPL_ERR_UNSUPPORTED; }
    if (m == 0 || n == 0) return CHPL_OK;
    if (ldc < m || lda < (opA == CHPL_OP_N ? m : k) || ldb < (opB == CHPL_OP_N ? k : n)) {
        set_error("leading dimension too small");
        return CHPL_ERR_INVALID;
    }
    if (k == 0 || *alpha == 0.0) return scale(st, C, ldc, m, n, *beta);
    if (!work) { set_error("work is NULL"); return CHPL_ERR_WORKSPACE; }
    const Moduli* M = moduli((int)num_moduli);
    const Layout y = layout(m, n, k, (int)num_moduli, workA != nullptr, workB != nullptr);
    uint8_t* w = static_cast<uint8_t*>(work);
    uint8_t* pa = workA ? static_cast<uint8_t*>(workA) : w + y.a_off;
    uint8_t* pb = workB ? static_cast<uint8_t*>(workB) : w + y.b_off;
    int32_t* shA = reinterpret_cast<int32_t*>(pa + y.a_shift);
    int8_t* resA = reinterpret_cast<int8_t*>(pa + y.a_res);
    int32_t* shB = reinterpret_cast<int32_t*>(pb + y.b_shift);
    int8_t* resB = reinterpret_cast<int8_t*>(pb + y.b_res);
    int8_t* scratch = reinterpret_cast<int8_t*>(w + y.scratch_off);
    void* tmp = w + y.tmp_off;

    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    if (phase_seconds) {
        for (auto& e : ev) CHPL_CUDA(cudaEventCreate(&e));
        CHPL_CUDA(cudaEventRecord(ev[0], st));
    }
    if (!(enable_skip_scalA && skip_scalA))
        CHPL_TRY(split(st, opA == CHPL_OP_T, A, lda, m, k, num_moduli, M->alpha, resA, y.mPad, y.kPad, shA, tmp));
    if (!(enable_skip_scalB && skip_scalB))
        CHPL_TRY(split(st, opB == CHPL_OP_N, B, ldb, n, k, num_moduli, M->beta, resB, y.nPad, y.kPad, shB, tmp));
    if (phase_seconds) CHPL_CUDA(cudaEventRecord(ev[1], st));
    CHPL_TRY(gemm_launch(st, 0, m, n, y.kPad, num_moduli, resA, y.mPad, resB, y.nPad, shA, shB, *alpha, *beta, C, ldc,
                         nullptr, 0, scratch, y.grid_max));
    if (phase_seconds) {
        CHPL_CUDA(cudaEventRecord(ev[2], st));
        CHPL_CUDA(cudaEventSynchronize(ev[2]));
        float t0 = 0.f, t1 = 0.f;
        CHPL_CUDA(cudaEventElapsedTime(&t0, ev[0], ev[1]));
        CHPL_CUDA(cudaEventElapsedTime(&t1, ev[1], ev[2]));
        phase_seconds[0] = t0 * 1e-3;
        phase_seconds[1] = t1 * 1e-3;
        for (auto& e : ev) cudaEventDestroy(e);
    }
    return CHPL_OK;
}
