/*
 * chpl.h -- C ABI of libchpl (chpl_b200), a B200-native (sm_100a) HPL engine.
 *
 * Conventions: every entry point returns an int status (CHPL_OK = 0, negative
 * on error; chpl_last_error_string() describes the last failure on the calling
 * thread).  Nothing aborts the process.  Matrices are FP64 column-major.
 * Device pointers are plain pointers; `stream` is a cudaStream_t passed as
 * void* (NULL = legacy default stream).  Calls are asynchronous on `stream`
 * unless stated otherwise.  Buffers are owned by the caller.
 *
 * Each declaration names the interface of Koyingtw/CHPL (file:line inside the
 * reference project) that it replaces.
 */
#ifndef CHPL_H
#define CHPL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CHPL_OK 0
#define CHPL_ERR_INVALID (-1)     /* bad argument */
#define CHPL_ERR_CUDA (-2)        /* CUDA runtime / driver error */
#define CHPL_ERR_TIMEOUT (-3)     /* a bounded device-side wait ran out */
#define CHPL_ERR_WORKSPACE (-4)   /* workspace or device memory too small */
#define CHPL_ERR_UNSUPPORTED (-5) /* valid request this build does not serve */
#define CHPL_ERR_SINGULAR (-6)    /* exact zero pivot */
#define CHPL_ERR_NCCL (-7)        /* NCCL error */
#define CHPL_ERR_NO_DEVICE (-8)   /* no sm_100 device */

#define CHPL_OP_N 0
#define CHPL_OP_T 1

/* matrix generators (chpl_hpl_config.generator) */
#define CHPL_GEN_CHPL 0   /* SplitMix64 hash of chpl_p2 / chpl_p4 (chpl_elem, src/chpl_p2.cu:66-73) */
#define CHPL_GEN_PHILOX 1 /* cuRAND Philox4_32_10 of chpl_single (hs_rand, src/chpl_single.cu:73-80) */

/* Human-readable description of the last error on this host thread. */
const char *chpl_last_error_string(void);
/* Library version string, e.g. "chpl_b200 0.1 (sm_100a)". */
const char *chpl_version(void);
/* Sticky device-side error (timeouts inside kernels) of the current device:
 * writes it to *status and clears it.  Synchronizes the device. */
int chpl_device_status(int *status);
/* Page-locked (pinned) host memory, portable across devices: host buffers of
 * chpl_hpl_run_host / chpl_matgen_host in it copy at the link's full
 * bandwidth.  No reference counterpart (the reference keeps every matrix on
 * the device). */
int chpl_host_alloc(size_t bytes, void **ptr);
int chpl_host_free(void *ptr);

/* ------------------------------------------------------------------------ */
/* Ozaki scheme II emulated DGEMM (trailing-matrix update)                   */
/* ------------------------------------------------------------------------ */

/*
 * Workspace bytes for chpl_oz2_gemm.  Replaces
 *   gemmul8::workSize<false, gemmul8::Backend::INT8>(m, n, k, num_moduli,
 *       enable_skip_scalA, enable_skip_scalB, &wsA, &wsB)
 * called at src/chpl_single.cu:367-369, src/chpl_p2.cu:755-757,
 * src/chpl_p4.cu:919-921.
 * *work_bytes: size of `work` when workA/workB are NULL (all parts inside);
 * *wsA / *wsB (may be NULL): sizes of the A part (int8 residues + scales of
 * op(A)) and B part, which the caller may instead place in workA / workB.
 * num_moduli in [2, 16]; k <= 131071.
 */
int chpl_oz2_worksize(size_t m, size_t n, size_t k, unsigned num_moduli, int enable_skip_scalA,
                      int enable_skip_scalB, size_t *work_bytes, size_t *wsA, size_t *wsB);

/*
 * C = alpha * op(A) * op(B) + beta * C, FP64 emulated with int8 tensor cores
 * (Ozaki scheme II, num_moduli moduli).  Replaces
 *   gemmul8::gemm<double, gemmul8::Backend::INT8>(handle, opA, opB, m, n, k,
 *       alpha, A, lda, B, ldb, beta, C, ldc, num_moduli, fastmode, work,
 *       workA, workB, enable_skip_scalA, enable_skip_scalB, skip_scalA,
 *       skip_scalB)
 * called at src/chpl_single.cu:641-649, src/chpl_p2.cu:1674-1683,
 * src/chpl_p4.cu:2340-2350 and 2362-2373 (the stream replaces the cuBLAS
 * handle, whose stream the reference sets at src/chpl_p2.cu:760-761).
 * skip_scalA = 1 reuses the residues of op(A) left in the A part by the
 * previous call with the same A, m, k, num_moduli (the per-panel reuse of
 * src/chpl_p2.cu:1642-1643,1684); likewise skip_scalB.
 * Scaling: power-of-two row/column scales from Cauchy-Schwarz bounds (the
 * 2-norms of the rows of op(A) and columns of op(B)), the fast mode of the
 * published method.  fastmode == 0 is accepted and uses the same rule (this
 * build has no separate accurate mode).
 * phase_seconds (NULL or double[4]): when non-NULL the call synchronizes and
 * reports {split, int8 GEMM + fused mod/CRT/unscale, 0, 0} in seconds --
 * the four phase times gemmul8::gemm returns (src/chpl_single.cu:651).
 */
int chpl_oz2_gemm(void *stream, int opA, int opB, size_t m, size_t n, size_t k, const double *alpha,
                  const double *A, size_t lda, const double *B, size_t ldb, const double *beta, double *C,
                  size_t ldc, unsigned num_moduli, int fastmode, void *work, void *workA, void *workB,
                  int enable_skip_scalA, int enable_skip_scalB, int skip_scalA, int skip_scalB,
                  double *phase_seconds);

/*
 * Pieces of chpl_oz2_gemm, exposed for verification (no reference
 * counterpart: GEMMul8 keeps them internal).  Layouts:
 *   rows residues  res[(l * ld_vec + i) * ld_k + h], i < m, h < k, l < L
 *   (K-major; ld_vec >= m, ld_k >= k, ld_k % 128 == 0; padding written 0),
 *   shift[i] such that op(A)[i,h] * 2^shift[i] rounds to the integer image.
 * chpl_oz2_split_rows: op(A) (m x k) -> residues of its rows.
 * chpl_oz2_split_cols: op(B) (k x n) -> residues of its columns.
 * chpl_oz2_products: per-modulus exact int32 products of split residues,
 *   P[l * ldp * n + i + j * ldp] = sum_h ra[l][i][h] * rb[l][j][h], through
 *   the same tcgen05 GEMM kernel as chpl_oz2_gemm (raw epilogue).
 *   ra/rb must have ld_vec multiples of 128 / 256 respectively.
 */
int chpl_oz2_split_rows(void *stream, int opA, size_t m, size_t k, const double *A, size_t lda,
                        unsigned num_moduli, int8_t *res, size_t ld_vec, size_t ld_k, int32_t *shift,
                        void *tmp);
int chpl_oz2_split_cols(void *stream, int opB, size_t k, size_t n, const double *B, size_t ldb,
                        unsigned num_moduli, int8_t *res, size_t ld_vec, size_t ld_k, int32_t *shift,
                        void *tmp);
/* bytes of `tmp` the split functions need for num_vectors vectors */
size_t chpl_oz2_split_tmp_bytes(size_t num_vectors);
int chpl_oz2_products(void *stream, size_t m, size_t n, size_t k, unsigned num_moduli, const int8_t *ra,
                      size_t lda_vec, const int8_t *rb, size_t ldb_vec, size_t ld_k, int32_t *P, size_t ldp);
/*
 * Allocation-free emulated GEMM.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory when they need the update --
 * hosts whose framework reserves the whole device memory pool up front, and
 * latency-sensitive callers that cannot take the synchronization a
 * cudaMalloc / cudaFree may imply.  Same operation and results as
 * chpl_oz2_gemm (fast mode, no skip flags, no phase times), with no `work`
 * argument: all scratch lives in a fixed 64 MiB device array inside libchpl,
 * which every GPU that loads the library keeps until process exit.  Sizes
 * whose scratch exceeds 64 MiB are rejected with CHPL_ERR_WORKSPACE (the
 * scratch is about L*(m_pad + n_pad)*k_pad bytes plus 2 MiB per modulus, with
 * m_pad, k_pad rounded up to 128 and n_pad to 256; e.g. m = n = k = 1024 at 12
 * moduli fits).  The first call on each device (and again after a
 * cudaDeviceReset, which gives the device a new context) looks up the array's
 * device address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture.  All calls on a device share the array
 * and it keeps the last call's contents, so calls that overlap on the GPU
 * (other streams, other host threads) race: serialize them.  Nothing is
 * allocated.  As for chpl_oz2_gemm, a device-side wait that runs out of time
 * leaves C undefined while the call itself has returned CHPL_OK: check
 * chpl_device_status after synchronizing.
 */
int chpl_oz2_gemm_noalloc(void *stream, int opA, int opB, size_t m, size_t n, size_t k, const double *alpha,
                          const double *A, size_t lda, const double *B, size_t ldb, const double *beta,
                          double *C, size_t ldc, unsigned num_moduli);
/* scaling exponents (alpha, beta) used for num_moduli (host-only query) */
int chpl_oz2_shift_bits(unsigned num_moduli, size_t k, int *alpha_bits, int *beta_bits);

/*
 * Ozaki scheme I emulated DGEMM, the reference's alternative engine
 * (HPLS_BACKEND=ozaki; oz_gemm and its kernels, src/chpl_single.cu:147-236,
 * 532-612): row / column power-of-two scales, six base-128 int8 digits per
 * entry, the six anti-diagonals of digit products as int32 products on the
 * tcgen05 int8 kernel, FP64 reconstruction.  C = alpha * A * B + beta * C,
 * column-major, no transposes, k <= 21845, n <= 65280 per call; C may alias B
 * when beta == 0.  `work` >= chpl_oz1_worksize bytes.
 */
int chpl_oz1_worksize(size_t m, size_t n, size_t k, size_t *work_bytes);
int chpl_oz1_gemm(void *stream, size_t m, size_t n, size_t k, double alpha, const double *A, size_t lda,
                  const double *B, size_t ldb, double beta, double *C, size_t ldc, void *work);

/* ------------------------------------------------------------------------ */
/* HPL building blocks                                                       */
/* ------------------------------------------------------------------------ */

/*
 * A[i + j*lda] = elem(seed, (grow(i)) * ncg + gcol(j)) for an m x n block,
 * elem = chpl_elem of src/chpl_p2.cu:66-73 (SplitMix64, [-0.5, 0.5)).
 * Global row of local row i: row0 + i (block-cyclic maps use the grid call
 * chpl_matgen_cyclic).  Replaces matgen2d_kernel (src/chpl_p2.cu:76-87).
 */
int chpl_matgen(void *stream, double *A, size_t lda, size_t m, size_t n, int64_t row0, int64_t col0,
                int64_t ncg, uint64_t seed);
/* The same block with chpl_single's generator: element index
 * (row0+i)*ncg + col0+j is the cuRAND Philox4_32_10 subsequence (offset 0,
 * seed), value curand_uniform_double - 0.5, computed through cuRAND's device
 * API.  Replaces matgen_kernel + hs_rand of src/chpl_single.cu:73-94 (called
 * there with ncg = N + 1). */
int chpl_matgen_philox(void *stream, double *A, size_t lda, size_t m, size_t n, int64_t row0, int64_t col0,
                       int64_t ncg, uint64_t seed);
/* Block-cyclic local piece of the N x (N+1) system for grid coordinate
 * (pr, qc) of a P x Q grid with block NB (src/chpl_p2.cu:615-626,951-957). */
int chpl_matgen_cyclic(void *stream, double *A, size_t lda, int64_t N, int64_t NB, int P, int Q, int pr,
                       int qc, uint64_t seed);
/* The generated N x (N+1) system [A | b] written into HOST memory Ab
 * (column-major, ldab >= N): generated on the current device in column blocks
 * of <= 256 MiB (the same elements as chpl_matgen) and copied out.
 * Synchronous.  Input preparation for chpl_hpl_run_host; the reference has
 * no host copy of the matrix (matgen2d_kernel, src/chpl_p2.cu:76-87). */
int chpl_matgen_host(int64_t N, uint64_t seed, double *Ab, size_t ldab);

/*
 * Row interchanges, LAPACK dlaswp semantics on columns [0, ncols) of A:
 * for i = k1..k2-1 (in order) swap rows i and ipiv[i] (0-based, absolute).
 * Applied as one gather/scatter of the net permutation built on the device
 * (no host synchronization).  Replaces apply_swaps + row_gather/scatter
 * (src/chpl_single.cu:489-518, 108-134).  `work` >= chpl_laswp_work_bytes.
 */
size_t chpl_laswp_work_bytes(int64_t nrows, int64_t nswaps);
int chpl_laswp(void *stream, double *A, size_t lda, int64_t ncols, int64_t k1, int64_t k2,
               const int64_t *ipiv, int64_t nrows, void *work);

/*
 * FP64 LU with partial pivoting of an m x n panel (m >= n), in place:
 * recursive (TRSM and Schur update on the FP64 kernels above), cooperative
 * base kernel with a warp-shuffle pivot search.  ipiv (device, n entries) receives
 * 0-based pivot rows relative to the panel, LAPACK order.  info (device int)
 * receives 0 or the 1-based column of the first exact zero pivot.
 * Replaces cusolverDnXgetrf of the panel (src/chpl_single.cu:668-679).
 */
size_t chpl_panel_getrf_work_bytes(int64_t m, int64_t n);
int chpl_panel_getrf_f64(void *stream, int64_t m, int64_t n, double *A, size_t lda, int64_t *ipiv,
                         int *info, void *work);

/*
 * FP64 BLAS of this library (sm_100a kernels; DGEMM on the FP64 tensor path,
 * mma.sync m16n8k8 .f64).  Column-major, device pointers, asynchronous on
 * `stream`, deterministic (fixed reduction orders).  They replace the cuBLAS
 * calls of the reference's solve path.
 *
 * C (m x n) = alpha * A (m x k) * B (k x n) + beta * C (beta == 0 never reads
 * C; C must not overlap A or B).  Replaces cublasDgemm at
 * src/chpl_single.cu:621-623 (native update) and 694-696 (inner panel
 * update), src/chpl_p2.cu:1377-1381, 1669-1673, 1697-1700.
 */
int chpl_dgemm(void *stream, int64_t m, int64_t n, int64_t k, double alpha, const double *A, size_t lda,
               const double *B, size_t ldb, double beta, double *C, size_t ldc);
/* B (n x nrhs) = L^-1 B with L unit lower triangular (its upper part is not
 * read).  Replaces cublasDtrsm at src/chpl_single.cu:689-691, 708-710 and
 * src/chpl_p2.cu:1211-1220 (inv(L11) against the identity). */
int chpl_dtrsm_llnu(void *stream, int64_t n, int64_t nrhs, const double *L, size_t ldl, double *B, size_t ldb);
/* X (n x n) = L^-1 for L unit lower triangular: X's upper part is set to
 * zero, its diagonal to one.  Recursive: X21 = -L22^-1 (L21 X11) on the DGEMM
 * and TRSM above, 64-wide leaves.  Replaces the trsm of the identity with
 * which the reference forms inv(L11) (src/chpl_p2.cu:1211-1220). */
int chpl_dtrtri_llnu(void *stream, int64_t n, const double *L, size_t ldl, double *X, size_t ldx);
/* x (n) = U^-1 x with U upper triangular, non-unit diagonal; work: n doubles
 * of device scratch.  Replaces cublasDtrsv at src/chpl_single.cu:724-725 (the
 * back solve, a one-column trsm there) and src/chpl_p2.cu:1851. */
int chpl_dtrsv_unn(void *stream, int64_t n, const double *U, size_t ldu, double *x, double *work);
/* y (m) = alpha * A (m x n) * x + beta * y (beta == 0 never reads y).
 * Replaces cublasDgemv at src/chpl_p2.cu:1870. */
int chpl_dgemv(void *stream, int64_t m, int64_t n, double alpha, const double *A, size_t lda, const double *x,
               double beta, double *y);

/*
 * HPL scaled residual of x (device, N) for the generated N x (N+1) system
 * (CHPL_GEN_CHPL, regenerated on the fly, b = column N): ||Ax-b||_oo /
 * (eps*(||A||_oo*||x||_oo+||b||_oo)*N), eps = 2^-53.  Synchronizes.
 * Replaces the verification of src/chpl_single.cu:762-817 /
 * src/chpl_p2.cu:1886-1932.
 */
int chpl_residual(void *stream, int64_t N, uint64_t seed, const double *x, double *resid);
/* The same residual for a system held in device memory: Ab is [A | b]
 * (N x (N+1), column-major, ldab >= N, b = column N).  Same reduction order
 * as chpl_residual, so a generated system gives the identical value.
 * Synchronizes.  Replaces the same verification
 * (src/chpl_single.cu:762-817) for systems that are not generated. */
int chpl_residual_matrix(void *stream, int64_t N, const double *Ab, size_t ldab, const double *x, double *resid);

/*
 * Failure-detection self-test (no reference counterpart): one bounded
 * device-side wait on something nothing signals -- kind 0: an mbarrier phase
 * (the wait every TMA / MMA / epilogue hand-off of the GEMM uses), kind 1: an
 * acquire poll of a flag in global memory (the panel's cross-CTA exchange).
 * Returns CHPL_ERR_TIMEOUT after limit_ns (<= 2 s) with the context still
 * usable.  Synchronizes the stream.
 */
int chpl_diag_bounded_wait(void *stream, int kind, uint64_t limit_ns);

/* ------------------------------------------------------------------------ */
/* HPL solver                                                                */
/* ------------------------------------------------------------------------ */
typedef struct chpl_hpl_config {
    int64_t N;          /* order (HPL.dat line 6) */
    int64_t NB;         /* panel width (HPL.dat line 8) */
    int P, Q;           /* process grid (rank = P*qc + pr) */
    int moduli;         /* CHPL2D_G8_MODULI / HPLS_G8_MODULI */
    int emulate;        /* CHPL2D_G8 / HPLS_BACKEND: 1 = Ozaki-II update (gemmul8), 0 = FP64 (native),
                           2 = Ozaki-I (ozaki; one GPU only) */
    int fast;           /* CHPL2D_G8_FAST / HPLS_G8_FAST */
    int64_t chunk;      /* column chunk of the update (CHPL2D_G8_NT / HPLS_G8_CHUNK), 0 = auto */
    int lookahead;      /* depth-1 lookahead on a high-priority stream (1) or serial (0, default) */
    int agg;            /* HPLS_AGG: panels per super-block; the bulk update runs with k = agg * NB
                           (src/chpl_single.cu:662); 0 = auto: k = 6144 for N >= 131072, 4096 for
                           N >= 65536, else k = NB (the deeper emulated updates cost residual margin
                           at small N) */
    int reserve_sms;    /* SMs left to the lookahead chain while the bulk update runs; -1 = auto */
    int trsm_mode;      /* U12 of a super-block: 0 = auto, 1 = inv(L) * A12 through the emulated GEMM,
                           2 = FP64 triangular solve */
    int panel_mode;     /* 0 = this library's FP64 panel kernel, 1 = cuSOLVER getrf (comparison) */
    uint64_t seed;      /* 42 */
    double threshold;   /* HPL.dat line 13 (16.0) */
    int verbose;        /* print the memory plan (MEM PLAN) and, for a host system streamed in, each
                           intake of column chunks (INGEST: step, columns, landed / reached ms) */
    int generator;      /* CHPL_GEN_CHPL (default; chpl_p2's matrix) or CHPL_GEN_PHILOX (chpl_single's matrix);
                           one-GPU runs only, the grid driver generates with CHPL_GEN_CHPL as chpl_p2 does */
} chpl_hpl_config;

typedef struct chpl_hpl_result {
    double time_s;      /* factor + solve, device time (matgen excluded, as HPL) */
    double tflops;      /* (2/3 N^3 + 2 N^2) / time_s / 1e12 */
    double resid;       /* scaled residual */
    int passed;         /* resid < threshold */
    double matgen_s;
    double phase_s[8];  /* per-stream busy time: panel, laswp, trsm, oz2 split, oz2 int8 GEMM + CRT,
                           FP64 update, back solve, communication */
    int64_t n_emulated; /* emulated update calls */
    int64_t n_launches; /* kernels of this library launched inside factor + solve */
    int64_t gemm_launches;      /* launches of the tcgen05 int8 GEMM kernel */
    double gemm_kernel_s;       /* their summed device time (CUDA events on their streams) */
    double gemm_int8_ops;       /* 2 * m * n * kPad * moduli summed over those launches */
    double gemm_fp64eq_flops;   /* 2 * m * n * k summed over those launches */
    int schedule;               /* grid runs: 0 = serial block steps, 1 = depth-1 lookahead */
} chpl_hpl_result;

/* Fill cfg with the defaults of chpl_single / chpl_p2 (src/chpl_p2.cu:570-584). */
void chpl_hpl_default_config(chpl_hpl_config *cfg);

/*
 * One HPL run on the current device (P = Q = 1): generate, factor and solve,
 * verify.  x_out (host, N doubles) may be NULL.  Replaces run_case of
 * chpl_single (src/chpl_single.cu:733-840).
 */
int chpl_hpl_run(const chpl_hpl_config *cfg, chpl_hpl_result *res, double *x_out);

/*
 * One solve of a caller-supplied system from HOST memory on the current
 * device (P = Q = 1): [A | b] (N x (N+1), column-major, ldab >= N, b = column
 * N) is copied to the device (page-locked memory from chpl_host_alloc copies
 * at full bandwidth; pageable memory works, slower), factored and solved with
 * the same kernels as chpl_hpl_run (cfg->seed is unused), and x is written to
 * x_out (host, N doubles; may be NULL).  With the serial schedule
 * (cfg->lookahead = 0) the copy runs in column chunks on its own stream while
 * the factorization works on the columns already present (a late chunk first
 * catches up on the steps the others have received); x is bit-identical to
 * chpl_hpl_run's on the same system, and res->time_s covers copy + factor +
 * solve (device time, res->matgen_s = 0).  With the lookahead the system is
 * copied first (res->matgen_s) and res->time_s is factor + solve.  verify = 1
 * copies [A | b] in again after the solve and computes the HPL scaled
 * residual against it (res->resid, res->passed); verify = 0 leaves
 * res->resid NaN and res->passed 0.  The host-buffer form of run_case
 * (src/chpl_single.cu:733-840), whose input the reference always generates
 * on the device (src/chpl_single.cu:750).
 */
int chpl_hpl_run_host(const chpl_hpl_config *cfg, const double *Ab, size_t ldab, int verify,
                      chpl_hpl_result *res, double *x_out);

/* ------------------------------------------------------------------------ */
/* P x Q process grid (one process per GPU, NCCL over NVLink)                */
/* ------------------------------------------------------------------------ */

/* NCCL unique id for the grid (rank 0 creates it and shares the bytes with
 * the other ranks by any host channel).  Replaces the MPI_Bcast of NCCL ids
 * of src/chpl_p2.cu:552-568.  len >= 128. */
int chpl_grid_unique_id(unsigned char *id, size_t len);
/* World, process-row and process-column communicators of rank `rank` of a
 * P x Q grid (pr = rank % P, qc = rank / P, src/chpl_p2.cu:528), on the
 * current device.  timeout_s bounds every host-side wait; past it the
 * communicators are aborted and calls return CHPL_ERR_TIMEOUT.
 * Replaces the MPI/NCCL bootstrap of src/chpl_p2.cu:520-568. */
int chpl_grid_create(int P, int Q, int rank, const unsigned char *id, size_t len, double timeout_s, void **grid);
/* One HPL solve on the grid (all ranks call it): block-cyclic generation,
 * factorization, distributed back substitution and residual.  res is the
 * same on every rank except time_s (this rank's device time).  x_out (host,
 * N) may be NULL.  Replaces main() of src/chpl_p2.cu (lines 518-1953). */
int chpl_grid_run(void *grid, const chpl_hpl_config *cfg, chpl_hpl_result *res, double *x_out);
int chpl_grid_destroy(void *grid);
/* Host-only: the row moves of one block column's interchanges (swaps
 * J+i <-> J+piv[i], i < K) for process row pr of P: local moves
 * (lsrc -> ldst), rows sent (snd) and received (rcv) across process rows,
 * each array >= 2K entries.  The reference builds the same lists on the
 * device (buildlists_kernel, src/chpl_p2.cu:255-300). */
int chpl_grid_plan_exchange(int64_t J, int64_t K, const int64_t *piv, int64_t NB, int P, int pr, int *lsrc,
                            int *ldst, int *nl, int *snd, int *ns, int *rcv, int *nr);

#ifdef __cplusplus
}
#endif

#endif /* CHPL_H */
