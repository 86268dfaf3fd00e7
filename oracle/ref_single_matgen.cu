// Harness around chpl_single's own generator kernel -- TEST INFRASTRUCTURE
// ONLY.  oracle/ref_build.py extracts hs_rand and matgen_kernel verbatim from
// the reference (src/chpl_single.cu) into oracle/_ref/single_matgen.inc
// (never committed) and compiles this file into
// oracle/_ref/libref_single_matgen.so for sm_100a.  The GPU tests compare this
// project's Philox generator with it, element for element.
#include <cstdint>
#include <curand_kernel.h>

#include "single_matgen.inc"

extern "C" int ref_single_matgen(double* A, int64_t nrows, int64_t col0, int64_t ncols, int64_t ld, uint64_t seed,
                                 uint64_t keyN, void* stream)
{
    const int64_t total = nrows * ncols;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (blocks < 1) blocks = 1;
    matgen_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(A, nrows, col0, ncols, ld, seed, keyN);
    return (int)cudaGetLastError();
}
