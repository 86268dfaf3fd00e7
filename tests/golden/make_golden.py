"""Generates the small golden fixtures under tests/golden/ from the oracle.

The reference itself cannot run in this container (no GPU, MPI or GEMMul8
source), so the fixtures are produced by the CPU restatement after it has been
pinned (tests/test_oracle.py: SplitMix64 published known answers, big-integer
CRT, LAPACK).  They freeze those outputs so that later changes to either the
oracle or the CUDA kernels are caught.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402


def main():
    np.savez_compressed(os.path.join(HERE, "matgen_N64_seed42.npz"), A=oracle.hpl_system(64, seed=42))
    rng = np.random.default_rng(2024)
    m, n, k = 40, 36, 160
    A = rng.uniform(-0.5, 0.5, (m, k)) * np.exp2(rng.integers(-20, 21, size=m))[:, None]
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    out = {"A": A, "B": B, "C": C}
    for L in (11, 12):
        a_bits, b_bits = oracle.oz2_shift_bits(L, k)
        sa = oracle.oz2_row_shift(A, a_bits)
        sb = oracle.oz2_col_shift(B, b_bits)
        out[f"sa{L}"] = sa
        out[f"sb{L}"] = sb
        out[f"ra{L}"] = oracle.oz2_split_rows(A, sa, L)
        out[f"rb{L}"] = oracle.oz2_split_cols(B, sb, L)
        out[f"C{L}"] = oracle.oz2_gemm(A, B, C, L, mode=1)
    np.savez_compressed(os.path.join(HERE, "oz2_m40_n36_k160.npz"), **out)
    make_oz1()
    x, ipiv, _ = oracle.hpl_solve(256, 32, L=0)
    np.savez_compressed(os.path.join(HERE, "hpl_N256_NB32.npz"), x=x, ipiv=ipiv,
                        resid=np.array([oracle.hpl_residual(x, 256)]))


def make_oz1():
    """The Ozaki-I engine's C -= A B and C = A B on rows 2^+-20 apart (the
    restatement is pinned to the reference's own Ozaki-I kernels on the GPU)."""
    rng = np.random.default_rng(2025)
    m, n, k = 48, 40, 200
    A = rng.uniform(-0.5, 0.5, (m, k)) * np.exp2(rng.integers(-20, 21, size=m))[:, None]
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    np.savez_compressed(os.path.join(HERE, "oz1_m48_n40_k200.npz"), A=A, B=B, C=C,
                        update=oracle.oz1_gemm(A, B, C), product=oracle.oz1_gemm(A, B, None, alpha=1.0, beta=0.0))


if __name__ == "__main__":
    main()
