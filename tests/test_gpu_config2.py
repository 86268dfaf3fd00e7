"""The standalone trailing update at its full size on a B200:
C(m x n) -= A(m x k) B(k x n), m = n = 32768, k = 4096, FP64 column-major,
entries uniform in [-0.5, 0.5) from the reference's generator (chpl_elem of
src/chpl_p2.cu:66-73 over each matrix's own index space; seeds 42, 43, 44 for
A, B, C), and a variant whose row i of A is scaled by 2^u_i, u_i
integer-uniform in [-20, 20] (seeded), to stress the exponent range.  At 11 and
12 moduli:

* the per-modulus int32 products of the residues, bit-exact against an
  independent integer GEMM on the same residues (cuBLAS int8 x int8 -> int32
  through torch._int_mm: exact integer arithmetic, so equality is the check);
* the emulated FP64 update against FP64 DGEMM (cuBLAS through torch) on the
  same inputs: max|dC| / (||A||_oo ||B||_oo) <= 1e-15 at 11 moduli, 1e-16 at 12.

The CPU oracle cannot finish these sizes in seconds; its bit-exact parity with
the GPU path is held at small sizes in test_gpu_oz2.py, and both checks here
are size-independent properties of the same kernels.
"""
import pytest
import torch

import oracle
from chpl_b200 import _lib, oz2
from gpu_util import empty_bytes

pytestmark = pytest.mark.gpu

M, N, K = 32768, 32768, 4096


def _generated(rows: int, cols: int, seed: int) -> torch.Tensor:
    """rows x cols column-major (tensor of shape (cols, rows)) from the generator."""
    L = _lib.load()
    t = torch.empty((cols, rows), dtype=torch.float64, device="cuda")
    _lib.check(L.chpl_matgen(0, t.data_ptr(), rows, rows, cols, 0, 0, cols, seed), "chpl_matgen")
    return t


@pytest.fixture(scope="module")
def operands(cuda):
    At = _generated(M, K, 42)          # At[h, i] = A[i, h]
    Bt = _generated(K, N, 43)          # Bt[j, h] = B[h, j]
    Ct = _generated(M, N, 44)          # Ct[j, i] = C[i, j]
    g = torch.Generator(device="cuda").manual_seed(42)
    u = torch.randint(-20, 21, (M,), generator=g, device="cuda").to(torch.float64)
    torch.cuda.synchronize()
    yield {"A": At, "B": Bt, "C": Ct, "row_scale": torch.exp2(u)}
    torch.cuda.empty_cache()


def _A(ops, scaled: bool) -> torch.Tensor:
    return ops["A"] * ops["row_scale"][None, :] if scaled else ops["A"]


@pytest.mark.parametrize("L", [11, 12])
@pytest.mark.parametrize("scaled", [False, True])
def test_config2_update_vs_fp64_dgemm(operands, L, scaled):
    At, Bt, Ct = _A(operands, scaled), operands["B"], operands["C"]
    tot, _, _ = oz2.workSize(M, N, K, L)
    work = empty_bytes(tot)
    got = Ct.clone()
    oz2.gemm(oz2.OP_N, oz2.OP_N, M, N, K, -1.0, At, M, Bt, K, 1.0, got, M, L, True, work)
    del work
    ref = torch.addmm(Ct, Bt, At, beta=1.0, alpha=-1.0)      # (C - A B)^T in FP64 (cuBLAS DGEMM)
    err = got.sub_(ref).abs_().max().item()
    del got, ref
    normA = At.abs().sum(dim=0).max().item()                 # ||A||_oo: largest row sum
    normB = Bt.abs().sum(dim=0).max().item()                 # ||B||_oo
    torch.cuda.empty_cache()
    ratio = err / (normA * normB)
    assert ratio <= (1e-15 if L == 11 else 1e-16), (L, scaled, ratio)


@pytest.mark.parametrize("L", [11, 12])
@pytest.mark.parametrize("scaled", [False, True])
def test_config2_products_bitexact(operands, L, scaled):
    At, Bt = _A(operands, scaled), operands["B"]
    ldk = K
    ra = torch.empty((L, M, ldk), dtype=torch.int8, device="cuda")     # rows of A, K-major
    rb = torch.empty((L, N, ldk), dtype=torch.int8, device="cuda")     # columns of B, K-major
    sa = torch.empty(M, dtype=torch.int32, device="cuda")
    sb = torch.empty(N, dtype=torch.int32, device="cuda")
    tmp = empty_bytes(oz2.split_tmp_bytes(max(M, N)))
    oz2.split_rows(oz2.OP_N, M, K, At, M, L, ra, M, ldk, sa, tmp)
    oz2.split_cols(oz2.OP_N, K, N, Bt, K, L, rb, N, ldk, sb, tmp)
    P = torch.empty((L, N, M), dtype=torch.int32, device="cuda")       # plane l: column-major M x N
    oz2.products(M, N, K, L, ra, M, rb, N, ldk, P, M)
    for l in range(L):
        ref = torch._int_mm(ra[l], rb[l].t())                          # (M x K) x (K x N), exact int32
        assert torch.equal(P[l].t(), ref), f"modulus {l}"
        del ref
    del ra, rb, P, tmp
    torch.cuda.empty_cache()


def test_config2_residues_in_range(operands):
    """Every residue lies in its modulus' symmetric range (a property the
    int32 accumulation bound relies on), at the full size."""
    L = 11
    At = operands["A"]
    ra = torch.empty((L, M, K), dtype=torch.int8, device="cuda")
    sa = torch.empty(M, dtype=torch.int32, device="cuda")
    tmp = empty_bytes(oz2.split_tmp_bytes(M))
    oz2.split_rows(oz2.OP_N, M, K, At, M, L, ra, M, K, sa, tmp)
    for l, md in enumerate(oracle.oz2_moduli(L)):
        hi = (md - 1) // 2
        assert int(ra[l].min()) >= hi - md + 1 and int(ra[l].max()) <= hi, f"modulus {md}"
    del ra
    torch.cuda.empty_cache()
