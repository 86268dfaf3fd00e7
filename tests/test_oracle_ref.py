"""Parity pins against the reference's own source (CPU).

oracle/ref_build.py cuts four self-contained pieces verbatim out of the
reference checkout and compiles them into oracle/_ref/ (git-ignored): the
generator chpl_elem (src/chpl_p2.cu), the swap resolution resolve_seq
(src/chpl_p2.cu), the scaled-residual reduction of run_case
(src/chpl_single.cu) and chpl_single's Philox generator kernel (GPU side,
tests/test_gpu_ref.py).  These tests hold the CPU oracle, the committed golden
fixtures and this library's host-side interchange planner to them, bit for
bit.  Where the libraries were never built (no reference checkout where the
repository was built) the tests skip.
"""
import json
import os

import numpy as np
import pytest

import oracle
from chpl_b200 import grid

HERE = os.path.dirname(os.path.abspath(__file__))
REF = oracle.ref_host()
pytestmark = pytest.mark.skipif(REF is None, reason="oracle/_ref not built (no reference checkout)")


def _ref_matgen(m, n, row0=0, col0=0, ncg=None, seed=42):
    A = np.zeros((n, m), dtype=np.float64)   # column-major m x n
    REF.ref_matgen(A.ctypes.data, m, m, n, row0, col0, ncg if ncg is not None else n, seed)
    return A.T


def test_fragments_were_cut_from_the_expected_functions():
    man = json.load(open(os.path.join(os.path.dirname(oracle.__file__), "_ref", "manifest.json")))
    assert set(man) == {"chpl_elem.inc", "resolve_seq.inc", "residual.inc", "single_matgen.inc", "single_oz1.inc"}
    assert man["chpl_elem.inc"]["file"] == "src/chpl_p2.cu"
    assert man["resolve_seq.inc"]["file"] == "src/chpl_p2.cu"
    assert man["residual.inc"]["file"] == "src/chpl_single.cu"
    assert man["single_matgen.inc"]["file"] == "src/chpl_single.cu"
    assert man["single_oz1.inc"]["file"] == "src/chpl_single.cu"
    for v in man.values():
        a, b = v["lines"]
        assert 0 < a < b


def test_generator_elements_equal_reference():
    rng = np.random.default_rng(5)
    seeds = [0, 1, 42, 2 ** 63, 2 ** 64 - 1] + [int(s) for s in rng.integers(0, 2 ** 63, 5)]
    idx = [0, 1, 2, 2 ** 32, 2 ** 62, 2 ** 64 - 2] + [int(i) for i in rng.integers(0, 2 ** 63, 200)]
    for s in seeds:
        for i in idx:
            a = oracle.lib().orc_elem(s, i)
            b = REF.ref_chpl_elem(s, i)
            assert np.float64(a).view(np.uint64) == np.float64(b).view(np.uint64), (s, i)


def test_generated_blocks_equal_reference():
    N = 300
    A = oracle.hpl_system(N, seed=42)
    assert np.array_equal(A, _ref_matgen(N, N + 1, ncg=N + 1, seed=42))
    # an interior block with its own row / column origin, as the block-cyclic generation uses
    B = oracle.matgen(70, 33, seed=7, row0=1000, col0=2000, ncg=5001)
    assert np.array_equal(B, _ref_matgen(70, 33, row0=1000, col0=2000, ncg=5001, seed=7))


def test_golden_matrix_fixture_is_the_reference_generator():
    g = np.load(os.path.join(HERE, "golden", "matgen_N64_seed42.npz"))["A"]
    assert np.array_equal(g, _ref_matgen(64, 65, ncg=65, seed=42))


def _ref_residual(y, rs, b, x):
    f = [np.ascontiguousarray(v, np.float64) for v in (y, rs, b, x)]
    return REF.ref_residual(*[v.ctypes.data for v in f], len(y))


def test_residual_formula_equals_reference():
    rng = np.random.default_rng(9)
    for N in (1, 2, 17, 1000):
        for scale in (1e-300, 1.0, 1e300):
            y = rng.standard_normal(N) * scale
            b = y + rng.standard_normal(N) * scale * 1e-14
            rs = np.abs(rng.standard_normal(N)) * N
            x = rng.standard_normal(N)
            a = oracle.hpl_residual_parts(y, rs, b, x)
            r = _ref_residual(y, rs, b, x)
            assert np.float64(a).view(np.uint64) == np.float64(r).view(np.uint64), (N, scale)
    # ties and zeros
    z = np.zeros(8)
    assert np.isnan(oracle.hpl_residual_parts(z, z, z, z)) and np.isnan(_ref_residual(z, z, z, z))


def test_golden_solution_residual_equals_reference():
    """The committed N = 256 solve: its residual recomputed by the reference's
    reduction (on the reference generator's matrix, with A x and the row sums
    summed in column order as the oracle does) equals the stored value."""
    g = np.load(os.path.join(HERE, "golden", "hpl_N256_NB32.npz"))
    N = 256
    Ab = _ref_matgen(N, N + 1, ncg=N + 1, seed=42)
    x = g["x"]
    y = np.zeros(N)
    rs = np.zeros(N)
    for c in range(N):        # sequential, no fused multiply-add: the oracle's loop order
        y = y + Ab[:, c] * x[c]
        rs = rs + np.abs(Ab[:, c])
    r = _ref_residual(y, rs, Ab[:, N], x)
    assert r == float(g["resid"][0])
    assert r == oracle.hpl_residual(x, N)


def _net_from_ref(piv_abs, base):
    top, below = oracle.ref_resolve_seq(np.asarray(piv_abs, np.int64), base)
    net = {base + i: int(t) for i, t in enumerate(top)}
    net.update(below)
    return {d: s for d, s in net.items() if d != s}


def _pivots(rng, K, span):
    return np.array([i + int(rng.integers(0, span - i)) for i in range(K)], dtype=np.int64)


def test_swap_resolution_matches_oracle_laswp():
    rng = np.random.default_rng(3)
    for K, span, base in ((1, 1, 0), (8, 8, 0), (16, 400, 100), (64, 70, 5), (200, 10000, 3000)):
        piv = _pivots(rng, K, span)
        ref = _net_from_ref(base + piv, base)
        ids = np.arange(base + span, dtype=np.float64).reshape(-1, 1)
        ipiv = np.arange(base + span, dtype=np.int64)     # absolute, indexed by row (dlaswp convention)
        ipiv[base:base + K] = base + piv
        got = oracle.laswp(ids.copy(), ipiv, base, base + K)[:, 0]
        mine = {int(d): int(s) for d, s in enumerate(got) if int(s) != d}
        assert mine == ref, (K, span)


def test_swap_resolution_matches_library_planner():
    """This library's host-side interchange planner (one process row: every
    move is local) produces the reference's net permutation."""
    rng = np.random.default_rng(4)
    for K, span, J in ((4, 4, 0), (32, 500, 1024), (256, 3000, 4096), (1024, 139264 - 8192, 8192)):
        piv = _pivots(rng, K, span)
        ref = _net_from_ref(J + piv, J)
        plan = grid.plan_exchange(J, K, piv, NB=1024, P=1, pr=0)
        mine = {int(d): int(s) for d, s in zip(plan["ldst"], plan["lsrc"])}
        assert mine == ref, (K, span)
        assert len(plan["snd"]) == 0 and len(plan["rcv"]) == 0
