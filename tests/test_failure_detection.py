"""Failure detection without a GPU fault.

Device side: every wait in the library's kernels is bounded; a wait on
something nothing signals (an mbarrier phase, a flag in global memory) ends
with CHPL_ERR_TIMEOUT after its limit, and the context stays usable.
Host side: the bootstrap of chpl_p2 gives up with an error when a rank never
shows up (CPU only, no device is touched before the bootstrap).  The grid's
collectives run under a host watchdog that aborts the NCCL communicators
(covered by design in hpl_grid.cu; no test kills a rank mid-collective).
"""
import os
import socket
import subprocess
import time

import numpy as np
import pytest

from chpl_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
P2 = os.path.join(ROOT, "chpl_b200", "bin", "chpl_p2")


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("rank", [0, 1])
def test_p2_bootstrap_gives_up_when_a_rank_never_joins(rank):
    env = dict(os.environ, WORLD_SIZE="2", RANK=str(rank), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
               CHPL_BOOTSTRAP_PORT=str(_port()), CHPL_BOOTSTRAP_TIMEOUT="2")
    t0 = time.monotonic()
    r = subprocess.run([P2], capture_output=True, text=True, env=env, timeout=60)
    el = time.monotonic() - t0
    assert r.returncode == 1
    assert ("not every rank fetched" in r.stderr) if rank == 0 else ("no NCCL id" in r.stderr)
    assert el < 30


@pytest.mark.gpu
@pytest.mark.parametrize("kind", [0, 1])
def test_bounded_wait_times_out_and_context_survives(cuda, kind):
    import torch

    import oracle
    from chpl_b200 import oz2
    from gpu_util import empty_bytes, from_dev, to_dev
    L = _lib.load()
    t0 = time.monotonic()
    rc = L.chpl_diag_bounded_wait(None, kind, 20_000_000)   # 20 ms
    el = time.monotonic() - t0
    assert rc == _lib.CHPL_ERR_TIMEOUT
    assert b"ran out" in L.chpl_last_error_string()
    assert 0.02 <= el < 5.0
    # the context is still usable: an emulated GEMM is bit-exact afterwards
    rng = np.random.default_rng(3)
    m, n, k, Lm = 200, 150, 300, 11
    A = rng.uniform(-0.5, 0.5, (m, k))
    B = rng.uniform(-0.5, 0.5, (k, n))
    C = rng.uniform(-0.5, 0.5, (m, n))
    dA, lda = to_dev(A)
    dB, ldb = to_dev(B)
    dC, ldc = to_dev(C)
    tot, _, _ = oz2.workSize(m, n, k, Lm)
    oz2.gemm(0, 0, m, n, k, -1.0, dA, lda, dB, ldb, 1.0, dC, ldc, Lm, True, empty_bytes(tot))
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(dC, m, n), oracle.oz2_gemm(A, B, C, Lm, mode=1))


def test_bounded_wait_rejects_bad_arguments():
    L = _lib.load()
    assert L.chpl_diag_bounded_wait(None, 2, 1000) == _lib.CHPL_ERR_INVALID
    assert L.chpl_diag_bounded_wait(None, 0, 0) == _lib.CHPL_ERR_INVALID
    assert L.chpl_diag_bounded_wait(None, 0, 3_000_000_000) == _lib.CHPL_ERR_INVALID
