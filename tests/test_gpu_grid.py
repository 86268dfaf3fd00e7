"""GPU tests of the P x Q grid driver (one process per GPU, NCCL).

The 1 x 1 grid runs in this process on one GPU; grids of 2 ranks (1 x 2,
2 x 1) and 4 ranks (2 x 2) run as spawned processes when the machine has that
many GPUs (NVLS off, as for every multi-rank test on this pool)."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from chpl_b200 import _lib, hpl

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, P, Q, N, NB, out, env=None, opts=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    os.environ.update(env or {})
    from chpl_b200 import grid
    dist = grid.init_from_env(timeout_s=300)
    g = grid.Grid(P, Q, timeout_s=120)
    o = dict(moduli=12, emulate=True)
    o.update(opts or {})
    r = g.run(hpl.Config(N=N, NB=NB, P=P, Q=Q, **o), want_x=True)
    g.close()
    out[rank] = (r.passed, r.resid, r.x)
    dist.barrier()
    dist.destroy_process_group()


def _run_spawned(P, Q, N, NB, env=None, opts=None):
    import torch.multiprocessing as mp
    world = P * Q
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        mp.start_processes(_worker, args=(world, _free_port(), P, Q, N, NB, out, env, opts), nprocs=world, join=True,
                           start_method="spawn")
        return dict(out)


def _reference_x(N):
    S = oracle.hpl_system(N)
    return np.linalg.solve(S[:, :N], S[:, N])


def _check_forward_error(x, N, resid):
    """x against the FP64 solution: to first order the forward error is at most
    cond_inf(A) times the normwise backward error, which the scaled residual
    gives as resid * eps * N (eps = 2^-53); the FP64 solution itself carries
    cond * eps.  A factor 2 covers the first-order terms."""
    S = oracle.hpl_system(N)
    A = S[:, :N]
    xs = np.linalg.solve(A, S[:, N])
    eps = 2.0 ** -53
    bound = 2.0 * np.linalg.cond(A, np.inf) * eps * (resid * N + 1.0)
    err = np.abs(x - xs).max() / np.abs(xs).max()
    assert err <= bound, (err, bound)


@pytest.mark.parametrize("moduli", [11, 12])
def test_grid_1x1_in_process(cuda, moduli):
    import torch.distributed as dist
    from chpl_b200 import grid
    if not dist.is_initialized():
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
        dist.init_process_group("gloo", rank=0, world_size=1)
    g = grid.Grid(1, 1)
    r = g.run(hpl.Config(N=4000, NB=256, P=1, Q=1, moduli=moduli, agg=2), want_x=True)
    g.close()
    assert r.passed, r.resid
    _check_forward_error(r.x, 4000, r.resid)


def test_grid_1x1_fp64_update(cuda):
    """CHPL2D_G8=0 (the reference's compiled-in default): the trailing update
    and U12 run in FP64 on the library's DGEMM, on the serial block steps."""
    import torch.distributed as dist
    from chpl_b200 import grid
    if not dist.is_initialized():
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
        dist.init_process_group("gloo", rank=0, world_size=1)
    g = grid.Grid(1, 1)
    r = g.run(hpl.Config(N=3000, NB=512, P=1, Q=1, emulate=False), want_x=True)
    # the Ozaki-I update is the one-GPU engine's only: an error, and the grid stays usable
    with pytest.raises(_lib.ChplError, match="Ozaki-I"):
        g.run(hpl.Config(N=2048, NB=256, P=1, Q=1, emulate=2))
    g.close()
    assert r.passed and r.resid < 1.0, r.resid
    # forward error of two backward-stable solves of a system with condition ~1e5
    assert np.allclose(r.x, _reference_x(3000), rtol=1e-7, atol=1e-9)


@pytest.mark.parametrize("moduli", [11, 12])
@pytest.mark.parametrize("grid_shape", [(1, 2), (2, 1)])
def test_grid_two_ranks(cuda, grid_shape, moduli):
    """Two ranks at the benchmark's 11 moduli and at 12, against the FP64
    solution of the same system."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    P, Q = grid_shape
    N, NB = 4000, 256
    out = _run_spawned(P, Q, N, NB, opts={"moduli": moduli})
    for rank in range(P * Q):
        passed, resid, x = out[rank]
        assert passed, resid
        _check_forward_error(x, N, resid)


@pytest.mark.parametrize("grid_shape", [(1, 2), (2, 1)])
def test_grid_two_ranks_fp64_update(cuda, grid_shape):
    """CHPL2D_G8=0 on two ranks: FP64 update, serial block steps."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    P, Q = grid_shape
    N, NB = 4000, 256
    out = _run_spawned(P, Q, N, NB, opts={"emulate": False})
    xs = _reference_x(N)
    for rank in range(P * Q):
        passed, resid, x = out[rank]
        assert passed and resid < 1.0, resid
        assert np.allclose(x, xs, rtol=1e-7, atol=1e-9)


@pytest.mark.parametrize("moduli", [11, 12])
def test_grid_2x2(cuda, moduli):
    if torch.cuda.device_count() < 4:
        pytest.skip("needs 4 GPUs")
    out = _run_spawned(2, 2, 5000, 256, opts={"moduli": moduli})
    for rank in range(4):
        passed, resid, x = out[rank]
        assert passed, resid
        _check_forward_error(x, 5000, resid)


def test_grid_1x2_lookahead_equals_serial(cuda):
    """The 1 x Q lookahead only reorders work (urgent block first, column
    chunks), so its solution is bit-identical to the serial block steps."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    N, NB = 4608, 512
    la = _run_spawned(1, 2, N, NB)
    se = _run_spawned(1, 2, N, NB, env={"CHPL_GRID_SERIAL": "1"})
    for rank in range(2):
        assert la[rank][0] and se[rank][0]
        assert np.array_equal(la[rank][2], se[rank][2])


@pytest.mark.parametrize("grid_shape,ngpu", [((2, 1), 2), ((2, 2), 4)])
def test_grid_p2_lookahead_equals_serial(cuda, grid_shape, ngpu):
    """The 2 x Q lookahead reorders work across three streams (urgent block,
    chunked gather / scatter, bulk exchanges on a second communicator); the
    solution is bit-identical to the serial block steps."""
    if torch.cuda.device_count() < ngpu:
        pytest.skip(f"needs {ngpu} GPUs")
    P, Q = grid_shape
    N, NB = 5000, 256
    la = _run_spawned(P, Q, N, NB)
    se = _run_spawned(P, Q, N, NB, env={"CHPL_GRID_SERIAL": "1"})
    for rank in range(P * Q):
        assert la[rank][0] and se[rank][0]
        assert np.array_equal(la[rank][2], se[rank][2])
        _check_forward_error(la[rank][2], N, la[rank][1])
