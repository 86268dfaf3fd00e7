"""CPU tests of the grid driver's host logic: interchange planning across a
2 x Q process grid, checked by gloo ranks that exchange rows of a
block-cyclic toy matrix exactly as the GPU path does with NCCL."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from chpl_b200 import grid


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _random_pivots(rng, K, rows_left):
    return np.array([i + rng.integers(0, rows_left - i) for i in range(K)], dtype=np.int64)


def test_plan_exchange_single_row_is_all_local():
    rng = np.random.default_rng(0)
    piv = _random_pivots(rng, 64, 500)
    pl = grid.plan_exchange(100, 64, piv, 64, 1, 0)
    assert len(pl["snd"]) == 0 and len(pl["rcv"]) == 0
    # applying the local moves reproduces the sequential swaps
    G = np.arange(1000.0)
    ref = G.copy()
    for i in range(64):
        a, b = 100 + i, 100 + piv[i]
        ref[[a, b]] = ref[[b, a]]
    out = G.copy()
    out[pl["ldst"]] = G[pl["lsrc"]]
    assert np.array_equal(out, ref)


def test_plan_rejects_bad_pivots():
    with pytest.raises(Exception):
        grid.plan_exchange(0, 4, np.array([0, 0, 5, 3]), 4, 2, 0)


def _worker(rank, world, port, N, NB, J, K, seed, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch
    P = world
    pr = rank
    rng = np.random.default_rng(seed)
    piv = _random_pivots(rng, K, N - J)
    Gm = np.arange(N * 3, dtype=np.float64).reshape(N, 3)   # global rows x 3 columns
    rows = [g for g in range(N) if (g // NB) % P == pr]
    local = Gm[rows].copy()
    pl = grid.plan_exchange(J, K, piv, NB, P, pr)
    send = local[pl["snd"]]
    tmp = local[pl["lsrc"]]
    # counts must pair up across the two process rows
    cnt = torch.tensor([len(pl["snd"]), len(pl["rcv"])], dtype=torch.int64)
    allc = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(allc, cnt)
    other = 1 - pr
    assert allc[pr][0].item() == allc[other][1].item()
    recv = torch.zeros((len(pl["rcv"]), 3), dtype=torch.float64)
    reqs = []
    if len(pl["snd"]):
        reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(send)), dst=other))
    if len(pl["rcv"]):
        reqs.append(dist.irecv(recv, src=other))
    for r in reqs:
        r.wait()
    local[pl["ldst"]] = tmp
    local[pl["rcv"]] = recv.numpy()
    # reference: sequential swaps on the global matrix
    ref = Gm.copy()
    for i in range(K):
        a, b = J + i, J + piv[i]
        ref[[a, b]] = ref[[b, a]]
    ok = np.array_equal(local, ref[rows])
    out[rank] = bool(ok)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("case", [(1000, 64, 128, 64, 1), (777, 32, 0, 32, 2), (4096, 256, 1024, 256, 3)])
def test_plan_exchange_two_process_rows_gloo(case):
    N, NB, J, K, seed = case
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        mp.start_processes(_worker, args=(2, _free_port(), N, NB, J, K, seed, out), nprocs=2, join=True,
                           start_method="spawn")
        assert out[0] and out[1]


def test_grid_shapes():
    assert grid.grid_shape(1) == (1, 1)
    assert grid.grid_shape(2) == (1, 2)
    assert grid.grid_shape(4) == (2, 2)
    assert grid.grid_shape(8) == (2, 4)
