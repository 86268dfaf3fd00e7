"""P x Q grid runs: one process per GPU, launched by torchrun (the chpl_p2 path).

The host side uses torch.distributed over gloo only for plumbing: sharing the
NCCL unique id, barriers and the max-over-ranks of the timings.  All matrix
traffic goes through the library's own NCCL communicators (world, process
row, process column; rank = P*qc + pr, src/chpl_p2.cu:528).
"""
from __future__ import annotations

import ctypes
import json
import os
import time
from datetime import timedelta

import numpy as np

from . import _lib, hpl


def grid_shape(world: int) -> tuple[int, int]:
    """Grid of a job with `world` GPUs: 1x1, 1x2, 2x2, 2x4 (P <= 2), else 1 x world."""
    return {1: (1, 1), 2: (1, 2), 4: (2, 2), 8: (2, 4)}.get(world, (1, world))


def plan_exchange(J: int, K: int, piv, NB: int, P: int, pr: int) -> dict:
    """Row moves of one block column's interchanges for process row pr (host only)."""
    L = _lib.load()
    p = np.ascontiguousarray(piv, dtype=np.int64)
    cap = max(2 * K, 1)
    bufs = {k: np.zeros(cap, dtype=np.int32) for k in ("lsrc", "ldst", "snd", "rcv")}
    nl, ns, nr = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.check(L.chpl_grid_plan_exchange(J, K, p.ctypes.data, NB, P, pr, bufs["lsrc"].ctypes.data,
                                         bufs["ldst"].ctypes.data, ctypes.byref(nl), bufs["snd"].ctypes.data,
                                         ctypes.byref(ns), bufs["rcv"].ctypes.data, ctypes.byref(nr)),
               "chpl_grid_plan_exchange")
    return {"lsrc": bufs["lsrc"][:nl.value], "ldst": bufs["ldst"][:nl.value], "snd": bufs["snd"][:ns.value],
            "rcv": bufs["rcv"][:nr.value]}


class Grid:
    """NCCL communicators of this rank; create on every rank of the job."""

    def __init__(self, P: int, Q: int, timeout_s: float = 300.0):
        import torch
        import torch.distributed as dist
        self.P, self.Q = P, Q
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        if P * Q != self.world:
            raise ValueError(f"grid {P}x{Q} needs {P * Q} ranks, job has {self.world}")
        L = _lib.load()
        idbuf = (ctypes.c_ubyte * 128)()
        if self.rank == 0:
            _lib.check(L.chpl_grid_unique_id(idbuf, 128), "chpl_grid_unique_id")
        obj = [bytes(idbuf) if self.rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        raw = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        h = ctypes.c_void_p()
        torch.cuda.synchronize()
        _lib.check(L.chpl_grid_create(P, Q, self.rank, raw, 128, timeout_s, ctypes.byref(h)), "chpl_grid_create")
        self.handle = h

    def run(self, cfg: hpl.Config, want_x: bool = False) -> hpl.Result:
        L = _lib.load()
        c = cfg.to_c()
        r = _lib.HplResult()
        x = np.empty(cfg.N, dtype=np.float64) if want_x else None
        _lib.check(L.chpl_grid_run(self.handle, ctypes.byref(c), ctypes.byref(r), x.ctypes.data if want_x else None),
                   "chpl_grid_run")
        return hpl.Result(N=cfg.N, NB=cfg.NB, P=cfg.P, Q=cfg.Q, time_s=r.time_s, tflops=r.tflops, resid=r.resid,
                          passed=bool(r.passed), threshold=cfg.threshold, matgen_s=r.matgen_s,
                          phases={p: r.phase_s[i] for i, p in enumerate(hpl.PHASES)}, n_emulated=r.n_emulated,
                          n_launches=r.n_launches, gemm_launches=r.gemm_launches, gemm_kernel_s=r.gemm_kernel_s,
                          gemm_int8_ops=r.gemm_int8_ops, gemm_fp64eq_flops=r.gemm_fp64eq_flops,
                          schedule=r.schedule, x=x)

    def close(self) -> None:
        if self.handle:
            _lib.load().chpl_grid_destroy(self.handle)
            self.handle = None


def init_from_env(timeout_s: float = 600.0):
    """torch.distributed over gloo from torchrun's environment; device = LOCAL_RANK."""
    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if not dist.is_initialized():
        dist.init_process_group("gloo", timeout=timedelta(seconds=timeout_s))
    return dist


def max_over_ranks(v: float) -> float:
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bench(a, workloads, metric, flops, ClockSampler, int8_peak_tops=None, traffic_per_unit=None,
          fp64_peak_tflops=None) -> None:
    """bench.py for N > 1 GPUs (driver contract): weak scaling, max over ranks."""
    import torch
    dist = init_from_env()
    world = dist.get_world_size()
    rank = dist.get_rank()
    P, Q = grid_shape(world)
    if getattr(a, "grid", ""):
        P, Q = (int(v) for v in a.grid.lower().split("x"))
    N, NB = workloads.get(world, (a.N or 65536, a.NB or 2048))[:2]
    if a.N:
        N, NB = a.N, a.NB or NB
    cfg = hpl.Config(N=N, NB=NB, P=P, Q=Q, moduli=a.moduli)
    g = Grid(P, Q)
    for _ in range(a.warmup):
        g.run(cfg)
    dist.barrier()
    torch.cuda.synchronize()
    res = []
    walls = []
    local = int(os.environ.get("LOCAL_RANK", "0"))
    with ClockSampler(local) as clk:
        dist.barrier()
        torch.cuda.synchronize()
        for _ in range(a.steps):
            t0 = time.perf_counter()
            r = g.run(cfg, want_x=True)
            walls.append(time.perf_counter() - t0)
            res.append(r)
        torch.cuda.synchronize()
        dist.barrier()
    solve = max_over_ranks(sum(r.time_s for r in res))
    wall = max_over_ranks(sum(walls))
    gk = sum(r.gemm_kernel_s for r in res)
    ops = sum(r.gemm_int8_ops for r in res)
    nl = sum(r.gemm_launches for r in res)
    launches = sum(r.n_launches for r in res)
    phases = {p: max_over_ranks(sum(r.phases[p] for r in res) / a.steps) for p in hpl.PHASES}
    # time each rank's solve spent outside its int8 GEMM kernel (panel, exchanges, waits for
    # other ranks, interchanges, splits): the largest and smallest over ranks, per step
    outside = (sum(r.time_s for r in res) - gk) / a.steps
    outside_max = max_over_ranks(outside)
    outside_min = -max_over_ranks(-outside)
    tpu = traffic_per_unit() if traffic_per_unit else None
    # the cuBLAS int8 denominator, measured after the solves (whose memory plan wants every free byte),
    # by every rank on its own GPU
    peak_burst, peak = int8_peak_tops(sustained_s=4.0) if int8_peak_tops else (None, None)
    fp64_peak = fp64_peak_tflops() if fp64_peak_tflops else None
    g.close()
    if rank == 0:
        out = {
            "metric": metric, "value": a.steps * flops(N) / solve / 1e12, "unit": "TFLOPS", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": solve / a.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": f"int8 tensor cores (Ozaki-II, {a.moduli} moduli) + fp64",
            "data": "synthetic (chpl SplitMix64 generator, seed 42)",
            "config": {"workload": f"HPL solve N={N} NB={NB} {P}x{Q} grid, {a.moduli} moduli", "N": N, "NB": NB,
                       "grid": f"{P}x{Q}", "parallelism": f"2D block-cyclic P{P}Q{Q}",
                       "schedule": "depth-1 lookahead" if all(r.schedule for r in res) else "serial block steps",
                       "l2": "inputs larger than L2",
                       "timed_region": "factor + back substitution (device events, max over ranks)"},
            "resid": max(r.resid for r in res), "passed": all(r.passed for r in res),
            "phases_s_max_over_ranks": phases,
            "outside_gemm_s_per_step": {"max_over_ranks": outside_max, "min_over_ranks": outside_min,
                                        "note": "solve time minus the rank's own int8 GEMM kernel time"},
            "hpl_roofline": ({"int8_tops_per_gpu": peak, "moduli": a.moduli,
                              "fp64eq_tflops": world * peak / a.moduli,
                              "frac": (a.steps * flops(N) / solve / 1e12) / (world * peak / a.moduli)}
                             if peak else None),
            "roofline": {"bound": "tensor", "achieved": ops / gk / 1e12 if gk else None, "peak": peak,
                         "unit": "TOPS (int8)",
                         "frac": (ops / gk / 1e12 / peak) if (gk and peak) else None,
                         "traffic": (tpu * ops / 2.0 / nl) if (tpu and nl) else None,
                         "kernel": "oz2_gemm_kernel (tcgen05 kind::i8 + fused CRT), rank 0",
                         "peak_source": "cuBLAS int8 GEMM 8192^3 launched back to back for 4 s on rank 0's GPU "
                                        "in this run (the sustained figure, for a kernel timed inside long solves)",
                         "peak_burst": peak_burst,
                         "launches": nl, "avg_launch_ms": gk / nl * 1e3 if nl else None},
            "e2e": {"value": a.steps * flops(N) / wall / 1e12, "unit": "TFLOPS",
                    "h2d_bytes_per_step": ctypes.sizeof(_lib.HplConfig),
                    "d2h_bytes_per_step": N * 8 + ctypes.sizeof(_lib.HplResult),
                    "note": "public API chpl_grid_run per step (wall clock, max over ranks): on-device "
                            "block-cyclic generation of the HPL system, solve, verification, x to the host; "
                            "no host copy of the ranks' local pieces (~144 GB each) is made"},
            "fp64_native": ({"peak_tflops_per_gpu": fp64_peak,
                             "x_peak_per_gpu": a.steps * flops(N) / solve / 1e12 / world / fp64_peak,
                             "source": "cuBLAS DGEMM 8192^3 (torch.matmul float64) on rank 0's GPU, this run"}
                            if fp64_peak else None),
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()
