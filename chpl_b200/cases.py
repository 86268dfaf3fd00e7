"""Single-case runner for timing and profiling (ncu) of the library's kernels.

    python -m chpl_b200.cases gemm --m 32768 --n 32768 --k 4096 --moduli 11 [--reps 3]
    python -m chpl_b200.cases hpl --N 65536 --NB 1024 [--no-lookahead]
    python -m chpl_b200.cases laswp --rows 139264 --cols 65536 --swaps 1024
    python -m chpl_b200.cases panel --m 139264 --n 1024
    python -m chpl_b200.cases dgemm --m 8192 --n 8192 --k 8192   (FP64 DGEMM, beside cuBLAS's)
    python -m chpl_b200.cases trsm --m 139264 --n 1024           (m right-hand sides)
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m chpl_b200.cases grid --N 131072 --NB 2048 --moduli 11 12

Prints one JSON line per case.  Inputs are uniform [-0.5, 0.5) (the
standalone update's distribution), generated on the device.
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch

from . import hpl, oz2


def gemm_case(m: int, n: int, k: int, L: int, reps: int, scaled: bool, sustain: float = 0.0) -> dict:
    g = torch.Generator(device="cuda")
    g.manual_seed(42)
    A = torch.rand(k, m, dtype=torch.float64, device="cuda", generator=g) - 0.5   # column-major m x k
    if scaled:
        u = torch.randint(-20, 21, (m,), device="cuda", generator=g).double()
        A *= torch.exp2(u)[None, :]
    B = torch.rand(n, k, dtype=torch.float64, device="cuda", generator=g) - 0.5   # column-major k x n
    C = torch.rand(n, m, dtype=torch.float64, device="cuda", generator=g) - 0.5   # column-major m x n
    tot, _, _ = oz2.workSize(m, n, k, L)
    work = torch.empty(tot, dtype=torch.uint8, device="cuda")
    best = None
    for _ in range(reps):
        ph = oz2.gemm(oz2.OP_N, oz2.OP_N, m, n, k, -1.0, A, m, B, k, 1.0, C, m, L, True, work, timed=True)
        if best is None or ph[0] + ph[1] < best[0] + best[1]:
            best = ph
    t = best[0] + best[1]
    out = {"case": "gemm", "m": m, "n": n, "k": k, "moduli": L, "split_ms": best[0] * 1e3, "gemm_ms": best[1] * 1e3,
           "fp64eq_tflops": 2.0 * m * n * k / t / 1e12,
           "kernel_int8_tops": 2.0 * m * n * (-(-k // 128) * 128) * L / best[1] / 1e12}
    if sustain > 0:
        # back-to-back updates for `sustain` seconds: the rate under the power cap
        import sys, os
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from bench import ClockSampler
        n_it = max(1, int(sustain / max(t, 1e-4)))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(torch.cuda.current_device()) as clk:
            e0.record()
            for _ in range(n_it):
                oz2.gemm(oz2.OP_N, oz2.OP_N, m, n, k, -1.0, A, m, B, k, 1.0, C, m, L, True, work)
            e1.record()
            torch.cuda.synchronize()
        ts = e0.elapsed_time(e1) * 1e-3
        out["sustained"] = {"iters": n_it, "s": ts, "fp64eq_tflops": n_it * 2.0 * m * n * k / ts / 1e12,
                            "clocks": clk.summary()}
    return out


def fp64_case(what: str, m: int, n: int, k: int, reps: int) -> dict:
    """This library's FP64 DGEMM (m x n x k, C -= A B) or TRSM (n x n unit
    lower against m right-hand sides) beside cuBLAS's on the same operands
    (torch), best of `reps`, CUDA events."""
    from . import _lib
    L = _lib.load()

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        best = 1e30
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1e-3)
        return best

    if what == "dgemm":
        A = torch.rand(k, m, dtype=torch.float64, device="cuda").t()   # column-major m x k
        B = torch.rand(n, k, dtype=torch.float64, device="cuda").t()
        C = torch.rand(n, m, dtype=torch.float64, device="cuda").t()
        t = timed(lambda: _lib.check(L.chpl_dgemm(None, m, n, k, -1.0, A.data_ptr(), m, B.data_ptr(), k, 1.0,
                                                  C.data_ptr(), m), "chpl_dgemm"))
        tc = timed(lambda: C.addmm_(A, B, alpha=-1.0))
        f = 2.0 * m * n * k
        return {"case": "dgemm", "m": m, "n": n, "k": k, "ms": t * 1e3, "tflops": f / t / 1e12,
                "cublas_ms": tc * 1e3, "cublas_tflops": f / tc / 1e12}
    Lm = torch.rand(n, n, dtype=torch.float64, device="cuda") / n     # column-major; unit lower part used
    Bm = torch.rand(m, n, dtype=torch.float64, device="cuda")          # n x m right-hand sides
    t = timed(lambda: _lib.check(L.chpl_dtrsm_llnu(None, n, m, Lm.data_ptr(), n, Bm.data_ptr(), n), "chpl_dtrsm"))
    Lt = torch.tril(Lm.t(), -1) + torch.eye(n, dtype=torch.float64, device="cuda")
    Bt = Bm.t().contiguous()
    tc = timed(lambda: torch.linalg.solve_triangular(Lt, Bt, upper=False, unitriangular=True))
    return {"case": "trsm", "n": n, "nrhs": m, "ms": t * 1e3, "tflops": n * n * m / t / 1e12, "cublas_ms": tc * 1e3}


def panel_case(m: int, n: int, reps: int) -> dict:
    import ctypes

    from . import _lib
    L = _lib.load()
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    A0 = torch.rand(n, m, dtype=torch.float64, device="cuda", generator=g) - 0.5   # column-major m x n
    A = A0.clone()
    piv = torch.zeros(n, dtype=torch.int64, device="cuda")
    info = torch.zeros(1, dtype=torch.int32, device="cuda")
    work = torch.empty(L.chpl_panel_getrf_work_bytes(m, n), dtype=torch.uint8, device="cuda")
    best = 1e30
    for _ in range(reps):
        A.copy_(A0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        _lib.check(L.chpl_panel_getrf_f64(0, m, n, A.data_ptr(), m, piv.data_ptr(), info.data_ptr(), work.data_ptr()),
                   "chpl_panel_getrf_f64")
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e-3)
    fl = m * n * n - n ** 3 / 3.0
    return {"case": "panel", "m": m, "n": n, "ms": best * 1e3, "fp64_tflops": fl / best / 1e12, "info": int(info.item())}


def ingest_case(N: int, NB: int, L: int) -> dict:
    """The same system solved from device-generated input and from pinned host
    memory (the copy streamed in by column chunks): device times, phases and the
    chunk timeline (printed by the library with verbose = 1)."""
    cfg = hpl.Config(N=N, NB=NB, moduli=L)
    a = hpl.run(cfg, want_x=True)
    with hpl.HostSystem(N) as S:
        S.generate(cfg.seed)
        vcfg = hpl.Config(N=N, NB=NB, moduli=L, verbose=True)
        t0 = time.perf_counter()
        b = hpl.run_host(vcfg, S, verify=False)
        wall = time.perf_counter() - t0
    return {"case": "ingest", "N": N, "NB": NB, "moduli": L, "resident_s": a.time_s, "host_s": b.time_s,
            "host_wall_s": wall, "x_equal": bool(np.array_equal(a.x, b.x)),
            "phases_resident": a.phases, "phases_host": b.phases}


def laswp_case(rows: int, cols: int, swaps: int, reps: int) -> dict:
    """Interchanges of `swaps` partial-pivoting rows (ipiv[i] uniform in [i, rows))
    on a rows x cols column-major matrix: plan + apply, as the solver's
    trailing-column interchanges.  Algorithmic bytes: 16 per moved element."""
    import ctypes

    import numpy as np

    from . import _lib
    L = _lib.load()
    rng = np.random.default_rng(1)
    ipiv = np.array([rng.integers(i, rows) for i in range(swaps)], dtype=np.int64)
    perm = np.arange(rows)
    for i, p in enumerate(ipiv):
        perm[i], perm[p] = perm[p], perm[i]
    moved = int(np.count_nonzero(perm != np.arange(rows)))
    A = torch.empty(cols, rows, dtype=torch.float64, device="cuda")
    A.copy_(torch.rand(cols, rows, dtype=torch.float64, device="cuda"))
    dpiv = torch.from_numpy(ipiv).cuda()
    work = torch.empty(L.chpl_laswp_work_bytes(rows, swaps), dtype=torch.uint8, device="cuda")
    best = 1e30
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        _lib.check(L.chpl_laswp(0, A.data_ptr(), rows, cols, 0, swaps, dpiv.data_ptr(), rows, work.data_ptr()),
                   "chpl_laswp")
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e-3)
    gb = 16.0 * moved * cols / 1e9
    return {"case": "laswp", "rows": rows, "cols": cols, "swaps": swaps, "moved_rows": moved, "ms": best * 1e3,
            "algorithmic_gb": gb, "gbs": gb / best}


def grid_case(N: int, NB: int, moduli: list[int], grid_shape: str) -> list[dict]:
    """The scaling-sweep case (N = 131072, NB = 2048 by default) on the job's grid (run under torchrun, one process per
    GPU): one solve per moduli count, with the per-phase device times (max over
    ranks), the time outside the int8 GEMM kernel (max / min over ranks) and
    the residual.  Rank 0 prints one JSON line per solve."""
    from . import grid
    dist = grid.init_from_env()
    world = dist.get_world_size()
    P, Q = grid.grid_shape(world)
    if grid_shape:
        P, Q = (int(v) for v in grid_shape.lower().split("x"))
    g = grid.Grid(P, Q)
    # module loading and NCCL channel set-up on a small system first, so the timed solves run warm
    g.run(hpl.Config(N=4 * NB * max(P, Q), NB=NB, P=P, Q=Q, moduli=moduli[0]))
    out = []
    for L in moduli:
        r = g.run(hpl.Config(N=N, NB=NB, P=P, Q=Q, moduli=L))
        outside = r.time_s - r.gemm_kernel_s
        row = {"case": "grid", "N": N, "NB": NB, "grid": f"{P}x{Q}", "moduli": L,
               "tflops": hpl.flops(N) / grid.max_over_ranks(r.time_s) / 1e12, "resid": r.resid,
               "passed": r.passed, "schedule": "lookahead" if r.schedule else "serial",
               "phases_max_over_ranks": {p: grid.max_over_ranks(v) for p, v in r.phases.items()},
               "phase_meaning": {"panel": "panel factorizations", "laswp": "interchanges incl. the exchange across "
                                 "process rows", "trsm": "U12 incl. its broadcast down the process columns",
                                 "oz2_split": "int8 residues of W", "oz2_gemm": "trailing update (int8 GEMM + CRT)",
                                 "back_solve": "distributed back substitution", "comm": "pivot / inv(L11) / W "
                                 "broadcasts"},
               "gemm_kernel_s_max_over_ranks": grid.max_over_ranks(r.gemm_kernel_s),
               # the reference's exposed-communication measure (src/chpl_p2.cu:1745-1753): wall minus update-busy time
               "outside_gemm_s": {"max": grid.max_over_ranks(outside), "min": -grid.max_over_ranks(-outside)}}
        out.append(row)
        if dist.get_rank() == 0:
            print(json.dumps(row), flush=True)
    g.close()
    dist.barrier()
    dist.destroy_process_group()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, default=32768)
    g.add_argument("--n", type=int, default=32768)
    g.add_argument("--k", type=int, default=4096)
    g.add_argument("--moduli", type=int, default=11)
    g.add_argument("--reps", type=int, default=3)
    g.add_argument("--scaled", action="store_true")
    g.add_argument("--sustain", type=float, default=0.0, help="also run back to back for this many seconds")
    for nm in ("dgemm", "trsm"):
        f = sub.add_parser(nm)
        f.add_argument("--m", type=int, default=8192, help="rows (dgemm) / right-hand sides (trsm)")
        f.add_argument("--n", type=int, default=8192)
        f.add_argument("--k", type=int, default=8192)
        f.add_argument("--reps", type=int, default=5)
    ig = sub.add_parser("ingest", help="host-buffer solve (streamed copy) beside the device-generated one")
    ig.add_argument("--N", type=int, default=139264)
    ig.add_argument("--NB", type=int, default=1024)
    ig.add_argument("--moduli", type=int, default=11)
    pn = sub.add_parser("panel")
    pn.add_argument("--m", type=int, default=65536)
    pn.add_argument("--n", type=int, default=1024)
    pn.add_argument("--reps", type=int, default=3)
    lw = sub.add_parser("laswp")
    lw.add_argument("--rows", type=int, default=139264)
    lw.add_argument("--cols", type=int, default=65536)
    lw.add_argument("--swaps", type=int, default=1024)
    lw.add_argument("--reps", type=int, default=5)
    gr = sub.add_parser("grid")
    gr.add_argument("--N", type=int, default=131072)
    gr.add_argument("--NB", type=int, default=2048)
    gr.add_argument("--moduli", type=int, nargs="+", default=[11, 12])
    gr.add_argument("--grid", default="", help="PxQ (default: 1x1, 1x2, 2x2, 2x4 by rank count)")
    h = sub.add_parser("hpl")
    h.add_argument("--N", type=int, default=16384)
    h.add_argument("--NB", type=int, default=1024)
    h.add_argument("--moduli", type=int, default=11)
    h.add_argument("--no-lookahead", action="store_true")
    h.add_argument("--fp64", action="store_true")
    h.add_argument("--agg", type=int, default=0)
    h.add_argument("--trsm-mode", type=int, default=0)
    h.add_argument("--reserve", type=int, default=-1)
    h.add_argument("--panel-mode", type=int, default=0)
    h.add_argument("--lookahead", action="store_true")
    h.add_argument("--ozaki", action="store_true", help="the Ozaki-I update (emulate = 2)")
    h.add_argument("--chunk", type=int, default=0)
    a = ap.parse_args()
    if a.what == "grid":
        grid_case(a.N, a.NB, a.moduli, a.grid)
        return
    torch.cuda.set_device(0)
    if a.what == "gemm":
        print(json.dumps(gemm_case(a.m, a.n, a.k, a.moduli, a.reps, a.scaled, a.sustain)), flush=True)
    elif a.what in ("dgemm", "trsm"):
        print(json.dumps(fp64_case(a.what, a.m, a.n, a.k, a.reps)), flush=True)
    elif a.what == "panel":
        print(json.dumps(panel_case(a.m, a.n, a.reps)), flush=True)
    elif a.what == "ingest":
        print(json.dumps(ingest_case(a.N, a.NB, a.moduli)), flush=True)
    elif a.what == "laswp":
        print(json.dumps(laswp_case(a.rows, a.cols, a.swaps, a.reps)), flush=True)
    else:
        r = hpl.run(hpl.Config(N=a.N, NB=a.NB, moduli=a.moduli, lookahead=a.lookahead and not a.no_lookahead,
                               emulate=0 if a.fp64 else 2 if a.ozaki else 1, chunk=a.chunk, agg=a.agg, trsm_mode=a.trsm_mode, reserve_sms=a.reserve,
                               panel_mode=a.panel_mode))
        print(json.dumps({"case": "hpl", "N": a.N, "NB": a.NB, "agg": a.agg, "trsm_mode": a.trsm_mode,
                          "lookahead": a.lookahead, "reserve": a.reserve, "ozaki": a.ozaki, "tflops": r.tflops, "time_s": r.time_s,
                          "resid": r.resid, "passed": r.passed, "phases": r.phases,
                          "gemm_int8_tops": r.gemm_int8_ops / r.gemm_kernel_s / 1e12 if r.gemm_kernel_s else None,
                          "gemm_launches": r.gemm_launches}), flush=True)


if __name__ == "__main__":
    main()
