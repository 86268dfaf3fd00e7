#!/usr/bin/env python
"""bench.py -- HPL FP64-equivalent TFLOPS on B200 (the reference's headline metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl chpl|reference]

One step = one HPL solve (factor + back substitution) of the generated system,
with the matrix generated in HBM before the step's timed region (HPL excludes
generation, src/chpl_single.cu:756-757, src/chpl_p2.cu:965-966).  Workload at
N=1: the single-GPU weak-scale solve (N=139264, NB=1024, 1x1 grid, 11 moduli, ~155 GB).
Multi-GPU runs are weak-scaled to ~155 GB per GPU on the grids 1x2, 2x2, 2x4
(config 4 at 8 GPUs: N=393216, NB=4096, P2Q4).

One JSON line is printed by rank 0.  --impl reference times the CPU baseline
(host FP64 LU, LAPACK dgetrf+dgetrs through OpenBLAS on all host cores) on a
bounded sample of the same generated system.
"""
from __future__ import annotations

import argparse
import csv
import ctypes
import io
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "HPL FP64-equiv TFLOPS (2/3N³+2N²)/t at 1/2/4/8 B200; scaled residual"
# per-GPU-count workloads: (N, NB, P, Q)
WORKLOADS = {
    1: (139264, 1024, 1, 1),
    2: (196608, 4096, 1, 2),
    4: (278528, 4096, 2, 2),
    8: (393216, 4096, 2, 4),
}
CPU_SAMPLE_N = 32768


def flops(N: int) -> float:
    return (2.0 / 3.0) * N ** 3 + 2.0 * N ** 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["chpl", "reference"], default="chpl")
    ap.add_argument("--N", type=int, default=0, help="override the order (profiling / small runs)")
    ap.add_argument("--NB", type=int, default=0)
    ap.add_argument("--moduli", type=int, default=11)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--lookahead", action="store_true", help="SM-reserving depth-1 lookahead (default: serial)")
    ap.add_argument("--grid", default="", help="process grid PxQ for N > 1 GPUs (default: 1x2, 2x2, 2x4)")
    ap.add_argument("--e2e-leg", action="store_true",
                    help="internal: the host-buffer end-to-end leg (run in a child process by the 1-GPU bench)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.p is not None:
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.p.kill()
                self.out, _ = self.p.communicate()

    def summary(self) -> dict:
        rows = [r for r in csv.reader(io.StringIO(getattr(self, "out", "") or "")) if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def f(x):
            try:
                return float(x.strip())
            except ValueError:
                return None
        load = [r for r in rows if (f(r[3]) or 0.0) > 300.0] or rows
        sm = [f(r[1]) for r in load if f(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": f(rows[0][2]),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(load),
                "power_w_max": max((f(r[3]) or 0.0) for r in rows),
                "power_w_median": statistics.median([f(r[3]) or 0.0 for r in load])}


# ----------------------------------------------------------------------------- helpers
def int8_peak_tops(sustained_s: float = 0.0):
    """cuBLAS int8 GEMM (torch._int_mm, 8192^3): the tensor-pipe denominator for
    the int8 kernel (MEASURED_PEAKS.json carries no int8 figure).  Returns the
    burst rate (best of 10 launches) and, when sustained_s > 0, also the rate of
    launches issued back to back for about sustained_s seconds -- the figure
    for a kernel timed inside a long step, as the GEMM inside an HPL solve is."""
    import torch
    n = 8192
    a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
    torch._int_mm(a, b)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 1e30
    for _ in range(10):
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e-3)
    burst = 2.0 * n ** 3 / best / 1e12
    sustained = None
    if sustained_s > 0:
        reps = max(1, int(sustained_s / best))
        e0.record()
        for _ in range(reps):
            torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        sustained = reps * 2.0 * n ** 3 / (e0.elapsed_time(e1) * 1e-3) / 1e12
    del a, b
    torch.cuda.empty_cache()
    return (burst, sustained) if sustained_s > 0 else burst


def fp64_peak_tflops() -> float:
    """Native FP64 rate of this GPU: cuBLAS DGEMM 8192^3 (torch.matmul), best
    of 5 -- the denominator of the "x native FP64 peak" figure."""
    import torch
    n = 8192
    a = torch.rand(n, n, dtype=torch.float64, device="cuda")
    b = torch.rand(n, n, dtype=torch.float64, device="cuda")
    c = a @ b
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 1e30
    for _ in range(5):
        e0.record()
        torch.matmul(a, b, out=c)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e-3)
    del a, b, c
    torch.cuda.empty_cache()
    return 2.0 * n ** 3 / best / 1e12


def measured_peaks() -> dict:
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return {}


def traffic_per_unit():
    """DRAM bytes per int8 multiply-add of the GEMM kernel from the committed
    ncu summary (profiles/oz2_gemm_kernel_m8192_n8192_k4096_L11.json), or None."""
    p = os.path.join(ROOT, "profiles", "oz2_gemm_kernel_m8192_n8192_k4096_L11.json")
    try:
        d = json.load(open(p))
        return d["dram_bytes"] / d["int8_macs"]
    except (OSError, ValueError, KeyError):
        return None


def cpu_baseline(N: int) -> dict:
    """Host FP64 LU (OpenBLAS via scipy) on the same generated system, N x (N+1)."""
    import oracle
    A = oracle.hpl_system_fast(N)
    t0 = time.perf_counter()
    x = oracle.lapack_hpl_solve(A)
    t = time.perf_counter() - t0
    del A
    r = oracle.hpl_residual_from(oracle.hpl_system_fast(N), x) if N <= 40000 else None
    return {"value": flops(N) / t / 1e12, "unit": "TFLOPS", "cores": os.cpu_count(), "kind": "port",
            "sample": f"HPL solve N={N} (same generator, seed 42): LAPACK dgetrf+dgetrs (OpenBLAS, "
                      f"{os.cpu_count()} threads), generation excluded, {t:.1f} s",
            "resid": r}


# ----------------------------------------------------------------------------- host-buffer end-to-end leg
E2E_MARGIN = 16 << 30      # host bytes left free beside the pinned [A|b]
E2E_MAX_STEPS = 2
E2E_WARM_N = 8192


def host_memory_available():
    """Bytes the host can still give this job: MemAvailable, capped by the
    cgroup's remaining limit when there is one (None if unknown)."""
    avail = None
    try:
        with open("/proc/meminfo") as f:
            for ln in f:
                if ln.startswith("MemAvailable:"):
                    avail = int(ln.split()[1]) * 1024
    except (OSError, ValueError):
        pass
    for lim_p, cur_p in (("/sys/fs/cgroup/memory.max", "/sys/fs/cgroup/memory.current"),
                         ("/sys/fs/cgroup/memory/memory.limit_in_bytes", "/sys/fs/cgroup/memory/memory.usage_in_bytes")):
        try:
            with open(lim_p) as f:
                lim = f.read().strip()
            with open(cur_p) as f:
                cur = int(f.read().strip())
        except (OSError, ValueError):
            continue
        if lim != "max" and int(lim) < (1 << 60):
            room = int(lim) - cur
            avail = room if avail is None else min(avail, room)
        break
    return avail


def e2e_order(N: int, NB: int):
    """Order of the host-buffer leg: N when its pinned [A|b] fits in host memory
    with a margin, else the largest multiple of NB that does; (None, why) when
    not even N = 16384 fits."""
    avail = host_memory_available()
    if avail is None:
        return None, "host memory size unknown"
    budget = (avail - E2E_MARGIN) / 1.05
    if N * (N + 1) * 8 <= budget:
        return N, None
    n = int((max(budget, 0.0) / 8.0) ** 0.5) // NB * NB
    why = (f"[A|b] of N={N} needs {N * (N + 1) * 8 / 2**30:.0f} GiB of pinned host memory, "
           f"{avail / 2**30:.0f} GiB available")
    return (n, why) if n >= 16384 else (None, why)


def run_e2e_leg(a) -> None:
    """Child process: chpl_hpl_run_host (the public host-buffer call) per step,
    wall clock; [A|b] in pinned host memory, copied in by the call and x
    copied out.  As in HPL (and the reference, src/chpl_single.cu:756-760) the
    verification is outside the timed region: one more call with verify=1
    after the timed steps reports the residual of the same solve."""
    try:   # if the host runs short of memory, this process is the one to go
        with open("/proc/self/oom_score_adj", "w") as f:
            f.write("1000")
    except OSError:
        pass
    from chpl_b200 import hpl
    N, NB = a.N, a.NB
    cfg = hpl.Config(N=N, NB=NB, moduli=a.moduli)
    t0 = time.perf_counter()
    S = hpl.HostSystem(N)
    S.generate(cfg.seed)
    setup = time.perf_counter() - t0
    wn = min(N, E2E_WARM_N)
    with hpl.HostSystem(wn) as W:       # warm-up at a small order: module load, allocator
        W.generate(cfg.seed)
        hpl.run_host(hpl.Config(N=wn, NB=min(NB, wn), moduli=a.moduli), W, verify=True)
    hpl.run_host(cfg, S, verify=False)  # and one untimed call at the full order (a first one ran ~2 s slower)
    walls, res = [], []
    vcfg = hpl.Config(N=N, NB=NB, moduli=a.moduli, verbose=True)   # prints the copy / intake timeline
    for _ in range(a.steps):
        t = time.perf_counter()
        r = hpl.run_host(vcfg, S, verify=False)
        walls.append(time.perf_counter() - t)
        res.append(r)
    chk = hpl.run_host(cfg, S, verify=True)     # untimed: the residual of this solve against the caller's [A | b]
    S.close()
    print(json.dumps({"value": a.steps * flops(N) / sum(walls) / 1e12, "steps": a.steps, "N": N, "NB": NB,
                      "wall_s": walls, "device_s": [r.time_s for r in res],
                      "resid": chk.resid, "passed": chk.passed,
                      "x_equal_to_timed_steps": all(bool(np.array_equal(chk.x, r.x)) for r in res),
                      "setup_s": setup, "launches": sum(r.n_launches for r in res)}), flush=True)


def e2e_host(a, N: int, NB: int, fallback: dict) -> dict:
    """The e2e figure through chpl_hpl_run_host in a child process (so a host
    that cannot hold the pinned system fails that process only).  Falls back to
    `fallback` (the generated-input public call) with the reason."""
    n, why = e2e_order(N, NB)
    if n is None:
        return dict(fallback, note=fallback["note"] + f"; host-buffer leg skipped: {why}")
    steps = max(1, min(a.steps, E2E_MAX_STEPS))
    cmd = [sys.executable, os.path.abspath(__file__), "--e2e-leg", "--N", str(n), "--NB", str(NB),
           "--moduli", str(a.moduli), "--steps", str(steps)]
    try:
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=1200)
        leg = json.loads(p.stdout.strip().splitlines()[-1]) if p.returncode == 0 and p.stdout.strip() else None
        if leg is not None:   # the last timed call's chunk timeline (intake step, landed / reached ms)
            lines = [ln[len("INGEST: "):] for ln in p.stdout.splitlines() if ln.startswith("INGEST: ")]
            steps0 = [i for i, ln in enumerate(lines) if ln.startswith("step 0 ")]
            leg["ingest"] = lines[steps0[-1]:] if steps0 else lines
        err = None if leg else f"child exited {p.returncode}: {(p.stderr or p.stdout).strip()[-300:]}"
    except (subprocess.TimeoutExpired, ValueError, IndexError) as ex:
        leg, err = None, f"{type(ex).__name__}: {ex}"
    if leg is None:
        return dict(fallback, note=fallback["note"] + f"; host-buffer leg failed: {err}")
    from chpl_b200 import _lib
    nb = n * (n + 1) * 8
    out = {"value": leg["value"], "unit": "TFLOPS", "h2d_bytes_per_step": nb + ctypes.sizeof(_lib.HplConfig),
           "d2h_bytes_per_step": n * 8 + ctypes.sizeof(_lib.HplResult), "steps": leg["steps"], "N": n, "NB": NB,
           "resid": leg["resid"], "passed": leg["passed"], "x_equal_to_timed_steps": leg.get("x_equal_to_timed_steps"),
           "wall_s_per_step": sum(leg["wall_s"]) / len(leg["wall_s"]),
           "device_copy_and_solve_s_per_step": sum(leg["device_s"]) / len(leg["device_s"]),
           "device_copy_and_solve_s": leg["device_s"], "ingest_timeline": leg.get("ingest"),
           "gpu_launches": leg["launches"],
           "note": "public host-buffer call chpl_hpl_run_host per step, wall clock: device allocation, [A|b] "
                   "host->device from pinned memory (streamed in column chunks while the factorization works on "
                   "the columns already present), factor + solve, x device->host; the HPL residual comes from "
                   "one more call with verification after the timed steps (HPL times the solve only); "
                   "warm-up at N=%d and one untimed call at N=%d" % (min(n, E2E_WARM_N), n)}
    if why:
        out["note"] += f"; order reduced from N={N}: {why}"
    return out


# ----------------------------------------------------------------------------- reference arm
def run_reference(a) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    N = a.N or CPU_SAMPLE_N
    times = []
    for i in range(a.warmup + a.steps):
        A = oracle.hpl_system_fast(N)
        t0 = time.perf_counter()
        oracle.lapack_hpl_solve(A)
        t = time.perf_counter() - t0
        if i >= a.warmup:
            times.append(t)
        del A
    tot = sum(times)
    v = a.steps * flops(N) / tot / 1e12
    wl = WORKLOADS.get(a.gpus, WORKLOADS[1])
    print(json.dumps({
        "metric": METRIC, "value": v, "unit": "TFLOPS", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": tot / a.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp64", "data": "synthetic (chpl SplitMix64 generator, seed 42)", "impl": "reference",
        "config": {"workload": f"HPL solve N={wl[0]} NB={wl[1]} {wl[2]}x{wl[3]} (sampled on the host at N={N})",
                   "grid": f"{wl[2]}x{wl[3]}"},
        "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"HPL solve N={N} per step, LAPACK dgetrf+dgetrs (OpenBLAS, "
                                   f"{os.cpu_count()} threads); the reference itself has no CPU path"},
        "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- chpl arm
def run_single(a) -> None:
    import torch

    from chpl_b200 import _lib, hpl
    N, NB = (a.N, a.NB or 1024) if a.N else WORKLOADS[1][:2]
    cfg = hpl.Config(N=N, NB=NB, moduli=a.moduli, lookahead=a.lookahead)
    torch.cuda.set_device(0)
    peak_burst, peak_i8 = int8_peak_tops(sustained_s=4.0)
    fp64_peak = fp64_peak_tflops()
    for _ in range(a.warmup):
        hpl.run(cfg)
    torch.cuda.synchronize()
    res = []
    walls = []
    with ClockSampler(0) as clk:
        torch.cuda.synchronize()
        for _ in range(a.steps):
            t0 = time.perf_counter()
            r = hpl.run(cfg, want_x=True)       # public API: generate, solve, verify, x -> host
            walls.append(time.perf_counter() - t0)
            res.append(r)
        torch.cuda.synchronize()
    solve = sum(r.time_s for r in res)
    value = a.steps * flops(N) / solve / 1e12
    gk = sum(r.gemm_kernel_s for r in res)
    ops = sum(r.gemm_int8_ops for r in res)
    nl = sum(r.gemm_launches for r in res)
    achieved = ops / gk / 1e12 if gk > 0 else None
    tpu = traffic_per_unit()
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak_i8, "unit": "TOPS (int8)",
            "frac": achieved / peak_i8 if achieved else None,
            "traffic": (tpu * ops / 2.0 / nl) if (tpu and nl) else None,
            "kernel": "oz2_gemm_kernel (tcgen05 kind::i8 + fused CRT)",
            "peak_source": "cuBLAS int8 GEMM 8192^3 measured in this run, launched back to back for 4 s (the "
                           "sustained figure: the kernel is timed inside solves of ~14 s under the power cap); "
                           "MEASURED_PEAKS.json has no int8 figure",
            "peak_burst": peak_burst, "frac_of_burst": achieved / peak_burst if achieved else None,
            "launches": nl, "avg_launch_ms": gk / nl * 1e3 if nl else None,
            "fp64eq_tflops_in_kernel": sum(r.gemm_fp64eq_flops for r in res) / gk / 1e12 if gk else None}
    phases = {p: sum(r.phases[p] for r in res) / a.steps for p in hpl.PHASES}
    outside = (solve - gk) / a.steps    # per step: everything the solve did outside the int8 GEMM kernel
    out = {
        "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": solve / a.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"int8 tensor cores (Ozaki-II, {a.moduli} moduli) + fp64",
        "data": "synthetic (chpl SplitMix64 generator, seed 42)",
        "config": {"workload": f"HPL solve N={N} NB={NB} 1x1 grid, {a.moduli} moduli (BASELINE config 3)"
                   if not a.N else f"HPL solve N={N} NB={NB} 1x1 grid, {a.moduli} moduli",
                   "N": N, "NB": NB, "grid": "1x1", "moduli": a.moduli, "lookahead": a.lookahead,
                   "l2": f"inputs larger than L2 ({N * (N + 1) * 8 / 1e9:.1f} GB matrix)",
                   "timed_region": "factor + back substitution per step (device events); generation excluded"},
        "resid": max(r.resid for r in res), "passed": all(r.passed for r in res),
        "phases_s": phases,
        "outside_gemm_s_per_step": outside,
        # the whole solve against the update's roofline: the int8 rate divided by the moduli count
        "hpl_roofline": {"int8_tops": peak_i8, "moduli": a.moduli, "fp64eq_tflops": peak_i8 / a.moduli,
                         "frac": value / (peak_i8 / a.moduli)},
        "roofline": roof,
        # the target "at least 3x the native FP64 peak per GPU", against cuBLAS DGEMM measured in this run
        "fp64_native": {"peak_tflops": fp64_peak, "x_peak": value / fp64_peak,
                        "source": "cuBLAS DGEMM 8192^3 (torch.matmul float64), best of 5, this run"},
        "e2e": None,
        "gpu_launches": sum(r.n_launches for r in res),
        "clocks": clk.summary(),
    }
    generated_e2e = {"value": a.steps * flops(N) / sum(walls) / 1e12, "unit": "TFLOPS",
                     "h2d_bytes_per_step": ctypes.sizeof(_lib.HplConfig),
                     "d2h_bytes_per_step": N * 8 + ctypes.sizeof(_lib.HplResult),
                     "note": "public API chpl_hpl_run per step (wall clock): allocation, on-device generation "
                             "of the HPL system, solve, verification, x to host"}
    out["e2e_generated"] = generated_e2e
    torch.cuda.empty_cache()
    out["e2e"] = e2e_host(a, N, NB, generated_e2e)
    if not a.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(CPU_SAMPLE_N)
    print(json.dumps(out), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
        return
    if a.e2e_leg:
        run_e2e_leg(a)
        return
    if a.gpus == 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        run_single(a)
        return
    from chpl_b200 import grid
    grid.bench(a, WORKLOADS, METRIC, flops, ClockSampler, int8_peak_tops, traffic_per_unit, fp64_peak_tflops)


if __name__ == "__main__":
    main()
