"""HPL solver front end: HPL.dat / environment configuration and runs.

Configuration sources, as in the reference:
  * HPL.dat lines 6 (N), 8 (NB) and 13 (threshold), with the fallback
    N=16384, NB=1024, 16.0 when the file has fewer than 13 lines
    (src/chpl_p2.cu:570-584); lines 11/12 give P and Q.
  * chpl_single: ``HPLS_NB HPLS_AGG HPLS_BACKEND HPLS_SEED HPLS_G8_MODULI
    HPLS_G8_FAST HPLS_G8_CHUNK HPLS_OZ_NT`` (src/chpl_single.cu:842-869).
  * chpl_p2 / grid: ``CHPL2D_G8 CHPL2D_G8_MODULI CHPL2D_G8_FAST CHPL2D_G8_NT``
    (src/chpl_p2.cu:685-691) with the launcher defaults of
    scripts/mpirun_chpl:107-126 (G8=1, 11 moduli, fast).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

from . import _lib


@dataclass
class HplDat:
    N: int = 16384
    NB: int = 1024
    threshold: float = 16.0
    P: int = 1
    Q: int = 1


def read_hpl_dat(path: str) -> HplDat:
    """Parse the fields CHPL reads from an HPL.dat file."""
    d = HplDat()
    try:
        with open(path) as f:
            lines = f.readlines()
    except OSError:
        return d
    if len(lines) > 12:
        first = [ln.split()[0] if ln.split() else "0" for ln in lines]
        d.N = int(first[5])
        d.NB = int(first[7])
        d.threshold = float(first[12])
        try:
            d.P = int(first[10])
            d.Q = int(first[11])
        except ValueError:
            pass
    return d


def write_hpl_dat(path: str, N: int, NB: int, P: int = 1, Q: int = 1, threshold: float = 16.0) -> None:
    """Standard 13-line HPL input (layout of scripts/HPL.dat, scripts/mpirun_chpl:84-104)."""
    with open(path, "w") as f:
        f.write("HPLinpack benchmark input file\n"
                "Innovative Computing Laboratory, University of Tennessee\n"
                "HPL.out      output file name (if any)\n"
                "6            device out (6=stdout,7=stderr,file)\n"
                "1            # of problems sizes (N)\n"
                f"{N:<12d} Ns\n"
                "1            # of NBs\n"
                f"{NB:<12d} NBs\n"
                "0            PMAP process mapping (0=Row-,1=Column-major)\n"
                "1            # of process grids (P x Q)\n"
                f"{P:<12d} Ps\n"
                f"{Q:<12d} Qs\n"
                f"{threshold:<12.1f} threshold\n")


def _env_int(env, name: str, default: int) -> int:
    v = env.get(name)
    return int(v) if v not in (None, "") else default


@dataclass
class Config:
    N: int = 16384
    NB: int = 1024
    P: int = 1
    Q: int = 1
    moduli: int = 11
    emulate: int = 1        # 0: FP64 update, 1: Ozaki-II, 2: Ozaki-I (one GPU only)
    fast: bool = True
    chunk: int = 0
    lookahead: bool = False
    agg: int = 0
    reserve_sms: int = -1
    trsm_mode: int = 0
    panel_mode: int = 0
    seed: int = 42
    threshold: float = 16.0
    verbose: bool = False
    generator: int = _lib.CHPL_GEN_CHPL    # CHPL_GEN_PHILOX: chpl_single's cuRAND Philox matrix

    def to_c(self) -> _lib.HplConfig:
        c = _lib.HplConfig()
        c.N, c.NB, c.P, c.Q = self.N, self.NB, self.P, self.Q
        c.moduli, c.emulate, c.fast, c.chunk = self.moduli, int(self.emulate), int(self.fast), self.chunk
        c.lookahead, c.seed, c.threshold, c.verbose = int(self.lookahead), self.seed, self.threshold, int(self.verbose)
        c.agg, c.reserve_sms, c.trsm_mode, c.panel_mode = self.agg, self.reserve_sms, self.trsm_mode, self.panel_mode
        c.generator = self.generator
        return c


def single_config_from_env(N: int, env=None) -> Config:
    """chpl_single's configuration (src/chpl_single.cu:842-869, launcher defaults
    scripts/mpirun_chpl:71-76).  HPLS_AGG groups panels into super-blocks whose
    trailing update runs with k = AGG * NB (0 = automatic: k = 6144 from
    N = 131072 up, 4096 from 65536, k = NB below, where deeper emulated
    updates cost residual margin).  The matrix is chpl_single's cuRAND Philox one
    (src/chpl_single.cu:73-80); HPLS_GEN=chpl (this build's switch) selects
    chpl_p2's SplitMix64 matrix instead."""
    env = os.environ if env is None else env
    backend = env.get("HPLS_BACKEND", "gemmul8")
    if backend not in ("native", "gemmul8", "ozaki"):
        raise ValueError(f"unknown HPLS_BACKEND '{backend}'")
    gen = env.get("HPLS_GEN", "philox")
    if gen not in ("philox", "chpl"):
        raise ValueError(f"unknown HPLS_GEN '{gen}'")
    c = Config(N=N, NB=_env_int(env, "HPLS_NB", 1024), moduli=_env_int(env, "HPLS_G8_MODULI", 11),
               emulate={"native": 0, "gemmul8": 1, "ozaki": 2}[backend], fast=bool(_env_int(env, "HPLS_G8_FAST", 1)),
               chunk=_env_int(env, "HPLS_OZ_NT" if backend == "ozaki" else "HPLS_G8_CHUNK", 0),
               seed=_env_int(env, "HPLS_SEED", 42),
               lookahead=bool(_env_int(env, "HPLS_LOOKAHEAD", 0)), agg=_env_int(env, "HPLS_AGG", 0),
               generator=_lib.CHPL_GEN_PHILOX if gen == "philox" else _lib.CHPL_GEN_CHPL)
    if c.N <= 0 or c.NB <= 0 or c.NB > c.N:
        raise ValueError("bad N/NB")
    return c


def grid_config_from_env(dat: HplDat, P: int, Q: int, env=None) -> Config:
    """chpl_p2's configuration: HPL.dat + CHPL2D_* switches (src/chpl_p2.cu:685-691)."""
    env = os.environ if env is None else env
    return Config(N=dat.N, NB=dat.NB, P=P, Q=Q, threshold=dat.threshold,
                  emulate=bool(_env_int(env, "CHPL2D_G8", 1)), moduli=_env_int(env, "CHPL2D_G8_MODULI", 11),
                  fast=bool(_env_int(env, "CHPL2D_G8_FAST", 1)), chunk=_env_int(env, "CHPL2D_G8_NT", 0),
                  lookahead=bool(_env_int(env, "CHPL2D_LOOKAHEAD", 0)))


@dataclass
class Result:
    N: int
    NB: int
    P: int
    Q: int
    time_s: float
    tflops: float
    resid: float
    passed: bool
    threshold: float
    matgen_s: float
    phases: dict = field(default_factory=dict)
    n_emulated: int = 0
    n_launches: int = 0
    gemm_launches: int = 0
    gemm_kernel_s: float = 0.0
    gemm_int8_ops: float = 0.0
    gemm_fp64eq_flops: float = 0.0
    schedule: int = 0
    x: np.ndarray | None = None


PHASES = ["panel", "laswp", "trsm", "oz2_split", "oz2_gemm", "update_fp64", "back_solve", "comm"]


def flops(N: int) -> float:
    """Operation count of the benchmark metric, 2/3 N^3 + 2 N^2 (the reference prints 3/2 N^2,
    src/chpl_p2.cu:1883)."""
    return (2.0 / 3.0) * N ** 3 + 2.0 * N ** 2


def run(cfg: Config, want_x: bool = False) -> Result:
    """One solve on the current CUDA device (P = Q = 1)."""
    L = _lib.load()
    c = cfg.to_c()
    r = _lib.HplResult()
    x = np.empty(cfg.N, dtype=np.float64) if want_x else None
    xp = x.ctypes.data if want_x else None
    _lib.check(L.chpl_hpl_run(ctypes.byref(c), ctypes.byref(r), xp), "chpl_hpl_run")
    return _result(cfg, r, x)


def _result(cfg: Config, r, x) -> Result:
    return Result(N=cfg.N, NB=cfg.NB, P=cfg.P, Q=cfg.Q, time_s=r.time_s, tflops=r.tflops, resid=r.resid,
                  passed=bool(r.passed), threshold=cfg.threshold, matgen_s=r.matgen_s,
                  phases={p: r.phase_s[i] for i, p in enumerate(PHASES)}, n_emulated=r.n_emulated,
                  n_launches=r.n_launches, gemm_launches=r.gemm_launches, gemm_kernel_s=r.gemm_kernel_s,
                  gemm_int8_ops=r.gemm_int8_ops, gemm_fp64eq_flops=r.gemm_fp64eq_flops, x=x)


class HostSystem:
    """[A | b] (N x (N+1), column-major) in page-locked host memory
    (chpl_host_alloc); ``array`` is a numpy view of shape (N+1, N): row j of
    the view is column j of the system."""

    def __init__(self, N: int):
        L = _lib.load()
        self.N = N
        self.ld = N
        self.nbytes = N * (N + 1) * 8
        p = ctypes.c_void_p()
        _lib.check(L.chpl_host_alloc(self.nbytes, ctypes.byref(p)), "chpl_host_alloc")
        self.ptr = p.value
        buf = (ctypes.c_double * (N * (N + 1))).from_address(self.ptr)
        self.array = np.frombuffer(buf, dtype=np.float64).reshape(N + 1, N)

    def generate(self, seed: int = 42) -> None:
        """The generated system of ``run`` (same elements), produced on the device."""
        _lib.check(_lib.load().chpl_matgen_host(self.N, seed, self.ptr, self.ld), "chpl_matgen_host")

    def close(self) -> None:
        if self.ptr:
            self.array = None
            _lib.load().chpl_host_free(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def run_host(cfg: Config, Ab, ldab: int | None = None, verify: bool = True, want_x: bool = True) -> Result:
    """One solve of a caller-supplied system read from host memory (P = Q = 1).

    ``Ab`` is a HostSystem, a numpy array holding [A | b] column-major (shape
    (N+1, ldab) C-contiguous, or (ldab, N+1) Fortran-ordered), or a raw host
    address with ``ldab`` given.  ``cfg.seed`` is not used."""
    L = _lib.load()
    if isinstance(Ab, HostSystem):
        ptr, ld = Ab.ptr, Ab.ld
    elif isinstance(Ab, np.ndarray):
        if Ab.dtype != np.float64:
            raise TypeError("Ab must be float64")
        if Ab.flags.c_contiguous and Ab.shape[0] == cfg.N + 1:
            ld = Ab.shape[1]
        elif Ab.flags.f_contiguous and Ab.ndim == 2 and Ab.shape[1] == cfg.N + 1:
            ld = Ab.shape[0]
        else:
            raise ValueError("Ab must hold the N+1 columns of [A | b] contiguously, column-major")
        ptr = Ab.ctypes.data
    else:
        if ldab is None:
            raise ValueError("ldab is required with a raw address")
        ptr, ld = int(Ab), ldab
    c = cfg.to_c()
    r = _lib.HplResult()
    x = np.empty(cfg.N, dtype=np.float64) if want_x else None
    _lib.check(L.chpl_hpl_run_host(ctypes.byref(c), ptr, ld if ldab is None else ldab, int(verify), ctypes.byref(r),
                                   x.ctypes.data if want_x else None), "chpl_hpl_run_host")
    return _result(cfg, r, x)


def format_single(res: Result, cfg: Config) -> str:
    """HPL-style report of chpl_single (src/chpl_single.cu:806-834)."""
    tag = "HPLS_" + ("native", "gemmul8", "ozaki")[int(cfg.emulate)]
    lines = ["=" * 58,
             "T/V                   N    NB   AGG      K           Time                 Gflops",
             "-" * 58,
             f"{tag:<16s}{res.N:8d} {res.NB:5d} {1:5d} {res.NB:6d} {res.time_s:14.2f}     {res.tflops * 1e3:18.4e}",
             "-" * 58,
             f"||Ax-b||_oo/(eps*(||A||_oo*||x||_oo+||b||_oo)*N)= {res.resid:13.7f} ...... "
             f"{'PASSED' if res.passed else 'FAILED'}",
             "-" * 58, "PHASE              sec     %wall"]
    for p in PHASES:
        v = res.phases.get(p, 0.0)
        lines.append(f"{p:<14s}{v:9.3f}   {100.0 * v / max(res.time_s, 1e-30):6.2f}%")
    if int(cfg.emulate) == 2:
        lines.append(f"wide_gemm calls: ozaki={res.n_emulated} (slices=6)")
    else:
        lines.append(f"wide_gemm calls: gemmul8={res.n_emulated} (moduli={cfg.moduli} fast={int(cfg.fast)})")
    lines.append("=" * 58)
    return "\n".join(lines)


def format_grid(res: Result) -> str:
    """HPL-style report of chpl_p2 (src/chpl_p2.cu:1938-1947)."""
    g = res.tflops * 1e3
    return "\n".join([
        "=" * 80,
        "T/V                N    NB     P     Q         Time          Gflops (   per GPU)",
        "-" * 80,
        f"{'WC2':<4s}{res.N:16d} {res.NB:5d} {res.P:5d} {res.Q:5d} {res.time_s:12.2f} {g:15.3e} "
        f"({g / (res.P * res.Q):10.3e})",
        "-" * 80,
        f"||Ax-b||_oo/(eps*(||A||_oo*||x||_oo+||b||_oo)*N)= {res.resid:16.12f} ...... "
        f"{'PASSED' if res.passed else 'FAILED'}"])
