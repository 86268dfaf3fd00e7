"""Launcher with the command line of the reference's scripts/mpirun_chpl, without MPI.

    python -m chpl_b200.launch -P <P> -Q <Q> (-N <N> [--NB <NB>] | -i <HPL.dat>) [--dry-run]

The grid picks the executable (scripts/mpirun_chpl:54-63): P = Q = 1 runs
``chpl_single N``; the grids of this build (P <= 2: 1x2, 1x4, 1x8, 2x1, 2x2,
2x4) run ``chpl_p2 <HPL.dat>`` with one process per GPU, started by
torchrun instead of mpirun (there is no MPI on a B200 box; chpl_p2 takes its
rank from torchrun's environment).  P = 4 is the reference's multi-node
chpl_p4, which this build does not have.

With -N the launcher writes a temporary 13-line HPL.dat (NB 4096 by default;
1024 for one GPU), as scripts/mpirun_chpl:84-104 does; with -i it reads N and
NB from the file (one GPU) or passes a copy whose P and Q lines carry -P and
-Q (grids).  Tuned defaults are exported only where the variable is unset
(scripts/mpirun_chpl:107-126), but they are this build's values, not the
ones the reference tuned for GEMMul8 on H200:

* one GPU: HPLS_NB 1024, HPLS_AGG 6 from N = 131072 up, 4 from 65536 and 1
  below (the residual margin of 11 moduli), HPLS_BACKEND gemmul8, HPLS_G8_MODULI 11,
  HPLS_G8_FAST 1, HPLS_G8_CHUNK 32768;
* grids: CHPL2D_G8 1, CHPL2D_G8_MODULI 11, CHPL2D_G8_FAST 1.

The reference's other knobs (CHPL2D_WCH, CHPL2D_PRESEL, CHPL2D_WS,
CHPL2D_XT, NCCL channel counts) steer machinery this build replaces and are
not set.  Environment: CHPL_BIN_DIR (directory of the executables, default
chpl_b200/bin), CHPL_LAUNCH_OPTS (extra torchrun options).
"""
from __future__ import annotations

import argparse
import os
import shlex
import socket
import subprocess
import sys
import tempfile

from . import hpl

HERE = os.path.dirname(os.path.abspath(__file__))
GRIDS = {(1, 2), (1, 4), (1, 8), (2, 1), (2, 2), (2, 4)}


class LaunchError(Exception):
    pass


def _parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="python -m chpl_b200.launch",
                                 description="Run chpl_single / chpl_p2 on a P x Q grid (no MPI).")
    ap.add_argument("-P", type=int, required=True, help="process rows (1 or 2)")
    ap.add_argument("-Q", type=int, required=True, help="process columns")
    ap.add_argument("-N", type=int, default=None, help="global matrix order")
    ap.add_argument("--NB", "-NB", type=int, default=None, help="block size (4096; 1024 for one GPU)")
    ap.add_argument("-i", dest="input", default=None, help="HPL.dat-style input (N, NB, threshold)")
    ap.add_argument("--dry-run", action="store_true", help="print the environment and command, run nothing")
    return ap


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def plan(P: int, Q: int, N: int | None, NB: int | None, input_path: str | None, env: dict) -> dict:
    """What to run: {"exe", "args", "env" (the exported defaults), "dat" (grid input text or None)}.
    Raises LaunchError on a request this build cannot serve."""
    if N is not None and input_path is not None:
        raise LaunchError("use either -N or -i, not both")
    bin_dir = env.get("CHPL_BIN_DIR") or os.path.join(HERE, "bin")
    if N is None and input_path is None:
        input_path = os.path.join(bin_dir, "HPL.dat")
    if input_path is not None and not os.path.isfile(input_path):
        raise LaunchError(f"input file not found: {input_path}")
    if P == 4:
        raise LaunchError("P=4 is the reference's multi-node chpl_p4, which this build does not have")
    exported: dict[str, str] = {}

    def default(name: str, value) -> None:
        if not env.get(name):
            exported[name] = str(value)

    if (P, Q) == (1, 1):
        if input_path is not None:
            dat = hpl.read_hpl_dat(input_path)
            N, NB = dat.N, dat.NB
        NB = NB or int(env.get("HPLS_NB") or 1024)
        if N is None or N <= 0 or NB <= 0 or NB > N:
            raise LaunchError(f"bad N/NB ({N}, {NB})")
        exported["HPLS_NB"] = str(NB)
        # the library's automatic depth (k = 6144 from N = 131072, 4096 from 65536)
        default("HPLS_AGG", max(1, (6144 if N >= 131072 else 4096) // NB) if N >= 65536 else 1)
        default("HPLS_BACKEND", "gemmul8")
        default("HPLS_G8_MODULI", 11)
        default("HPLS_G8_FAST", 1)
        default("HPLS_G8_CHUNK", 32768)
        return {"exe": os.path.join(bin_dir, "chpl_single"), "args": [str(N)], "env": exported, "dat": None,
                "nproc": 1}
    if (P, Q) not in GRIDS:
        raise LaunchError(f"grid {P}x{Q} is not one of this build's grids (1x1, "
                          + ", ".join(f"{p}x{q}" for p, q in sorted(GRIDS)) + ")")
    if input_path is not None:
        d = hpl.read_hpl_dat(input_path)
        N, NB, thr = d.N, d.NB, d.threshold
    else:
        NB, thr = NB or 4096, 16.0
    if N is None or N <= 0 or NB <= 0:
        raise LaunchError(f"bad N/NB ({N}, {NB})")
    default("CHPL2D_G8", 1)
    default("CHPL2D_G8_MODULI", 11)
    default("CHPL2D_G8_FAST", 1)
    with tempfile.NamedTemporaryFile("r", suffix=".dat") as t:
        hpl.write_hpl_dat(t.name, N, NB, P, Q, thr)
        text = t.read()
    return {"exe": os.path.join(bin_dir, "chpl_p2"), "args": [], "env": exported, "dat": text, "nproc": P * Q}


def command(pl: dict, dat_path: str | None, env: dict) -> list[str]:
    if pl["nproc"] == 1:
        return [pl["exe"]] + pl["args"]
    extra = shlex.split(env.get("CHPL_LAUNCH_OPTS", ""))
    return ([sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(pl["nproc"]),
             "--master-addr", "127.0.0.1", "--master-port", str(_free_port())] + extra
            + ["--no-python", pl["exe"], dat_path or "HPL.dat"])


def main(argv=None) -> int:
    a = _parser().parse_args(argv)
    env = dict(os.environ)
    try:
        pl = plan(a.P, a.Q, a.N, a.NB, a.input, env)
    except LaunchError as e:
        print(f"chpl_b200.launch: {e}", file=sys.stderr)
        return 1
    if not a.dry_run and not os.access(pl["exe"], os.X_OK):
        print(f"chpl_b200.launch: executable not found: {pl['exe']} (python -m chpl_b200.build)", file=sys.stderr)
        return 1
    env.update(pl["env"])
    if pl["dat"] is None:
        cmd = command(pl, None, env)
        if a.dry_run:
            for k in sorted(v for v in env if v.startswith("HPLS_")):
                print(f"{k}={env[k]}")
            print(" ".join(cmd))
            return 0
        os.execve(cmd[0], cmd, env)
    with tempfile.NamedTemporaryFile("w", prefix="chpl_HPL.", suffix=".dat", delete=False) as f:
        f.write(pl["dat"])
        dat_path = f.name
    try:
        cmd = command(pl, dat_path, env)
        if a.dry_run:
            for k in sorted(v for v in env if v.startswith(("CHPL2D_", "NCCL_"))):
                print(f"{k}={env[k]}")
            print(" ".join(cmd))
            sys.stdout.write(pl["dat"])
            return 0
        return subprocess.call(cmd, env=env)
    finally:
        os.unlink(dat_path)


if __name__ == "__main__":
    sys.exit(main())
