"""Build libchpl.so (and the chpl_single / chpl_p2 executables) in-tree for sm_100a.

    python -m chpl_b200.build [--force] [--verbose]

Objects go to chpl_b200/_build/, the library to chpl_b200/libchpl.so and the
executables to chpl_b200/bin/.  nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
BIN = os.path.join(HERE, "bin")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libchpl.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
                  "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]
LIB_SOURCES = ["capi.cu", "oz2.cu", "oz2_noalloc.cu", "oz1.cu", "fp64.cu", "hpl_kernels.cu", "panel.cu", "hpl_single.cu",
               "hpl_grid.cu", "diag.cu"]
def _nccl_dir() -> str:
    """NCCL bundled with torch (the same library torch.distributed loads), so
    one NCCL lives in the process; falls back to the system copy."""
    try:
        import nvidia.nccl as _n  # noqa: F401
        d = os.path.join(os.path.dirname(list(_n.__path__)[0]), "nccl")
        if os.path.exists(os.path.join(d, "lib", "libnccl.so.2")):
            return d
    except ImportError:
        pass
    return ""


NCCL_DIR = _nccl_dir()
NCCL_INC = ["-I", os.path.join(NCCL_DIR, "include")] if NCCL_DIR else []
NCCL_LINK = (["-L", os.path.join(NCCL_DIR, "lib"), "-l:libnccl.so.2", "-Xlinker", "-rpath," + os.path.join(NCCL_DIR, "lib")]
             if NCCL_DIR else ["-lnccl"])
LINK = ["-cudart", "shared"] + NCCL_LINK + ["-Xlinker", "-rpath," + os.path.join(CUDA, "lib64")]
EXES = {"chpl_single": "chpl_single_main.cpp", "chpl_p2": "chpl_p2_main.cpp"}


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith((".h", ".hpp"))]
    return hs


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:6])} ...")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(BIN, exist_ok=True)
    hdrs = _headers()
    flags = NVFLAGS + NCCL_INC + (extra_flags or [])
    objs = []
    jobs = []
    for src in LIB_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            jobs.append([NVCC] + flags + ["-c", s, "-o", o])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda c: _run(c, verbose), jobs))
    if force or _newer(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + LINK, verbose)
    for exe, src in EXES.items():
        s = os.path.join(CSRC, src)
        out = os.path.join(BIN, exe)
        if os.path.exists(s) and (force or _newer(out, [s, LIB] + hdrs)):
            _run(["g++", "-O2", "-std=c++17", "-I", INCLUDE, s, "-o", out, "-L", HERE, "-lchpl",
                  "-Wl,-rpath,$ORIGIN/..", "-Wl,-rpath," + os.path.join(CUDA, "lib64"),
                  "-I", os.path.join(CUDA, "include"), "-L" + os.path.join(CUDA, "lib64"), "-lcublas", "-lcudart", "-lpthread",
                  "-ldl", "-Wall"], verbose)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
