"""Builds oracle/_ref/ from the reference's own source -- TEST INFRASTRUCTURE ONLY.

The reference (Koyingtw/CHPL) cannot be built as a whole here: its CMake
build needs MPI and the GEMMul8 submodule, which is empty.  Four pieces of it
are self-contained, though, and are what parity of this project's generator,
interchange planning, residual and Ozaki-I engine hangs on.  This recipe cuts them out of the
reference checkout (located by CHPL_REFERENCE_ROOT) by pattern, writes them
verbatim into oracle/_ref/ (git-ignored: reference source never enters this
repository's history) and compiles them with this project's harnesses:

  chpl_elem.inc      src/chpl_p2.cu     chpl_elem: the SplitMix64 generator of
                                        chpl_p2 / chpl_p4
  resolve_seq.inc    src/chpl_p2.cu     resolve_seq: a pivot sequence -> its
                                        net row permutation
  residual.inc       src/chpl_single.cu the scaled-residual reduction of
                                        run_case (norms and the formula)
  single_matgen.inc  src/chpl_single.cu hs_rand + matgen_kernel: chpl_single's
                                        cuRAND Philox generator
  single_oz1.inc     src/chpl_single.cu ozrowscale_kernel .. ozrecon_kernel:
                                        chpl_single's Ozaki-I scales, digit
                                        slices and reconstruction

  oracle/_ref/libref_host.so           g++ on oracle/ref_host.cpp (the first three)
  oracle/_ref/libref_single_matgen.so  nvcc (sm_100a) on oracle/ref_single_matgen.cu
  oracle/_ref/libref_oz1.so            nvcc (sm_100a) on oracle/ref_oz1.cu

oracle/_ref/manifest.json records the file and line range of each fragment.
The built libraries travel with the repository snapshot to a GPU machine
(they are not ignored for that), where the reference checkout is absent.

    python -m oracle.ref_build        # or oracle.build_ref()
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def reference_root() -> str:
    return os.environ.get("CHPL_REFERENCE_ROOT", "/root/reference")


def available() -> bool:
    r = reference_root()
    return all(os.path.exists(os.path.join(r, "src", f)) for f in ("chpl_p2.cu", "chpl_single.cu"))


def _cut(lines: list[str], start: str, end) -> tuple[int, int]:
    """(first, last) 0-based line range: the first line matching `start`, up to
    and including the first line after it for which end(line) holds."""
    s = next((i for i, ln in enumerate(lines) if re.search(start, ln)), None)
    if s is None:
        raise RuntimeError(f"reference fragment not found: {start!r}")
    e = next((i for i in range(s, len(lines)) if end(lines[i])), None)
    if e is None:
        raise RuntimeError(f"end of reference fragment not found after {start!r}")
    return s, e


def _closing_brace(ln: str) -> bool:
    return ln.rstrip("\n") == "}"


# name -> (file, start pattern, end rule)
FRAGMENTS = {
    "chpl_elem.inc": ("src/chpl_p2.cu", r"^__device__ __forceinline__ double chpl_elem\(", _closing_brace),
    "resolve_seq.inc": ("src/chpl_p2.cu", r"^static void resolve_seq\(", _closing_brace),
    "residual.inc": ("src/chpl_single.cu", r"^\s*double resid0 = 0\.0, AnormI",
                     lambda ln: re.search(r"const double resid1 =", ln) is not None),
}


def _extract(root: str) -> dict:
    os.makedirs(OUT, exist_ok=True)
    manifest = {}
    cache: dict[str, list[str]] = {}

    def lines_of(rel):
        if rel not in cache:
            with open(os.path.join(root, rel)) as f:
                cache[rel] = f.readlines()
        return cache[rel]

    def write(name, rel, s, e):
        text = "".join(lines_of(rel)[s:e + 1])
        with open(os.path.join(OUT, name), "w") as f:
            f.write(f"// extracted verbatim from {rel}:{s + 1}-{e + 1} of the reference checkout\n")
            f.write(text)
        manifest[name] = {"file": rel, "lines": [s + 1, e + 1], "sha256": hashlib.sha256(text.encode()).hexdigest()}

    for name, (rel, start, end) in FRAGMENTS.items():
        s, e = _cut(lines_of(rel), start, end)
        write(name, rel, s, e)
    # chpl_single's generator: hs_rand through the end of matgen_kernel
    L = lines_of("src/chpl_single.cu")
    s, _ = _cut(L, r"^__device__ __forceinline__ double hs_rand\(", _closing_brace)
    _, e = _cut(L, r"^__global__ void matgen_kernel\(", _closing_brace)
    write("single_matgen.inc", "src/chpl_single.cu", s, e)
    # chpl_single's Ozaki-I kernels: ozrowscale_kernel through the end of ozrecon_kernel
    s, _ = _cut(L, r"^__global__ void ozrowscale_kernel\(", _closing_brace)
    _, e = _cut(L, r"^__global__ void ozrecon_kernel\(", _closing_brace)
    write("single_oz1.inc", "src/chpl_single.cu", s, e)
    with open(os.path.join(OUT, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return manifest


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"oracle/_ref build step failed: {' '.join(cmd[:4])} ...")


def build(force: bool = False) -> bool:
    """Extract and compile; False (nothing done) when the reference checkout is
    absent, as on a GPU machine, where the libraries built here are used."""
    if not available():
        return False
    host_so = os.path.join(OUT, "libref_host.so")
    dev_so = os.path.join(OUT, "libref_single_matgen.so")
    oz1_so = os.path.join(OUT, "libref_oz1.so")
    deps = [os.path.join(HERE, f) for f in ("ref_build.py", "ref_host.cpp", "ref_single_matgen.cu", "ref_oz1.cu")]
    newest = max(os.path.getmtime(d) for d in deps)
    if not force and all(os.path.exists(p) and os.path.getmtime(p) >= newest for p in (host_so, dev_so, oz1_so)):
        return True
    _extract(reference_root())
    _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-I", OUT,
          os.path.join(HERE, "ref_host.cpp"), "-o", host_so])
    _run([os.path.join(CUDA, "bin", "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
          "-shared", "-Xcompiler", "-fPIC", "-cudart", "shared", "-I", OUT, os.path.join(HERE, "ref_single_matgen.cu"),
          "-o", dev_so])
    _run([os.path.join(CUDA, "bin", "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
          "-shared", "-Xcompiler", "-fPIC", "-cudart", "shared", "-I", OUT, os.path.join(HERE, "ref_oz1.cu"),
          "-o", oz1_so])
    return True


if __name__ == "__main__":
    print("built" if build(force="--force" in sys.argv) else "reference checkout absent: nothing built")
