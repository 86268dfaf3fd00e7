"""CPU checks of the C ABI: libchpl.so loads and exports every function that
include/chpl.h declares (no GPU work is issued)."""
import ctypes
import os
import re
import subprocess

import pytest

from chpl_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header: str) -> list[str]:
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(chpl_[a-z0-9_]+)\s*\(", text)))


def test_library_present_and_loads():
    assert os.path.exists(_lib.LIB_PATH), "build the library first (python -m chpl_b200.build)"
    _lib.load()


def test_every_declared_symbol_is_exported():
    names = _declared("chpl.h")
    assert len(names) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (chpl_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for n in names:
        assert getattr(lib, n) is not None


def test_bindings_cover_header():
    assert sorted(_lib.SIGNATURES) == _declared("chpl.h")


def test_host_only_entry_points():
    """Entry points that need no device: version, error string, sizes."""
    L = _lib.load()
    assert b"sm_100a" in L.chpl_version()
    assert L.chpl_last_error_string() is not None
    tot, wa, wb = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    assert L.chpl_oz2_worksize(1000, 2000, 512, 11, 1, 0, ctypes.byref(tot), ctypes.byref(wa), ctypes.byref(wb)) == 0
    # A part: shifts + 11 planes of 1024 x 512 int8; B part: 11 planes of 2048 x 512
    assert wa.value >= 11 * 1024 * 512 and wb.value >= 11 * 2048 * 512
    assert tot.value >= wa.value + wb.value
    assert L.chpl_oz2_worksize(10, 10, 10, 1, 0, 0, ctypes.byref(tot), None, None) == _lib.CHPL_ERR_INVALID
    assert L.chpl_oz2_worksize(10, 10, 131072, 11, 0, 0, ctypes.byref(tot), None, None) == _lib.CHPL_ERR_UNSUPPORTED
    a, b = ctypes.c_int(), ctypes.c_int()
    assert L.chpl_oz2_shift_bits(11, 4096, ctypes.byref(a), ctypes.byref(b)) == 0
    assert (a.value, b.value) == (43, 43)
    assert L.chpl_laswp_work_bytes(1000, 1024) >= 2 * 1024 * 8
    # Ozaki-I: digits of A (1024 x 6k) and B (6 planes of 512 x 6k), six int32 products of m x n
    w = ctypes.c_size_t()
    assert L.chpl_oz1_worksize(1000, 300, 4096, ctypes.byref(w)) == 0
    assert w.value >= 1024 * 6 * 4096 + 6 * 512 * 6 * 4096 + 6 * 1000 * 300 * 4
    assert L.chpl_oz1_worksize(64, 64, 21845, ctypes.byref(w)) == 0
    assert L.chpl_oz1_worksize(64, 64, 21846, ctypes.byref(w)) == _lib.CHPL_ERR_UNSUPPORTED
    assert L.chpl_oz1_worksize(64, 64, 64, None) == _lib.CHPL_ERR_INVALID


def test_shift_bits_agree_with_oracle():
    import oracle
    L = _lib.load()
    for nm in range(2, 17):
        a, b = ctypes.c_int(), ctypes.c_int()
        assert L.chpl_oz2_shift_bits(nm, 1000, ctypes.byref(a), ctypes.byref(b)) == 0
        assert (a.value, b.value) == oracle.oz2_shift_bits(nm, 1000)


def test_gemm_entry_points_validate_before_early_return():
    """A bad moduli count or k is an error even when there is nothing to
    compute (m, n or k zero); these checks run before any CUDA call."""
    L = _lib.load()
    a, b = ctypes.c_double(1.0), ctypes.c_double(1.0)
    for m, n, k in ((4, 4, 0), (0, 4, 4), (4, 0, 4)):
        rc = L.chpl_oz2_gemm(None, 0, 0, m, n, k, ctypes.byref(a), None, 4, None, 4, ctypes.byref(b), None, 4, 1, 1,
                             None, None, None, 0, 0, 0, 0, None)
        assert rc == _lib.CHPL_ERR_INVALID, (m, n, k)
        rc = L.chpl_oz2_gemm_noalloc(None, 0, 0, m, n, k, ctypes.byref(a), None, 4, None, 4, ctypes.byref(b), None, 4,
                                     17)
        assert rc == _lib.CHPL_ERR_INVALID, (m, n, k)
    rc = L.chpl_oz2_gemm(None, 0, 0, 4, 4, 131072, ctypes.byref(a), None, 4, None, 131072, ctypes.byref(b), None, 4, 11,
                         1, None, None, None, 0, 0, 0, 0, None)
    assert rc == _lib.CHPL_ERR_UNSUPPORTED
    # Ozaki-I: leading dimensions and NULL matrices are checked before any CUDA call
    assert L.chpl_oz1_gemm(None, 8, 8, 8, -1.0, None, 4, None, 8, 1.0, None, 8, None) == _lib.CHPL_ERR_INVALID
    assert L.chpl_oz1_gemm(None, 8, 8, 8, -1.0, None, 8, None, 8, 1.0, None, 8, None) == _lib.CHPL_ERR_INVALID


def test_default_config():
    L = _lib.load()
    c = _lib.HplConfig()
    L.chpl_hpl_default_config(ctypes.byref(c))
    assert (c.N, c.NB, c.P, c.Q, c.moduli, c.emulate, c.fast, c.seed) == (16384, 1024, 1, 1, 11, 1, 1, 42)
    assert c.threshold == 16.0


def test_invalid_config_rejected_without_gpu():
    L = _lib.load()
    c = _lib.HplConfig()
    L.chpl_hpl_default_config(ctypes.byref(c))
    c.N = -5
    r = _lib.HplResult()
    assert L.chpl_hpl_run(ctypes.byref(c), ctypes.byref(r), None) == _lib.CHPL_ERR_INVALID
    assert b"N" in L.chpl_last_error_string()


def test_host_entry_points_reject_bad_arguments_without_gpu():
    """Argument checks of the host-buffer entry points run before any CUDA call."""
    L = _lib.load()
    c = _lib.HplConfig()
    L.chpl_hpl_default_config(ctypes.byref(c))
    c.N = 100
    r = _lib.HplResult()
    assert L.chpl_hpl_run_host(ctypes.byref(c), None, 100, 1, ctypes.byref(r), None) == _lib.CHPL_ERR_INVALID
    buf = (ctypes.c_double * 16)()
    assert L.chpl_hpl_run_host(ctypes.byref(c), buf, 99, 1, ctypes.byref(r), None) == _lib.CHPL_ERR_INVALID
    assert b"ldab" in L.chpl_last_error_string()
    assert L.chpl_matgen_host(0, 42, buf, 1) == _lib.CHPL_ERR_INVALID
    assert L.chpl_matgen_host(10, 42, buf, 9) == _lib.CHPL_ERR_INVALID
    p = ctypes.c_void_p()
    assert L.chpl_host_alloc(0, ctypes.byref(p)) == _lib.CHPL_ERR_INVALID
    assert L.chpl_host_free(None) == _lib.CHPL_OK
    res = ctypes.c_double()
    assert L.chpl_residual_matrix(None, 10, None, 10, None, ctypes.byref(res)) == _lib.CHPL_ERR_INVALID


def test_header_is_plain_c_and_links(tmp_path):
    """include/chpl.h compiles as C99 (no C++ in the ABI) and a C program links
    against libchpl.so and calls its host-only entry points."""
    src = tmp_path / "abi.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "chpl.h"
int main(void) {
    chpl_hpl_config c;
    chpl_hpl_result r;
    size_t tot = 0, wa = 0, wb = 0;
    int a = 0, b = 0;
    chpl_hpl_default_config(&c);
    if (c.N != 16384 || c.NB != 1024 || c.moduli != 11) return 2;
    if (chpl_oz2_worksize(4096, 4096, 4096, 11, 1, 0, &tot, &wa, &wb) != CHPL_OK || tot < wa + wb) return 3;
    if (chpl_oz2_shift_bits(11, 4096, &a, &b) != CHPL_OK || a != 43 || b != 43) return 4;
    c.N = -1;
    if (chpl_hpl_run(&c, &r, NULL) != CHPL_ERR_INVALID) return 5;
    if (strstr(chpl_version(), "sm_100a") == NULL) return 6;
    printf("ok %s\n", chpl_version());
    return 0;
}
''')
    exe = tmp_path / "abi"
    libdir = os.path.dirname(_lib.LIB_PATH)
    cc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                         "-o", str(exe), "-L", libdir, "-lchpl", f"-Wl,-rpath,{libdir}"],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.startswith("ok"), (run.returncode, run.stdout, run.stderr)


def test_host_buffer_api_fails_loudly_without_a_gpu():
    """No silent host fallback: without a device the pinned allocation and the
    host-buffer solve raise ChplError (CUDA error), never compute on the CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import numpy as np
    from chpl_b200 import hpl
    with pytest.raises(_lib.ChplError):
        hpl.HostSystem(64)
    Ab = np.zeros((65, 64))
    with pytest.raises(_lib.ChplError):
        hpl.run_host(hpl.Config(N=64, NB=16), Ab)
