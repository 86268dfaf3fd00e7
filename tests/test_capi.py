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


def test_shift_bits_agree_with_oracle():
    import oracle
    L = _lib.load()
    for nm in range(2, 17):
        a, b = ctypes.c_int(), ctypes.c_int()
        assert L.chpl_oz2_shift_bits(nm, 1000, ctypes.byref(a), ctypes.byref(b)) == 0
        assert (a.value, b.value) == oracle.oz2_shift_bits(nm, 1000)


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
