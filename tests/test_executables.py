"""The drop-in executables chpl_single and chpl_p2 (C++ over the C ABI).

CPU: they are built and their argument / environment errors exit before any
device work, with the reference's usage text and exit status
(src/chpl_single.cu:950-965).  GPU: a solve through each executable prints
the reference's report lines and PASSED; the GEMM self-check passes.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "chpl_b200", "bin")
SINGLE = os.path.join(BIN, "chpl_single")
P2 = os.path.join(BIN, "chpl_p2")


def _run(cmd, env=None, timeout=600):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run(cmd, capture_output=True, text=True, env=e, timeout=timeout)


def test_executables_built():
    assert os.access(SINGLE, os.X_OK) and os.access(P2, os.X_OK)


def test_single_usage():
    r = _run([SINGLE])
    assert r.returncode == 1
    assert "usage: chpl_single N" in r.stderr


def test_single_rejects_backend():
    r = _run([SINGLE, "4096"], env={"HPLS_BACKEND": "bogus"})
    assert r.returncode == 1 and "unknown HPLS_BACKEND" in r.stderr


def test_single_ozaki_backend_configuration():
    """HPLS_BACKEND=ozaki selects the Ozaki-I update; HPLS_OZ_NT its column tile."""
    r = _run([SINGLE, "8192"], env={"CHPL_DRY_RUN": "1", "HPLS_BACKEND": "ozaki", "HPLS_NB": "512", "HPLS_OZ_NT": "1024"})
    assert r.returncode == 0, r.stderr
    assert "backend=ozaki" in r.stdout and "chunk=1024" in r.stdout


def test_single_rejects_bad_sizes():
    r = _run([SINGLE, "1000"], env={"HPLS_NB": "2048"})
    assert r.returncode == 1 and "bad N/NB/AGG" in r.stderr


def test_p2_rejects_odd_rank_count():
    r = _run([P2], env={"WORLD_SIZE": "3", "RANK": "0"})
    assert r.returncode == 1 and "even number of ranks" in r.stderr


def test_single_reads_hpl_dat(tmp_path):
    """chpl_single HPL.dat: N, NB and threshold from lines 6, 8 and 13; the
    reference's chpl_single takes only N (its launcher translates the file)."""
    sys.path.insert(0, ROOT)
    from chpl_b200 import hpl
    p = tmp_path / "HPL.dat"
    hpl.write_hpl_dat(str(p), 139264, 1024, 1, 1, 12.5)
    r = _run([SINGLE, str(p)], env={"CHPL_DRY_RUN": "1", "HPLS_BACKEND": "gemmul8", "HPLS_NB": "2048"})
    assert r.returncode == 0, r.stderr
    assert "N=139264 NB=1024 AGG=6 backend=gemmul8" in r.stdout and "threshold=12.5" in r.stdout
    r = _run([SINGLE, "65536"], env={"CHPL_DRY_RUN": "1"})
    assert r.returncode == 0 and "N=65536 NB=2048 AGG=6 backend=native moduli=14" in r.stdout
    short = tmp_path / "short.dat"
    short.write_text("x\n")
    r = _run([SINGLE, str(short)])
    assert r.returncode == 1 and "cannot read N/NB/threshold" in r.stderr


def _dat(path, N, NB):
    sys.path.insert(0, ROOT)
    from chpl_b200 import hpl
    hpl.write_hpl_dat(str(path), N, NB)


@pytest.mark.gpu
def test_single_solve(cuda):
    env = {"HPLS_BACKEND": "gemmul8", "HPLS_NB": "512", "HPLS_AGG": "4", "HPLS_G8_MODULI": "12"}
    r = _run([SINGLE, "6144"], env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "HPLS_gemmul8" in r.stdout and "PASSED" in r.stdout


@pytest.mark.gpu
def test_single_native_solve(cuda):
    r = _run([SINGLE, "4096"], env={"HPLS_BACKEND": "native", "HPLS_NB": "512", "HPLS_AGG": "2"})
    assert r.returncode == 0, r.stdout + r.stderr
    assert "HPLS_native" in r.stdout and "PASSED" in r.stdout


@pytest.mark.gpu
def test_single_gemmtest(cuda):
    r = _run([SINGLE, "--gemmtest", "1500", "1024", "900"])
    assert r.returncode == 0, r.stdout + r.stderr
    assert "GEMMTEST_PASS" in r.stdout


@pytest.mark.gpu
def test_single_ozaki_gemmtest_and_solve(cuda):
    """HPLS_BACKEND=ozaki: the reference's gemmtest form (n in tiles of nt
    columns) and a whole solve through the Ozaki-I update."""
    r = _run([SINGLE, "--gemmtest", "1500", "1024", "900", "256"], env={"HPLS_BACKEND": "ozaki"})
    assert r.returncode == 0, r.stdout + r.stderr
    assert "GEMMTEST_PASS" in r.stdout and "(ozaki)" in r.stdout
    r = _run([SINGLE, "8192"], env={"HPLS_BACKEND": "ozaki", "HPLS_NB": "512", "HPLS_AGG": "4", "HPLS_OZ_NT": "512"})
    assert r.returncode == 0, r.stdout + r.stderr
    assert "HPLS_ozaki" in r.stdout and "PASSED" in r.stdout and "wide_gemm calls: ozaki=" in r.stdout


@pytest.mark.gpu
def test_p2_one_rank(cuda, tmp_path):
    dat = tmp_path / "HPL.dat"
    _dat(dat, 5000, 512)
    r = _run([P2, str(dat)], env={"WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0", "CHPL2D_G8_MODULI": "12"})
    assert r.returncode == 0, r.stdout + r.stderr
    assert "WC2" in r.stdout and "PASSED" in r.stdout


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.gpu
def test_p2_two_ranks(cuda, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    dat = tmp_path / "HPL.dat"
    _dat(dat, 6000, 512)
    port = _port()
    procs = []
    for rank in range(2):
        e = dict(os.environ, WORLD_SIZE="2", RANK=str(rank), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                 CHPL_BOOTSTRAP_PORT=str(port), CHPL2D_G8_MODULI="12", NCCL_NVLS_ENABLE="0",
                 CHPL_BOOTSTRAP_TIMEOUT="60")
        procs.append(subprocess.Popen([P2, str(dat)], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, env=e))
    outs = [p.communicate(timeout=600) for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    assert "WC2" in outs[0][0] and "PASSED" in outs[0][0]
