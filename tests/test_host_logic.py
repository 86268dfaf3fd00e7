"""CPU tests of the host-side logic: HPL.dat and environment configuration,
block-cyclic maps, flop count, report formats."""
import os

import numpy as np
import pytest

from chpl_b200 import hpl


def test_read_hpl_dat_fields(tmp_path):
    p = tmp_path / "HPL.dat"
    hpl.write_hpl_dat(str(p), 393216, 4096, 2, 4, 16.0)
    d = hpl.read_hpl_dat(str(p))
    assert (d.N, d.NB, d.P, d.Q, d.threshold) == (393216, 4096, 2, 4, 16.0)


def test_read_hpl_dat_fallback(tmp_path):
    # fewer than 13 lines or missing file: N=16384, NB=1024, 16.0 (src/chpl_p2.cu:570-584)
    p = tmp_path / "short.dat"
    p.write_text("a\nb\n")
    d = hpl.read_hpl_dat(str(p))
    assert (d.N, d.NB, d.threshold) == (16384, 1024, 16.0)
    d = hpl.read_hpl_dat(str(tmp_path / "missing.dat"))
    assert (d.N, d.NB) == (16384, 1024)


def test_reference_hpl_dat_layout(tmp_path):
    """The 13-line layout of scripts/HPL.dat (N on line 6, NB on 8, threshold on 13)."""
    text = ("HPLinpack benchmark input file\nInnovative Computing Laboratory, University of Tennessee\n"
            "HPL.out      output file name (if any)\n6            device out (6=stdout,7=stderr,file)\n"
            "1            # of problems sizes (N)\n460800       Ns\n1            # of NBs\n4096         NBs\n"
            "0            PMAP process mapping (0=Row-,1=Column-major)\n1            # of process grids (P x Q)\n"
            "4            Ps\n4            Qs\n16.0         threshold\n")
    p = tmp_path / "HPL.dat"
    p.write_text(text)
    d = hpl.read_hpl_dat(str(p))
    assert (d.N, d.NB, d.P, d.Q, d.threshold) == (460800, 4096, 4, 4, 16.0)


def test_single_env_config():
    env = {"HPLS_NB": "512", "HPLS_BACKEND": "gemmul8", "HPLS_G8_MODULI": "12", "HPLS_G8_FAST": "1",
           "HPLS_G8_CHUNK": "3072", "HPLS_SEED": "7"}
    c = hpl.single_config_from_env(8192, env)
    assert (c.N, c.NB, c.moduli, c.fast, c.chunk, c.seed, c.emulate) == (8192, 512, 12, True, 3072, 7, True)
    assert hpl.single_config_from_env(2000, {"HPLS_BACKEND": "native"}).emulate == 0
    # HPLS_BACKEND=ozaki: the Ozaki-I update (emulate = 2), HPLS_OZ_NT columns per call
    c = hpl.single_config_from_env(8192, {"HPLS_BACKEND": "ozaki", "HPLS_OZ_NT": "512", "HPLS_G8_CHUNK": "3072"})
    assert (c.emulate, c.chunk, c.to_c().emulate) == (2, 512, 2)
    assert hpl.format_single(hpl.Result(N=8192, NB=512, P=1, Q=1, time_s=1.0, tflops=1.0, resid=0.5, passed=True,
                                        threshold=16.0, matgen_s=0.0),
                             c).splitlines()[3].startswith("HPLS_ozaki")
    with pytest.raises(ValueError):
        hpl.single_config_from_env(2000, {"HPLS_BACKEND": "bogus"})
    with pytest.raises(ValueError):
        hpl.single_config_from_env(100, {"HPLS_NB": "200"})


def test_grid_env_config():
    d = hpl.HplDat(N=131072, NB=2048, threshold=16.0)
    c = hpl.grid_config_from_env(d, 2, 4, {"CHPL2D_G8": "1", "CHPL2D_G8_MODULI": "12"})
    assert (c.N, c.NB, c.P, c.Q, c.moduli, c.emulate) == (131072, 2048, 2, 4, 12, True)
    assert hpl.grid_config_from_env(d, 1, 2, {"CHPL2D_G8": "0"}).emulate is False
    # launcher default (scripts/mpirun_chpl:107-126): 11 moduli, fast
    c = hpl.grid_config_from_env(d, 1, 1, {})
    assert (c.moduli, c.fast, c.emulate) == (11, True, True)


def test_flop_count():
    assert hpl.flops(1000) == pytest.approx(2.0 / 3.0 * 1e9 + 2e6)


def test_report_formats():
    r = hpl.Result(N=1000, NB=128, P=2, Q=4, time_s=1.5, tflops=0.5, resid=1.25, passed=True, threshold=16.0,
                   matgen_s=0.1)
    s = hpl.format_grid(r)
    assert "WC2" in s and "PASSED" in s and "1000" in s
    s = hpl.format_single(r, hpl.Config(N=1000, NB=128))
    assert "HPLS_gemmul8" in s and "PASSED" in s


def test_bench_e2e_order_follows_host_memory(monkeypatch):
    """The host-buffer leg runs at the bench's N when the pinned [A|b] fits in
    host memory with a margin, at the largest multiple of NB that fits
    otherwise, and not at all below N = 16384."""
    import bench
    GiB = 1 << 30
    need = 139264 * 139265 * 8
    monkeypatch.setattr(bench, "host_memory_available", lambda: need + 40 * GiB)
    assert bench.e2e_order(139264, 1024) == (139264, None)
    monkeypatch.setattr(bench, "host_memory_available", lambda: 62 * GiB)
    n, why = bench.e2e_order(139264, 1024)
    assert n % 1024 == 0 and 16384 <= n < 139264 and n * (n + 1) * 8 <= (62 - 16) * GiB / 1.05
    assert "pinned host memory" in why
    monkeypatch.setattr(bench, "host_memory_available", lambda: 17 * GiB)
    assert bench.e2e_order(139264, 1024)[0] is None
    monkeypatch.setattr(bench, "host_memory_available", lambda: None)
    assert bench.e2e_order(139264, 1024) == (None, "host memory size unknown")


def test_bench_host_memory_reads_meminfo():
    import bench
    v = bench.host_memory_available()
    assert v is None or v > 0



def test_bench_reference_arm_contract():
    """`bench.py --impl reference` (the CPU arm the driver compares against)
    prints one JSON line with the contract's keys, on the bench's own metric."""
    import json
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--N", "1024",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=300, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
