"""CPU tests of the launcher (python -m chpl_b200.launch), the MPI-free
counterpart of the reference's scripts/mpirun_chpl, and of chpl_p2's grid
choice.  Nothing here touches a GPU: dry runs, and chpl_p2 with
CHPL_DRY_RUN=1, which exits before any device or network work."""
import os
import subprocess
import sys

import pytest

from chpl_b200 import hpl, launch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
P2 = os.path.join(ROOT, "chpl_b200", "bin", "chpl_p2")


def _run(args, env=None):
    e = dict(os.environ)
    for k in list(e):
        if k.startswith(("HPLS_", "CHPL2D_", "CHPL_DRY")):
            del e[k]
    e.update(env or {})
    return subprocess.run([sys.executable, "-m", "chpl_b200.launch"] + args, capture_output=True, text=True,
                          cwd=ROOT, env=e, timeout=120)


def test_single_gpu_defaults_follow_the_order():
    big = launch.plan(1, 1, 139264, None, None, {})
    assert big["exe"].endswith("chpl_single") and big["args"] == ["139264"]
    assert big["env"] == {"HPLS_NB": "1024", "HPLS_AGG": "6", "HPLS_BACKEND": "gemmul8", "HPLS_G8_MODULI": "11",
                          "HPLS_G8_FAST": "1", "HPLS_G8_CHUNK": "32768"}
    assert launch.plan(1, 1, 65536, None, None, {})["env"]["HPLS_AGG"] == "4"
    small = launch.plan(1, 1, 16384, None, None, {})
    assert small["env"]["HPLS_AGG"] == "1"          # 11 moduli keep their residual margin
    assert launch.plan(1, 1, 8192, 512, None, {})["env"]["HPLS_NB"] == "512"


def test_user_settings_win_over_defaults():
    pl = launch.plan(1, 1, 139264, None, None, {"HPLS_G8_MODULI": "12", "HPLS_AGG": "8", "HPLS_NB": "2048"})
    assert "HPLS_G8_MODULI" not in pl["env"] and "HPLS_AGG" not in pl["env"]
    assert pl["env"]["HPLS_NB"] == "2048"
    g = launch.plan(2, 4, 393216, None, None, {"CHPL2D_G8_MODULI": "12"})
    assert "CHPL2D_G8_MODULI" not in g["env"] and g["env"]["CHPL2D_G8"] == "1"


def test_grid_writes_the_input_file(tmp_path):
    g = launch.plan(2, 4, 393216, None, None, {})
    assert g["exe"].endswith("chpl_p2") and g["nproc"] == 8
    p = tmp_path / "HPL.dat"
    p.write_text(g["dat"])
    d = hpl.read_hpl_dat(str(p))
    assert (d.N, d.NB, d.P, d.Q, d.threshold) == (393216, 4096, 2, 4, 16.0)
    cmd = launch.command(g, str(p), {})
    assert cmd[1:3] == ["-m", "torch.distributed.run"] and "--no-python" in cmd and cmd[-1] == str(p)
    assert cmd[cmd.index("--nproc-per-node") + 1] == "8" and cmd[cmd.index("--master-addr") + 1] == "127.0.0.1"


def test_input_file_keeps_its_fields_and_takes_the_grid(tmp_path):
    src = tmp_path / "in.dat"
    hpl.write_hpl_dat(str(src), 131072, 2048, 4, 4, 8.0)
    g = launch.plan(1, 2, None, None, str(src), {})
    out = tmp_path / "out.dat"
    out.write_text(g["dat"])
    d = hpl.read_hpl_dat(str(out))
    assert (d.N, d.NB, d.P, d.Q, d.threshold) == (131072, 2048, 1, 2, 8.0)
    one = launch.plan(1, 1, None, None, str(src), {})
    assert one["args"] == ["131072"] and one["env"]["HPLS_NB"] == "2048"


@pytest.mark.parametrize("args,msg", [
    ((4, 4, 65536, None, None), "chpl_p4"),
    ((1, 3, 65536, None, None), "not one of this build's grids"),
    ((2, 8, 65536, None, None), "not one of this build's grids"),
    ((1, 1, 100, 200, None), "bad N/NB"),
])
def test_rejected_requests(args, msg):
    with pytest.raises(launch.LaunchError, match=msg):
        launch.plan(*args, {})


def test_rejects_both_inputs_and_missing_file(tmp_path):
    src = tmp_path / "in.dat"
    hpl.write_hpl_dat(str(src), 8192, 512)
    with pytest.raises(launch.LaunchError, match="either -N or -i"):
        launch.plan(1, 1, 8192, None, str(src), {})
    with pytest.raises(launch.LaunchError, match="not found"):
        launch.plan(2, 2, None, None, str(tmp_path / "missing.dat"), {})


def test_dry_run_cli():
    r = _run(["-P", "1", "-Q", "1", "-N", "139264", "--dry-run"])
    assert r.returncode == 0, r.stderr
    assert "HPLS_AGG=6" in r.stdout and r.stdout.strip().splitlines()[-1].endswith("chpl_single 139264")
    r = _run(["-P", "2", "-Q", "2", "-N", "278528", "--dry-run"])
    assert r.returncode == 0 and "CHPL2D_G8=1" in r.stdout and "278528" in r.stdout
    r = _run(["-P", "4", "-Q", "4", "-N", "65536"])
    assert r.returncode == 1 and "chpl_p4" in r.stderr


def test_chpl_p2_takes_the_grid_from_hpl_dat(tmp_path):
    dat = tmp_path / "HPL.dat"
    hpl.write_hpl_dat(str(dat), 196608, 4096, 1, 2)
    base = {"CHPL_DRY_RUN": "1", "RANK": "0"}
    out = subprocess.run([P2, str(dat)], env=dict(os.environ, WORLD_SIZE="2", **base), capture_output=True,
                         text=True, timeout=60)
    assert out.returncode == 0 and "grid 1x2 N=196608 NB=4096" in out.stdout
    # P x Q not matching the rank count: the reference's fixed P = 2
    out = subprocess.run([P2, str(dat)], env=dict(os.environ, WORLD_SIZE="8", **base), capture_output=True,
                         text=True, timeout=60)
    assert out.returncode == 0 and "grid 2x4" in out.stdout


def test_launcher_starts_ranks_through_torchrun():
    """The whole chain on CPU: launcher -> torchrun (2 processes) -> chpl_p2,
    which reads its rank from torchrun's environment and the grid from the
    launcher's HPL.dat, then stops before any GPU work (dry run)."""
    r = _run(["-P", "1", "-Q", "2", "-N", "65536"], env={"CHPL_DRY_RUN": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert "[chpl_p2] grid 1x2 N=65536 NB=4096 threshold=16 moduli=11 ranks=2" in r.stdout
