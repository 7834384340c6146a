"""The abft_gemm driver's command line (the reference's flags, core/cli.cuh:7-86,
plus this project's extensions): malformed flags and values are refused with
a message before any CUDA call, so these checks run without a GPU."""
import os
import subprocess

import pytest

from conftest import PKG_NAME, ROOT

DRIVER = os.path.join(ROOT, PKG_NAME, "abft_gemm")

pytestmark = pytest.mark.skipif(not os.path.exists(DRIVER), reason="driver not built")


def run(*args, cwd=None):
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    return subprocess.run([DRIVER, *args], capture_output=True, text=True, timeout=60, env=env, cwd=cwd)


@pytest.mark.parametrize("args,msg", [
    (["64", "--inject", "bogus"], "--inject must be none, add or swifi"),
    (["64", "--swifi-zone"], "unknown or incomplete flag --swifi-zone"),
    (["64", "--grid", "2"], "unknown or incomplete flag --grid"),
    (["64", "--dist", "cauchy"], "--dist must be uniform or normal"),
    (["64", "--correct", "later"], "--correct must be inloop or drain"),
    (["64", "--verify-priority", "urgent"], "--verify-priority must be low, default or high"),
    (["64", "--inject-seed-mode", "random"], "--inject-seed-mode must be reference or json"),
    (["64", "--turbo"], "unknown or incomplete flag --turbo"),
    (["0"], "matrix sizes must be positive"),
    (["64", "32", "-5"], "unknown or incomplete flag -5"),
])
def test_bad_flags_are_refused(args, msg):
    r = run(*args)
    assert r.returncode == 2, (r.returncode, r.stderr)
    assert msg in r.stderr


def test_grid_must_match_world(tmp_path):
    r = run("64", "--grid", "2", "2", cwd=str(tmp_path))
    assert r.returncode == 1 and "does not match" in r.stderr


def test_help_lists_reference_flags_and_extensions():
    r = run("--help")
    assert r.returncode == 0
    for flag in ("--inject", "--swifi-zone", "--baseline", "--threshold", "--frags-per-rank", "--frag-cap", "--grid",
                 "--repeats", "--warmups", "--samples", "--reseed-per-trial", "--seed-a", "--seed-b", "--csv",
                 "--calibrate", "--calibration-safety", "--calib-diffs", "--dist", "--add-delta",
                 "--relative-threshold", "--correct", "--verify-priority", "--csv-extra", "--graph",
                 "--inject-seed-mode"):
        assert flag in r.stdout, flag


def test_sweep_commands_are_valid_driver_invocations(tmp_path):
    """The throughput sweep (the reference's example_run.sh protocol: per size
    --baseline, --inject none, --inject add) builds driver command lines that
    the driver accepts: on a machine without a GPU each stops at the first CUDA
    call (exit 1), never at argument parsing (exit 2)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("abft_sweep", os.path.join(ROOT, PKG_NAME, "sweep.py"))
    sweep = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sweep)
    k = sweep.knobs({"SIZES": "64 96", "F": "4", "SAMPLES": "1", "WARMUPS": "0",
                     "OUT_CSV": str(tmp_path / "m.csv")})
    runs = sweep.commands(k, ["--graph"])
    assert [label for label, _ in runs] == [f"S = {s}, {m}" for s in (64, 96) for m, _ in sweep.MODES]
    for label, argv in runs:
        assert argv[0] == DRIVER and "--graph" in argv and "--csv" in argv
        r = run(*argv[1:], cwd=str(tmp_path))
        assert r.returncode in (0, 1), (label, r.returncode, r.stderr)
        assert "flag" not in r.stderr and "must be" not in r.stderr, (label, r.stderr)
    multi = sweep.commands(dict(k, NP=8))
    assert all("--nproc-per-node=8" in argv and DRIVER in argv for _, argv in multi)
    # the rendezvous port is chosen at launch, one per run
    assert all(sweep.PORT_ARG in argv for _, argv in multi)
    launched = sweep.launch_argv(multi[0][1])
    port = [a for a in launched if a.startswith("--master-port=")]
    assert len(port) == 1 and int(port[0].split("=")[1]) > 0 and sweep.PORT_ARG not in launched
