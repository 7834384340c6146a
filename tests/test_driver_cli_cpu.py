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
