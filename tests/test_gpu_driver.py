"""abft_gemm (this project) against the reference binary rebuilt for sm_100a
(oracle/_ref/abft_gemm_ref, single rank): same flags, same seeds, same cuBLAS
build -> every non-timing CSV column (confusion matrix, restore count,
threshold, geometry) must be identical."""
import csv
import os
import subprocess

import numpy as np
import pytest

import refharness
from conftest import PKG_NAME, ROOT

DRIVER = os.path.join(ROOT, PKG_NAME, "abft_gemm")
TIMING_COLS = {"baseline_min_ms", "baseline_median_ms", "baseline_mean_ms", "baseline_max_ms",
               "baseline_gflops_min", "baseline_gflops_median", "baseline_gflops_mean", "baseline_gflops_max",
               "protected_min_ms", "protected_median_ms", "protected_mean_ms", "protected_max_ms",
               "protected_gflops_min", "protected_gflops_median", "protected_gflops_mean", "protected_gflops_max",
               "overhead_pct"}

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(refharness.REF_DRIVER), reason="reference binary not built")]

CASES = [
    ["1024", "--inject", "add", "--threshold", "0.01024"],
    ["1024", "--inject", "swifi", "--threshold", "0.01024"],
    ["1024", "--inject", "swifi"],                                     # formula threshold
    ["1024", "--inject", "none", "--threshold", "0.01024"],
    ["1024", "--baseline"],
    ["1100", "300", "1030", "--inject", "swifi", "--swifi-zone", "exponent", "--threshold", "0.003"],
    ["2048", "--inject", "swifi", "--swifi-zone", "sig_high", "--threshold", "0.02", "--frags-per-rank", "8"],
    ["1024", "--inject", "swifi", "--reseed-per-trial", "--threshold", "0.01024"],
    ["4096", "1024", "2048", "--inject", "add", "--threshold", "0.04", "--frag-cap", "1000000"],
    ["1024", "--calibrate"],
    ["1100", "300", "1030", "--calibrate", "--calibration-safety", "4", "--frags-per-rank", "3"],
]


# The workloads' own shapes (rank tiles of the tile-geometry table), with the
# relative threshold 1e-5 * K * max|A| * max|B| computed on the host from the
# inputs both binaries draw (the reference has no relative-threshold flag, so
# both get it as --threshold). (label, M, K, N, flags, trial protocol)
SHAPE_CASES = [
    ("4096^3 swifi any, F=4, 20 iterations", 4096, 4096, 4096, ["--inject", "swifi", "--swifi-zone", "any"],
     ["--repeats", "20", "--samples", "1", "--warmups", "1"]),
    ("16384^3 swifi any, one GPU", 16384, 16384, 16384, ["--inject", "swifi", "--swifi-zone", "any"],
     ["--repeats", "3", "--samples", "1", "--warmups", "1"]),
    ("tall 16384x1024 K=4096, add", 16384, 4096, 1024, ["--inject", "add"],
     ["--repeats", "5", "--samples", "1", "--warmups", "1"]),
    ("wide 1024x16384 K=16384, add", 1024, 16384, 16384, ["--inject", "add"],
     ["--repeats", "5", "--samples", "1", "--warmups", "1"]),
    ("8192^3 2x4 rank-tile shape 4096x2048 K=8192, add", 4096, 8192, 2048, ["--inject", "add"],
     ["--repeats", "5", "--samples", "1", "--warmups", "1"]),
]


def relative_tau(orc, M, K, N, seed_a=123456, seed_b=987654):
    A = orc.fill_random(M * K, seed_a)
    a = float(np.abs(A).max())
    del A
    B = orc.fill_random(K * N, seed_b)
    b = float(np.abs(B).max())
    return 1e-5 * K * a * b


def run(binary, args, csv_path, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    diffs = csv_path + ".diffs"
    r = subprocess.run([binary] + args + ["--csv", csv_path, "--calib-diffs", diffs], capture_output=True, text=True,
                       timeout=600, env=env)
    assert r.returncode == 0, (binary, r.stdout[-2000:], r.stderr[-2000:])
    with open(csv_path) as f:
        rows = list(csv.DictReader(f))
    assert len(rows) == 1
    return rows[0], r.stdout


@pytest.mark.parametrize("case", CASES, ids=[" ".join(c) for c in CASES])
def test_driver_matches_reference_binary(case, tmp_path):
    common = ["--repeats", "10", "--samples", "2", "--warmups", "1"]
    ours, out_ours = run(DRIVER, case + common, str(tmp_path / "ours.csv"))
    ref, out_ref = run(refharness.REF_DRIVER, case + common, str(tmp_path / "ref.csv"))
    assert list(ours.keys()) == list(ref.keys())
    for k in ref:
        if k not in TIMING_COLS:
            assert ours[k] == ref[k], (k, ours[k], ref[k])
    if "--calibrate" in case:
        a = open(str(tmp_path / "ours.csv.diffs")).read()
        b = open(str(tmp_path / "ref.csv.diffs")).read()
        assert a.splitlines()[0] == "abs_diff" and len(a.splitlines()) > 1000
        assert a == b  # every |actual - expected|, printed with 8 significant digits
        assert "Suggested threshold" in out_ours
    else:
        assert "TP / TN / FP / FN" in out_ours


@pytest.mark.parametrize("label,M,K,N,flags,protocol", SHAPE_CASES, ids=[c[0] for c in SHAPE_CASES])
def test_driver_matches_reference_at_workload_shapes(label, M, K, N, flags, protocol, orc, tmp_path):
    tau = relative_tau(orc, M, K, N)
    case = [str(M), str(K), str(N)] + flags + ["--threshold", "%.17g" % tau] + protocol
    ours, out_ours = run(DRIVER, case, str(tmp_path / "ours.csv"))
    ref, _ = run(refharness.REF_DRIVER, case, str(tmp_path / "ref.csv"))
    assert list(ours.keys()) == list(ref.keys())
    for k in ref:
        if k not in TIMING_COLS:
            assert ours[k] == ref[k], (k, ours[k], ref[k])
    tp, fn = int(ours["TP"]), int(ours["FN"])
    assert tp + fn == int(protocol[1]) * int(protocol[3])  # one injected fragment per recorded iteration
    if "add" in flags:
        assert fn == 0 and int(ours["FP"]) == 0


def test_driver_rejects_bad_flags(tmp_path):
    r = subprocess.run([DRIVER, "64", "--inject", "bogus"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "inject" in r.stderr
    r = subprocess.run([DRIVER, "64", "--grid", "2", "2"], capture_output=True, text=True, timeout=60,
                       cwd=str(tmp_path))
    assert r.returncode == 1 and "does not match" in r.stderr
