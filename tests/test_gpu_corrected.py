"""Corrected C against a fault-free SGEMM, as the abft_gemm driver reports it
with --csv-extra (corrected_max_rel_err = max |C - C_clean| / max |C_clean| over
the final buffers of the last trial).

The single-rank 1024^3 workload as specified for it: A and B uniform[-1,1]
from seed 0, one +1.0 fault per iteration at an (i, j) uniform over the tile
from seed 1 + iteration, threshold 1e-5 * K * max|A| * max|B|. Every fault must
be detected and corrected to within 1e-5 of the fault-free C, in-loop and in
the post-loop drain alike; without faults the final C is the clean C exactly.
"""
import csv
import os
import subprocess

import pytest

from conftest import PKG_NAME, ROOT

DRIVER = os.path.join(ROOT, PKG_NAME, "abft_gemm")

pytestmark = pytest.mark.gpu


def run_driver(args, tmp_path):
    out = str(tmp_path / "m.csv")
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    r = subprocess.run([DRIVER] + args + ["--csv-extra", "--csv", out], capture_output=True, text=True,
                       timeout=600, env=env)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])
    rows = list(csv.DictReader(open(out)))
    assert len(rows) == 1
    return rows[0], r.stdout


WORKLOAD = ["1024", "--seed-a", "0", "--seed-b", "0", "--relative-threshold", "1e-5", "--repeats", "10",
            "--samples", "2", "--warmups", "1"]


@pytest.mark.parametrize("correct", ["inloop", "drain"])
def test_additive_faults_corrected_within_1e5(correct, tmp_path):
    row, out = run_driver(WORKLOAD + ["--inject", "add", "--add-delta", "1.0", "--inject-seed-mode", "json",
                                      "--correct", correct], tmp_path)
    tp, tn, fp, fn = (int(row[k]) for k in ("TP", "TN", "FP", "FN"))
    assert (tp, fp, fn) == (2 * 10, 0, 0) and tn == 2 * 10 * 3
    assert row["correct_mode"] == correct
    assert float(row["encode_ms"]) > 0.0
    err = float(row["corrected_max_rel_err"])
    assert 0.0 <= err <= 1e-5, err
    assert "Corrected C vs fault-free" in out


def test_no_faults_leave_clean_c(tmp_path):
    row, _ = run_driver(WORKLOAD + ["--inject", "none"], tmp_path)
    assert int(row["TP"]) == int(row["FP"]) == int(row["FN"]) == 0
    assert float(row["corrected_max_rel_err"]) == 0.0
