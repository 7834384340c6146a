"""Metrics, report and CSV formatting against the reference's own metrics
module (fixtures from oracle/_ref/host_probe, tests/golden/host_golden.json)."""
import importlib
import os
import struct

import pytest

from conftest import PKG_NAME


@pytest.fixture(scope="module")
def metrics():
    return importlib.import_module(f"{PKG_NAME}.metrics")


def d2hex(x):
    return struct.pack(">d", x).hex()


def test_stats_of(metrics, host_golden):
    for c in host_golden["stats_of"]:
        t = metrics.stats_of(c["samples"])
        got = [d2hex(t.min_ms), d2hex(t.median_ms), d2hex(t.mean_ms), d2hex(t.max_ms), str(t.n_samples)]
        assert got == c["bits"]


def build(metrics, args):
    (scheme, inject, zone, bo, cal, M, K, N, Pr, Pc, F, repeats, tau, TP, TN, FP, FN, restored,
     bmin, bmed, bmean, bmax) = args
    T = metrics.Timing
    base = T(bmin, bmed, bmean, bmax, 0)
    prot = T(bmin * 1.25, bmed * 1.25, bmean * 1.25, bmax * 1.25, 0)
    calib = (0.125, 10.0, 1.25) if cal else (0.0, 0.0, 0.0)
    return metrics.make_metrics(scheme, inject, zone, bo, cal, M, K, N, Pr, Pc, F, repeats, tau, base, prot,
                                (TP, TN, FP, FN), restored, calib)


def test_report_and_csv_match_reference(metrics, host_golden, tmp_path):
    for i, c in enumerate(host_golden["metrics"]):
        m = build(metrics, c["args"])
        assert metrics.report(m) == c["stdout"]
        path = str(tmp_path / f"m{i}.csv")
        metrics.csv_append(m, path)
        assert open(path).read() == c["csv"]


def test_csv_appends_without_second_header(metrics, host_golden, tmp_path):
    c = host_golden["metrics"][0]
    m = build(metrics, c["args"])
    path = str(tmp_path / "twice.csv")
    metrics.csv_append(m, path)
    metrics.csv_append(m, path)
    lines = open(path).read().splitlines()
    assert len(lines) == 3 and lines[1] == lines[2]
    assert len(lines[0].split(",")) == 41


def test_csv_extra_columns(metrics, host_golden, tmp_path):
    m = build(metrics, host_golden["metrics"][1]["args"])
    path = str(tmp_path / "extra.csv")
    metrics.csv_append(m, path, "correct_mode,dist", "drain,normal")
    header, row = open(path).read().splitlines()
    assert header.endswith(",correct_mode,dist") and row.endswith(",drain,normal")
    assert len(header.split(",")) == 43 and len(row.split(",")) == 43


def test_derived_metrics(metrics):
    T = metrics.Timing
    m = metrics.make_metrics("online", "swifi", "any", 0, 0, 4096, 4096, 4096, 1, 1, 4, 20, 0.04,
                             T(2.0, 2.5, 2.6, 3.0, 5), T(2.1, 2.55, 2.7, 3.2, 5), (45, 300, 0, 55), 40)
    assert m.recall == pytest.approx(45 / 100)
    assert m.precision == pytest.approx(1.0)
    assert m.correction_precision_pct == pytest.approx(100 * 40 / 45)
    assert m.overhead_pct == pytest.approx(2.0)
    assert m.baseline_gflops_median == pytest.approx(2 * 4096 ** 3 / (2.5 * 1e6))
