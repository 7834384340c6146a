"""Multi-GPU runs (skipped with fewer than 2 visible GPUs): the Python stack
over NCCL with per-rank oracle parity, and the abft_gemm driver on 2 ranks."""
import csv
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import PKG_NAME, ROOT

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def free_ports(n):
    """The first of n free consecutive loopback ports."""
    for _ in range(50):
        base = free_port()
        if base + n >= 65535:
            continue
        socks = []
        try:
            for p in range(base, base + n):
                s = socket.socket()
                socks.append(s)
                s.bind(("127.0.0.1", p))
            return base
        except OSError:
            continue
        finally:
            for s in socks:
                s.close()
    raise RuntimeError("no free port range")


def torchrun(n, args, timeout=600, env_extra=None):
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={free_port()}"] + args
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    env.update(env_extra or {})
    return subprocess.run(cmd, capture_output=True, text=True, timeout=timeout + 60, env=env, cwd=ROOT)


def test_python_stack_two_ranks():
    r = torchrun(2, [os.path.join(ROOT, "tests", "multi_rank_worker.py")])
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    d = json.loads(line)
    assert d["ranks_ok"] == 2, d
    assert sum(d["cm"]) == 2 * 8 * 4  # every fragment of every iteration on both ranks decided once


@pytest.mark.parametrize("grid", [["1", "2"], ["2", "1"]])
def test_driver_two_ranks(grid, tmp_path):
    drv = os.path.join(ROOT, PKG_NAME, "abft_gemm")
    out = str(tmp_path / "m.csv")
    r = torchrun(2, ["--no-python", drv, "2048", "1024", "2048", "--grid", *grid, "--inject", "add",
                     "--threshold", "0.02", "--repeats", "6", "--samples", "2", "--warmups", "1", "--csv", out])
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    row = list(csv.DictReader(open(out)))[0]
    assert (row["Pr"], row["Pc"]) == tuple(grid)
    # one additive fault per rank per iteration, all detected
    assert int(row["TP"]) == 2 * 6 * 2 and int(row["FN"]) == 0
    assert int(row["TP"]) + int(row["TN"]) + int(row["FP"]) + int(row["FN"]) == 2 * 6 * 2 * 4


NGPU = torch.cuda.device_count()
GRIDS = {4: ("2", "2"), 8: ("2", "4")}


@pytest.mark.skipif(NGPU < 4, reason="needs 4 GPUs")
def test_python_stack_all_gpus():
    """4 or 8 ranks: a 2x2 or 2x4 grid, row and column panels both travel."""
    n = 8 if NGPU >= 8 else 4
    r = torchrun(n, [os.path.join(ROOT, "tests", "multi_rank_worker.py")])
    assert r.returncode == 0, r.stderr[-3000:]
    d = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert d["ranks_ok"] == n and tuple(str(x) for x in d["grid"]) == GRIDS[n], d
    assert sum(d["cm"]) == n * 8 * 4


@pytest.mark.skipif(NGPU < 4, reason="needs 4 GPUs")
def test_driver_all_gpus_graph_swifi(tmp_path):
    n = 8 if NGPU >= 8 else 4
    drv = os.path.join(ROOT, PKG_NAME, "abft_gemm")
    out = str(tmp_path / "m.csv")
    r = torchrun(n, ["--no-python", drv, "4096", "--inject", "swifi", "--graph", "--repeats", "6", "--samples", "2",
                     "--warmups", "1", "--csv", out])
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    row = list(csv.DictReader(open(out)))[0]
    assert (row["Pr"], row["Pc"]) == GRIDS[n]
    assert int(row["TP"]) + int(row["TN"]) + int(row["FP"]) + int(row["FN"]) == n * 6 * 2 * 4
    assert int(row["FP"]) == 0 and int(row["TP"]) + int(row["FN"]) == n * 6 * 2


REF_MPI = os.path.join(ROOT, "oracle", "_ref", "abft_gemm_ref_mpi")
TIMING_COLS = {"baseline_min_ms", "baseline_median_ms", "baseline_mean_ms", "baseline_max_ms",
               "baseline_gflops_min", "baseline_gflops_median", "baseline_gflops_mean", "baseline_gflops_max",
               "protected_min_ms", "protected_median_ms", "protected_mean_ms", "protected_max_ms",
               "protected_gflops_min", "protected_gflops_median", "protected_gflops_mean", "protected_gflops_max",
               "overhead_pct"}


@pytest.mark.skipif(not os.path.exists(REF_MPI), reason="multi-rank reference driver not built")
@pytest.mark.parametrize("grid", [["1", "2"], ["2", "1"]])
def test_reference_binary_two_ranks(grid, tmp_path):
    """The reference driver itself as two ranks (its MPI calls carried by the
    loopback stand-in, one GPU per rank) against abft_gemm with the same grid,
    flags and seeds: every non-timing CSV column (confusion matrix, restore
    count, threshold, geometry) must be equal."""
    args = ["2048", "1024", "2048", "--grid", *grid, "--inject", "swifi", "--threshold", "0.02", "--repeats", "6",
            "--samples", "2", "--warmups", "1"]
    ref_csv, ours_csv = str(tmp_path / "ref.csv"), str(tmp_path / "ours.csv")
    # the reference picks its GPU from OMPI_COMM_WORLD_LOCAL_RANK (main.cu:43-47)
    wrap = 'OMPI_COMM_WORLD_LOCAL_RANK=$LOCAL_RANK exec "$0" "$@"'
    r = torchrun(2, ["--no-python", "bash", "-c", wrap, REF_MPI] + args + ["--csv", ref_csv],
                 env_extra={"ABFT_MPI_STUB_PORT": str(free_ports(2)), "ABFT_MPI_STUB_TIMEOUT": "120"})
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    drv = os.path.join(ROOT, PKG_NAME, "abft_gemm")
    r = torchrun(2, ["--no-python", drv] + args + ["--csv", ours_csv])
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    ref = list(csv.DictReader(open(ref_csv)))[0]
    ours = list(csv.DictReader(open(ours_csv)))[0]
    assert list(ours.keys()) == list(ref.keys())
    for k in ref:
        if k not in TIMING_COLS:
            assert ours[k] == ref[k], (k, ours[k], ref[k])
    assert (ref["Pr"], ref["Pc"]) == tuple(grid) and int(ref["TP"]) + int(ref["FN"]) == 2 * 6 * 2


def relative_tau(n):
    """1e-5 * K * max|A| * max|B| of the global n^3 inputs both drivers draw."""
    import numpy as np
    import oracle
    a = float(np.abs(oracle.fill_random(n * n, 123456)).max())
    b = float(np.abs(oracle.fill_random(n * n, 987654)).max())
    return 1e-5 * n * a * b


@pytest.mark.skipif(not os.path.exists(REF_MPI), reason="multi-rank reference driver not built")
@pytest.mark.skipif(NGPU < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("size,inject,repeats", [(8192, "add", 5), (16384, "swifi", 3)], ids=["8192-add", "16384-swifi"])
def test_reference_binary_all_gpus(size, inject, repeats, tmp_path):
    """The multi-GPU workloads against the reference driver itself, one rank
    per GPU on the 2x4 grid (2x2 with 4 GPUs): global 8192^3 with an additive
    fault on every rank every iteration, and global 16384^3 with SWIFI flips;
    relative threshold 1e-5 * K * max|A| * max|B| given to both. Every
    non-timing CSV column (confusion matrix summed over ranks, restore count,
    threshold, geometry) must be equal."""
    n = 8 if NGPU >= 8 else 4
    args = [str(size), "--grid", *GRIDS[n], "--inject", inject, "--threshold", "%.17g" % relative_tau(size),
            "--repeats", str(repeats), "--samples", "1", "--warmups", "1"]
    ref_csv, ours_csv = str(tmp_path / "ref.csv"), str(tmp_path / "ours.csv")
    wrap = 'OMPI_COMM_WORLD_LOCAL_RANK=$LOCAL_RANK exec "$0" "$@"'
    r = torchrun(n, ["--no-python", "bash", "-c", wrap, REF_MPI] + args + ["--csv", ref_csv], timeout=900,
                 env_extra={"ABFT_MPI_STUB_PORT": str(free_ports(n)), "ABFT_MPI_STUB_TIMEOUT": "300"})
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    drv = os.path.join(ROOT, PKG_NAME, "abft_gemm")
    r = torchrun(n, ["--no-python", drv] + args + ["--csv", ours_csv], timeout=900)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    ref = list(csv.DictReader(open(ref_csv)))[0]
    ours = list(csv.DictReader(open(ours_csv)))[0]
    assert list(ours.keys()) == list(ref.keys())
    for k in ref:
        if k not in TIMING_COLS:
            assert ours[k] == ref[k], (k, ours[k], ref[k])
    assert (ref["Pr"], ref["Pc"]) == GRIDS[n]
    assert int(ref["TP"]) + int(ref["FN"]) == n * repeats  # one injected fragment per rank per iteration
    if inject == "add":
        assert int(ref["FN"]) == 0 and int(ref["FP"]) == 0
