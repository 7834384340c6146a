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


def torchrun(n, args, timeout=600):
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={free_port()}"] + args
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
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
