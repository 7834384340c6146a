"""Run the reference binary (the reference's main.cu built for sm_100a) and
this project's abft_gemm with identical flags and print a markdown table of
GFLOPS, overhead and the confusion matrix of each.

One rank (default): oracle/_ref/abft_gemm_ref on the single-GPU workloads.
--ranks N (2, 4 or 8): oracle/_ref/abft_gemm_ref_mpi (the reference over the
loopback MPI stand-in) and abft_gemm, both launched by torchrun with one rank
per GPU, on the multi-rank workloads: the global 8192^3 additive workload and
the 16384^3 SWIFI sweep on the near-square grid of N ranks.

MEASUREMENT INFRASTRUCTURE ONLY (not part of the product). Needs GPUs.

    python oracle/compare_reference.py [--quick] [--ranks N] [--dry-run] > table.md
"""
import argparse
import csv
import os
import socket
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref", "abft_gemm_ref")
REF_MPI = os.path.join(HERE, "_ref", "abft_gemm_ref_mpi")
GRIDS = {2: ("1", "2"), 4: ("2", "2"), 8: ("2", "4")}
OURS = os.path.join(ROOT, "asynchronous_abft_for_mpi-cuda_architectures_b200", "abft_gemm")

# (label, sizes/flags). Thresholds: 1e-5 * K * max|A| * max|B| with max|.| ~ 1 for uniform[-1,1].
WORKLOADS = [
    ("1024^3, add", ["1024", "--inject", "add", "--threshold", "0.01024"]),
    ("1024^3, none", ["1024", "--inject", "none", "--threshold", "0.01024"]),
    ("4096^3, swifi any", ["4096", "--inject", "swifi", "--threshold", "0.04096"]),
    ("4096^3, add", ["4096", "--inject", "add", "--threshold", "0.04096"]),
    ("4096x8192x2048 (8192^3 rank tile of a 2x4 grid), add", ["4096", "8192", "2048", "--inject", "add",
                                                               "--threshold", "0.08192"]),
    ("16384x4096x1024 (tall-skinny), add", ["16384", "4096", "1024", "--inject", "add", "--threshold", "0.04096"]),
    ("1024x16384x16384 (wide), add", ["1024", "16384", "16384", "--inject", "add", "--threshold", "0.16384"]),
    ("16384^3, swifi any", ["16384", "--inject", "swifi", "--threshold", "0.16384"]),
]


def multi_rank_workloads(n):
    """Global sizes on the grid of n ranks; thresholds 1e-5 * K * max|A| * max|B|."""
    Pr, Pc = GRIDS[n]
    g = ["--grid", Pr, Pc]
    return [
        (f"8192^3 on {Pr}x{Pc}, add (every rank, every iteration)",
         ["8192"] + g + ["--inject", "add", "--threshold", "0.08192"]),
        (f"16384^3 on {Pr}x{Pc}, swifi any", ["16384"] + g + ["--inject", "swifi", "--threshold", "0.16384"]),
    ]


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def command(binary, args, ranks, mpi_port):
    """The command line and extra environment of one run (torchrun for several ranks)."""
    if ranks == 1:
        return [binary] + args, {}
    launch = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={ranks}",
              "--master-addr=127.0.0.1", f"--master-port={free_port()}", "--no-python"]
    if binary == REF_MPI:
        # the reference picks its GPU from OMPI_COMM_WORLD_LOCAL_RANK (main.cu:43-47)
        wrap = 'OMPI_COMM_WORLD_LOCAL_RANK=$LOCAL_RANK exec "$0" "$@"'
        return launch + ["bash", "-c", wrap, binary] + args, {"ABFT_MPI_STUB_PORT": str(mpi_port)}
    return launch + [binary] + args, {}


def run(binary, args, common, ranks=1, dry_run=False):
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "m.csv")
        cmd, extra = command(binary, args + common + ["--csv", path], ranks, free_port())
        if dry_run:
            print(" ".join(f"{k}={v}" for k, v in extra.items()), " ".join(cmd), file=sys.stderr)
            return None, "dry run"
        r = subprocess.run(["timeout", "-k", "60", "1800"] + cmd, capture_output=True, text=True, timeout=1900,
                           env=dict(os.environ, **extra))
        if r.returncode != 0:
            return None, (r.stderr or r.stdout)[-300:]
        return list(csv.DictReader(open(path)))[0], ""


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true", help="fewer samples and the small workloads only")
    ap.add_argument("--ranks", type=int, default=1, choices=[1, 2, 4, 8], help="ranks (one GPU each)")
    ap.add_argument("--dry-run", action="store_true", help="print the commands instead of running them")
    a = ap.parse_args()
    workloads = WORKLOADS if a.ranks == 1 else multi_rank_workloads(a.ranks)
    ref = REF if a.ranks == 1 else REF_MPI
    print("| workload | impl | baseline GFLOPS (med) | protected GFLOPS (med) | overhead % | TP/TN/FP/FN | restored |")
    print("|---|---|---|---|---|---|---|")
    for label, args in workloads:
        big = "16384" in args
        if a.quick and big:
            continue
        common = ["--repeats", "5", "--samples", "3", "--warmups", "1"] if big else \
            ["--repeats", "20", "--samples", "5", "--warmups", "2"]
        runs = [("reference (sm_100a build)", ref, []), ("this project", OURS, []),
                ("this project, --graph", OURS, ["--graph"])]
        for name, binary, extra in runs:
            row, err = run(binary, args + extra, common, a.ranks, a.dry_run)
            if row is None:
                print(f"| {label} | {name} | failed: {err.strip()} | | | | |")
                continue
            cm = "/".join(row[k] for k in ("TP", "TN", "FP", "FN"))
            print(f"| {label} | {name} | {float(row['baseline_gflops_median']):.0f} | "
                  f"{float(row['protected_gflops_median']):.0f} | {float(row['overhead_pct']):.2f} | {cm} | "
                  f"{row['correction_precision_pct']} |", flush=True)


if __name__ == "__main__":
    main()
