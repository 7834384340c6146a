"""Run the reference binary (oracle/_ref/abft_gemm_ref, the reference's main.cu
built for sm_100a, one rank) and this project's abft_gemm with identical flags
on the single-GPU workloads, and print a markdown table of GFLOPS, overhead and
the confusion matrix of each.

MEASUREMENT INFRASTRUCTURE ONLY (not part of the product). Needs a GPU.

    python oracle/compare_reference.py [--quick] > table.md
"""
import argparse
import csv
import os
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref", "abft_gemm_ref")
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


def run(binary, args, common):
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "m.csv")
        r = subprocess.run([binary] + args + common + ["--csv", path], capture_output=True, text=True,
                           timeout=1800)
        if r.returncode != 0:
            return None, (r.stderr or r.stdout)[-300:]
        return list(csv.DictReader(open(path)))[0], ""


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true", help="fewer samples and the small workloads only")
    a = ap.parse_args()
    print("| workload | impl | baseline GFLOPS (med) | protected GFLOPS (med) | overhead % | TP/TN/FP/FN | restored |")
    print("|---|---|---|---|---|---|---|")
    for label, args in WORKLOADS:
        big = "16384" in args
        if a.quick and big:
            continue
        common = ["--repeats", "5", "--samples", "3", "--warmups", "1"] if big else \
            ["--repeats", "20", "--samples", "5", "--warmups", "2"]
        runs = [("reference (sm_100a build)", REF, []), ("this project", OURS, []),
                ("this project, --graph", OURS, ["--graph"])]
        for name, binary, extra in runs:
            row, err = run(binary, args + extra, common)
            if row is None:
                print(f"| {label} | {name} | failed: {err.strip()} | | | | |")
                continue
            cm = "/".join(row[k] for k in ("TP", "TN", "FP", "FN"))
            print(f"| {label} | {name} | {float(row['baseline_gflops_median']):.0f} | "
                  f"{float(row['protected_gflops_median']):.0f} | {float(row['overhead_pct']):.2f} | {cm} | "
                  f"{row['correction_precision_pct']} |", flush=True)


if __name__ == "__main__":
    main()
