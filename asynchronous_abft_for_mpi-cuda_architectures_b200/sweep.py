"""Throughput sweep with the abft_gemm driver: for every size, the unprotected
pass, the protected loop without faults and the protected loop with an
additive fault per iteration, all appended to one metrics CSV. The same knobs
and three-mode protocol as the reference's scripts/example_run.sh (which ran
the reference binary under mpirun), so existing sweeps and CSV consumers carry
over; several ranks are launched with torchrun, one per GPU.

    NP=8 SIZES="4096 8192" python asynchronous_abft_for_mpi-cuda_architectures_b200/sweep.py [--dry-run]

Environment knobs (defaults): NP (1), SIZES ("1024 2048 4096"), F (8), SAMPLES
(10), WARMUPS (2), R (1), OUT_CSV (abft_metrics.csv), TAU (1.0; the threshold
does not matter for a throughput sweep). Extra arguments after "--" go to
every driver run (e.g. -- --graph).
"""
import os
import shlex
import socket
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
DRIVER = os.path.join(PKG_DIR, "abft_gemm")

# torchrun's rendezvous port is chosen when a run starts (a port picked when
# the list is built could be taken by then): this argument marks its place.
PORT_ARG = "--master-port={port}"

MODES = [("baseline", ["--baseline"]), ("online, no fault", ["--inject", "none"]),
         ("online, additive fault", ["--inject", "add"])]


def knobs(env):
    return {
        "NP": int(env.get("NP", "1")),
        "SIZES": [int(s) for s in env.get("SIZES", "1024 2048 4096").split()],
        "F": int(env.get("F", "8")),
        "SAMPLES": int(env.get("SAMPLES", "10")),
        "WARMUPS": int(env.get("WARMUPS", "2")),
        "R": int(env.get("R", "1")),
        "OUT_CSV": env.get("OUT_CSV", "abft_metrics.csv"),
        "TAU": env.get("TAU", "1.0"),
    }


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def commands(k, extra=()):
    """(label, argv) of every run of the sweep, in order; a multi-rank argv
    holds PORT_ARG, which launch_argv fills in."""
    common = ["--frags-per-rank", str(k["F"]), "--samples", str(k["SAMPLES"]), "--warmups", str(k["WARMUPS"]),
              "--repeats", str(k["R"]), "--csv", k["OUT_CSV"]]
    out = []
    for size in k["SIZES"]:
        for label, mode in MODES:
            args = [str(size)] * 3 + mode + ([] if mode == ["--baseline"] else ["--threshold", k["TAU"]])
            args += common + list(extra)
            if k["NP"] > 1:
                argv = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={k['NP']}",
                        "--master-addr=127.0.0.1", PORT_ARG, "--no-python", DRIVER] + args
            else:
                argv = [DRIVER] + args
            out.append((f"S = {size}, {label}", argv))
    return out


def launch_argv(argv):
    """argv with a free loopback port in place of PORT_ARG, chosen now."""
    return [a.format(port=free_port()) if a == PORT_ARG else a for a in argv]


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    dry = "--dry-run" in argv
    extra = argv[argv.index("--") + 1:] if "--" in argv else []
    k = knobs(os.environ)
    runs = commands(k, extra)
    if not dry:
        if not os.path.exists(DRIVER):
            sys.exit(f"{DRIVER} is missing: build it with python {os.path.join(PKG_DIR, 'build.py')}")
        if os.path.exists(k["OUT_CSV"]):
            os.remove(k["OUT_CSV"])
    print(f"=== Throughput sweep: sizes {' '.join(map(str, k['SIZES']))}, {k['NP']} rank(s), "
          f"{k['SAMPLES']} samples per phase ===", flush=True)
    for label, cmd in runs:
        print(f"--- {label}: {shlex.join(cmd)}", flush=True)
        if not dry:
            r = subprocess.run(launch_argv(cmd))
            if r.returncode != 0:
                sys.exit(f"run failed ({r.returncode}): {label}")
    print(f"CSV: {os.path.abspath(k['OUT_CSV'])} (baseline_gflops_mean / protected_gflops_mean per row; "
          "overhead_pct relative to the unprotected pass)")


if __name__ == "__main__":
    main()
