"""Driver for oracle/_ref/kernel_harness: the reference's own kernels on the GPU.

File formats are documented in oracle/ref_harness/kernel_harness.cu.
"""
import os
import subprocess
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "kernel_harness")
REF_DRIVER = os.path.join(ROOT, "oracle", "_ref", "abft_gemm_ref")


def available():
    return os.path.exists(HARNESS)


def run_verify(A, B, C, F, tau, injected, golden=None):
    M, K = A.shape
    N = B.shape[1]
    with tempfile.TemporaryDirectory() as td:
        fi, fo = os.path.join(td, "in.bin"), os.path.join(td, "out.bin")
        with open(fi, "wb") as f:
            np.array([M, K, N, F, 1 if golden is not None else 0], np.int32).tofile(f)
            np.asarray(injected, np.int32).tofile(f)
            np.asarray(tau, np.float64).tofile(f)
            for a in (A, B, C):
                np.ascontiguousarray(a, np.float32).tofile(f)
            if golden is not None:
                np.ascontiguousarray(golden, np.float32).tofile(f)
        subprocess.run([HARNESS, "verify", fi, fo], check=True, timeout=300)
        raw = open(fo, "rb").read()
    out = {}
    pos = 0

    def take(name, dtype, n):
        nonlocal pos
        nb = np.dtype(dtype).itemsize * n
        out[name] = np.frombuffer(raw[pos:pos + nb], dtype=dtype).copy()
        pos += nb

    take("colSumA", np.float64, K)
    take("expRow", np.float64, N)
    take("actRow", np.float64, N)
    take("errcol", np.int32, F)
    take("rowdiff", np.float64, F)
    take("rowSumB", np.float64, F * K)
    take("expCol", np.float64, F * M)
    take("actCol", np.float64, F * M)
    take("C", np.float32, M * N)
    take("cm", np.int32, 4)
    take("n_restored", np.int32, 1)
    out["rowSumB"] = out["rowSumB"].reshape(F, K)
    out["expCol"] = out["expCol"].reshape(F, M)
    out["actCol"] = out["actCol"].reshape(F, M)
    out["C"] = out["C"].reshape(M, N)
    return out


def run_inject(C, F, frag, seed, mode, zone="any"):
    M, N = C.shape
    with tempfile.TemporaryDirectory() as td:
        fi, fo = os.path.join(td, "in.bin"), os.path.join(td, "out.bin")
        with open(fi, "wb") as f:
            np.array([M, N, F, frag, 0], np.int32).tofile(f)
            np.array([seed], np.uint64).tofile(f)
            np.array([0 if mode == "add" else 1, len(zone)], np.int32).tofile(f)
            f.write(zone.encode())
            np.ascontiguousarray(C, np.float32).tofile(f)
        subprocess.run([HARNESS, "inject", fi, fo], check=True, timeout=300)
        raw = open(fo, "rb").read()
    rcb = np.frombuffer(raw[:12], np.int32)
    ba = np.frombuffer(raw[12:20], np.float32)
    Cout = np.frombuffer(raw[20:], np.float32).reshape(M, N).copy()
    return tuple(int(x) for x in rcb), tuple(float(x) for x in ba), Cout
