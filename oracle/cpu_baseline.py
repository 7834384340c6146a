"""CPU baseline of the protected SGEMM: the reference's algorithm on host cores.

TEST AND CPU-BASELINE INFRASTRUCTURE ONLY: bench.py's CPU-baseline leg and its
`--impl reference` arm call this; the product never does. One protected
iteration = the SGEMM of the rank tile (numpy/BLAS, all host threads) followed
by the reference's verification exactly as pass_online_loop runs it
(pipeline/passes.cuh:139-203): injection, actualRow + detect per fragment and,
after a detection, the reference's on-demand localisation (rowSumB_f, A .
rowSumB_f, actualCol) and correction, all from oracle/abft_oracle.cpp
(OpenMP across columns / rows; each sum stays sequential).
"""
import os
import time

import numpy as np

from . import oracle as orc


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def inject(C, seed, counts, offsets, mode, lo, hi):
    """The reference's fault of one iteration (pipeline/passes.cuh:149-170,
    kernels/swifi.cuh:61-114) applied to C in place; returns the fragment (-1:
    none)."""
    if mode not in ("add", "swifi"):
        return -1
    frag = orc.inject_frag(seed, len(counts))
    Cf = C[:, offsets[frag]:]
    if mode == "add":
        r, c, _ = orc.inject_position(seed, frag, C.shape[0], counts[frag])
        Cf[r, c] = np.float32(Cf[r, c] + np.float32(1.0e6))
    else:
        r, c, b = orc.inject_position(seed, frag, C.shape[0], counts[frag], lo, hi)
        Cf.view(np.uint32)[r, c] ^= np.uint32(1 << b)
    return frag


def protected_iterations(A, B, counts, offsets, tau, mode, zone, base_seed, rank, iters, golden=None,
                         time_budget_s=None):
    """Run up to `iters` protected iterations (stop early once time_budget_s is spent).

    Returns dict(iters, seconds, flops, cm, n_restored). Encode (colSumA,
    expectedRow) runs before the clock starts, as in the reference.
    """
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    counts = np.ascontiguousarray(counts, np.int32)
    offsets = np.ascontiguousarray(offsets, np.int32)
    M_b, K = A.shape
    N_b = B.shape[1]
    F = len(counts)
    colSumA = orc.col_checksum_A(A)
    expRow = orc.expected_row(colSumA, B)
    lo, hi = orc.swifi_zone_range(zone)
    cm = np.zeros(4, np.int64)
    nr = 0
    done = 0
    t0 = time.perf_counter()
    for it in range(iters):
        C = np.matmul(A, B)
        frag = inject(C, orc.inject_seed(base_seed, rank, it), counts, offsets, mode, lo, hi)
        c4, n, _, _, _ = orc.verify_iteration(C, A, B, counts, offsets, expRow, tau, frag,
                                              mode in ("add", "swifi"), expCol=None, golden=golden)
        cm += c4
        nr += n
        done += 1
        if time_budget_s is not None and time.perf_counter() - t0 >= time_budget_s:
            break
    secs = time.perf_counter() - t0
    return dict(iters=done, seconds=secs, flops=2.0 * M_b * N_b * K * done, cm=cm.tolist(), n_restored=nr)


def abft_only(C_clean, A, B, counts, offsets, tau, mode, zone, base_seed, rank, time_budget_s=5.0, max_reps=5):
    """The ABFT work alone on the host cores, on a given fault-free C (e.g. the
    GPU's own SGEMM output): the encode (colSumA, expectedRow) once, then the
    verification of one iteration (that iteration's planted fault, actualRow +
    detect on every fragment and the reference's on-demand localisation and
    correction) repeated on fresh copies until time_budget_s is spent.

    Returns dict(encode_ms, verify_ms (mean per iteration), reps)."""
    C_clean = np.ascontiguousarray(C_clean, np.float32)
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    counts = np.ascontiguousarray(counts, np.int32)
    offsets = np.ascontiguousarray(offsets, np.int32)
    lo, hi = orc.swifi_zone_range(zone)
    t0 = time.perf_counter()
    expRow = orc.expected_row(orc.col_checksum_A(A), B)
    encode_s = time.perf_counter() - t0
    total, reps = 0.0, 0
    while reps < max_reps:
        C = C_clean.copy()
        frag = inject(C, orc.inject_seed(base_seed, rank, reps), counts, offsets, mode, lo, hi)
        t = time.perf_counter()
        orc.verify_iteration(C, A, B, counts, offsets, expRow, tau, frag, mode in ("add", "swifi"), expCol=None)
        total += time.perf_counter() - t
        reps += 1
        if total >= time_budget_s:
            break
    return dict(encode_ms=encode_s * 1e3, verify_ms=total / reps * 1e3, reps=reps)
