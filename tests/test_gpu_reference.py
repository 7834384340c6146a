"""Pin the oracle (and the new kernels) against the reference's OWN kernels,
compiled from the reference sources for sm_100a (oracle/_ref/kernel_harness),
run on the GPU on identical inputs."""
import numpy as np
import pytest
import torch

import refharness
from gpu_cases import add_fault, flip, product_f64, tiles
from test_gpu_kernels import run_gpu_iteration, run_oracle_iteration

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refharness.available(), reason="oracle/_ref not built (make -C oracle ref)")]

CASES = [(64, 80, 48, 1), (257, 129, 515, 4), (1024, 512, 1024, 4), (600, 300, 1030, 3)]


def bits(a):
    return np.ascontiguousarray(a).view(np.uint64 if a.dtype == np.float64 else np.uint32)


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_kernels(case, orc):
    M, K, N, F = case
    A, B = tiles(orc, M, K, N, 41, 42)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    rng = np.random.default_rng(3)
    inj_f = F - 1
    r = int(rng.integers(0, M))
    c = int(offsets[inj_f] + rng.integers(0, counts[inj_f]))
    C = add_fault(C0, r, c, 2.0)
    tau = [1e-5 * K] * F
    injected = [1 if f == inj_f else 0 for f in range(F)]
    ref = run = refharness.run_verify(A, B, C, F, tau, injected, golden=C0)
    colSumA, expRow, rowSumB, expCol = orc.encode(A, B, counts, offsets)
    assert np.array_equal(bits(ref["colSumA"]), bits(colSumA))
    assert np.array_equal(bits(ref["expRow"]), bits(expRow))
    assert np.array_equal(bits(ref["actRow"]), bits(orc.actual_row(C)))
    o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, inj_f, golden=C0)
    assert list(run["errcol"]) == list(o["ec"])
    assert np.array_equal(bits(run["rowdiff"]), bits(o["rd"]))
    for f in range(F):
        if o["ec"][f] >= 0:  # the reference's localisation scratch is only valid after a detection
            assert np.array_equal(bits(ref["rowSumB"][f]), bits(rowSumB[f]))
            assert np.array_equal(bits(ref["expCol"][f]), bits(expCol[f]))
            assert np.array_equal(bits(ref["actCol"][f]), bits(orc.actual_col(C[:, offsets[f]:offsets[f] + counts[f]])))
    assert np.array_equal(bits(ref["C"]), bits(o["C"]))
    assert list(ref["cm"]) == list(o["cm"])
    assert int(ref["n_restored"][0]) == o["nr"]


@pytest.mark.parametrize("case", CASES[:3])
def test_new_kernels_match_reference_kernels(case, abft, orc):
    M, K, N, F = case
    A, B = tiles(orc, M, K, N, 43, 44)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    tau = [0.0] * F  # every noisy column is a candidate: the hardest arg-max
    injected = [0] * F
    ref = refharness.run_verify(A, B, C0, F, tau, injected, golden=None)
    g = run_gpu_iteration(abft, torch, A, B, C0, counts, offsets, tau, -1)
    assert list(g["ec"]) == list(ref["errcol"])
    assert np.array_equal(bits(g["rd"]), bits(ref["rowdiff"]))
    assert np.array_equal(bits(g["C"]), bits(ref["C"]))
    assert list(g["cm"]) == list(ref["cm"])


def test_exact_ties_match_reference(abft, orc):
    M, K, N, F = 600, 16, 1030, 2
    A = np.zeros((M, K), np.float32)
    _, B = tiles(orc, M, K, N)
    counts, offsets = orc.split_dim(N, F)
    C = np.zeros((M, N), np.float32)
    for k, c in enumerate([1, 2, 3, 258, 259]):
        C[(7 * k + 3) % M, c] = 3.0
    tau = [0.5] * F
    ref = refharness.run_verify(A, B, C, F, tau, [1, 0])
    g = run_gpu_iteration(abft, torch, A, B, C, counts, offsets, tau, 0)
    assert list(g["ec"]) == list(ref["errcol"])
    assert np.array_equal(bits(g["C"]), bits(ref["C"]))


@pytest.mark.parametrize("mode,zone", [("add", "any"), ("swifi", "any"), ("swifi", "exponent"), ("swifi", "sig_low")])
def test_injection_draws_match_reference(mode, zone, abft, orc):
    """The reference's injectors, run on the GPU, hit the element and bit that
    the new injection plan predicts."""
    M, N, F = 300, 260, 3
    C = orc.fill_random(M * N, 5).reshape(M, N)
    counts, offsets = orc.split_dim(N, F)
    for it in range(6):
        base = 1000 + it
        seed = orc.inject_seed(base, 0, it)
        frag = orc.inject_frag(seed, F)
        (row, col, bit), (before, after), Cout = refharness.run_inject(C, F, frag, seed, mode, zone)
        f, r, c, b = abft.injection_plan(base, 0, it, counts, M, mode, zone)
        assert (f, r, c) == (frag, row, col)
        if mode == "swifi":
            assert b == bit
            want = flip(C, r, offsets[f] + c, b)
        else:
            want = add_fault(C, r, offsets[f] + c, 1.0e6)
        assert np.array_equal(bits(Cout), bits(want))
