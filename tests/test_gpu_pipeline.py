"""GPU parity of the online pipeline (pass_online_loop) against the oracle.

The SGEMM is cuBLAS on the GPU; the oracle replays the reference's decision
path on the GPU's own fault-free C (every iteration recomputes the same C), so
every decision, counter, injection and final buffer must be bit-identical.
"""
import numpy as np
import pytest
import torch

from gpu_cases import tiles

pytestmark = pytest.mark.gpu


def make_session(abft, orc, M, K, N, F, seed_a=123456, seed_b=987654, tau=None, max_iters=64, dist="uniform"):
    A, B = tiles(orc, M, K, N, seed_a, seed_b, dist)
    counts, offsets = orc.split_dim(N, F)
    s = abft.OnlineSession(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), counts=counts, offsets=offsets,
                           max_iters=max_iters)
    if tau is None:
        tau = [abft.relative_threshold(A, B, K)] * F
    s.set_tau(tau)
    s.baseline(1)
    torch.cuda.synchronize()
    C_clean = s.C[0].cpu().numpy().copy()
    return s, A, B, counts, offsets, np.asarray(s.tau), C_clean


def compare(s, res, o, repeats, check_injections=True):
    assert res["cm"] == list(o["cm"])
    assert res["n_restored"] == o["n_restored"]
    n = min(repeats, s.max_iters)
    ec, er, rd = s.read_log(n)
    assert np.array_equal(ec, o["errcol"][:n])
    assert np.array_equal(er, o["errrow"][:n])
    assert np.array_equal(rd.view(np.uint64), o["rowdiff"][:n].view(np.uint64))
    if check_injections:
        inj, _ = s.read_injections(n)
        want = o["inj"][:n].copy()
        assert np.array_equal(inj[want[:, 0] >= 0], want[want[:, 0] >= 0])
    torch.cuda.synchronize()
    assert np.array_equal(s.C[0].cpu().numpy().view(np.uint32), o["buf0"].view(np.uint32))
    if repeats > 1:
        assert np.array_equal(s.C[1].cpu().numpy().view(np.uint32), o["buf1"].view(np.uint32))


@pytest.mark.parametrize("mode,zone", [("none", "any"), ("add", "any"), ("swifi", "any"), ("swifi", "exponent"),
                                       ("swifi", "sig_low"), ("swifi", "sign"), ("swifi", "sig_high")])
def test_online_1024_cube(mode, zone, abft, orc):
    """1024^3, F = 4, 10 iterations (the single-rank 1024^3 workload)."""
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 1024, 1024, 1024, 4)
    golden = torch.from_numpy(C0).cuda() if mode == "swifi" else None
    s.set_golden(golden)
    base = 123456 + 987654 + 2 * 31337
    res = s.online(mode, zone, base_seed=base, repeats=10, log=True)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, mode, zone, 1.0e6, base, 0, 10,
                        golden=C0 if mode == "swifi" else None)
    compare(s, res, o, 10)
    if mode == "add":
        assert res["cm"][0] == 10 and res["cm"][3] == 0  # every additive fault detected
    s.close()


@pytest.mark.parametrize("correct", ["inloop", "drain"])
def test_drain_equals_inloop(correct, abft, orc):
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 512, 384, 768, 4, 1, 2)
    s.set_golden(torch.from_numpy(C0).cuda())
    res = s.online("swifi", "exponent", base_seed=99, repeats=9, log=True, correct=correct)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "swifi", "exponent", 1.0e6, 99, 0, 9, golden=C0)
    compare(s, res, o, 9)
    s.close()


def test_uneven_fragments_and_rank(abft, orc):
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 1100, 300, 1030, 3, 5, 7)
    s.set_golden(torch.from_numpy(C0).cuda())
    res = s.online("swifi", "any", base_seed=4242, rank=5, repeats=12, log=True)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "swifi", "any", 1.0e6, 4242, 5, 12, golden=C0)
    compare(s, res, o, 12)
    s.close()


def test_formula_threshold_and_normal_inputs(abft, orc):
    """Reference default threshold (gamma_K formula) and normal(0,1) inputs."""
    M, K, N, F = 2048, 1024, 1024, 4
    A, B = tiles(orc, M, K, N, 21, 22, "normal")
    counts, offsets = orc.split_dim(N, F)
    tau = abft.frag_thresholds(A, B, counts, offsets)
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, M, K, N, F, 21, 22, tau=tau, dist="normal")
    res = s.online("add", base_seed=7, repeats=6, log=True)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "add", "any", 1.0e6, 7, 0, 6)
    compare(s, res, o, 6)
    s.close()


@pytest.mark.parametrize("M,K,N", [(16384, 4096, 1024), (1024, 16384, 16384)], ids=["tall", "wide"])
def test_workload_shapes_normal_inputs(M, K, N, abft, orc):
    """The non-square workload shapes with normal(0,1) inputs (tall: 16384 x
    1024 tile, K = 4096; wide: 1024 x 16384 tile, K = 16384), F = 4, threshold
    1e-5 * K * max|A| * max|B|: the reference's additive faults (+1e6) and the
    workload's +1.0 at a seeded tile-uniform (i, j). The reference cannot draw
    normal inputs, so the oracle replays every decision on the GPU's own C;
    counters, logs and final buffers must be bit-identical."""
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, M, K, N, 4, dist="normal", max_iters=8)
    # the wide tile's C rows are 64 KB: the session pads their pitch
    assert s.C[0].stride(0) == abft.c_pitch(N) == (N + 32 if N == 16384 else N)
    assert tau[0] == 1e-5 * K * float(np.abs(A).max()) * float(np.abs(B).max())
    res = s.online("add", base_seed=11, repeats=4, log=True)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "add", "any", 1.0e6, 11, 0, 4)
    compare(s, res, o, 4)
    assert res["cm"][0] == 4
    res = s.online("add", add_delta=1.0, base_seed=1, repeats=4, log=True, seed_scheme="tile")
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "add", "any", 1.0, 1, 0, 4, seed_scheme="tile")
    compare(s, res, o, 4)
    s.close()


def test_add_delta_one_restores_clean_c(abft, orc):
    """+1.0 faults (the 1024^3 workload's fault size) with a golden C: every
    fault is detected, located and corrected back to within tau of the
    fault-free value, bit-identically to the oracle."""
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 1024, 1024, 1024, 4, 0, 0)
    s.set_golden(torch.from_numpy(C0).cuda())
    res = s.online("add", add_delta=1.0, base_seed=1, repeats=10, log=True)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "add", "any", 1.0, 1, 0, 10, golden=C0)
    compare(s, res, o, 10)
    assert res["cm"][0] == 10 and res["n_restored"] == 10
    torch.cuda.synchronize()
    err = np.abs(s.C[1].cpu().numpy().astype(np.float64) - C0).max() / np.abs(C0).max()
    assert err <= 1e-5
    s.close()


def test_repeats_beyond_log_capacity(abft, orc):
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 256, 256, 512, 4, max_iters=4)
    res = s.online("add", base_seed=3, repeats=11, log=True)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "add", "any", 1.0e6, 3, 0, 11)
    compare(s, res, o, 11)
    s.close()


def test_baseline_and_run_host(abft, orc):
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 768, 512, 1024, 4, 31, 32)
    ms, hms = s.baseline(3)
    assert ms > 0 and hms > 0
    hA = torch.from_numpy(A).pin_memory()
    hB = torch.from_numpy(B).pin_memory()
    hC = torch.empty((768, 1024), dtype=torch.float32).pin_memory()
    res = s.run_host(hA, hB, hC, "add", base_seed=17, repeats=3)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "add", "any", 1.0e6, 17, 0, 3)
    assert res["cm"] == list(o["cm"])
    assert np.array_equal(hC.numpy().view(np.uint32), o["buf0"].view(np.uint32))
    assert res["e2e_ms"] > 0
    s.close()


@pytest.mark.parametrize("mode,correct,repeats", [("swifi", "inloop", 5), ("swifi", "drain", 5), ("add", "inloop", 4),
                                                  ("none", "inloop", 1)])
def test_run_host_overlapped_copies(mode, correct, repeats, abft, orc):
    """run_host uploads B one fragment at a time and (in-loop correction)
    downloads each final fragment as soon as it is checked: uneven fragments,
    every element of the host output written, repeated calls stay exact."""
    M, K, N, F = 1100, 300, 1030, 3
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, M, K, N, F, 5, 7, max_iters=8)
    golden = C0 if mode == "swifi" else None
    s.set_golden(torch.from_numpy(C0).cuda() if golden is not None else None)
    hA = torch.from_numpy(A).pin_memory()
    hB = torch.from_numpy(B).pin_memory()
    for trial in range(2):
        base = 41 + trial * 31337
        s.A.zero_()
        s.B.zero_()
        torch.cuda.synchronize()
        hC = torch.full((M, N), float("nan"), dtype=torch.float32).pin_memory()
        res = s.run_host(hA, hB, hC, mode, base_seed=base, rank=1, repeats=repeats, correct=correct)
        # drain correction ends with the same buffers as in-loop correction
        o = orc.online_loop(C0, A, B, counts, offsets, tau, mode, "any", 1.0e6, base, 1, repeats, golden=golden)
        assert res["cm"] == list(o["cm"])
        assert res["n_restored"] == o["n_restored"]
        want = o["buf0"] if (repeats - 1) % 2 == 0 else o["buf1"]
        assert np.array_equal(hC.numpy().view(np.uint32), want.view(np.uint32))
    s.close()


@pytest.mark.parametrize("kernel", ["ldg", "tma"])
@pytest.mark.parametrize("mode,zone,correct", [("swifi", "any", "inloop"), ("add", "any", "inloop"),
                                                ("none", "any", "inloop"), ("swifi", "exponent", "drain")])
def test_graph_mode_matches_oracle(mode, zone, correct, kernel, abft, orc):
    """The loop replayed as a CUDA graph (injection applied inside the verify
    kernel from the device plan table) gives the same decisions, logs and
    buffers, trial after trial with different seeds; with either verify body."""
    abft.set_verify_kernel(kernel)
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 1024, 512, 1024, 4, 3, 4, max_iters=12)
    golden = torch.from_numpy(C0).cuda() if mode == "swifi" else None
    s.set_golden(golden)
    for trial in range(3):
        base = 777 + trial * 31337
        res = s.online(mode, zone, base_seed=base, repeats=12, log=True, correct=correct, graph=True)
        o = orc.online_loop(C0, A, B, counts, offsets, tau, mode, zone, 1.0e6, base, 0, 12,
                            golden=C0 if mode == "swifi" else None)
        compare(s, res, o, 12)
        # localisation runs (as a conditional graph node) only for detected fragments
        detected = res["cm"][0] + res["cm"][2] if mode != "none" else 0
        drain_kernel = 1 if (mode != "none" and correct == "drain") else 0
        assert res["kernel_launches"] == 4 * 12 + detected + drain_kernel
    s.close()
    abft.set_verify_kernel("auto")


def test_graph_mode_uneven_and_small_fragments(abft, orc):
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 1100, 300, 1030, 3, 5, 7, max_iters=9)
    s.set_golden(torch.from_numpy(C0).cuda())
    res = s.online("swifi", "any", base_seed=91, rank=3, repeats=9, log=True, graph=True)
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "swifi", "any", 1.0e6, 91, 3, 9, golden=C0)
    compare(s, res, o, 9)
    with pytest.raises(abft.AbftError):
        s.online("add", repeats=10, graph=True)  # beyond the plan table
    s.close()


@pytest.mark.parametrize("graph", [False, True])
def test_tile_seed_scheme(graph, abft, orc):
    """1024^3 with +1.0 faults at (i, j) uniform over the tile from seed 1 + iteration."""
    s, A, B, counts, offsets, tau, C0 = make_session(abft, orc, 1024, 1024, 1024, 4, 0, 0, max_iters=10)
    s.set_golden(torch.from_numpy(C0).cuda())
    res = s.online("add", add_delta=1.0, base_seed=1, repeats=10, log=True, graph=graph, seed_scheme="tile")
    o = orc.online_loop(C0, A, B, counts, offsets, tau, "add", "any", 1.0, 1, 0, 10, golden=C0,
                        seed_scheme="tile")
    compare(s, res, o, 10)
    assert res["cm"][0] == 10 and res["n_restored"] == 10
    s.close()


@pytest.mark.parametrize("mode,correct,repeats", [("add", "inloop", 6), ("swifi", "drain", 5), ("swifi", "inloop", 5),
                                                  ("none", "inloop", 4)])
def test_run_host_steps(mode, correct, repeats, abft, orc):
    """Four steps on four different inputs in one run_host_steps call (inputs
    of step k+1 copied while step k computes, a second device copy of A and B
    reused from step 2 on): every step's counters and final C equal a
    separate run_host call on the same inputs and the oracle's replay on that
    step's own fault-free C, bit for bit."""
    M, K, N, F = 768, 512, 1024, 4
    s, A0, B0, counts, offsets, tau, _ = make_session(abft, orc, M, K, N, F, 31, 32)
    steps = [tiles(orc, M, K, N, 100 + k, 200 + k) for k in range(4)]
    seeds = [1000 + 31337 * k for k in range(4)]
    hAs = [torch.from_numpy(A).pin_memory() for A, _ in steps]
    hBs = [torch.from_numpy(B).pin_memory() for _, B in steps]
    want = []
    for k, (A, B) in enumerate(steps):
        # the oracle replays the step on the GPU's own fault-free C of its inputs
        s.A.copy_(hAs[k].cuda())
        s.B.copy_(hBs[k].cuda())
        torch.cuda.synchronize()  # the session's streams are not ordered after torch's
        s.baseline(1)
        torch.cuda.synchronize()
        clean = s.C[0].cpu().numpy().copy()
        o = orc.online_loop(clean, A, B, counts, offsets, tau, mode, "any", 1.0e6, seeds[k], 0, repeats)
        hC = torch.empty((M, N), dtype=torch.float32).pin_memory()
        r = s.run_host(hAs[k], hBs[k], hC, mode, "any", base_seed=seeds[k], repeats=repeats, correct=correct)
        assert r["cm"] == list(o["cm"])
        want.append((r, hC.numpy().copy(), o))
    hCs = [torch.zeros((M, N), dtype=torch.float32).pin_memory() for _ in range(4)]
    got, e2e = s.run_host_steps(hAs, hBs, hCs, seeds, mode, "any", repeats=repeats, correct=correct)
    assert e2e > 0 and len(got) == 4
    fin = "buf1" if (repeats - 1) & 1 else "buf0"
    for k in range(4):
        r, c_single, o = want[k]
        assert got[k]["cm"] == r["cm"] == list(o["cm"]), k
        assert got[k]["n_restored"] == r["n_restored"]
        assert got[k]["verify_launches"] == repeats * F
        h = hCs[k].numpy()
        assert np.array_equal(h.view(np.uint32), c_single.view(np.uint32)), k
        assert np.array_equal(h.view(np.uint32), o[fin].view(np.uint32)), k
    if mode != "none":
        assert sum(g["cm"][0] for g in got) > 0
    # a second call reuses the session's step resources; one host buffer may serve every step
    one = torch.zeros((M, N), dtype=torch.float32).pin_memory()
    got2, _ = s.run_host_steps(hAs[:3], hBs[:3], [one] * 3, seeds[:3], mode, "any", repeats=repeats, correct=correct)
    assert [g["cm"] for g in got2] == [g["cm"] for g in got[:3]]
    assert np.array_equal(one.numpy().view(np.uint32), hCs[2].numpy().view(np.uint32))
    # the workspace now holds the last step's checksums: an online call encodes its own inputs again
    s.A.copy_(hAs[0].cuda())
    s.B.copy_(hBs[0].cuda())
    torch.cuda.synchronize()
    res = s.online("add", base_seed=5, repeats=2)
    assert res["cm"][0] == 2 and res["cm"][2] == 0
    s.close()
