"""Seeded random parity sweep of the online loop (GPU) against the oracle:
random tile shapes (odd and tiny sizes included), fault modes, SWIFI zones,
correction modes, host-enqueued or graph loop and either verify body. Every
decision, counter, log entry and final buffer must be bit-identical."""
import numpy as np
import pytest
import torch

from gpu_cases import tiles

pytestmark = pytest.mark.gpu

ZONES = ["any", "sign", "exponent", "sig_high", "sig_low"]


def cases(n=64, seed=20261201):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        M = int(rng.choice([int(rng.integers(1, 40)), int(rng.integers(40, 1200))]))
        N = int(rng.choice([int(rng.integers(1, 40)), int(rng.integers(40, 1500))]))
        if i % 3 == 0:
            N = 4 * max(1, N // 4)  # 16-byte aligned rows: the vector and TMA paths
        K = int(rng.integers(1, 300))
        F = int(min(N, rng.integers(1, 6)))
        mode = str(rng.choice(["none", "add", "swifi"]))
        zone = str(rng.choice(ZONES)) if mode == "swifi" else "any"
        correct = str(rng.choice(["inloop", "drain"]))
        graph = bool(rng.integers(0, 2))
        kernel = str(rng.choice(["ldg", "tma"]))
        repeats = int(rng.integers(1, 7))
        out.append((i, M, K, N, F, mode, zone, correct, graph, kernel, repeats))
    return out


@pytest.mark.parametrize("case", cases(), ids=lambda c: f"case{c[0]}")
def test_random_online_loop(case, abft, orc):
    i, M, K, N, F, mode, zone, correct, graph, kernel, repeats = case
    prev = abft.set_verify_kernel(kernel)
    try:
        A, B = tiles(orc, M, K, N, 1000 + i, 2000 + i)
        counts, offsets = orc.split_dim(N, F)
        s = abft.OnlineSession(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), counts=counts,
                               offsets=offsets, max_iters=8)
        tau = [max(abft.relative_threshold(A, B, K), 1e-30)] * F
        s.set_tau(tau)
        s.baseline(1)
        torch.cuda.synchronize()
        C0 = s.C[0].cpu().numpy().copy()
        golden = C0 if mode == "swifi" else None
        s.set_golden(torch.from_numpy(C0).cuda() if golden is not None else None)
        base = 777 + 31 * i
        res = s.online(mode, zone, base_seed=base, rank=i % 3, repeats=repeats, log=True, correct=correct,
                       graph=graph)
        o = orc.online_loop(C0, A, B, counts, offsets, np.asarray(s.tau), mode, zone, 1.0e6, base, i % 3, repeats,
                            golden=golden)
        assert res["cm"] == list(o["cm"])
        assert res["n_restored"] == o["n_restored"]
        ec, er, rd = s.read_log(repeats)
        assert np.array_equal(ec, o["errcol"]) and np.array_equal(er, o["errrow"])
        assert np.array_equal(rd.view(np.uint64), o["rowdiff"].view(np.uint64))
        torch.cuda.synchronize()
        assert np.array_equal(s.C[0].cpu().numpy().view(np.uint32), o["buf0"].view(np.uint32))
        if repeats > 1:
            assert np.array_equal(s.C[1].cpu().numpy().view(np.uint32), o["buf1"].view(np.uint32))
        s.close()
    finally:
        abft.set_verify_kernel(prev)
