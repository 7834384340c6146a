"""One rank of the multi-GPU parity check (launched by torchrun from
tests/test_gpu_multi.py). Panels travel over NCCL from rank 0; every rank runs
the protected loop on its tile and checks its own decisions against the oracle;
rank 0 prints one JSON line with the all-reduced results."""
import importlib
import json
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = "asynchronous_abft_for_mpi-cuda_architectures_b200"


def main():
    import oracle
    abft = importlib.import_module(PKG)
    dmod = importlib.import_module(f"{PKG}.distributed")
    rank, world, local = dmod.init_from_env(timeout_s=120)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    grid = dmod.Grid2D(world, rank)
    M, K, N = grid.Pr * 640 + 3, 384, grid.Pc * 1030
    A_full = B_full = None
    if rank == 0:
        A_full = torch.from_numpy(abft.fill_random(M * K, 17).reshape(M, K)).to(dev)
        B_full = torch.from_numpy(abft.fill_random(K * N, 18).reshape(K, N)).to(dev)
    A, B = dmod.distribute_panels(grid, M, K, N, A_full, B_full, dev)
    t = abft.rank_tile(M, K, N, grid.Pr, grid.Pc, rank, 4)
    s = abft.OnlineSession(A, B, counts=t.counts, offsets=t.offsets, max_iters=8)
    tau = 1e-5 * K
    s.set_tau([tau] * t.F)
    s.baseline(1)
    torch.cuda.synchronize()
    C0 = s.C[0].cpu().numpy().copy()
    s.set_golden(torch.from_numpy(C0).to(dev))
    base = 4242
    res = s.online("swifi", "any", base_seed=base, rank=rank, repeats=8, log=True)
    An, Bn = A.cpu().numpy(), B.cpu().numpy()
    want = oracle.online_loop(C0, An, Bn, t.counts, t.offsets, np.full(t.F, tau), "swifi", "any", 1.0e6, base,
                              rank, 8, golden=C0)
    ec, er, rd = s.read_log(8)
    ok = (res["cm"] == list(want["cm"]) and res["n_restored"] == want["n_restored"]
          and np.array_equal(ec, want["errcol"]) and np.array_equal(er, want["errrow"])
          and np.array_equal(rd.view(np.uint64), want["rowdiff"].view(np.uint64)))
    # the stripes this rank received are the ones rank 0 generated
    A_ref = abft.fill_random(M * K, 17).reshape(M, K)[t.row_off:t.row_off + t.M_b]
    ok = ok and np.array_equal(An, A_ref)
    tot = dmod.allreduce(list(res["cm"]) + [res["n_restored"], int(ok)], "sum", dev)
    s.close()
    if rank == 0:
        print(json.dumps({"world": world, "grid": [grid.Pr, grid.Pc], "cm": tot[:4], "restored": tot[4],
                          "ranks_ok": tot[5]}), flush=True)
    dmod.shutdown()


if __name__ == "__main__":
    main()
