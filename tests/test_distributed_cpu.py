"""Multi-rank plumbing on CPU (gloo): panel distribution over the Pr x Pc grid
and the metric reductions, with world sizes 2, 3, 4, 6 and 8 (grids 1x2, 1x3,
2x2, 2x3, 2x4), tiles ragged where the sizes do not divide."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG_NAME, ROOT


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def worker(rank, world, port, M, K, N, q):
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        abft = importlib.import_module(PKG_NAME)
        dmod = importlib.import_module(f"{PKG_NAME}.distributed")
        r, w, _ = dmod.init_from_env(backend="gloo", timeout_s=60)
        grid = dmod.Grid2D(w, r)
        A_full = B_full = None
        if r == 0:
            A_full = torch.from_numpy(abft.fill_random(M * K, 1).reshape(M, K))
            B_full = torch.from_numpy(abft.fill_random(K * N, 2).reshape(K, N))
        A, B = dmod.distribute_panels(grid, M, K, N, A_full, B_full, device=torch.device("cpu"))
        t = abft.rank_tile(M, K, N, grid.Pr, grid.Pc, r)
        A_ref = abft.fill_random(M * K, 1).reshape(M, K)[t.row_off:t.row_off + t.M_b]
        B_ref = abft.fill_random(K * N, 2).reshape(K, N)[:, t.col_off:t.col_off + t.N_b]
        ok = np.array_equal(A.numpy(), A_ref) and np.array_equal(B.numpy(), B_ref)
        sums = dmod.allreduce([1, r, 10 * r], "sum")
        maxs = dmod.allreduce([float(r), -float(r)], "max")
        dmod.barrier()
        q.put((r, ok, sums, maxs, (grid.Pr, grid.Pc, grid.pr, grid.pc)))
        dmod.shutdown()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, repr(e), None, None))


@pytest.mark.parametrize("world,shape", [(2, (300, 40, 517)), (3, (97, 21, 302)), (4, (301, 33, 250)),
                                         (6, (301, 29, 1000)), (8, (257, 17, 130))])
def test_panels_and_reductions(world, shape):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, *shape, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    results.sort()
    for r, ok, sums, maxs, g in results:
        assert ok is True, (r, sums)
        assert sums == [world, sum(range(world)), 10 * sum(range(world))]
        assert maxs == [world - 1, 0.0]
    Pr, Pc = results[0][4][:2]
    assert Pr * Pc == world
