"""Multi-rank plumbing over torch.distributed (NCCL on GPUs, gloo on CPU).

Replaces the reference's host-staged MPI (distribution/grid.cuh:31-91,
metrics/metrics.cuh:67-102): A and B panels travel device to device, the
confusion matrix is summed and timings are max-reduced on device tensors.
Every rank must call these functions in the same order.
"""
import datetime
import os

import torch
import torch.distributed as dist

from . import host


def init_from_env(backend=None, timeout_s=120):
    """Initialise the default process group from torchrun's environment.

    Returns (rank, world, local_rank). A world of 1 needs no process group.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kw)
    return rank, world, local


class Grid2D:
    """Pr x Pc rank grid (main.cu:32-37) with the panel groups the distribution needs.

    a_groups[pr] holds rank 0 and the ranks of grid row pr (they receive A stripe pr);
    b_groups[pc] holds rank 0 and the ranks of grid column pc (B stripe pc). All ranks
    create every group, in the same order.
    """

    def __init__(self, world, rank, Pr=None, Pc=None):
        if Pr is None or Pc is None:
            Pr, Pc = host.choose_grid(world)
        if Pr * Pc != world:
            raise ValueError(f"grid {Pr}x{Pc} does not match world size {world}")
        self.Pr, self.Pc, self.world, self.rank = Pr, Pc, world, rank
        self.pr, self.pc = rank // Pc, rank % Pc
        self.a_groups, self.b_groups = [], []
        if world > 1 and dist.is_initialized():
            for pr in range(Pr):
                members = sorted({0} | {pr * Pc + c for c in range(Pc)})
                self.a_groups.append((members, dist.new_group(members)))
            for pc in range(Pc):
                members = sorted({0} | {r * Pc + pc for r in range(Pr)})
                self.b_groups.append((members, dist.new_group(members)))


def distribute_panels(grid, M, K, N, A_full=None, B_full=None, device=None):
    """Return this rank's A stripe (M_b x K) and B stripe (K x N_b) on `device`.

    Rank 0 passes the full row-major A (M x K) and B (K x N) as device tensors;
    the stripes are broadcast from rank 0 inside each panel group.
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    rc, ro = host.split_dim(M, grid.Pr)
    cc, co = host.split_dim(N, grid.Pc)
    M_b, N_b = int(rc[grid.pr]), int(cc[grid.pc])
    A_mine = B_mine = None
    for pr, (members, g) in enumerate(grid.a_groups or [([0], None)]):
        if grid.rank not in members:
            continue
        rows = int(rc[pr])
        if grid.rank == 0:
            buf = A_full[int(ro[pr]):int(ro[pr]) + rows].contiguous()
        else:
            buf = torch.empty((rows, K), dtype=torch.float32, device=device)
        if g is not None:
            dist.broadcast(buf, src=0, group=g)
        if pr == grid.pr:
            A_mine = buf
    for pc, (members, g) in enumerate(grid.b_groups or [([0], None)]):
        if grid.rank not in members:
            continue
        cols = int(cc[pc])
        if grid.rank == 0:
            buf = B_full[:, int(co[pc]):int(co[pc]) + cols].contiguous()
        else:
            buf = torch.empty((K, cols), dtype=torch.float32, device=device)
        if g is not None:
            dist.broadcast(buf, src=0, group=g)
        if pc == grid.pc:
            B_mine = buf
    assert A_mine is not None and A_mine.shape == (M_b, K)
    assert B_mine is not None and B_mine.shape == (K, N_b)
    return A_mine, B_mine


def allreduce(values, op="sum", device=None, dtype=torch.float64):
    """All-reduce a small list of numbers; identity without a process group."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(values)
    backend = dist.get_backend()
    dev = device if backend == "nccl" else torch.device("cpu")
    t = torch.tensor(list(values), dtype=dtype, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX)
    return t.cpu().tolist()


def barrier(device=None):
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[device.index if device is not None else torch.cuda.current_device()])
        else:
            dist.barrier()


def shutdown():
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
