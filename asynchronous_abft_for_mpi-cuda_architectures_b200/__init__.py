"""B200-native asynchronous ABFT layer around SGEMM.

The compute path is libabft_b200.so (hand-written sm_100a kernels, C ABI in
include/abft_b200.h, C++ pipeline around cuBLAS SGEMM). This package is the
Python front end: ctypes bindings, the per-rank OnlineSession and the
torch.distributed (NCCL) plumbing for multi-GPU runs. Importing it without the
built library raises ImportError; there is no CPU fallback.
"""
from ._lib import (ADD_FAULT_DELTA, CORRECT_DRAIN, CORRECT_INLOOP, DRIVER_PATH, HEADER_PATH, INJECT_ADD,
                   INJECT_NONE, INJECT_SWIFI, LIB_PATH, SIGNATURES, AbftError, lib)
from . import host
from .host import (choose_grid, fill_random, frag_count, frag_thresholds, injection_plan, rank_tile,
                   relative_threshold, split_dim, swifi_zone_range, threshold_formula)

__all__ = [
    "ADD_FAULT_DELTA", "CORRECT_DRAIN", "CORRECT_INLOOP", "DRIVER_PATH", "HEADER_PATH", "INJECT_ADD", "INJECT_NONE",
    "INJECT_SWIFI", "LIB_PATH", "SIGNATURES", "AbftError", "lib", "host", "choose_grid", "fill_random",
    "frag_count", "frag_thresholds", "injection_plan", "rank_tile", "relative_threshold", "split_dim",
    "swifi_zone_range", "threshold_formula",
]


def __getattr__(name):
    # torch-dependent parts load lazily so that host helpers work without CUDA
    if name in ("OnlineSession",):
        from .session import OnlineSession
        return OnlineSession
    if name in ("kernels", "session", "distributed"):
        import importlib
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
