"""B200-native asynchronous ABFT layer around SGEMM.

The compute path is libabft_b200.so (hand-written sm_100a kernels, C ABI in
include/abft_b200.h, C++ pipeline around cuBLAS SGEMM). This package is the
Python front end: ctypes bindings, the per-rank OnlineSession and the
torch.distributed (NCCL) plumbing for multi-GPU runs. Importing it without the
built library raises ImportError; there is no CPU fallback.
"""
from ._lib import (ADD_FAULT_DELTA, CORRECT_DRAIN, CORRECT_INLOOP, DRIVER_PATH, HEADER_PATH, INJECT_ADD,
                   INJECT_NONE, INJECT_SWIFI, LIB_PATH, SIGNATURES, AbftError, call, lib)
from . import _lib, host
from .host import (c_pitch, choose_grid, fill_random, frag_count, frag_thresholds, injection_plan, rank_tile,
                   relative_threshold, split_dim, swifi_zone_range, threshold_formula)


VERIFY_KERNELS = {"auto": 0, "ldg": 1, "tma": 2}


def set_verify_kernel(which):
    """Verify body for every later verify launch in this process: "auto" (the
    body that is faster inside the protected loop: 128-bit loads), "ldg"
    (128-bit loads) or "tma" (bulk tensor copies through shared memory).
    Returns the previous setting."""
    prev = lib.abft_set_verify_kernel(VERIFY_KERNELS[which])
    if prev < 0:
        raise AbftError("abft_set_verify_kernel", prev, _lib.last_error())
    return {v: k for k, v in VERIFY_KERNELS.items()}[prev]


__all__ = [
    "ADD_FAULT_DELTA", "CORRECT_DRAIN", "CORRECT_INLOOP", "DRIVER_PATH", "HEADER_PATH", "INJECT_ADD", "INJECT_NONE",
    "INJECT_SWIFI", "LIB_PATH", "SIGNATURES", "AbftError", "lib", "host", "choose_grid", "fill_random",
    "c_pitch", "frag_count", "frag_thresholds", "injection_plan", "rank_tile", "relative_threshold", "split_dim",
    "swifi_zone_range", "threshold_formula", "call", "set_verify_kernel", "VERIFY_KERNELS",
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
