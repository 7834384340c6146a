"""Host helpers through the C ABI: inputs, grid geometry, thresholds, injection plan.

These mirror the reference's host code (core/common.cuh, distribution/grid.cuh,
main.cu, kernels/swifi.cuh) and are bit-identical to it.
"""
import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import INJECT_ADD, INJECT_NONE, INJECT_SWIFI, call, lib


def _iptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))


def _dptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def fill_random(n, seed, dist="uniform", out=None):
    """fill_random (core/common.cuh:57-61): mt19937_64 + uniform_real_distribution<float>(-1, 1).

    dist="normal" draws std::normal_distribution<float>(0, 1) instead.
    """
    out = np.empty(int(n), np.float32) if out is None else out
    assert out.dtype == np.float32 and out.flags.c_contiguous and out.size == int(n)
    call("abft_fill_random", out.ctypes.data, int(n), int(seed), 1 if dist == "normal" else 0)
    return out


def choose_grid(world):
    """choose_grid (distribution/grid.cuh:7-12): near-square Pr x Pc."""
    pr, pc = ctypes.c_int(), ctypes.c_int()
    call("abft_choose_grid", int(world), ctypes.byref(pr), ctypes.byref(pc))
    return pr.value, pc.value


def split_dim(total, parts):
    """split_dim (distribution/grid.cuh:15-28): the first total % parts parts get one more."""
    c = np.zeros(parts, np.int32)
    o = np.zeros(parts, np.int32)
    call("abft_split_dim", int(total), int(parts), _iptr(c), _iptr(o))
    return c, o


def frag_count(M, K, N, M_b, N_b, frags_per_rank=4, frag_cap=0):
    """Fragments per rank (main.cu:55-69)."""
    F = lib.abft_frag_count(int(M), int(K), int(N), int(M_b), int(N_b), int(frags_per_rank), int(frag_cap))
    if F < 1:
        raise ValueError("bad fragment parameters")
    return F


def c_pitch(n):
    """Row pitch (floats) the sessions allocate for an n-column C: n, or
    n + 32 when n * 4 bytes is a multiple of 64 KB (a fragment that is a
    quarter of a 64 KB row streams ~9 % slower through the verify kernel
    when every row starts at the same offset modulo 64 KB)."""
    ld = lib.abft_c_pitch(int(n))
    if ld < 1:
        raise ValueError(f"bad column count {n}")
    return int(ld)


@dataclass
class RankTile:
    """Geometry of one rank's tile on a Pr x Pc grid (main.cu:32-54)."""
    rank: int
    Pr: int
    Pc: int
    pr: int
    pc: int
    M_b: int
    N_b: int
    row_off: int
    col_off: int
    K: int
    F: int
    counts: np.ndarray
    offsets: np.ndarray


def rank_tile(M, K, N, Pr, Pc, rank, frags_per_rank=4, frag_cap=0):
    pr, pc = rank // Pc, rank % Pc
    rc, ro = split_dim(M, Pr)
    cc, co = split_dim(N, Pc)
    M_b, N_b = int(rc[pr]), int(cc[pc])
    F = frag_count(M, K, N, M_b, N_b, frags_per_rank, frag_cap)
    counts, offsets = split_dim(N_b, F)
    return RankTile(rank, Pr, Pc, pr, pc, M_b, N_b, int(ro[pr]), int(co[pc]), K, F, counts, offsets)


def matrix_inf_norm(M):
    M = np.ascontiguousarray(M, np.float32)
    return lib.abft_matrix_inf_norm(M.ctypes.data, M.shape[0], M.shape[1], M.shape[1])


def threshold_formula(k, nA, nB):
    return lib.abft_threshold_formula(int(k), float(nA), float(nB))


def frag_thresholds(A, B, counts, offsets, override=-1.0):
    """Per-fragment thresholds (main.cu:147-164); override > 0 replaces the formula."""
    counts = np.ascontiguousarray(counts, np.int32)
    offsets = np.ascontiguousarray(offsets, np.int32)
    out = np.zeros(len(counts), np.float64)
    if override > 0:
        call("abft_frag_thresholds", None, 0, 0, 0, None, 0, len(counts), _iptr(counts), _iptr(offsets),
             float(override), _dptr(out))
        return out
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    call("abft_frag_thresholds", A.ctypes.data, A.shape[0], A.shape[1], A.shape[1], B.ctypes.data, B.shape[1],
         len(counts), _iptr(counts), _iptr(offsets), -1.0, _dptr(out))
    return out


def relative_threshold(A, B, K, rel=1e-5):
    """The relative threshold rel * K * max|A| * max|B| of the benchmark workloads."""
    return float(rel) * float(K) * float(np.abs(A).max()) * float(np.abs(B).max())


def swifi_zone_range(zone):
    lo, hi = ctypes.c_int(), ctypes.c_int()
    call("abft_swifi_zone_range", zone.encode(), ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


MODES = {"none": INJECT_NONE, "add": INJECT_ADD, "swifi": INJECT_SWIFI}


def injection_plan_tile(seed, M_b, counts, offsets, mode, zone="any"):
    """Tile-uniform scheme: (frag, row, col, bit) from mt19937_64(seed), j uniform over the tile."""
    counts = np.ascontiguousarray(counts, np.int32)
    offsets = np.ascontiguousarray(offsets, np.int32)
    lo, hi = swifi_zone_range(zone)
    r = [ctypes.c_int() for _ in range(4)]
    call("abft_injection_plan_tile", int(seed), int(M_b), len(counts), _iptr(counts), _iptr(offsets),
         MODES[mode] if isinstance(mode, str) else int(mode), lo, hi, *[ctypes.byref(x) for x in r])
    return tuple(x.value for x in r)


def injection_plan(base_seed, rank, it, counts, M_b, mode, zone="any"):
    """(frag, row, col, bit) injected at iteration `it` (-1s when nothing is injected)."""
    counts = np.ascontiguousarray(counts, np.int32)
    lo, hi = swifi_zone_range(zone)
    r = [ctypes.c_int() for _ in range(4)]
    call("abft_injection_plan", int(base_seed), int(rank), int(it), len(counts), int(M_b), _iptr(counts),
         MODES[mode] if isinstance(mode, str) else int(mode), lo, hi, *[ctypes.byref(x) for x in r])
    return tuple(x.value for x in r)
