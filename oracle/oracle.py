"""ctypes/numpy front end of the CPU oracle (oracle/abft_oracle.cpp).

TEST INFRASTRUCTURE ONLY (the tests' reference of correctness, and the timed
CPU arm of bench.py). The arithmetic lives in the C++ file, which restates the
reference's kernels in the reference's evaluation order; this module only
marshals numpy arrays.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
REF_DIR = os.path.join(_HERE, "_ref")

_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_longlong
_U64 = ctypes.c_uint64
_D = ctypes.c_double
_F = ctypes.c_float

_SIGS = {
    "oracle_fill_random": (None, [_P, _L, _U64, _I]),
    "oracle_choose_grid": (None, [_I, _P, _P]),
    "oracle_split_dim": (None, [_I, _I, _P, _P]),
    "oracle_frag_count": (_I, [_I, _I, _I, _I, _I, _I, _L]),
    "oracle_matrix_inf_norm": (_D, [_P, _I, _I, _L]),
    "oracle_threshold_formula": (_D, [_I, _D, _D]),
    "oracle_frag_thresholds": (None, [_P, _I, _I, _L, _P, _L, _I, _P, _P, _D, _P]),
    "oracle_col_checksum_A": (None, [_P, _L, _I, _I, _P]),
    "oracle_expected_row": (None, [_P, _P, _L, _I, _I, _P]),
    "oracle_row_checksum_B": (None, [_P, _L, _I, _I, _P]),
    "oracle_expected_col": (None, [_P, _L, _P, _I, _I, _P]),
    "oracle_actual_row": (None, [_P, _L, _I, _I, _P]),
    "oracle_actual_col": (None, [_P, _L, _I, _I, _P]),
    "oracle_argmax256": (_I, [_P, _P, _I, _D]),
    "oracle_detect_row": (None, [_P, _P, _I, _D, _I, _P, _P, _P]),
    "oracle_locate_correct": (_I, [_P, _P, _I, _D, _I, _D, _P, _L, _P, _L, _I, _I, _P]),
    "oracle_swifi_zone_range": (None, [ctypes.c_char_p, _P, _P]),
    "oracle_inject_seed": (_U64, [_U64, _I, _I]),
    "oracle_inject_frag": (_I, [_U64, _I]),
    "oracle_inject_position": (None, [_U64, _I, _I, _I, _I, _I, _P, _P, _P]),
    "oracle_inject_position_tile": (None, [_U64, _I, _I, _P, _P, _I, _I, _P, _P, _P, _P]),
    "oracle_inject_add": (None, [_P, _L, _I, _I, _F]),
    "oracle_inject_bitflip": (None, [_P, _L, _I, _I, _I]),
    "oracle_encode": (None, [_P, _L, _P, _L, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
    "oracle_verify_iteration": (None, [_P, _L, _P, _L, _P, _L, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I,
                                       _P, _L, _P, _P, _P, _P, _P]),
    "oracle_online_loop": (None, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _I, _I, _I, _F, _U64, _I, _I,
                                  _P, _P, _P, _P, _P, _P, _P, _P, _P, _I]),
}


def build():
    """Compile liboracle.so (and the reference tools when the checkout exists)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            subprocess.run(["make", "-s", "-C", _HERE, "oracle"], check=True)
        _lib = ctypes.CDLL(_LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- inputs ---
def fill_random(n, seed, dist="uniform"):
    out = np.empty(int(n), dtype=np.float32)
    lib().oracle_fill_random(_p(out), int(n), int(seed), 1 if dist == "normal" else 0)
    return out


def choose_grid(world):
    pr, pc = _I(), _I()
    lib().oracle_choose_grid(int(world), ctypes.byref(pr), ctypes.byref(pc))
    return pr.value, pc.value


def split_dim(total, parts):
    c = np.zeros(parts, np.int32)
    o = np.zeros(parts, np.int32)
    lib().oracle_split_dim(int(total), int(parts), _p(c), _p(o))
    return c, o


def frag_count(M, K, N, M_b, N_b, frags_per_rank, frag_cap=0):
    return lib().oracle_frag_count(M, K, N, M_b, N_b, frags_per_rank, frag_cap)


def matrix_inf_norm(M):
    M = _c(M, np.float32)
    return lib().oracle_matrix_inf_norm(_p(M), M.shape[0], M.shape[1], M.shape[1])


def threshold_formula(k, nA, nB):
    return lib().oracle_threshold_formula(int(k), float(nA), float(nB))


def frag_thresholds(A, B, counts, offsets, override=-1.0):
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    counts = _c(counts, np.int32)
    offsets = _c(offsets, np.int32)
    out = np.zeros(len(counts), np.float64)
    lib().oracle_frag_thresholds(_p(A), A.shape[0], A.shape[1], A.shape[1], _p(B), B.shape[1], len(counts),
                                 _p(counts), _p(offsets), float(override), _p(out))
    return out


# ---------------------------------------------------------------- encode ---
def col_checksum_A(A):
    A = _c(A, np.float32)
    out = np.zeros(A.shape[1], np.float64)
    lib().oracle_col_checksum_A(_p(A), A.shape[1], A.shape[0], A.shape[1], _p(out))
    return out


def expected_row(colSumA, B):
    """expectedRow over every column of B (K x N)."""
    colSumA = _c(colSumA, np.float64)
    B = _c(B, np.float32)
    out = np.zeros(B.shape[1], np.float64)
    lib().oracle_expected_row(_p(colSumA), _p(B), B.shape[1], B.shape[0], B.shape[1], _p(out))
    return out


def row_checksum_B(B):
    B = _c(B, np.float32)
    out = np.zeros(B.shape[0], np.float64)
    lib().oracle_row_checksum_B(_p(B), B.shape[1], B.shape[0], B.shape[1], _p(out))
    return out


def expected_col(A, rowSumB):
    A = _c(A, np.float32)
    rowSumB = _c(rowSumB, np.float64)
    out = np.zeros(A.shape[0], np.float64)
    lib().oracle_expected_col(_p(A), A.shape[1], _p(rowSumB), A.shape[0], A.shape[1], _p(out))
    return out


def encode(A, B, counts, offsets):
    """colSumA[K], expRow[N_b], rowSumB[F,K], expCol[F,M_b] for one rank tile."""
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    counts = _c(counts, np.int32)
    offsets = _c(offsets, np.int32)
    M_b, K = A.shape
    N_b = B.shape[1]
    F = len(counts)
    colSumA = np.zeros(K, np.float64)
    expRow = np.zeros(N_b, np.float64)
    rowSumB = np.zeros((F, K), np.float64)
    expCol = np.zeros((F, M_b), np.float64)
    lib().oracle_encode(_p(A), K, _p(B), N_b, M_b, K, F, _p(counts), _p(offsets), _p(colSumA), _p(expRow),
                        _p(rowSumB), _p(expCol))
    return colSumA, expRow, rowSumB, expCol


# ---------------------------------------------------------------- verify ---
def actual_row(C):
    C = _c(C, np.float32)
    out = np.zeros(C.shape[1], np.float64)
    lib().oracle_actual_row(_p(C), C.shape[1], C.shape[0], C.shape[1], _p(out))
    return out


def actual_col(C):
    C = _c(C, np.float32)
    out = np.zeros(C.shape[0], np.float64)
    lib().oracle_actual_col(_p(C), C.shape[1], C.shape[0], C.shape[1], _p(out))
    return out


def argmax256(expected, actual, tau):
    e = _c(expected, np.float64)
    a = _c(actual, np.float64)
    return lib().oracle_argmax256(_p(e), _p(a), len(e), float(tau))


def detect_row(expected, actual, tau, injected):
    e = _c(expected, np.float64)
    a = _c(actual, np.float64)
    ec, rd = _I(), _D()
    cm = np.zeros(4, np.int32)
    lib().oracle_detect_row(_p(e), _p(a), len(e), float(tau), int(injected), ctypes.byref(ec), ctypes.byref(rd),
                            _p(cm))
    return ec.value, rd.value, cm


def swifi_zone_range(zone):
    lo, hi = _I(), _I()
    lib().oracle_swifi_zone_range(zone.encode(), ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def inject_seed(base_seed, rank, it):
    return lib().oracle_inject_seed(int(base_seed), int(rank), int(it))


def inject_frag(seed, F):
    return lib().oracle_inject_frag(int(seed), int(F))


def inject_position(seed, frag, M_b, N_f, lo=1, hi=0):
    r, c, b = _I(), _I(), _I()
    lib().oracle_inject_position(int(seed), int(frag), int(M_b), int(N_f), int(lo), int(hi), ctypes.byref(r),
                                 ctypes.byref(c), ctypes.byref(b))
    return r.value, c.value, b.value


def inject_position_tile(seed, M_b, counts, offsets, lo=1, hi=0):
    counts = _c(counts, np.int32)
    offsets = _c(offsets, np.int32)
    f, r, c, b = _I(), _I(), _I(), _I()
    lib().oracle_inject_position_tile(int(seed), int(M_b), len(counts), _p(counts), _p(offsets), int(lo), int(hi),
                                      ctypes.byref(f), ctypes.byref(r), ctypes.byref(c), ctypes.byref(b))
    return f.value, r.value, c.value, b.value


def verify_iteration(C, A, B, counts, offsets, expRow, tau, inject_frag=-1, do_localize=True, expCol=None,
                     golden=None):
    """Verify half of one online iteration on a rank tile C (modified in place).

    Returns (cm[4], n_restored, errcol[F], errrow[F], rowdiff[F]).
    """
    assert C.dtype == np.float32 and C.flags.c_contiguous
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    counts = _c(counts, np.int32)
    offsets = _c(offsets, np.int32)
    expRow = _c(expRow, np.float64)
    tau = _c(tau, np.float64)
    F = len(counts)
    M_b, N_b = C.shape
    K = A.shape[1]
    cm = np.zeros(4, np.int32)
    nr = np.zeros(1, np.int32)
    ec = np.zeros(F, np.int32)
    er = np.zeros(F, np.int32)
    rd = np.zeros(F, np.float64)
    expCol = _c(expCol, np.float64) if expCol is not None else None
    golden = _c(golden, np.float32) if golden is not None else None
    lib().oracle_verify_iteration(_p(C), N_b, _p(A), K, _p(B), B.shape[1], M_b, K, F, _p(counts), _p(offsets),
                                  _p(expRow), _p(expCol), _p(tau), int(inject_frag), int(bool(do_localize)),
                                  _p(golden), N_b, _p(cm), _p(nr), _p(ec), _p(er), _p(rd))
    return cm, int(nr[0]), ec, er, rd


MODES = {"none": 0, "add": 1, "swifi": 2}


def online_loop(C_clean, A, B, counts, offsets, tau, mode="none", zone="any", add_delta=1.0e6, base_seed=0,
                rank=0, repeats=1, golden=None, seed_scheme="reference"):
    """Decision path of the reference's online loop for one rank, on the CPU."""
    C_clean = _c(C_clean, np.float32)
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    counts = _c(counts, np.int32)
    offsets = _c(offsets, np.int32)
    tau = _c(tau, np.float64)
    M_b, N_b = C_clean.shape
    K = A.shape[1]
    F = len(counts)
    lo, hi = swifi_zone_range(zone)
    buf0 = np.zeros_like(C_clean)
    buf1 = np.zeros_like(C_clean)
    cm = np.zeros(4, np.int32)
    nr = np.zeros(1, np.int32)
    inj = np.full((repeats, 4), -1, np.int32)
    ec = np.zeros((repeats, F), np.int32)
    er = np.zeros((repeats, F), np.int32)
    rd = np.zeros((repeats, F), np.float64)
    golden = _c(golden, np.float32) if golden is not None else None
    lib().oracle_online_loop(_p(C_clean), _p(A), _p(B), M_b, K, N_b, F, _p(counts), _p(offsets), _p(tau),
                             MODES[mode], lo, hi, float(add_delta), int(base_seed), int(rank), int(repeats),
                             _p(golden), _p(buf0), _p(buf1), _p(cm), _p(nr), _p(inj), _p(ec), _p(er), _p(rd),
                             1 if seed_scheme == "tile" else 0)
    return dict(buf0=buf0, buf1=buf1, cm=cm, n_restored=int(nr[0]), inj=inj, errcol=ec, errrow=er, rowdiff=rd)
