"""ctypes binding of libabft_b200.so (the C ABI declared in include/abft_b200.h).

The shared library is built in-tree by build.py. There is no fallback: if the
library is missing or fails to load, importing this package raises.
"""
import ctypes
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libabft_b200.so")
DRIVER_PATH = os.path.join(PKG_DIR, "abft_gemm")
HEADER_PATH = os.path.join(os.path.dirname(PKG_DIR), "include", "abft_b200.h")

ABFT_OK = 0
ABFT_ERR_ARG = -1
ABFT_ERR_CUDA = -2
ABFT_ERR_CUBLAS = -3
ABFT_ERR_STATE = -4

INJECT_NONE = 0
INJECT_ADD = 1
INJECT_SWIFI = 2
CORRECT_INLOOP = 0
CORRECT_DRAIN = 1
ADD_FAULT_DELTA = 1.0e6


class AbftError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, fn, rc, msg):
        super().__init__(f"{fn} failed ({rc}): {msg}")
        self.rc = rc


class SessionCfg(ctypes.Structure):
    _fields_ = [
        ("M_b", ctypes.c_int), ("N_b", ctypes.c_int), ("K", ctypes.c_int), ("F", ctypes.c_int),
        ("counts", ctypes.POINTER(ctypes.c_int)), ("offsets", ctypes.POINTER(ctypes.c_int)),
        ("dA", ctypes.c_void_p), ("lda", ctypes.c_int64),
        ("dB", ctypes.c_void_p), ("ldb", ctypes.c_int64),
        ("dC0", ctypes.c_void_p), ("dC1", ctypes.c_void_p), ("ldc", ctypes.c_int64),
        ("verify_priority", ctypes.c_int), ("max_iters", ctypes.c_int),
    ]


class OnlineArgs(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int), ("zone_lo", ctypes.c_int), ("zone_hi", ctypes.c_int),
        ("add_delta", ctypes.c_float), ("base_seed", ctypes.c_uint64), ("rank", ctypes.c_int),
        ("repeats", ctypes.c_int), ("correct_mode", ctypes.c_int), ("log", ctypes.c_int),
        ("profile", ctypes.c_int), ("graph", ctypes.c_int), ("seed_scheme", ctypes.c_int),
    ]


class OnlineResult(ctypes.Structure):
    _fields_ = [
        ("device_ms", ctypes.c_double), ("host_ms", ctypes.c_double), ("cm", ctypes.c_int * 4),
        ("n_restored", ctypes.c_int), ("kernel_launches", ctypes.c_int), ("verify_launches", ctypes.c_int),
        ("verify_ms_sum", ctypes.c_double), ("verify_ms_max", ctypes.c_double),
    ]


class Timing(ctypes.Structure):
    _fields_ = [("min_ms", ctypes.c_double), ("median_ms", ctypes.c_double), ("mean_ms", ctypes.c_double),
                ("max_ms", ctypes.c_double), ("n_samples", ctypes.c_int)]


class Metrics(ctypes.Structure):
    _fields_ = [
        ("scheme", ctypes.c_char * 16), ("inject", ctypes.c_char * 16), ("swifi_zone", ctypes.c_char * 16),
        ("baseline_only", ctypes.c_int), ("calibrate", ctypes.c_int),
        ("M", ctypes.c_int), ("K", ctypes.c_int), ("N", ctypes.c_int), ("Pr", ctypes.c_int), ("Pc", ctypes.c_int),
        ("frags_per_rank", ctypes.c_int), ("num_fragments_total", ctypes.c_int), ("repeats", ctypes.c_int),
        ("threshold_used", ctypes.c_double), ("baseline", Timing), ("protected_", Timing),
        ("cm", ctypes.c_int * 4), ("n_restored", ctypes.c_int),
        ("calib_max_diff", ctypes.c_double), ("calib_safety_factor", ctypes.c_double),
        ("calib_suggested_tau", ctypes.c_double),
        ("overhead_pct", ctypes.c_double), ("recall", ctypes.c_double), ("precision", ctypes.c_double),
        ("correction_precision_pct", ctypes.c_double),
        ("baseline_gflops_min", ctypes.c_double), ("baseline_gflops_median", ctypes.c_double),
        ("baseline_gflops_mean", ctypes.c_double), ("baseline_gflops_max", ctypes.c_double),
        ("protected_gflops_min", ctypes.c_double), ("protected_gflops_median", ctypes.c_double),
        ("protected_gflops_mean", ctypes.c_double), ("protected_gflops_max", ctypes.c_double),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64
_D = ctypes.c_double
_F = ctypes.c_float
_IP = ctypes.POINTER(ctypes.c_int)
_DP = ctypes.POINTER(ctypes.c_double)

# name -> (restype, argtypes). Every symbol of include/abft_b200.h.
SIGNATURES = {
    "abft_last_error": (ctypes.c_char_p, []),
    "abft_version": (_I, []),
    "abft_fill_random": (_I, [_P, _I64, _U64, _I]),
    "abft_choose_grid": (_I, [_I, _IP, _IP]),
    "abft_split_dim": (_I, [_I, _I, _IP, _IP]),
    "abft_frag_count": (_I, [_I, _I, _I, _I, _I, _I, _I64]),
    "abft_c_pitch": (_I64, [_I]),
    "abft_matrix_inf_norm": (_D, [_P, _I, _I, _I64]),
    "abft_threshold_formula": (_D, [_I, _D, _D]),
    "abft_frag_thresholds": (_I, [_P, _I, _I, _I64, _P, _I64, _I, _IP, _IP, _D, _DP]),
    "abft_swifi_zone_range": (_I, [ctypes.c_char_p, _IP, _IP]),
    "abft_injection_plan": (_I, [_U64, _I, _I, _I, _I, _IP, _I, _I, _I, _IP, _IP, _IP, _IP]),
    "abft_injection_plan_tile": (_I, [_U64, _I, _I, _IP, _IP, _I, _I, _I, _IP, _IP, _IP, _IP]),
    "abft_ws_bytes": (ctypes.c_size_t, [_I, _I, _I, _I, _IP, _I]),
    "abft_ws_create": (_I, [_I, _I, _I, _I, _IP, _IP, _I, _P, ctypes.c_size_t, ctypes.POINTER(_P)]),
    "abft_ws_destroy": (_I, [_P]),
    "abft_ws_reset_counters": (_I, [_P, _P]),
    "abft_ws_counters_device": (_P, [_P]),
    "abft_ws_read_counters": (_I, [_P, _IP, _IP]),
    "abft_ws_read_log": (_I, [_P, _I, _IP, _IP, _DP]),
    "abft_ws_read_checksums": (_I, [_P, _DP, _DP, _DP, _DP]),
    "abft_encode": (_I, [_P, _P, _I64, _P, _I64, _P]),
    "abft_verify": (_I, [_P, _P, _I64, _I, _D, _I, _I, _P]),
    "abft_calibrate": (_I, [_P, _P, _I64, _I, _P, _P]),
    "abft_verify_noalloc": (_I, [_P, _I64, _I, _I, _P, _D, _I, _P, _P, _P, _P]),
    "abft_set_verify_kernel": (_I, [_I]),
    "abft_set_wait_limit": (_I, [_I]),
    "abft_localize_correct": (_I, [_P, _P, _I64, _I, _D, _I, _P, _I64, _I, _I, _P]),
    "abft_drain": (_I, [_P, _P, _P, _I64, _P, _I64, _I, _P]),
    "abft_inject_add": (_I, [_P, _I64, _I, _I, _F, _P]),
    "abft_inject_bitflip": (_I, [_P, _I64, _I, _I, _I, _P]),
    "abft_sgemm": (_I, [_P, _P, _I, _P, _I, _P, _I, _I, _I, _I]),
    "abft_session_create": (_I, [ctypes.POINTER(SessionCfg), ctypes.POINTER(_P)]),
    "abft_session_destroy": (_I, [_P]),
    "abft_session_ws": (_P, [_P]),
    "abft_session_set_tau": (_I, [_P, _DP]),
    "abft_session_set_golden": (_I, [_P, _P, _I64]),
    "abft_session_encode": (_I, [_P, _DP]),
    "abft_session_baseline": (_I, [_P, _I, _I, _DP, _DP]),
    "abft_session_baseline_monolithic": (_I, [_P, _I, _I, _DP, _DP]),
    "abft_session_online": (_I, [_P, ctypes.POINTER(OnlineArgs), ctypes.POINTER(OnlineResult)]),
    "abft_session_read_injections": (_I, [_P, _I, _IP, ctypes.POINTER(ctypes.c_float)]),
    "abft_session_run_host": (_I, [_P, _P, _P, _P, ctypes.POINTER(OnlineArgs), ctypes.POINTER(OnlineResult),
                                   _DP]),
    "abft_session_run_host_steps": (_I, [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P),
                                         ctypes.POINTER(OnlineArgs), ctypes.POINTER(_U64),
                                         ctypes.POINTER(OnlineResult), _DP]),
    "abft_stats_of": (_I, [_DP, _I, ctypes.POINTER(Timing)]),
    "abft_metrics_finalize": (_I, [ctypes.POINTER(Metrics)]),
    "abft_metrics_report": (_I, [ctypes.POINTER(Metrics), ctypes.c_char_p, ctypes.c_size_t]),
    "abft_metrics_csv_append": (_I, [ctypes.POINTER(Metrics), ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python {os.path.join(PKG_DIR, 'build.py')}` "
            "(or __graft_entry__.build()). There is no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error():
    msg = lib.abft_last_error()
    return msg.decode() if msg else ""


def check(rc, fn="abft call"):
    if rc != ABFT_OK:
        raise AbftError(fn, rc, last_error())
    return rc


def call(name, *args):
    """Call C-ABI function `name`, raising AbftError on a negative status."""
    rc = getattr(lib, name)(*args)
    check(rc, name)
    return rc
