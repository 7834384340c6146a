"""Metrics, stdout report and CSV through the C ABI (metrics/metrics.cuh of the reference)."""
import ctypes

from ._lib import Metrics, Timing, call, lib


def stats_of(samples):
    """stats_of (core/common.cuh:86-106): min, median (sorted[n/2]), mean, max."""
    arr = (ctypes.c_double * len(samples))(*samples)
    t = Timing()
    call("abft_stats_of", arr, len(samples), ctypes.byref(t))
    return t


def make_metrics(scheme, inject, zone, baseline_only, calibrate, M, K, N, Pr, Pc, F, repeats, tau, baseline,
                 protected, cm, n_restored, calib=(0.0, 0.0, 0.0)):
    m = Metrics()
    m.scheme, m.inject, m.swifi_zone = scheme.encode(), inject.encode(), zone.encode()
    m.baseline_only, m.calibrate = int(baseline_only), int(calibrate)
    m.M, m.K, m.N, m.Pr, m.Pc = M, K, N, Pr, Pc
    m.frags_per_rank, m.num_fragments_total, m.repeats = F, Pr * Pc * F, repeats
    m.threshold_used = tau
    m.baseline, m.protected_ = baseline, protected
    for i in range(4):
        m.cm[i] = int(cm[i])
    m.n_restored = int(n_restored)
    m.calib_max_diff, m.calib_safety_factor, m.calib_suggested_tau = calib
    call("abft_metrics_finalize", ctypes.byref(m))
    return m


def report(m):
    n = lib.abft_metrics_report(ctypes.byref(m), None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    lib.abft_metrics_report(ctypes.byref(m), buf, n + 1)
    return buf.value.decode()


def csv_append(m, path, extra_header=None, extra_values=None):
    call("abft_metrics_csv_append", ctypes.byref(m), path.encode(),
         extra_header.encode() if extra_header else None, extra_values.encode() if extra_values else None)
