"""CPU property check of the summation rules that make the parallel checksum
kernels bit-exact (csrc/abft_kernels.cu: cert_window and run_shortcut),
restated here in Python and tested against IEEE double arithmetic on
adversarial float32 data.

The reference sums each column sequentially in double
(kernels/abft_stepwise.cuh:43-52). The kernels sum in parallel, in an order
fixed by the launch, and rely on two claims:

* cert_window: with T the float32 sum of |x| (any order) and p the ulp
  exponent of the smallest nonzero |x|, T * (1 + 4n 2^-24) <= 2^(p+53) makes
  every order's double sum equal the sequential one bit for bit (window 0);
  otherwise |d_seq - d| <= window for d = |S - E| computed from any order's
  sum S and any expected value E.
* run_shortcut: a run of terms may be added to the sequential sum s in one
  step when (i) s and every term are multiples of 2^p and |s| + sum|x| stays
  within 2^(p+53) (no partial sum rounds), or (ii) every |x| < ulp(s) / 4
  (every add rounds back to s).
"""
import math
import struct

import numpy as np

TWO = 2.0


def f32_bits(x):
    return np.asarray(x, np.float32).view(np.uint32)


def seq_sum(xs, s=0.0):
    for v in xs:
        s = s + float(v)
    return s


def cert_window(S, T, mbm1, n, d):
    """Python restatement of cert_window (double S, float T, uint32 mbm1)."""
    if not math.isfinite(S):
        return 0.0
    nz = (int(mbm1) + 1) & 0xffffffff
    if nz == 0:
        return 0.0
    if n > (1 << 21):
        return math.inf
    e = max(nz >> 23, 1)
    tb = float(T) * (1.0 + 4.0 * n * TWO ** -24)
    limit = TWO ** (e - 97)
    if tb <= limit:
        return 0.0
    E = 2.0 * n * TWO ** -53 * tb * (1.0 + TWO ** -30)
    w = E * (1.0 + TWO ** -40) + d * TWO ** -51 + TWO ** -1000
    return w if w > 0.0 else math.inf


def lowbit_exp(s):
    b = struct.unpack("<Q", struct.pack("<d", s))[0]
    e = (b >> 52) & 0x7ff
    m = b & ((1 << 52) - 1)
    if e == 0:
        return -1074 + ((m & -m).bit_length() - 1)
    m |= 1 << 52
    return (e - 1075) + ((m & -m).bit_length() - 1)


def run_shortcut(s, S, T, amax, mbm1):
    """Python restatement of run_shortcut: (applied, new s)."""
    if amax >= 0x7f800000 or not math.isfinite(s):
        return False, s
    none = 1 << 30
    p = none if mbm1 == 0xffffffff else max((mbm1 + 1) >> 23, 1) - 150
    if s != 0.0:
        p = min(p, lowbit_exp(s))
    if p == none:
        return True, s
    if p + 53 <= 1023 and (abs(s) + T) * (1.0 + TWO ** -40) <= TWO ** (p + 53):
        return True, s + S
    if s != 0.0:
        es = (struct.unpack("<Q", struct.pack("<d", s))[0] >> 52) & 0x7ff
        if es >= 55 and float(np.uint32(amax).view(np.float32)) < TWO ** (es - 1077):
            return True, s
    return False, s


def stats(xs, rng):
    """Float32 |x|-sum in a random order, and the smallest (|x| bits - 1)."""
    a = np.abs(xs[rng.permutation(len(xs))])
    T = np.cumsum(a, dtype=np.float32)[-1] if len(a) else np.float32(0)
    bits = f32_bits(np.abs(xs)).astype(np.int64) - 1
    mbm1 = int(np.min(bits & 0xffffffff)) if len(xs) else 0xffffffff
    return T, mbm1


def column(rng, kind, n):
    if kind == "uniform":
        x = rng.uniform(-1, 1, n)
    elif kind == "sgemm":
        x = rng.normal(0, 20, n)
    elif kind == "mixed":
        x = rng.normal(0, 1, n) * np.exp2(rng.integers(-60, 61, n))
    elif kind == "huge":
        x = rng.uniform(-1, 1, n)
        x[rng.integers(0, n)] = 2.0 ** 60
    elif kind == "tiny":
        x = rng.normal(0, 20, n)
        x[rng.integers(0, n)] = 2.0 ** -60
    elif kind == "grid":
        x = rng.integers(-1000, 1001, n) * 2.0 ** -10
    elif kind == "cancel":
        h = rng.normal(0, 1e6, (n + 1) // 2)
        x = np.concatenate([h, -h])[:n] + rng.normal(0, 1e-3, n)
    elif kind == "denormal":
        x = rng.normal(0, 1, n) * 1e-40
    else:  # zeros mixed with values
        x = rng.uniform(-1, 1, n) * (rng.random(n) < 0.3)
    return np.asarray(x, np.float32)


KINDS = ["uniform", "sgemm", "mixed", "huge", "tiny", "grid", "cancel", "denormal", "sparse"]


def test_certified_sums_are_exact_and_windows_hold():
    rng = np.random.default_rng(20261202)
    certified = uncertified = 0
    for trial in range(900):
        kind = KINDS[trial % len(KINDS)]
        n = int(rng.choice([1, 2, 31, 128, 1000, 4096]))
        xs = column(rng, kind, n)
        seq = seq_sum(xs)
        T, mbm1 = stats(xs, rng)
        d64 = xs.astype(np.float64)
        orders = [
            seq_sum(xs[::-1]),
            seq_sum(xs[rng.permutation(n)]),
            float(np.sum(d64)),                                     # pairwise
            seq_sum([seq_sum(xs[k::32]) for k in range(32)]),       # per-lane partials, then combined
            math.fsum(d64),                                         # the exact sum, rounded once
        ]
        for S in orders:
            for E in (seq, seq + 1.0, seq - 3.5e-3 * (abs(seq) + 1.0), 0.0):
                d = abs(S - E)
                w = cert_window(S, T, mbm1, n, d)
                d_ref = abs(seq - E)
                assert abs(d_ref - d) <= w, (kind, n, S, seq, E, w)
                if w == 0.0:
                    assert S == seq and d == d_ref, (kind, n, S, seq)
                    certified += 1
                else:
                    uncertified += 1
    assert certified > 100 and uncertified > 100


def test_run_shortcut_gives_the_sequential_sum():
    rng = np.random.default_rng(7)
    applied = {"exact": 0, "absorbed": 0}
    for trial in range(1500):
        kind = KINDS[trial % len(KINDS)]
        run = column(rng, kind, int(rng.choice([32, 128])))
        s = float(rng.choice([0.0, float(rng.normal(0, 10)), float(rng.integers(-50, 50)) * 2.0 ** -8,
                              2.0 ** int(rng.integers(20, 90)), -(2.0 ** 60) * 1.5]))
        want = seq_sum(run, s)
        a = np.abs(run.astype(np.float64))
        S = float(np.sum(run.astype(np.float64)))
        T = float(np.sum(a))
        bits = f32_bits(np.abs(run)).astype(np.int64)
        amax = int(bits.max())
        mbm1 = int(np.min((bits - 1) & 0xffffffff))
        ok, got = run_shortcut(s, S, T, amax, mbm1)
        if ok:
            assert got == want and math.copysign(1, got) == math.copysign(1, want) or got == want == 0.0, \
                (kind, s, got, want)
            applied["absorbed" if got == s and any(run != 0) else "exact"] += 1
    assert applied["exact"] > 50 and applied["absorbed"] > 20, applied
