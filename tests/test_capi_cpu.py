"""CPU checks of the C ABI: the library loads, exports every symbol that
include/abft_b200.h declares, and its host helpers reject bad arguments.
No CUDA call is made."""
import ctypes
import re

import numpy as np
import pytest


def declared_functions(header_path):
    text = open(header_path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w\s\*]*?\b(abft_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(abft):
    names = declared_functions(abft.HEADER_PATH)
    assert len(names) >= 30
    lib = ctypes.CDLL(abft.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers all of them
    assert sorted(abft.SIGNATURES) == names


def test_version_and_error_channel(abft):
    assert abft.lib.abft_version() >= 10000
    with pytest.raises(abft.AbftError) as e:
        abft.split_dim(10, 0)
    assert "split_dim" in str(e.value)
    with pytest.raises(abft.AbftError):
        abft.choose_grid(0)
    with pytest.raises(abft.AbftError):
        abft.host.call("abft_injection_plan", 0, 0, 0, 0, 4, None, 1, 0, 31, None, None, None, None)


def test_swifi_plan_rejects_bad_zone(abft):
    counts = np.array([4, 4], np.int32)
    p = counts.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    outs = [ctypes.c_int() for _ in range(4)]
    rc = abft.lib.abft_injection_plan(1, 0, 0, 2, 8, p, abft.INJECT_SWIFI, 5, 40, *[ctypes.byref(o) for o in outs])
    assert rc == -1


def test_rank_tiles_cover_the_matrix(abft):
    for world in (1, 2, 4, 8, 6):
        Pr, Pc = abft.choose_grid(world)
        M, K, N = 1000, 64, 1030
        cover = np.zeros((M, N), np.int32)
        for r in range(world):
            t = abft.rank_tile(M, K, N, Pr, Pc, r)
            cover[t.row_off:t.row_off + t.M_b, t.col_off:t.col_off + t.N_b] += 1
            assert t.F == 4 and sum(t.counts) == t.N_b
        assert (cover == 1).all()


def test_frag_policy(abft):
    assert abft.frag_count(512, 512, 512, 512, 512, 4) == 1          # small-matrix rule
    assert abft.frag_count(1024, 1024, 1024, 1024, 1024, 4) == 4
    assert abft.frag_count(4096, 4096, 4096, 4096, 4096, 4, frag_cap=1 << 20) == 16
    assert abft.frag_count(4096, 4096, 4096, 4096, 3, 4) == 3          # never more than N_b


def test_c_pitch_pads_64k_multiples_only(abft):
    # a dense 64 KB (or 128 KB ...) pitch gets 32 floats more; others stay dense
    assert abft.c_pitch(16384) == 16416
    assert abft.c_pitch(32768) == 32800
    for n in (1, 256, 1000, 1024, 4096, 8192, 12288, 16385):
        assert abft.c_pitch(n) == n
    with pytest.raises(ValueError):
        abft.c_pitch(0)


def test_tile_injection_scheme_matches_oracle(abft, orc):
    """The tile-uniform scheme (seed 1 + iteration, (i, j) uniform over the tile)."""
    counts, offsets = abft.split_dim(1030, 3)
    for seed in range(1, 40):
        for mode, zone in (("add", "any"), ("swifi", "any"), ("swifi", "exponent")):
            got = abft.host.injection_plan_tile(seed, 777, counts, offsets, mode, zone)
            lo, hi = (1, 0) if mode == "add" else orc.swifi_zone_range(zone)
            want = orc.inject_position_tile(seed, 777, counts, offsets, lo, hi)
            assert got == want
            f, r, c, b = got
            assert 0 <= r < 777 and 0 <= c < counts[f]
    assert abft.host.injection_plan_tile(5, 10, counts, offsets, "none") == (-1, -1, -1, -1)


def test_verify_kernel_selector(abft):
    assert abft.set_verify_kernel("ldg") == "auto"
    assert abft.set_verify_kernel("tma") == "ldg"
    assert abft.set_verify_kernel("auto") == "tma"
    assert abft.lib.abft_set_verify_kernel(3) == -1
    assert "abft_set_verify_kernel" in abft._lib.last_error()
    with pytest.raises(KeyError):
        abft.set_verify_kernel("fast")


def test_device_entry_points_reject_bad_arguments(abft):
    """Every device-side entry point validates its arguments before touching
    CUDA and reports ABFT_ERR_ARG with a message (the reference aborted the
    job instead; core/common.cuh:22-50). Only argument checks run here."""
    lib = abft.lib
    ERR = abft._lib.ABFT_ERR_ARG
    fake = ctypes.c_void_p(256)  # never dereferenced: each call fails its checks first
    out = ctypes.c_void_p()
    i4 = (ctypes.c_int * 4)(4, 4, 4, 4)
    o4 = (ctypes.c_int * 4)(0, 4, 8, 12)
    cases = [
        ("abft_ws_create", (0, 16, 8, 4, i4, o4, 1, None, 0, ctypes.byref(out))),      # M_b < 1
        ("abft_ws_create", (16, 15, 8, 4, i4, o4, 1, None, 0, ctypes.byref(out))),     # fragment 3 past N_b
        ("abft_ws_create", (16, 16, 8, 4, i4, o4, -1, None, 0, ctypes.byref(out))),    # max_iters < 0
        ("abft_ws_create", (16, 16, 8, 0, i4, o4, 1, None, 0, ctypes.byref(out))),     # F < 1
        ("abft_encode", (None, fake, 8, fake, 16, None)),
        ("abft_verify", (None, fake, 16, 0, 1.0, 0, -1, None)),
        ("abft_calibrate", (None, fake, 16, 0, fake, None)),
        ("abft_localize_correct", (None, fake, 16, 0, 1.0, 0, None, 0, -1, 0, None)),
        ("abft_drain", (None, fake, fake, 16, None, 0, 4, None)),
        ("abft_verify_noalloc", (None, 16, 8, 8, fake, 1.0, 0, fake, fake, fake, None)),
        ("abft_verify_noalloc", (fake, 4, 8, 8, fake, 1.0, 0, fake, fake, fake, None)),   # ldc < N
        ("abft_verify_noalloc", (fake, 16, 0, 8, fake, 1.0, 0, fake, fake, fake, None)),  # M < 1
        ("abft_inject_add", (None, 16, 0, 0, 1.0, None)),
        ("abft_inject_add", (fake, 16, 0, 16, 1.0, None)),          # col outside the row
        ("abft_inject_add", (fake, 16, -1, 0, 1.0, None)),
        ("abft_inject_bitflip", (fake, 16, 0, 0, 32, None)),        # bit outside 0..31
        ("abft_inject_bitflip", (fake, 16, 0, 0, -1, None)),
        ("abft_sgemm", (None, fake, 8, fake, 16, fake, 16, 8, 16, 8)),
        ("abft_session_create", (None, ctypes.byref(out))),
        ("abft_session_online", (None, None, None)),
        ("abft_session_baseline", (None, 1, 0, None, None)),
        ("abft_session_set_tau", (None, None)),
        ("abft_ws_read_counters", (None, None, None)),
        ("abft_ws_read_log", (None, 1, None, None, None)),
        ("abft_ws_reset_counters", (None, None)),
    ]
    for name, args in cases:
        rc = getattr(lib, name)(*args)
        assert rc == ERR, (name, rc)
        assert abft._lib.last_error(), name
    assert out.value is None  # no workspace or session was handed out
    # a session configuration with a zero tile edge is refused before any CUDA call
    cfg = abft._lib.SessionCfg(M_b=0, N_b=16, K=8, F=4, counts=i4, offsets=o4, dA=256, lda=8, dB=256, ldb=16,
                               dC0=256, dC1=256, ldc=16, verify_priority=-1, max_iters=1)
    assert lib.abft_session_create(ctypes.byref(cfg), ctypes.byref(out)) == ERR and out.value is None
    assert lib.abft_ws_bytes(16, 16, 8, 4, i4, 1) > 0
    assert lib.abft_ws_bytes(0, 16, 8, 4, i4, 1) == 0


def test_session_arguments_are_validated(abft):
    """Online-loop options are checked on the host before any call: an unknown
    correction mode, seed scheme or injection mode is an error."""
    from importlib import import_module
    OnlineSession = import_module(abft.__name__ + ".session").OnlineSession
    ok = OnlineSession._args(None, "swifi", "exponent", 1.0, 7, 2, 5, "drain", True, graph=True, seed_scheme="tile")
    assert (ok.mode, ok.zone_lo, ok.zone_hi, ok.correct_mode, ok.seed_scheme) == (abft.INJECT_SWIFI, 23, 30,
                                                                                    abft.CORRECT_DRAIN, 1)
    for bad in (dict(correct="later"), dict(seed_scheme="json")):
        kw = dict(correct="inloop", seed_scheme="reference")
        kw.update(bad)
        with pytest.raises(ValueError):
            OnlineSession._args(None, "add", "any", 1.0, 0, 0, 1, kw["correct"], False,
                                seed_scheme=kw["seed_scheme"])
    with pytest.raises(KeyError):
        OnlineSession._args(None, "flip", "any", 1.0, 0, 0, 1, "inloop", False)
    # an unknown SWIFI zone means the whole word, as in the reference (kernels/swifi.cuh:25-31)
    z = OnlineSession._args(None, "swifi", "mantissa", 1.0, 0, 0, 1, "inloop", False)
    assert (z.zone_lo, z.zone_hi) == (0, 31)


C_CLIENT = r"""
#include "abft_b200.h"
#include <stdio.h>
int main(void) {
    int counts[4], offsets[4], Pr = 0, Pc = 0;
    if (abft_split_dim(1030, 4, counts, offsets) != ABFT_OK) return 1;
    if (abft_choose_grid(8, &Pr, &Pc) != ABFT_OK || Pr * Pc != 8) return 2;
    if (abft_verify(NULL, NULL, 0, 0, 1.0, 0, -1, NULL) != ABFT_ERR_ARG) return 3;
    printf("%d %d %d %d %dx%d\n", counts[0], counts[1], counts[2], counts[3], Pr, Pc);
    return 0;
}
"""


def test_header_is_a_plain_c_abi(abft, tmp_path):
    """include/abft_b200.h compiles as strict C99 and a C program links and
    calls libabft_b200.so (what a cgo / JNI / ctypes binding needs)."""
    import os
    import subprocess
    src = tmp_path / "client.c"
    src.write_text(C_CLIENT)
    exe = str(tmp_path / "client")
    libdir = os.path.dirname(abft.LIB_PATH)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I",
                        os.path.dirname(abft.HEADER_PATH), "-o", exe, str(src), "-L", libdir, "-labft_b200",
                        f"-Wl,-rpath,{libdir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.returncode, r.stderr)
    assert r.stdout.split() == ["258", "258", "257", "257", "2x4"]
