"""abft_verify_noalloc: the verify entry point that allocates nothing.

It serves callers that must not allocate device memory while they run (a
fault-tolerance hook inside another library's hot loop, a service whose device
memory is fixed at start-up): cudaMalloc/cudaFree can synchronise the device
and can fail under memory pressure. Its scratch is a static device array in
the library (at most 4096 columns per fragment), shared by every call.

The test calls it through the C ABI and checks that its decisions (errcol,
rowdiff, confusion-matrix increments) equal the workspace-based abft_verify
bit for bit, on two calls in a row, twice over. This file sorts last so that a
run stopping at the first failure has already run every other test; it passes
alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_cases import add_fault, flip, product_f64, tiles

pytestmark = pytest.mark.gpu


def call_noalloc(abft, C, off, nf, exp_dev, tau, injected, out_ec, out_rd, out_cm):
    stream = torch.cuda.current_stream().cuda_stream
    Cf = C.data_ptr() + 4 * off
    rc = abft.lib.abft_verify_noalloc(ctypes.c_void_p(Cf), C.stride(0), C.shape[0], nf,
                                      ctypes.c_void_p(exp_dev.data_ptr() + 8 * off), float(tau), int(injected),
                                      ctypes.c_void_p(out_ec.data_ptr()), ctypes.c_void_p(out_rd.data_ptr()),
                                      ctypes.c_void_p(out_cm.data_ptr()), ctypes.c_void_p(stream))
    assert rc == 0, abft._lib.last_error()


def test_noalloc_matches_workspace_verify(abft, orc):
    M, K, N, F = 2048, 512, 2048, 2
    A, B = tiles(orc, M, K, N, 71, 72)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    kern = abft.kernels
    ws = kern.Workspace(M, N, K, counts, offsets, max_iters=2)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    kern.encode(ws, dA, dB)
    torch.cuda.synchronize()
    exp_dev = torch.from_numpy(ws.read_checksums()[1]).cuda()

    rounds = [
        (add_fault(C0, 100, offsets[1] + 7, 2.0), 1, 1e-5 * K),   # fault in fragment 1
        (flip(C0, 1500, 33, 27), 0, 1e-5 * K),                      # exponent flip in fragment 0
        (C0, -1, 0.0),                                              # tau = 0: arg-max over rounding noise
    ]
    out_ec = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_rd = torch.zeros(1, dtype=torch.float64, device="cuda")
    out_cm = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws.reset_counters()
    for it, (C, inj_f, tau) in enumerate(rounds[:2] + rounds[2:]):
        dC = torch.from_numpy(np.ascontiguousarray(C)).cuda()
        got_ec, got_rd = [], []
        for f in range(F):  # two calls in a row, one per fragment
            kern.verify(ws, dC, f, tau, injected=(f == inj_f), it=min(it, 1))
            call_noalloc(abft, dC, int(offsets[f]), int(counts[f]), exp_dev, tau, f == inj_f, out_ec, out_rd, out_cm)
            torch.cuda.synchronize()
            got_ec.append(int(out_ec.item()))
            got_rd.append(float(out_rd.item()))
        want_ec, _, want_rd = ws.read_log(min(it, 1) + 1)
        assert got_ec == list(want_ec[min(it, 1)])
        assert np.array_equal(np.array(got_rd).view(np.uint64), want_rd[min(it, 1)].view(np.uint64))
        cm, _ = ws.counters()
        assert out_cm.cpu().tolist() == cm.tolist()
    ws.close()


def test_noalloc_rejects_wide_fragments(abft):
    C = torch.zeros((4, 4100), dtype=torch.float32, device="cuda")
    e = torch.zeros(4100, dtype=torch.float64, device="cuda")
    ec = torch.zeros(1, dtype=torch.int32, device="cuda")
    rd = torch.zeros(1, dtype=torch.float64, device="cuda")
    cm = torch.zeros(4, dtype=torch.int32, device="cuda")
    rc = abft.lib.abft_verify_noalloc(ctypes.c_void_p(C.data_ptr()), 4100, 4, 4100, ctypes.c_void_p(e.data_ptr()),
                                      1.0, 0, ctypes.c_void_p(ec.data_ptr()), ctypes.c_void_p(rd.data_ptr()),
                                      ctypes.c_void_p(cm.data_ptr()), None)
    assert rc == abft._lib.ABFT_ERR_ARG
    assert "4096" in abft._lib.last_error()


def test_noalloc_width_changes_match_oracle(abft, orc):
    """Calls of different widths in a row (a narrow fragment, the full
    4096-column maximum, the narrow one again) each start from clean scratch:
    every result equals the oracle's decision directly (errcol, rowdiff bits,
    confusion-matrix increment)."""
    M, K, N = 384, 96, 4096
    A, B = tiles(orc, M, K, N, 81, 82)
    C0 = product_f64(A, B)
    expRow = orc.expected_row(orc.col_checksum_A(A), B)
    exp_dev = torch.from_numpy(expRow).cuda()
    tau = 1e-5 * K
    cases = [
        # (column offset, width, fault (row, column, delta) or None, tau, injected)
        (128, 200, (10, 128 + 57, 2.0), tau, True),
        (0, 4096, (300, 4000, -5.0), tau, True),
        (128, 200, None, tau, False),
        (0, 4096, None, 0.0, False),     # tau = 0: the arg-max over rounding noise of every column
        (128, 200, (17, 128 + 3, 0.5), tau, True),
    ]
    out_ec = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_rd = torch.zeros(1, dtype=torch.float64, device="cuda")
    out_cm = torch.zeros(4, dtype=torch.int32, device="cuda")
    want_cm = np.zeros(4, np.int64)
    for off, nf, fault, t, injected in cases:
        C = C0 if fault is None else add_fault(C0, fault[0], fault[1], fault[2])
        dC = torch.from_numpy(np.ascontiguousarray(C)).cuda()
        call_noalloc(abft, dC, off, nf, exp_dev, t, injected, out_ec, out_rd, out_cm)
        torch.cuda.synchronize()
        w_ec, w_rd, w_cm = orc.detect_row(expRow[off:off + nf], orc.actual_row(C[:, off:off + nf]), t, injected)
        want_cm += w_cm
        assert int(out_ec.item()) == w_ec, (off, nf, fault)
        assert np.float64(out_rd.item()).view(np.uint64) == np.float64(w_rd).view(np.uint64)
        assert out_cm.cpu().numpy().tolist() == want_cm.tolist()
        if fault is not None:
            assert w_ec == fault[1] - off
