"""The TMA verify body's bounded waits: a wait that gives up leaves an error
status for the host and a usable context.

Each wait of the TMA-staged verify for a bulk tensor copy polls at most a set
number of times (abft_set_wait_limit). With the limit at 0 every such wait in
the streaming loop gives up at once; the kernel then waits, with the default
limit, for the copies it already issued (they all land), adds nothing and
finishes its arrival protocol. The counter read must return ABFT_ERR_CUDA
with the wait message, and the next verify in the same context, with the
default limit, must equal the oracle bit for bit. Nothing here faults, traps
or waits without a bound: every copy lands and every wait ends.
"""
import numpy as np
import pytest
import torch

from gpu_cases import add_fault, product_f64, tiles

pytestmark = pytest.mark.gpu

DEFAULT_LIMIT = 1 << 20


def test_wait_limit_failure_path(abft, orc):
    M, K, N, F = 512, 64, 1024, 2  # 512-column fragments: a tensor map describes them, so the TMA body runs
    A, B = tiles(orc, M, K, N, 31, 32)
    counts, offsets = orc.split_dim(N, F)
    C = add_fault(product_f64(A, B), 200, int(offsets[1]) + 17, 3.0)
    tau = 1e-5 * K
    _, expRow, _, _ = orc.encode(A, B, counts, offsets)
    kern = abft.kernels
    ws = kern.Workspace(M, N, K, counts, offsets, max_iters=2)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.from_numpy(np.ascontiguousarray(C)).cuda()
    kern.encode(ws, dA, dB)
    prev_kernel = abft.set_verify_kernel("tma")
    try:
        prev = abft.lib.abft_set_wait_limit(0)
        assert prev == DEFAULT_LIMIT
        try:
            ws.reset_counters()
            for f in range(F):
                kern.verify(ws, dC, f, tau, injected=(f == 1), it=0)
            torch.cuda.synchronize()
            with pytest.raises(abft.AbftError) as err:
                ws.counters()
            assert err.value.rc == abft._lib.ABFT_ERR_CUDA
            assert "wait limit" in str(err.value)
        finally:
            assert abft.lib.abft_set_wait_limit(prev) == 0
        assert abft.lib.abft_set_wait_limit(-1) == abft._lib.ABFT_ERR_ARG

        # Same context, default limit: the next launches start from clean
        # accumulators and match the oracle bit for bit.
        ws.reset_counters()
        for f in range(F):
            kern.verify(ws, dC, f, tau, injected=(f == 1), it=1)
        torch.cuda.synchronize()
        cm, _ = ws.counters()
        ec, _, rd = ws.read_log(2)
        want_cm = np.zeros(4, np.int64)
        for f in range(F):
            o, n = int(offsets[f]), int(counts[f])
            w_ec, w_rd, w_cm = orc.detect_row(expRow[o:o + n], orc.actual_row(C[:, o:o + n]), tau, f == 1)
            assert int(ec[1][f]) == w_ec
            assert np.float64(rd[1][f]).view(np.uint64) == np.float64(w_rd).view(np.uint64)
            want_cm += w_cm
        assert ec[1][1] == 17 and ec[1][0] == -1
        assert cm.tolist() == want_cm.tolist()
    finally:
        abft.set_verify_kernel(prev_kernel)
    ws.close()
