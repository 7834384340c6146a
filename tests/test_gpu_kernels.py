"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Bar: bit-exact. Checksums (colSumA, expectedRow, rowSumB_f, expectedCol_f),
detected column, rowdiff, located row, corrected C and the counters must equal
the oracle's restatement of the reference kernels bit for bit.
"""
import numpy as np
import pytest

from gpu_cases import add_fault, flip, product_f64, tiles

pytestmark = pytest.mark.gpu

SHAPES = [
    # M, K, N, F
    (64, 80, 48, 1),
    (257, 129, 515, 4),      # uneven fragments, N_f not a multiple of 4 -> scalar path
    (1100, 300, 1030, 3),
    (1024, 1024, 1024, 4),   # 1024^3 rank tile, F = 4
    (33, 7, 9, 2),
    (2048, 64, 512, 4),
    (1000, 96, 1032, 3),     # 16-byte aligned fragments of 344 columns: ragged last box in x and y
    (70000, 16, 128, 1),     # tall: more row boxes per CTA than ring stages
    (64, 8, 6400, 1),        # wide: the last CTA's d / w arrays do not fit in shared memory
    (1, 1, 1, 1),            # degenerate tiles
    (1, 3, 5, 1),
    (5, 1, 7, 2),
    (2, 2, 4, 4),            # one column per fragment
]


@pytest.fixture(autouse=True, params=["ldg", "tma"])
def verify_kernel(request, abft):
    """Every test runs with each verify body forced (TMA falls back to LDG for
    fragments a tensor map cannot describe)."""
    abft.set_verify_kernel(request.param)
    yield request.param
    abft.set_verify_kernel("auto")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    return torch


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_gpu_iteration(abft, torch, A, B, C, counts, offsets, tau, inject_frag, golden=None, localize=True):
    kern = abft.kernels
    M, K = A.shape
    N = B.shape[1]
    ws = kern.Workspace(M, N, K, counts, offsets, max_iters=1)
    dA, dB, dC = to_dev(torch, A), to_dev(torch, B), to_dev(torch, C)
    dG = to_dev(torch, golden) if golden is not None else None
    kern.encode(ws, dA, dB)
    ws.reset_counters()
    for f in range(len(counts)):
        kern.verify(ws, dC, f, tau[f], injected=(f == inject_frag), it=0)
        if localize:
            kern.localize_correct(ws, dC, f, tau[f], injected=(f == inject_frag), golden=dG, it=0)
    torch.cuda.synchronize()
    cm, nr = ws.counters()
    ec, er, rd = ws.read_log(1)
    sums = ws.read_checksums()
    out = dC.cpu().numpy()
    ws.close()
    return dict(cm=cm, nr=nr, ec=ec[0], er=er[0], rd=rd[0], C=out, sums=sums)


def run_oracle_iteration(orc, A, B, C, counts, offsets, tau, inject_frag, golden=None, localize=True):
    colSumA, expRow, rowSumB, expCol = orc.encode(A, B, counts, offsets)
    Cc = C.copy()
    cm, nr, ec, er, rd = orc.verify_iteration(Cc, A, B, counts, offsets, expRow, tau, inject_frag, localize,
                                              expCol=expCol, golden=golden)
    return dict(cm=cm, nr=nr, ec=ec, er=er, rd=rd, C=Cc, sums=(colSumA, expRow, rowSumB, expCol))


def assert_same(g, o):
    assert list(g["cm"]) == list(o["cm"])
    assert g["nr"] == o["nr"]
    assert list(g["ec"]) == list(o["ec"])
    assert list(g["er"]) == list(o["er"])
    assert g["rd"].view(np.uint64).tolist() == o["rd"].view(np.uint64).tolist()
    assert np.array_equal(g["C"].view(np.uint32), o["C"].view(np.uint32))


@pytest.mark.parametrize("shape", SHAPES)
def test_encode_bit_exact(shape, abft, orc, torch_cuda):
    M, K, N, F = shape
    A, B = tiles(orc, M, K, N)
    counts, offsets = orc.split_dim(N, F)
    C = product_f64(A, B)
    g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, [1e30] * F, -1, localize=False)
    o = orc.encode(A, B, counts, offsets)
    for got, want, name in zip(g["sums"], o, ["colSumA", "expRow", "rowSumB", "expCol"]):
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), name


def test_encode_strided_and_unaligned(abft, orc, torch_cuda):
    """Tiles that are views: leading dimensions larger than the width, base not 16-byte aligned."""
    torch = torch_cuda
    M, K, N, F = 300, 200, 260, 3
    Aw, Bw = tiles(orc, M, K + 7, N + 5, 11, 12)
    counts, offsets = orc.split_dim(N, F)
    dAw, dBw = to_dev(torch, Aw), to_dev(torch, Bw)
    dA, dB = dAw[:, 1:K + 1], dBw[:, 3:N + 3]
    A, B = Aw[:, 1:K + 1], Bw[:, 3:N + 3]
    ws = abft.kernels.Workspace(M, N, K, counts, offsets)
    abft.kernels.encode(ws, dA, dB)
    torch.cuda.synchronize()
    got = ws.read_checksums()
    want = orc.encode(A, B, counts, offsets)
    for g, w in zip(got, want):
        assert np.array_equal(g.view(np.uint64), w.view(np.uint64))


@pytest.mark.parametrize("pad,shift", [(12, 4), (5, 1)])
def test_verify_localize_on_views(pad, shift, abft, orc, torch_cuda):
    """C as a view into a wider buffer (leading dimension > width): 16-byte
    aligned with ldc % 4 == 0 (the TMA body takes it), or shifted by one float
    (128-bit loads impossible). Decisions and corrections equal the oracle's
    and the padding around the view is never written."""
    torch = torch_cuda
    M, K, N, F = 700, 64, 1032, 3
    A, B = tiles(orc, M, K, N, 81, 82)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    tau = [1e-2] * F
    kern = abft.kernels
    dA, dB, dG = to_dev(torch, A), to_dev(torch, B), to_dev(torch, C0)
    for f in range(F):
        C = add_fault(C0, 123 + f, offsets[f] + 7 * f + 1, 1.0e6)
        Cw = np.full((M, N + pad), np.nan, np.float32)
        Cw[:, shift:shift + N] = C
        dCw = to_dev(torch, Cw)
        dC = dCw[:, shift:shift + N]
        ws = kern.Workspace(M, N, K, counts, offsets, max_iters=1)
        kern.encode(ws, dA, dB)
        ws.reset_counters()
        for g in range(F):
            kern.verify(ws, dC, g, tau[g], injected=(g == f), it=0)
            kern.localize_correct(ws, dC, g, tau[g], injected=(g == f), golden=dG, it=0)
        torch.cuda.synchronize()
        cm, nr = ws.counters()
        ec, er, rd = ws.read_log(1)
        out = dCw.cpu().numpy()
        ws.close()
        o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, f, golden=C0)
        assert_same(dict(cm=cm, nr=nr, ec=ec[0], er=er[0], rd=rd[0], C=np.ascontiguousarray(out[:, shift:shift + N])),
                    o)
        assert np.isnan(out[:, :shift]).all() and np.isnan(out[:, shift + N:]).all()


@pytest.mark.parametrize("shape", SHAPES)
def test_clean_tile_no_detection(shape, abft, orc, torch_cuda):
    M, K, N, F = shape
    A, B = tiles(orc, M, K, N, 3, 4)
    counts, offsets = orc.split_dim(N, F)
    C = product_f64(A, B)
    tau = [1e-5 * K] * F
    g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, -1)
    o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, -1)
    assert_same(g, o)


@pytest.mark.parametrize("shape", SHAPES)
def test_additive_fault_every_fragment(shape, abft, orc, torch_cuda):
    M, K, N, F = shape
    A, B = tiles(orc, M, K, N, 5, 6)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    rng = np.random.default_rng(1)
    for f in range(F):
        r = int(rng.integers(0, M))
        c = int(offsets[f] + rng.integers(0, counts[f]))
        for delta in (1.0e6, 1.0, 0.03125):
            C = add_fault(C0, r, c, delta)
            tau = [1e-5 * K] * F
            g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, f, golden=C0)
            o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, f, golden=C0)
            assert_same(g, o)


@pytest.mark.parametrize("shape", [(257, 129, 515, 4), (1024, 1024, 1024, 4), (1000, 96, 1032, 3)])
def test_bitflips_all_bits(shape, abft, orc, torch_cuda):
    M, K, N, F = shape
    A, B = tiles(orc, M, K, N, 7, 8)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    rng = np.random.default_rng(2)
    tau = [1e-5 * K] * F
    for bit in range(32):
        f = int(rng.integers(0, F))
        r = int(rng.integers(0, M))
        c = int(offsets[f] + rng.integers(0, counts[f]))
        C = flip(C0, r, c, bit)
        g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, f, golden=C0)
        o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, f, golden=C0)
        assert_same(g, o)


@pytest.mark.parametrize("shape", [(257, 129, 515, 4), (1024, 1024, 1024, 4), (2048, 64, 512, 4)])
def test_zero_threshold_noise_argmax(shape, abft, orc, torch_cuda):
    """tau = 0: every noisy column is a candidate; the arg-max over pure rounding
    noise must still be the reference's (exact values, exact tie rule)."""
    M, K, N, F = shape
    A, B = tiles(orc, M, K, N, 9, 10)
    counts, offsets = orc.split_dim(N, F)
    C = product_f64(A, B)
    tau = [0.0] * F
    g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, -1)
    o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, -1)
    assert_same(g, o)


def test_exact_ties(abft, orc, torch_cuda):
    """A = 0 makes every expected checksum 0, so equal faults give exactly equal
    |actual - expected|: the winner is decided by the reference's tree rule."""
    M, K, N, F = 600, 16, 1030, 2
    A = np.zeros((M, K), np.float32)
    _, B = tiles(orc, M, K, N)
    counts, offsets = orc.split_dim(N, F)
    for cols in ([1, 2, 3], [0, 256, 257, 513], [5, 261, 517], [255, 511, 300, 44]):
        C = np.zeros((M, N), np.float32)
        for k, c in enumerate(cols):
            C[(7 * k + 3) % M, c] = 3.0
            C[(7 * k + 3) % M, offsets[1] + c % counts[1]] = 3.0
        tau = [0.5] * F
        g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, 0)
        o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, 0)
        assert_same(g, o)


@pytest.mark.parametrize("row,col,fault", [(9700, 1234, "add"), (100, 4095, "add"), (7424, 7, "add"),
                                           (9727, 2048, "flip"), (5000, 3000, "flip")])
def test_verify_one_batch_tail_units(row, col, fault, abft, orc, torch_cuda):
    """A fragment large enough that the verify schedule ends in one-batch
    units (9728 x 4096: 18 CTAs per column group, each with at least four
    128-row units, so rows from 7424 on are read in 64-row units): faults in
    the bulk rows and in the tail rows are detected, located and corrected
    exactly as by the oracle."""
    M, K, N, F = 9728, 16, 4096, 1
    A, B = tiles(orc, M, K, N, 31, 32)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    C = add_fault(C0, row, col, 64.0) if fault == "add" else flip(C0, row, col, 30)
    tau = [1.0]
    g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, 0)
    o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, 0)
    assert_same(g, o)
    assert o["ec"][0] == col and o["er"][0] == row


@pytest.mark.parametrize("rows", [[5, 261], [261, 5], [64, 128], [128, 64, 517, 773], [1, 257, 513, 769, 1025],
                                  [200, 100, 300], [1099, 0], [3, 10, 17, 24]])
def test_exact_row_ties(rows, abft, orc, torch_cuda):
    """Equal faults in several rows of one fragment (A = 0, so every faulty row
    has exactly the same |actual - expected|): the localised row is decided by
    the reference's scan-and-tree order alone - across row blocks, within one
    slot (rows j and j + 256) and between slots (bit-reversed slot order)."""
    M, K, N, F = 1100, 16, 1030, 2
    A = np.zeros((M, K), np.float32)
    _, B = tiles(orc, M, K, N)
    counts, offsets = orc.split_dim(N, F)
    C = np.zeros((M, N), np.float32)
    for k, r in enumerate(rows):
        C[r, 3 + 11 * k] = 3.0
    tau = [0.5] * F
    g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, 0)
    o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, 0)
    assert_same(g, o)
    assert o["er"][0] in rows


def test_uncertified_sum_uses_sequential_value(abft, orc, torch_cuda):
    """Columns whose parallel double sum differs from the sequential one:
    2^30 followed by many 2^-27 terms. Each sequential add rounds the small
    term away; a parallel partial of 16 or more small terms survives."""
    M, K, N, F = 4096, 8, 256, 1
    A = np.zeros((M, K), np.float32)
    _, B = tiles(orc, M, K, N)
    counts, offsets = orc.split_dim(N, F)
    C = np.zeros((M, N), np.float32)
    C[0, 17] = 2.0 ** 30
    C[1:, 17] = 2.0 ** -27
    C[5, 40] = 2.0 ** 29
    C[6:, 40] = 2.0 ** -28
    seq = orc.actual_row(C)
    assert seq[17] == 2.0 ** 30 and seq[40] == 2.0 ** 29  # the reference's values
    assert float(C[:, 17].astype(np.float64).sum()) != 2.0 ** 30  # an unordered sum differs
    for tau in (0.5, 2.0 ** 30 + 2.0 ** -22, 2.0 ** 29 + 1.0):
        g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, [tau], 0)
        o = run_oracle_iteration(orc, A, B, C, counts, offsets, [tau], 0)
        assert_same(g, o)


def test_nonfinite_values(abft, orc, torch_cuda):
    M, K, N, F = 512, 32, 384, 3
    A, B = tiles(orc, M, K, N, 13, 14)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    tau = [1e-3] * F
    for val in (np.inf, -np.inf, np.nan, 3.0e38):
        for f in range(F):
            C = C0.copy()
            C[100, offsets[f] + 5] = val
            g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, f, golden=C0)
            o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, f, golden=C0)
            assert_same(g, o)
    C = C0.copy()
    C[3, 4] = np.inf
    C[9, 4] = -np.inf
    g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, 0, golden=C0)
    o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, 0, golden=C0)
    assert_same(g, o)


def test_multiple_faults_one_fragment(abft, orc, torch_cuda):
    """Two faults in one fragment (outside the single-fault model): decisions
    still follow the reference exactly."""
    M, K, N, F = 1024, 256, 1024, 4
    A, B = tiles(orc, M, K, N, 15, 16)
    counts, offsets = orc.split_dim(N, F)
    C0 = product_f64(A, B)
    C = add_fault(add_fault(C0, 10, 20, 5.0), 700, 20, 6.0)
    C = add_fault(C, 11, 100, 5.5)
    tau = [1e-5 * K] * F
    g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, tau, 0, golden=C0)
    o = run_oracle_iteration(orc, A, B, C, counts, offsets, tau, 0, golden=C0)
    assert_same(g, o)


def test_injectors(abft, torch_cuda):
    torch = torch_cuda
    C = torch.zeros((8, 12), dtype=torch.float32, device="cuda")
    C[3, 5] = 1.5
    abft.kernels.inject_add(C, 3, 5, 1.0e6)
    abft.kernels.inject_bitflip(C, 2, 7, 30)
    torch.cuda.synchronize()
    h = C.cpu().numpy()
    assert h[3, 5] == np.float32(np.float32(1.5) + np.float32(1.0e6))
    assert h[2, 7].view(np.uint32) == np.uint32(1 << 30)


def test_bad_arguments_raise(abft, torch_cuda):
    torch = torch_cuda
    with pytest.raises(abft.AbftError):
        abft.kernels.Workspace(0, 4, 4, [4], [0])
    with pytest.raises(abft.AbftError):
        abft.kernels.Workspace(4, 4, 4, [3, 3], [0, 3])  # fragment beyond the tile
    ws = abft.kernels.Workspace(4, 4, 4, [4], [0])
    C = torch.zeros((4, 4), device="cuda")
    with pytest.raises(abft.AbftError):
        abft.kernels.verify(ws, C, 1, 1.0)  # fragment index out of range
    with pytest.raises(abft.AbftError):
        abft.kernels.inject_bitflip(C, 0, 0, 32)
    ws.close()


@pytest.mark.parametrize("shape", [(257, 129, 515, 4), (1024, 1024, 1024, 4), (4096, 8, 256, 1)])
def test_calibrate_exact_diffs(shape, abft, orc, torch_cuda):
    """|actualRow - expectedRow| of every column (pass_calibrate), bit-exact,
    including columns whose parallel sum is not certified."""
    torch = torch_cuda
    M, K, N, F = shape
    A, B = tiles(orc, M, K, N, 61, 62)
    counts, offsets = orc.split_dim(N, F)
    C = product_f64(A, B)
    if M == 4096:  # force uncertified columns: one huge term followed by many tiny ones
        C[0, 3] = 2.0 ** 30
        C[1:, 3] = 2.0 ** -27
        C[7, 100] = 1.0e30
    ws = abft.kernels.Workspace(M, N, K, counts, offsets)
    dA, dB, dC = to_dev(torch, A), to_dev(torch, B), to_dev(torch, C)
    abft.kernels.encode(ws, dA, dB)
    got = [abft.kernels.calibrate(ws, dC, f).cpu().numpy() for f in range(F)]
    torch.cuda.synchronize()
    _, expRow, _, _ = orc.encode(A, B, counts, offsets)
    act = orc.actual_row(C)
    want = np.abs(act - expRow)
    for f in range(F):
        w = want[offsets[f]:offsets[f] + counts[f]]
        assert np.array_equal(got[f].view(np.uint64), w.view(np.uint64))
    ws.close()


def adversarial(rng, n, kind):
    """One line of n float32 terms built to defeat the any-order certificate."""
    x = (rng.standard_normal(n) * 30).astype(np.float32)
    r = int(rng.integers(0, n))
    if kind == 1:
        x[r] *= np.float32(2.0 ** -40)                      # one tiny term
    elif kind == 2:
        x[r] *= np.float32(2.0 ** 40)                       # one huge term
    elif kind == 3:
        r2 = int(rng.integers(r, n))
        x[r], x[r2] = 3.0e30, -3.0e30                        # huge, later cancelled
    elif kind == 4:
        idx = rng.integers(0, n, 7)
        x[idx] = (rng.integers(1, 1 << 20, 7) * np.float32(2.0 ** -149)).astype(np.float32)  # subnormals
    elif kind == 5:
        x *= np.exp2(rng.integers(-60, 61, n)).astype(np.float32)   # magnitudes over 2^+-60
    elif kind == 6:
        x[0] = 1.0e30                                         # absorbs everything after it
    elif kind == 7:
        k = np.arange(n)
        x = ((1.0 + (k % 97) * 2.0 ** -23) * np.where(k % 2, -1.0, 1.0)).astype(np.float32)
    elif kind == 8:
        x[:] = -0.0
        x[r] = 1.5
    elif kind == 9:
        x[:] = 2.0 ** -27
        x[0] = 2.0 ** 30
    elif kind == 10:
        x[n // 2] = 1.0e35
        x[-1] = -1.0e35
    elif kind == 11:
        x *= np.float32(2.0 ** -100)
        x[r] = 7.0
    elif kind == 12:
        h = n // 3                                            # a hard stretch, then plain terms
        x[:h] *= np.exp2(rng.integers(-60, 61, h)).astype(np.float32)
    return x


@pytest.mark.parametrize("M", [3000, 257])
def test_exact_chain_adversarial_columns(M, abft, orc, torch_cuda):
    """Calibration re-sums every uncertified column in the reference's order:
    each must equal the sequential double sum bit for bit, whatever mix of
    tiny, huge, subnormal, cancelling and absorbed terms the column holds."""
    torch = torch_cuda
    rng = np.random.default_rng(2024 + M)
    K, N, F = 16, 512, 2
    A, B = tiles(orc, M, K, N, 71, 72)
    counts, offsets = orc.split_dim(N, F)
    C = np.empty((M, N), np.float32)
    for j in range(N):
        C[:, j] = adversarial(rng, M, j % 13)
    ws = abft.kernels.Workspace(M, N, K, counts, offsets)
    dA, dB, dC = to_dev(torch, A), to_dev(torch, B), to_dev(torch, C)
    abft.kernels.encode(ws, dA, dB)
    got = [abft.kernels.calibrate(ws, dC, f).cpu().numpy() for f in range(F)]
    torch.cuda.synchronize()
    _, expRow, _, _ = orc.encode(A, B, counts, offsets)
    want = np.abs(orc.actual_row(C) - expRow)
    for f in range(F):
        w = want[offsets[f]:offsets[f] + counts[f]]
        assert np.array_equal(got[f].view(np.uint64), w.view(np.uint64))
    ws.close()


@pytest.mark.parametrize("M,K,N,F", [(3000, 257, 1200, 3), (300, 1536, 700, 2)])
def test_encode_adversarial_sums(M, K, N, F, abft, orc, torch_cuda):
    """rowSumB_f runs as certified parallel row sums (per warp) with the
    reference-order re-sum for rows the certificate does not cover. Rows of B
    and columns of A built to defeat the certificate (tiny, huge, subnormal,
    cancelling, absorbed terms) must give checksums bit-identical to the
    reference's sequential ones, and so must the FMA chains that use them as
    weights."""
    torch = torch_cuda
    rng = np.random.default_rng(4040 + M)
    A = np.empty((M, K), np.float32)
    for k in range(K):
        A[:, k] = adversarial(rng, M, k % 13)
    B = np.empty((K, N), np.float32)
    for k in range(K):
        B[k, :] = adversarial(rng, N, (3 * k) % 13)
    counts, offsets = orc.split_dim(N, F)
    ws = abft.kernels.Workspace(M, N, K, counts, offsets)
    abft.kernels.encode(ws, to_dev(torch, A), to_dev(torch, B))
    torch.cuda.synchronize()
    got = ws.read_checksums()
    want = orc.encode(A, B, counts, offsets)
    for g, w, name in zip(got, want, ["colSumA", "expRow", "rowSumB", "expCol"]):
        assert np.array_equal(g.view(np.uint64), w.view(np.uint64)), name
    # the patterns make the order matter: the reference's sequential row sums
    # differ from the exactly rounded ones in some rows of B
    import math
    seq = orc.row_checksum_B(B[:, offsets[0]:offsets[0] + counts[0]])
    exact = np.array([math.fsum(B[k, offsets[0]:offsets[0] + counts[0]].astype(np.float64)) for k in range(K)])
    assert (seq != exact).any()
    ws.close()


def test_exact_chain_adversarial_rows(abft, orc, torch_cuda):
    """The same patterns along rows, with a fault to localise: the row arg-max
    re-sums its uncertified candidate rows exactly."""
    rng = np.random.default_rng(77)
    M, K, N, F = 600, 16, 1200, 2
    A, B = tiles(orc, M, K, N, 73, 74)
    counts, offsets = orc.split_dim(N, F)
    C0 = np.empty((M, N), np.float32)
    for i in range(M):
        C0[i, :] = adversarial(rng, N, i % 13)
    for f, (r, c) in enumerate([(37, 5), (300, 200)]):
        C = add_fault(C0, r, offsets[f] + c, 1.0e6)
        for tau in (1.0e3, 1.0e5):
            g = run_gpu_iteration(abft, torch_cuda, A, B, C, counts, offsets, [tau] * F, f, golden=C0)
            o = run_oracle_iteration(orc, A, B, C, counts, offsets, [tau] * F, f, golden=C0)
            assert_same(g, o)


def test_caller_owned_workspace_memory(abft, orc, torch_cuda):
    """A workspace placed in caller-owned device memory (any dtype; the size
    counts in bytes) gives the same checksums and decisions as one that
    allocates its own; a buffer one byte short is refused."""
    import ctypes
    torch = torch_cuda
    M, K, N, F = 1024, 256, 768, 3
    A, B = tiles(orc, M, K, N, 5, 6, "uniform")
    counts, offsets = orc.split_dim(N, F)
    c32 = np.ascontiguousarray(counts, np.int32)
    need = abft.lib.abft_ws_bytes(M, N, K, F, c32.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), 1)
    assert need > 0
    with pytest.raises(abft.AbftError):
        abft.kernels.Workspace(M, N, K, counts, offsets, max_iters=1,
                               device_buffer=torch.empty(need - 1, dtype=torch.uint8, device="cuda"))
    mem = torch.empty((need + 3) // 4, dtype=torch.float32, device="cuda")
    ws_own = abft.kernels.Workspace(M, N, K, counts, offsets, max_iters=1)
    ws_ext = abft.kernels.Workspace(M, N, K, counts, offsets, max_iters=1, device_buffer=mem)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    C0 = product_f64(A, B)
    res = []
    for ws in (ws_own, ws_ext):
        dC = to_dev(torch, add_fault(C0, 700, int(offsets[1]) + 9, 3.0))
        abft.kernels.encode(ws, dA, dB)
        ws.reset_counters()
        for f in range(F):
            abft.kernels.verify(ws, dC, f, 1e-5 * K, injected=(f == 1), it=0)
            abft.kernels.localize_correct(ws, dC, f, 1e-5 * K, injected=(f == 1), it=0)
        torch.cuda.synchronize()
        cm, _ = ws.counters()
        ec, er, rd = ws.read_log(1)
        res.append((ws.read_checksums(), cm, ec, er, rd, dC.cpu().numpy()))
    ws_own.close()
    ws_ext.close()
    (s0, cm0, ec0, er0, rd0, c0), (s1, cm1, ec1, er1, rd1, c1) = res
    for a, b in zip(s0, s1):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))
    assert list(cm0) == list(cm1) == [1, F - 1, 0, 0]
    assert np.array_equal(ec0, ec1) and np.array_equal(er0, er1) and int(er0[0][1]) == 700
    assert np.array_equal(rd0.view(np.uint64), rd1.view(np.uint64))
    assert np.array_equal(c0.view(np.uint32), c1.view(np.uint32))
