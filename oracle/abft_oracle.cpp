// CPU oracle: a plain restatement of the reference's ABFT arithmetic.
//
// TEST INFRASTRUCTURE ONLY. Nothing in the product links, loads or calls this
// file: tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it
// as the reference of correctness (and as the timed CPU arm), nothing else.
//
// Every function restates one piece of FaridRojas/Asynchronous_ABFT_for_MPI-
// CUDA_Architectures in the reference's own evaluation order, so that results
// are bit-identical to the reference for the same inputs:
//   * each checksum is a sequential double sum in the reference's loop order;
//   * the reference's `s += x * y` forms compile (nvcc, default -fmad=true) to
//     a fused multiply-add, so they are written std::fma here, and this file is
//     compiled with -ffp-contract=off so that nothing else is fused;
//   * the arg-max of k_detect_row / k_locate_correct is emulated slot by slot:
//     256 strided per-thread scans followed by the same shared-memory tree;
//   * random numbers come from libstdc++'s std::mt19937_64 and distributions,
//     the generator and library the reference uses.
// Pinning: tests/test_oracle_golden.py checks these functions against fixtures
// produced by the reference's own host code (tests/golden/make_golden.py runs
// oracle/_ref/host_probe) and, on a GPU, against the reference's own kernels
// (oracle/_ref/kernel_harness).

#include <cmath>
#include <cfloat>
#include <cstdint>
#include <cstring>
#include <random>
#include <string>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef long long i64;

extern "C" {

// ---------------------------------------------------------------- inputs ---

// core/common.cuh:57-61 (fill_random). dist=1 is the normal(0,1) extension
// used by the non-square workloads; it follows the same generator discipline.
void oracle_fill_random(float* out, i64 n, uint64_t seed, int dist) {
    std::mt19937_64 gen(seed);
    if (dist == 1) {
        std::normal_distribution<float> d(0.0f, 1.0f);
        for (i64 i = 0; i < n; ++i) out[i] = d(gen);
    } else {
        std::uniform_real_distribution<float> d(-1.0f, 1.0f);
        for (i64 i = 0; i < n; ++i) out[i] = d(gen);
    }
}

// ------------------------------------------------------------------ grid ---

// distribution/grid.cuh:7-12
void oracle_choose_grid(int world, int* Pr, int* Pc) {
    int pr = (int)std::sqrt((double)world);
    while (pr > 1 && (world % pr != 0)) --pr;
    if (pr < 1) pr = 1;
    *Pr = pr;
    *Pc = world / pr;
}

// distribution/grid.cuh:15-28
void oracle_split_dim(int total, int parts, int* counts, int* offsets) {
    int base = total / parts, rem = total % parts, off = 0;
    for (int i = 0; i < parts; ++i) {
        counts[i] = base + (i < rem ? 1 : 0);
        offsets[i] = off;
        off += counts[i];
    }
}

// main.cu:55-69: fragments per rank.
int oracle_frag_count(int M, int K, int N, int M_b, int N_b, int frags_per_rank, i64 frag_cap) {
    int F = std::min(frags_per_rank, N_b);
    bool small = std::max(M, std::max(K, N)) < 1024;
    if (small) F = 1;
    if (!small && frag_cap > 0) {
        i64 elems = (i64)M_b * (i64)N_b;
        int need = (int)((elems + frag_cap - 1) / frag_cap);
        if (need > F) F = std::min(need, N_b);
    }
    return F;
}

// ------------------------------------------------------------ thresholds ---

// core/common.cuh:64-74
double oracle_matrix_inf_norm(const float* M, int rows, int cols, i64 ld) {
    double mx = 0.0;
    for (int i = 0; i < rows; ++i) {
        double rs = 0.0;
        for (int j = 0; j < cols; ++j) rs += std::abs((double)M[(i64)i * ld + j]);
        mx = std::max(mx, rs);
    }
    return mx;
}

// core/common.cuh:77-83
double oracle_threshold_formula(int k, double nA, double nB) {
    const double eps = (double)FLT_EPSILON;
    double denom = 1.0 - (double)k * eps;
    if (denom <= 0.0) denom = 1.0;
    double g = ((double)k * eps) / denom;
    return g * nA * nB;
}

// main.cu:148-164: one threshold per fragment (override if > 0).
void oracle_frag_thresholds(const float* A, int M_b, int K, i64 lda, const float* B, i64 ldb, int F,
                            const int* counts, const int* offsets, double override_tau, double* out) {
    double nA = oracle_matrix_inf_norm(A, M_b, K, lda);
    for (int f = 0; f < F; ++f) {
        if (override_tau > 0.0) { out[f] = override_tau; continue; }
        double mx = 0.0;
        for (int k = 0; k < K; ++k) {
            double rs = 0.0;
            for (int j = 0; j < counts[f]; ++j) rs += std::abs((double)B[(i64)k * ldb + offsets[f] + j]);
            if (rs > mx) mx = rs;
        }
        out[f] = oracle_threshold_formula(K, nA, mx);
    }
}

// --------------------------------------------------------------- encode ----

// kernels/abft_stepwise.cuh:9-18 (k_col_checksum_A): colSumA[k] = sum_i A[i,k].
void oracle_col_checksum_A(const float* A, i64 lda, int M, int K, double* out) {
    for (int k = 0; k < K; ++k) out[k] = 0.0;
    for (int i = 0; i < M; ++i) {
        const float* r = A + (i64)i * lda;
        for (int k = 0; k < K; ++k) out[k] += (double)r[k];
    }
}

// kernels/abft_stepwise.cuh:31-41 (k_expected_row): fused multiply-add chain over k.
void oracle_expected_row(const double* colSumA, const float* B, i64 ldb, int K, int N, double* out) {
    for (int j = 0; j < N; ++j) out[j] = 0.0;
    for (int k = 0; k < K; ++k) {
        const float* r = B + (i64)k * ldb;
        const double a = colSumA[k];
        for (int j = 0; j < N; ++j) out[j] = std::fma(a, (double)r[j], out[j]);
    }
}

// kernels/abft_stepwise.cuh:121-132 (k_row_checksum_B_g): rowSumB[k] = sum_j B[k,j].
void oracle_row_checksum_B(const float* B, i64 ldb, int K, int N, double* out) {
#pragma omp parallel for schedule(static)
    for (int k = 0; k < K; ++k) {
        double s = 0.0;
        const float* r = B + (i64)k * ldb;
        for (int j = 0; j < N; ++j) s += (double)r[j];
        out[k] = s;
    }
}

// kernels/abft_stepwise.cuh:134-146 (k_expected_col_g): fused multiply-add chain over k.
void oracle_expected_col(const float* A, i64 lda, const double* rowSumB, int M, int K, double* out) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < M; ++i) {
        double s = 0.0;
        const float* r = A + (i64)i * lda;
        for (int k = 0; k < K; ++k) s = std::fma((double)r[k], rowSumB[k], s);
        out[i] = s;
    }
}

// --------------------------------------------------------------- verify ----

// kernels/abft_stepwise.cuh:43-52 (k_actual_row): actualRow[j] = sum_i C[i,j], i ascending.
// Row-outer loop keeps each column's sum in ascending-i order; columns are split
// across threads, never the sum itself.
void oracle_actual_row(const float* C, i64 ldc, int M, int N, double* out) {
#pragma omp parallel
    {
#ifdef _OPENMP
        int t = omp_get_thread_num(), nt = omp_get_num_threads();
#else
        int t = 0, nt = 1;
#endif
        int per = (N + nt - 1) / nt;
        int j0 = t * per, j1 = std::min(N, j0 + per);
        for (int j = j0; j < j1; ++j) out[j] = 0.0;
        for (int i = 0; i < M; ++i) {
            const float* r = C + (i64)i * ldc;
            for (int j = j0; j < j1; ++j) out[j] += (double)r[j];
        }
    }
}

// kernels/abft_stepwise.cuh:148-159 (k_actual_col_g): actualCol[i] = sum_j C[i,j], j ascending.
void oracle_actual_col(const float* C, i64 ldc, int M, int N, double* out) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < M; ++i) {
        double s = 0.0;
        const float* r = C + (i64)i * ldc;
        for (int j = 0; j < N; ++j) s += (double)r[j];
        out[i] = s;
    }
}

// The arg-max of k_detect_row (abft_stepwise.cuh:85-110) and k_locate_correct
// (:174-187), launched with one block of 256 threads: thread t scans
// j = t, t+256, ... keeping the first j with d > tau && d > best (best starts
// at 0.0), then a shared-memory tree keeps the right operand only when it is
// strictly larger. Returns -1 when no element passes.
int oracle_argmax256(const double* expected, const double* actual, int n, double tau) {
    double sd[256];
    int sj[256];
    for (int t = 0; t < 256; ++t) {
        double best = 0.0;
        int bj = -1;
        for (int j = t; j < n; j += 256) {
            double d = std::fabs(actual[j] - expected[j]);
            if (d > tau && d > best) { best = d; bj = j; }
        }
        sd[t] = best;
        sj[t] = bj;
    }
    for (int s = 128; s > 0; s >>= 1)
        for (int t = 0; t < s; ++t)
            if (sd[t + s] > sd[t]) { sd[t] = sd[t + s]; sj[t] = sj[t + s]; }
    return sj[0];
}

// k_detect_row (abft_stepwise.cuh:85-118): errcol, rowdiff and the CM bucket
// {0:TP, 1:TN, 2:FP, 3:FN}.
void oracle_detect_row(const double* expected, const double* actual, int n, double tau, int injected,
                       int* errcol, double* rowdiff, int* cm) {
    int ec = oracle_argmax256(expected, actual, n, tau);
    *errcol = ec;
    *rowdiff = (ec >= 0) ? (actual[ec] - expected[ec]) : 0.0;
    int det = ec >= 0;
    int idx = injected ? (det ? 0 : 3) : (det ? 2 : 1);
    if (cm) cm[idx] += 1;
}

// k_locate_correct (abft_stepwise.cuh:162-206). C_frag points at the
// fragment's first column; golden (may be null) at the full tile. Returns the
// located row (-1 = none).
int oracle_locate_correct(const double* expCol, const double* actCol, int M, double tau, int errcol,
                          double rowdiff, float* C_frag, i64 ldc, const float* golden, i64 ldg,
                          int frag_off, int injected, int* n_restored) {
    if (errcol < 0) return -1;
    int er = oracle_argmax256(expCol, actCol, M, tau);
    if (er >= 0) {
        float c = (float)((double)C_frag[(i64)er * ldc + errcol] - rowdiff);
        C_frag[(i64)er * ldc + errcol] = c;
        if (injected && golden) {
            float g = golden[(i64)er * ldg + frag_off + errcol];
            if (std::fabs((double)c - (double)g) <= tau && n_restored) *n_restored += 1;
        }
    }
    return er;
}

// ------------------------------------------------------------ injection ----

// kernels/swifi.cuh:25-31
void oracle_swifi_zone_range(const char* zone, int* lo, int* hi) {
    std::string z(zone ? zone : "");
    if (z == "sign") { *lo = 31; *hi = 31; }
    else if (z == "exponent") { *lo = 23; *hi = 30; }
    else if (z == "sig_high") { *lo = 13; *hi = 22; }
    else if (z == "sig_low") { *lo = 0; *hi = 12; }
    else { *lo = 0; *hi = 31; }
}

// pipeline/passes.cuh:148-156: per-(rank, iteration) seed and injected fragment.
uint64_t oracle_inject_seed(uint64_t base_seed, int rank, int it) {
    return base_seed + (uint64_t)rank * 7919ull + (uint64_t)it * 104729ull;
}
int oracle_inject_frag(uint64_t inject_seed, int F) {
    std::mt19937_64 rng(inject_seed);
    std::uniform_int_distribution<int> d(0, F - 1);
    return d(rng);
}

// kernels/swifi.cuh:67-71 and :91-98: row, col (and bit when lo <= hi) drawn in
// that order from mt19937_64(seed + frag). bit is -1 when lo > hi (additive).
void oracle_inject_position(uint64_t inject_seed, int frag, int M_b, int N_f, int lo, int hi, int* row,
                            int* col, int* bit) {
    std::mt19937_64 gen(inject_seed + (uint64_t)frag);
    std::uniform_int_distribution<int> rd(0, M_b - 1);
    std::uniform_int_distribution<int> cd(0, N_f - 1);
    *row = rd(gen);
    *col = cd(gen);
    if (lo <= hi) {
        std::uniform_int_distribution<int> bd(lo, hi);
        *bit = bd(gen);
    } else {
        *bit = -1;
    }
}

// Tile-uniform scheme (the 1024^3 workload's wording, an extension the
// reference cannot express): mt19937_64(seed) draws i uniform over the M_b
// rows and j uniform over the whole N_b-column tile (then the bit when
// lo <= hi); the fragment is the one that holds column j.
void oracle_inject_position_tile(uint64_t seed, int M_b, int F, const int* counts, const int* offsets, int lo,
                                 int hi, int* frag, int* row, int* col, int* bit) {
    int N_b = 0;
    for (int f = 0; f < F; ++f) N_b = std::max(N_b, offsets[f] + counts[f]);
    std::mt19937_64 gen(seed);
    std::uniform_int_distribution<int> rd(0, M_b - 1);
    std::uniform_int_distribution<int> cd(0, N_b - 1);
    *row = rd(gen);
    const int j = cd(gen);
    *bit = -1;
    if (lo <= hi) {
        std::uniform_int_distribution<int> bd(lo, hi);
        *bit = bd(gen);
    }
    *frag = 0;
    for (int f = 0; f < F; ++f)
        if (j >= offsets[f] && j < offsets[f] + counts[f]) *frag = f;
    *col = j - offsets[*frag];
}

// kernels/swifi.cuh:55-59 and :33-40
void oracle_inject_add(float* C, i64 ldc, int row, int col, float delta) { C[(i64)row * ldc + col] += delta; }
void oracle_inject_bitflip(float* C, i64 ldc, int row, int col, int bit) {
    uint32_t u;
    std::memcpy(&u, &C[(i64)row * ldc + col], 4);
    u ^= (1u << bit);
    std::memcpy(&C[(i64)row * ldc + col], &u, 4);
}

// -------------------------------------------------------- whole passes -----

// Encode for one rank tile, all fragments: colSumA[K], expRow[N_b] (absolute
// column index), and, when rowSumB/expCol are non-null, the localisation
// checksums per fragment rowSumB[F*K], expCol[F*M_b] that the reference
// recomputes after each detection (abft_stepwise.cuh:230-233).
void oracle_encode(const float* A, i64 lda, const float* B, i64 ldb, int M_b, int K, int F, const int* counts,
                   const int* offsets, double* colSumA, double* expRow, double* rowSumB, double* expCol) {
    oracle_col_checksum_A(A, lda, M_b, K, colSumA);
    for (int f = 0; f < F; ++f) {
        oracle_expected_row(colSumA, B + offsets[f], ldb, K, counts[f], expRow + offsets[f]);
        if (rowSumB && expCol) {
            oracle_row_checksum_B(B + offsets[f], ldb, K, counts[f], rowSumB + (i64)f * K);
            oracle_expected_col(A, lda, rowSumB + (i64)f * K, M_b, K, expCol + (i64)f * M_b);
        }
    }
}

// The verify half of one pass_online_loop iteration (passes.cuh:180-198) on a
// rank tile C (ld ldc) that already carries this iteration's fault. When
// expCol is null the localisation checksums are recomputed from A and B after
// each detection, as the reference does; otherwise they are taken from expCol.
// Per fragment f the decision is written to errcol[f], errrow[f], rowdiff[f].
void oracle_verify_iteration(float* C, i64 ldc, const float* A, i64 lda, const float* B, i64 ldb, int M_b,
                             int K, int F, const int* counts, const int* offsets, const double* expRow,
                             const double* expCol, const double* tau, int inject_frag, int do_localize,
                             const float* golden, i64 ldg, int* cm, int* n_restored, int* errcol, int* errrow,
                             double* rowdiff) {
    int nfmax = 0;
    for (int f = 0; f < F; ++f) nfmax = std::max(nfmax, counts[f]);
    std::vector<double> act(nfmax), actCol(M_b), rsb, ec_on_demand;
    for (int f = 0; f < F; ++f) {
        int injected = (f == inject_frag) ? 1 : 0;
        float* Cf = C + offsets[f];
        oracle_actual_row(Cf, ldc, M_b, counts[f], act.data());
        int ec;
        double rd;
        oracle_detect_row(expRow + offsets[f], act.data(), counts[f], tau[f], injected, &ec, &rd, cm);
        int er = -1;
        if (do_localize && ec >= 0) {
            const double* ecol;
            if (expCol) {
                ecol = expCol + (i64)f * M_b;
            } else {
                rsb.resize(K);
                ec_on_demand.resize(M_b);
                oracle_row_checksum_B(B + offsets[f], ldb, K, counts[f], rsb.data());
                oracle_expected_col(A, lda, rsb.data(), M_b, K, ec_on_demand.data());
                ecol = ec_on_demand.data();
            }
            oracle_actual_col(Cf, ldc, M_b, counts[f], actCol.data());
            er = oracle_locate_correct(ecol, actCol.data(), M_b, tau[f], ec, rd, Cf, ldc, golden, ldg, offsets[f],
                                       injected, n_restored);
        }
        if (errcol) errcol[f] = ec;
        if (errrow) errrow[f] = er;
        if (rowdiff) rowdiff[f] = rd;
    }
}

// Decision path of pass_online_loop (passes.cuh:90-227) for `repeats`
// iterations on one rank, given the fault-free SGEMM output C_clean (M_b x N_b,
// ld N_b) that every iteration reproduces. mode: 0 none, 1 add, 2 swifi.
// Outputs: the two double-buffer tiles after the loop (buf0/buf1, M_b*N_b),
// cm[4] and n_restored (accumulated), and per-iteration logs:
//   inj[it*4 + {0,1,2,3}] = inject frag, row, col, bit (-1 when none)
//   errcol/errrow/rowdiff[it*F + f].
void oracle_online_loop(const float* C_clean, const float* A, const float* B, int M_b, int K, int N_b, int F,
                        const int* counts, const int* offsets, const double* tau, int mode, int zone_lo,
                        int zone_hi, float add_delta, uint64_t base_seed, int rank, int repeats,
                        const float* golden, float* buf0, float* buf1, int* cm, int* n_restored, int* inj,
                        int* errcol, int* errrow, double* rowdiff, int seed_scheme) {
    const i64 tile = (i64)M_b * N_b;
    std::vector<double> colSumA(K), expRow(N_b), rowSumB((i64)F * K), expCol((i64)F * M_b);
    oracle_encode(A, K, B, N_b, M_b, K, F, counts, offsets, colSumA.data(), expRow.data(), rowSumB.data(),
                  expCol.data());
    float* bufs[2] = {buf0, buf1};
    const int inject_on = (mode == 1 || mode == 2);
    for (int it = 0; it < repeats; ++it) {
        float* C = bufs[it % 2];
        std::memcpy(C, C_clean, sizeof(float) * tile);
        int frag = -1, row = -1, col = -1, bit = -1;
        uint64_t seed = oracle_inject_seed(base_seed, rank, it);
        if (inject_on && seed_scheme == 1) {
            oracle_inject_position_tile(base_seed + (uint64_t)it, M_b, F, counts, offsets, mode == 2 ? zone_lo : 1,
                                        mode == 2 ? zone_hi : 0, &frag, &row, &col, &bit);
            if (mode == 1) oracle_inject_add(C + offsets[frag], N_b, row, col, add_delta);
            else oracle_inject_bitflip(C + offsets[frag], N_b, row, col, bit);
        } else if (inject_on) {
            frag = oracle_inject_frag(seed, F);
            if (mode == 1) {
                oracle_inject_position(seed, frag, M_b, counts[frag], 1, 0, &row, &col, &bit);
                oracle_inject_add(C + offsets[frag], N_b, row, col, add_delta);
            } else {
                oracle_inject_position(seed, frag, M_b, counts[frag], zone_lo, zone_hi, &row, &col, &bit);
                oracle_inject_bitflip(C + offsets[frag], N_b, row, col, bit);
            }
        }
        if (inj) {
            inj[it * 4 + 0] = frag; inj[it * 4 + 1] = row; inj[it * 4 + 2] = col; inj[it * 4 + 3] = bit;
        }
        oracle_verify_iteration(C, N_b, A, K, B, N_b, M_b, K, F, counts, offsets, expRow.data(), expCol.data(), tau,
                                frag, inject_on, golden, N_b, cm, n_restored, errcol ? errcol + (i64)it * F : nullptr,
                                errrow ? errrow + (i64)it * F : nullptr, rowdiff ? rowdiff + (i64)it * F : nullptr);
    }
}

}  // extern "C"
