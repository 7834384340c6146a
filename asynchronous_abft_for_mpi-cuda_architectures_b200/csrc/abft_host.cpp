// Host helpers of the C ABI: input generation, grid geometry, thresholds and
// the injection plan. Compiled with -ffp-contract=off and no -march flag so
// that every double operation rounds exactly like the reference's x86-64 host
// code; random numbers come from libstdc++'s std::mt19937_64 and
// distributions, the generator and library the reference uses.

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <random>
#include <string>
#include <algorithm>

#include "abft_b200.h"

namespace abft {
void set_error(const std::string& msg);
}
using abft::set_error;

extern "C" {

// core/common.cuh:57-61
int abft_fill_random(float* out, int64_t n, uint64_t seed, int dist) {
    if (!out || n < 0 || (dist != 0 && dist != 1)) {
        set_error("abft_fill_random: bad argument");
        return ABFT_ERR_ARG;
    }
    std::mt19937_64 gen(seed);
    if (dist == 1) {
        std::normal_distribution<float> d(0.0f, 1.0f);
        for (int64_t i = 0; i < n; ++i) out[i] = d(gen);
    } else {
        std::uniform_real_distribution<float> d(-1.0f, 1.0f);
        for (int64_t i = 0; i < n; ++i) out[i] = d(gen);
    }
    return ABFT_OK;
}

// distribution/grid.cuh:7-12
int abft_choose_grid(int world, int* Pr, int* Pc) {
    if (world < 1 || !Pr || !Pc) {
        set_error("abft_choose_grid: world must be >= 1");
        return ABFT_ERR_ARG;
    }
    int pr = (int)std::sqrt((double)world);
    while (pr > 1 && (world % pr != 0)) --pr;
    if (pr < 1) pr = 1;
    *Pr = pr;
    *Pc = world / pr;
    return ABFT_OK;
}

// distribution/grid.cuh:15-28
int abft_split_dim(int total, int parts, int* counts, int* offsets) {
    if (total < 0 || parts < 1 || !counts || !offsets) {
        set_error("abft_split_dim: bad argument");
        return ABFT_ERR_ARG;
    }
    const int base = total / parts, rem = total % parts;
    int off = 0;
    for (int i = 0; i < parts; ++i) {
        counts[i] = base + (i < rem ? 1 : 0);
        offsets[i] = off;
        off += counts[i];
    }
    return ABFT_OK;
}

// main.cu:55-69
int abft_frag_count(int M, int K, int N, int M_b, int N_b, int frags_per_rank, int64_t frag_cap) {
    if (frags_per_rank < 1 || N_b < 1) {
        set_error("abft_frag_count: bad argument");
        return ABFT_ERR_ARG;
    }
    int F = std::min(frags_per_rank, N_b);
    const bool small = std::max(M, std::max(K, N)) < 1024;
    if (small) F = 1;
    if (!small && frag_cap > 0) {
        const int64_t elems = (int64_t)M_b * (int64_t)N_b;
        const int need = (int)((elems + frag_cap - 1) / frag_cap);
        if (need > F) F = std::min(need, N_b);
    }
    return F;
}

int64_t abft_c_pitch(int n) {
    if (n < 1) {
        set_error("abft_c_pitch: n must be >= 1");
        return -1;
    }
    const int64_t bytes = 4 * (int64_t)n;
    return (bytes % 65536 == 0) ? (int64_t)n + 32 : (int64_t)n;
}

// core/common.cuh:64-74
double abft_matrix_inf_norm(const float* M, int rows, int cols, int64_t ld) {
    double mx = 0.0;
    for (int i = 0; i < rows; ++i) {
        double rs = 0.0;
        for (int j = 0; j < cols; ++j) rs += std::abs(static_cast<double>(M[(int64_t)i * ld + j]));
        mx = std::max(mx, rs);
    }
    return mx;
}

// core/common.cuh:77-83
double abft_threshold_formula(int k, double nA, double nB) {
    const double eps = static_cast<double>(FLT_EPSILON);
    double denom = 1.0 - static_cast<double>(k) * eps;
    if (denom <= 0.0) denom = 1.0;
    const double g = (static_cast<double>(k) * eps) / denom;
    return g * nA * nB;
}

// main.cu:147-164
int abft_frag_thresholds(const float* A, int M_b, int K, int64_t lda, const float* B, int64_t ldb, int F,
                         const int* counts, const int* offsets, double override_tau, double* tau) {
    if (!tau || F < 1 || !counts || !offsets || (override_tau <= 0.0 && (!A || !B))) {
        set_error("abft_frag_thresholds: bad argument");
        return ABFT_ERR_ARG;
    }
    if (override_tau > 0.0) {
        for (int f = 0; f < F; ++f) tau[f] = override_tau;
        return ABFT_OK;
    }
    const double nA = abft_matrix_inf_norm(A, M_b, K, lda);
    for (int f = 0; f < F; ++f) {
        double mx = 0.0;
        for (int k = 0; k < K; ++k) {
            double rs = 0.0;
            const float* row = B + (int64_t)k * ldb + offsets[f];
            for (int j = 0; j < counts[f]; ++j) rs += std::abs(static_cast<double>(row[j]));
            if (rs > mx) mx = rs;
        }
        tau[f] = abft_threshold_formula(K, nA, mx);
    }
    return ABFT_OK;
}

// kernels/swifi.cuh:25-31
int abft_swifi_zone_range(const char* zone, int* lo, int* hi) {
    if (!lo || !hi) {
        set_error("abft_swifi_zone_range: bad argument");
        return ABFT_ERR_ARG;
    }
    const std::string z(zone ? zone : "");
    if (z == "sign") { *lo = 31; *hi = 31; }
    else if (z == "exponent") { *lo = 23; *hi = 30; }
    else if (z == "sig_high") { *lo = 13; *hi = 22; }
    else if (z == "sig_low") { *lo = 0; *hi = 12; }
    else { *lo = 0; *hi = 31; }
    return ABFT_OK;
}

// pipeline/passes.cuh:148-156 and kernels/swifi.cuh:67-71, :91-98
int abft_injection_plan(uint64_t base_seed, int rank, int it, int F, int M_b, const int* counts, int mode,
                        int zone_lo, int zone_hi, int* frag, int* row, int* col, int* bit) {
    if (!frag || !row || !col || !bit || F < 1 || M_b < 1 || !counts ||
        (mode == ABFT_INJECT_SWIFI && (zone_lo < 0 || zone_hi > 31 || zone_lo > zone_hi))) {
        set_error("abft_injection_plan: bad argument");
        return ABFT_ERR_ARG;
    }
    *frag = *row = *col = *bit = -1;
    if (mode != ABFT_INJECT_ADD && mode != ABFT_INJECT_SWIFI) return ABFT_OK;
    const uint64_t seed = base_seed + (uint64_t)rank * 7919ull + (uint64_t)it * 104729ull;
    std::mt19937_64 rng(seed);
    std::uniform_int_distribution<int> fd(0, F - 1);
    const int f = fd(rng);
    std::mt19937_64 gen(seed + static_cast<uint64_t>(f));
    std::uniform_int_distribution<int> rd(0, M_b - 1);
    std::uniform_int_distribution<int> cd(0, counts[f] - 1);
    *frag = f;
    *row = rd(gen);
    *col = cd(gen);
    if (mode == ABFT_INJECT_SWIFI) {
        std::uniform_int_distribution<int> bd(zone_lo, zone_hi);
        *bit = bd(gen);
    }
    return ABFT_OK;
}

int abft_injection_plan_tile(uint64_t seed, int M_b, int F, const int* counts, const int* offsets, int mode,
                             int zone_lo, int zone_hi, int* frag, int* row, int* col, int* bit) {
    if (!frag || !row || !col || !bit || F < 1 || M_b < 1 || !counts || !offsets ||
        (mode == ABFT_INJECT_SWIFI && (zone_lo < 0 || zone_hi > 31 || zone_lo > zone_hi))) {
        set_error("abft_injection_plan_tile: bad argument");
        return ABFT_ERR_ARG;
    }
    *frag = *row = *col = *bit = -1;
    if (mode != ABFT_INJECT_ADD && mode != ABFT_INJECT_SWIFI) return ABFT_OK;
    int N_b = 0;
    for (int f = 0; f < F; ++f) N_b = std::max(N_b, offsets[f] + counts[f]);
    std::mt19937_64 gen(seed);
    std::uniform_int_distribution<int> rd(0, M_b - 1);
    std::uniform_int_distribution<int> cd(0, N_b - 1);
    *row = rd(gen);
    const int j = cd(gen);
    if (mode == ABFT_INJECT_SWIFI) {
        std::uniform_int_distribution<int> bd(zone_lo, zone_hi);
        *bit = bd(gen);
    }
    int fr = 0;
    for (int f = 0; f < F; ++f)
        if (j >= offsets[f] && j < offsets[f] + counts[f]) fr = f;
    *frag = fr;
    *col = j - offsets[fr];
    return ABFT_OK;
}

}  // extern "C"
