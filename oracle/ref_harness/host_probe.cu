// Host-side probe of the reference's own helper functions.
//
// TEST INFRASTRUCTURE ONLY. Compiled by oracle/Makefile from the reference
// sources where they lie (include path = the reference checkout) into
// oracle/_ref/host_probe. It calls the reference's host functions directly and
// prints their results, so that the fixtures in tests/golden/ come from the
// reference itself rather than from a restatement:
//   fill_random            core/common.cuh:57-61
//   matrix_inf_norm        core/common.cuh:64-74
//   compute_threshold_formula core/common.cuh:77-83
//   stats_of               core/common.cuh:86-106
//   choose_grid/split_dim  distribution/grid.cuh:7-28
//   swifi_zone_range       kernels/swifi.cuh:25-31
//   inject_add_constant    kernels/swifi.cuh:61-76 (row/col draws)
//   finalize_metrics, print_metrics, log_metrics_csv  metrics/metrics.cuh:132-254
// The inline call-site logic of main.cu / passes.cuh that is not a function
// (per-fragment threshold loop main.cu:147-164, inject_frag draw
// passes.cuh:148-156, F policy main.cu:55-69) is restated here line for line
// and marked as such.
//
// It refuses to run when a GPU is visible: inject_add_constant launches a
// one-thread kernel on the pointer it is given, and this probe passes none.
// Without a device the launch is rejected by the runtime before anything runs.

#include "core/common.cuh"
#include "core/types.cuh"
#include "distribution/grid.cuh"
#include "kernels/swifi.cuh"
#include "metrics/metrics.cuh"

#include <cinttypes>
#include <cstdio>
#include <cstring>

static uint32_t fbits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static uint64_t dbits(double d) { uint64_t u; std::memcpy(&u, &d, 8); return u; }

static int usage() {
    std::fprintf(stderr, "host_probe MODE ARGS (see source)\n");
    return 2;
}

int main(int argc, char** argv) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) == cudaSuccess && ndev > 0) {
        std::fprintf(stderr, "host_probe: a GPU is visible; this probe runs on CPU-only hosts\n");
        return 4;
    }
    (void)cudaGetLastError();
    if (argc < 2) return usage();
    std::string mode = argv[1];

    if (mode == "fill" && argc == 5) {
        // fill SEED TOTAL NPRINT : fill a vector of TOTAL values, print first NPRINT bit patterns
        // and an order-sensitive hash of all TOTAL values.
        uint64_t seed = std::strtoull(argv[2], nullptr, 10);
        size_t total = std::strtoull(argv[3], nullptr, 10);
        size_t np = std::strtoull(argv[4], nullptr, 10);
        std::vector<float> v(total);
        fill_random(v, seed);
        uint64_t h = 1469598103934665603ull;
        for (size_t i = 0; i < total; ++i) { h ^= fbits(v[i]); h *= 1099511628211ull; }
        std::printf("hash %" PRIu64 "\n", h);
        for (size_t i = 0; i < np && i < total; ++i) std::printf("%08x\n", fbits(v[i]));
        return 0;
    }
    if (mode == "grid" && argc == 3) {
        int Pr = 0, Pc = 0;
        choose_grid(std::atoi(argv[2]), Pr, Pc);
        std::printf("%d %d\n", Pr, Pc);
        return 0;
    }
    if (mode == "split" && argc == 4) {
        std::vector<int> c, o;
        split_dim(std::atoi(argv[2]), std::atoi(argv[3]), c, o);
        for (size_t i = 0; i < c.size(); ++i) std::printf("%d %d\n", c[i], o[i]);
        return 0;
    }
    if (mode == "zone" && argc == 3) {
        int lo, hi;
        swifi_zone_range(argv[2], lo, hi);
        std::printf("%d %d\n", lo, hi);
        return 0;
    }
    if (mode == "formula" && argc == 5) {
        // formula K NORM_A NORM_B (norms given as %a hex-floats or decimals)
        double t = compute_threshold_formula(std::atoi(argv[2]), std::strtod(argv[3], nullptr),
                                             std::strtod(argv[4], nullptr));
        std::printf("%016" PRIx64 "\n", dbits(t));
        return 0;
    }
    if (mode == "thresholds" && argc == 9) {
        // thresholds M K N SEED_A SEED_B F OVERRIDE : single-rank regen_inputs threshold part.
        int M = std::atoi(argv[2]), K = std::atoi(argv[3]), N = std::atoi(argv[4]);
        uint64_t sa = std::strtoull(argv[5], nullptr, 10), sb = std::strtoull(argv[6], nullptr, 10);
        int frags = std::atoi(argv[7]);
        double ovr = std::strtod(argv[8], nullptr);
        // F policy, restated from main.cu:55-61 (frag_cap off)
        int F = std::min(frags, N);
        if (std::max(M, std::max(K, N)) < 1024) F = 1;
        std::vector<int> cc, co;
        split_dim(N, F, cc, co);
        std::vector<float> A((size_t)M * K), B((size_t)K * N);
        fill_random(A, sa);
        fill_random(B, sb);
        double norm_A = matrix_inf_norm(A.data(), M, K, K);
        std::printf("F %d\n", F);
        std::printf("normA %016" PRIx64 "\n", dbits(norm_A));
        // per-fragment loop restated from main.cu:149-164
        for (int f = 0; f < F; ++f) {
            double th;
            if (ovr > 0.0) th = ovr;
            else {
                double mx = 0.0;
                for (int k = 0; k < K; ++k) {
                    double rs = 0.0;
                    for (int j = 0; j < cc[f]; ++j) rs += std::abs((double)B[(size_t)k * N + co[f] + j]);
                    if (rs > mx) mx = rs;
                }
                th = compute_threshold_formula(K, norm_A, mx);
            }
            std::printf("tau %d %016" PRIx64 "\n", f, dbits(th));
        }
        return 0;
    }
    if (mode == "inject" && argc >= 7) {
        // inject BASE_SEED RANK IT M_B NF_0 [NF_1 ...] : inject_frag draw (restated,
        // passes.cuh:148-156) then the reference's own inject_add_constant row/col draws.
        uint64_t base = std::strtoull(argv[2], nullptr, 10);
        int rank = std::atoi(argv[3]);
        int it = std::atoi(argv[4]);
        int M_b = std::atoi(argv[5]);
        std::vector<int> nf;
        for (int i = 6; i < argc; ++i) nf.push_back(std::atoi(argv[i]));
        int F = (int)nf.size();
        uint64_t inject_seed = base + (uint64_t)rank * 7919ull + (uint64_t)it * 104729ull;
        std::mt19937_64 rng(inject_seed);
        std::uniform_int_distribution<int> d(0, F - 1);
        int frag = d(rng);
        InjectionInfo info = inject_add_constant(nullptr, 1, M_b, nf[frag], frag, inject_seed, 0);
        (void)cudaGetLastError();
        std::printf("%d %d %d\n", frag, info.row, info.col);
        return 0;
    }
    if (mode == "stats" && argc >= 3) {
        std::vector<double> s;
        for (int i = 2; i < argc; ++i) s.push_back(std::strtod(argv[i], nullptr));
        TimingStats t = stats_of(s);
        std::printf("%016" PRIx64 " %016" PRIx64 " %016" PRIx64 " %016" PRIx64 " %d\n", dbits(t.min_ms),
                    dbits(t.median_ms), dbits(t.mean_ms), dbits(t.max_ms), t.n_samples);
        return 0;
    }
    if (mode == "metrics" && argc == 3 + 22) {
        // metrics CSV_PATH scheme inject zone baseline_only calibrate M K N Pr Pc F repeats tau
        //         TP TN FP FN restored  bmin bmed bmean bmax  (protected = baseline * 1.25)
        int a = 2;
        std::string path = argv[a++];
        ExperimentMetrics m{};
        m.scheme = argv[a++]; m.inject = argv[a++]; m.swifi_zone = argv[a++];
        m.baseline_only = std::atoi(argv[a++]) != 0; m.calibrate = std::atoi(argv[a++]) != 0;
        m.M = std::atoi(argv[a++]); m.K = std::atoi(argv[a++]); m.N = std::atoi(argv[a++]);
        m.Pr = std::atoi(argv[a++]); m.Pc = std::atoi(argv[a++]);
        m.frags_per_rank = std::atoi(argv[a++]);
        m.num_fragments_total = m.Pr * m.Pc * m.frags_per_rank;
        m.repeats = std::atoi(argv[a++]);
        m.threshold_used = std::strtod(argv[a++], nullptr);
        m.cm.TP = std::atoi(argv[a++]); m.cm.TN = std::atoi(argv[a++]);
        m.cm.FP = std::atoi(argv[a++]); m.cm.FN = std::atoi(argv[a++]);
        m.n_successfully_restored = std::atoi(argv[a++]);
        m.baseline.min_ms = std::strtod(argv[a++], nullptr);
        m.baseline.median_ms = std::strtod(argv[a++], nullptr);
        m.baseline.mean_ms = std::strtod(argv[a++], nullptr);
        m.baseline.max_ms = std::strtod(argv[a++], nullptr);
        m.protected_.min_ms = m.baseline.min_ms * 1.25;
        m.protected_.median_ms = m.baseline.median_ms * 1.25;
        m.protected_.mean_ms = m.baseline.mean_ms * 1.25;
        m.protected_.max_ms = m.baseline.max_ms * 1.25;
        if (m.calibrate) {
            m.calib_max_diff = 0.125;
            m.calib_safety_factor = 10.0;
            m.calib_suggested_tau = 1.25;
        }
        finalize_metrics(m);
        print_metrics(m);
        log_metrics_csv(m, path);
        return 0;
    }
    return usage();
}
