// Metrics, report and CSV of the C ABI, formatted like the reference's
// metrics module so that existing CSV consumers keep working.

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <sstream>
#include <string>
#include <vector>

#include "abft_b200.h"

namespace abft {
void set_error(const std::string& msg);
}
using abft::set_error;

namespace {

double gflops(double ms, int M, int N, int K) {
    if (ms <= 0.0) return 0.0;
    const double flops = 2.0 * (double)M * (double)N * (double)K;
    return flops / (ms * 1e6);
}

}  // namespace

extern "C" {

int abft_stats_of(const double* samples, int n, abft_timing* out) {
    if (!out || n < 0 || (n > 0 && !samples)) {
        set_error("abft_stats_of: bad argument");
        return ABFT_ERR_ARG;
    }
    *out = abft_timing{};
    out->n_samples = n;
    if (n == 0) return ABFT_OK;
    std::vector<double> s(samples, samples + n);
    double sum = 0.0;
    for (double v : s) sum += v;
    out->mean_ms = sum / s.size();
    std::sort(s.begin(), s.end());
    out->min_ms = s.front();
    out->max_ms = s.back();
    out->median_ms = s[s.size() / 2];
    return ABFT_OK;
}

int abft_metrics_finalize(abft_metrics* m) {
    if (!m) {
        set_error("abft_metrics_finalize: NULL");
        return ABFT_ERR_ARG;
    }
    const double tb = m->baseline.median_ms, tp = m->protected_.median_ms;
    m->overhead_pct = (tb > 0.0) ? ((tp - tb) / tb) * 100.0 : 0.0;
    const int TP = m->cm[0], FP = m->cm[2], FN = m->cm[3];
    m->recall = (TP + FN > 0) ? static_cast<double>(TP) / (TP + FN) : 0.0;
    m->precision = (TP + FP > 0) ? static_cast<double>(TP) / (TP + FP) : 0.0;
    m->correction_precision_pct = (TP > 0) ? (static_cast<double>(m->n_restored) / TP) * 100.0 : 0.0;
    m->baseline_gflops_median = gflops(m->baseline.median_ms, m->M, m->N, m->K);
    m->baseline_gflops_max = gflops(m->baseline.min_ms, m->M, m->N, m->K);
    m->baseline_gflops_min = gflops(m->baseline.max_ms, m->M, m->N, m->K);
    m->baseline_gflops_mean = gflops(m->baseline.mean_ms, m->M, m->N, m->K);
    m->protected_gflops_median = gflops(m->protected_.median_ms, m->M, m->N, m->K);
    m->protected_gflops_max = gflops(m->protected_.min_ms, m->M, m->N, m->K);
    m->protected_gflops_min = gflops(m->protected_.max_ms, m->M, m->N, m->K);
    m->protected_gflops_mean = gflops(m->protected_.mean_ms, m->M, m->N, m->K);
    return ABFT_OK;
}

int abft_metrics_report(const abft_metrics* m, char* buf, size_t cap) {
    if (!m) {
        set_error("abft_metrics_report: NULL");
        return ABFT_ERR_ARG;
    }
    std::ostringstream o;
    o << std::fixed << std::setprecision(4);
    o << "\n========== EXPERIMENT METRICS (global) ==========\n";
    const std::string inject(m->inject), zone(m->swifi_zone), scheme(m->scheme);
    if (m->calibrate) {
        o << "Mode              : CALIBRATION\n";
    } else if (m->baseline_only) {
        o << "Mode              : BASELINE\n";
    } else {
        o << "Mode              : " << scheme << " / inject=" << inject;
        if (inject == "swifi") o << " (zone=" << zone << ")";
        o << "\n";
    }
    o << "M x K x N         : " << m->M << " x " << m->K << " x " << m->N << "\n";
    o << "Process grid      : " << m->Pr << " x " << m->Pc << "\n";
    o << "Frags per rank    : " << m->frags_per_rank << "\n";
    o << "Total fragments   : " << m->num_fragments_total << "\n";
    o << "Repeats           : " << m->repeats << "\n";
    if (!m->calibrate) o << "Threshold used    : " << m->threshold_used << "\n";
    o << "--- Timing (worst rank) ---\n";
    o << "Baseline   min/med/max : " << m->baseline.min_ms << " / " << m->baseline.median_ms << " / "
      << m->baseline.max_ms << "  ms\n";
    o << "Baseline   GFLOPS (med): " << m->baseline_gflops_median << "  (min " << m->baseline_gflops_min << ", max "
      << m->baseline_gflops_max << ")\n";
    if (!m->calibrate) {
        o << "Protected  min/med/max : " << m->protected_.min_ms << " / " << m->protected_.median_ms << " / "
          << m->protected_.max_ms << "  ms\n";
        o << "Protected  GFLOPS (med): " << m->protected_gflops_median << "  (min " << m->protected_gflops_min
          << ", max " << m->protected_gflops_max << ")\n";
        o << "Overhead (median)      : " << m->overhead_pct << " %\n";
    }
    if (m->calibrate) {
        o << "--- Calibration ---\n";
        o << "Max |actual-expected|  : " << m->calib_max_diff << "\n";
        o << "Safety factor          : " << m->calib_safety_factor << "\n";
        o << "Suggested threshold    : " << m->calib_suggested_tau << "\n";
        o << "\n=> Re-run with:  --threshold " << m->calib_suggested_tau << "\n";
    } else {
        o << "--- Confusion Matrix (global) ---\n";
        o << "TP / TN / FP / FN     : " << m->cm[0] << " / " << m->cm[1] << " / " << m->cm[2] << " / " << m->cm[3]
          << "\n";
        o << "Recall                : " << m->recall << "\n";
        o << "Detection precision   : " << m->precision << "\n";
        o << "Correction precision  : " << m->correction_precision_pct << " %\n";
    }
    o << "==================================================\n\n";
    const std::string s = o.str();
    if (buf && cap > 0) {
        const size_t n = std::min(cap - 1, s.size());
        std::memcpy(buf, s.data(), n);
        buf[n] = '\0';
    }
    return (int)s.size();
}

int abft_metrics_csv_append(const abft_metrics* m, const char* path, const char* extra_header,
                            const char* extra_values) {
    if (!m || !path || (!extra_header != !extra_values)) {
        set_error("abft_metrics_csv_append: bad argument");
        return ABFT_ERR_ARG;
    }
    bool write_header = false;
    {
        std::ifstream test(path);
        if (!test.good()) write_header = true;
    }
    std::ofstream ofs(path, std::ios::app);
    if (!ofs.is_open()) {
        set_error(std::string("cannot open ") + path + " for CSV logging");
        return ABFT_ERR_ARG;
    }
    if (write_header) {
        ofs << "scheme,inject,swifi_zone,baseline_only,calibrate,"
               "M,K,N,Pr,Pc,frags_per_rank,num_fragments_total,repeats,"
               "threshold_used,"
               "baseline_min_ms,baseline_median_ms,baseline_mean_ms,baseline_max_ms,"
               "baseline_gflops_min,baseline_gflops_median,baseline_gflops_mean,baseline_gflops_max,"
               "protected_min_ms,protected_median_ms,protected_mean_ms,protected_max_ms,"
               "protected_gflops_min,protected_gflops_median,protected_gflops_mean,protected_gflops_max,"
               "overhead_pct,"
               "TP,TN,FP,FN,recall,precision,correction_precision_pct,"
               "calib_max_diff,calib_safety_factor,calib_suggested_tau";
        if (extra_header) ofs << "," << extra_header;
        ofs << "\n";
    }
    ofs << std::fixed << std::setprecision(6);
    ofs << m->scheme << "," << m->inject << "," << m->swifi_zone << "," << (m->baseline_only ? 1 : 0) << ","
        << (m->calibrate ? 1 : 0) << "," << m->M << "," << m->K << "," << m->N << "," << m->Pr << "," << m->Pc << ","
        << m->frags_per_rank << "," << m->num_fragments_total << "," << m->repeats << "," << m->threshold_used << ","
        << m->baseline.min_ms << "," << m->baseline.median_ms << "," << m->baseline.mean_ms << ","
        << m->baseline.max_ms << "," << m->baseline_gflops_min << "," << m->baseline_gflops_median << ","
        << m->baseline_gflops_mean << "," << m->baseline_gflops_max << "," << m->protected_.min_ms << ","
        << m->protected_.median_ms << "," << m->protected_.mean_ms << "," << m->protected_.max_ms << ","
        << m->protected_gflops_min << "," << m->protected_gflops_median << "," << m->protected_gflops_mean << ","
        << m->protected_gflops_max << "," << m->overhead_pct << "," << m->cm[0] << "," << m->cm[1] << ","
        << m->cm[2] << "," << m->cm[3] << "," << m->recall << "," << m->precision << ","
        << m->correction_precision_pct << "," << m->calib_max_diff << "," << m->calib_safety_factor << ","
        << m->calib_suggested_tau;
    if (extra_values) ofs << "," << extra_values;
    ofs << "\n";
    return ABFT_OK;
}

}  // extern "C"
