// Internal declarations shared by the kernels, the C ABI and the pipeline.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace abft {

constexpr int kThreads = 256;    // threads of the verify / localise CTAs
constexpr int kWarps = kThreads / 32;
constexpr int kGroupCols = 128;  // columns per verify CTA: 32 lanes x 4 columns
constexpr int kMaxChunks = 1024; // row chunks per column group (verify grid.y)
constexpr int kVerifySmemMax = 64 * 1024;  // verify dynamic shared memory cap
// Arrival and work state of one verify launch, in WsDev::vcnt (all zero
// between launches; G = number of column groups):
//   [0, 2)                  one 64-bit word: column groups that have finished (low
//                           half; the last one decides the fragment) and, in the
//                           high half, how many of them hold a column whose
//                           |actual - expected| may exceed tau
//   [kArriveGroup + g]      CTAs of column group g that have finished (the last one
//                           finishes the group)
//   [kArriveGroup + G + g]  next unit of rows of column group g to hand out
constexpr int kArriveGroup = 2;
constexpr int vcnt_ints(int groups) { return kArriveGroup + 2 * groups; }
// Columns of the per-column verify accumulators: the widest fragment,
// rounded up to whole column groups.
constexpr int acc_columns(int nfmax) { return (nfmax + kGroupCols - 1) / kGroupCols * kGroupCols; }

// Per-fragment decision record (the reference's dErrCol[f] / dRowDiff[f],
// plus the located row).
struct FragRecord {
    int errcol;
    int errrow;
    double rowdiff;
};

struct DecisionLog {
    int errcol;
    int errrow;
    double rowdiff;
};

struct InjectLog {
    int frag, row, col, bit;
    float before, after;
};

// Injection of one iteration, read on the device in graph mode (frag -1: none).
struct InjectPlan {
    int frag, row, col, bit;
};

struct PendingFix {
    int it, f, er, ec, injected, off;
    double rowdiff;
    double tau;
    float c_fault;
    float pad;
};

struct Counters {
    int cm[4];       // TP, TN, FP, FN
    int n_restored;
    int n_pending;
    int fault;  // a verify kernel's bounded wait for a bulk copy ran out (or its ring was misplaced)
    int pad;
};

// Device-side workspace pointers (plain struct, passed by value to kernels).
struct WsDev {
    double* colSumA;   // [K]
    double* expRow;    // [N_b]  absolute column index
    double* rowSumB;   // [F][K]
    double* expCol;    // [F][M_b]
    FragRecord* rec;   // [F]
    Counters* ctr;
    // per-column accumulators of the verify kernel: double sum, float sum of
    // |x| and the smallest (|x| bits - 1) (0xffffffff when every term is 0)
    double* vacc_s;    // [nacc]
    float* vacc_t;     // [nacc]
    uint32_t* vacc_m;  // [nacc]
    double* vact;      // [nacc]
    double* vd;
    double* vw;
    int* vcnt;         // [vcnt_ints(groups_max)], 8-byte aligned
    // localisation: per row block, its best row under the reference's
    // arg-max order (-1: no row above tau) and that row's |actual - expected|
    double* lbd;       // [M_b] (at most M_b / kWarps blocks)
    int* lbr;          // [M_b]
    int* lcnt;         // [1]
    DecisionLog* dlog; // [max_iters][F]
    InjectLog* ilog;   // [max_iters]
    PendingFix* pend;  // [max_iters * F]
    InjectPlan* plan;  // [max_iters]
};

}  // namespace abft

// The opaque handle of the C ABI.
struct abft_ws {
    int device = 0;
    int sms = 148;
    int M_b = 0, N_b = 0, K = 0, F = 0, nfmax = 0, nacc = 0, max_iters = 0;
    std::vector<int> counts, offsets;
    void* base = nullptr;
    size_t bytes = 0;
    bool owns = false;
    abft::WsDev d{};
};

namespace abft {

// Error reporting (thread-local last error).
void set_error(const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

struct WsLayout {
    size_t colSumA, expRow, rowSumB, expCol, rec, ctr, vacc_s, vacc_t, vacc_m, vact, vd, vw, vcnt, lbd, lbr, lcnt, dlog, ilog,
        pend, plan, total;
};
WsLayout ws_layout(int M_b, int N_b, int K, int F, int nfmax, int max_iters);

// Kernel launchers (enqueue only). Return ABFT_OK or a negative status.
int launch_encode(abft_ws* ws, const float* dA, int64_t lda, const float* dB, int64_t ldb, cudaStream_t st,
                  int* launches);
// plan_it >= 0 selects graph mode: the injection of iteration plan_it is read
// from ws->d.plan on the device (verify applies it, log_inj logs it). cond:
// a graph conditional handle the kernel sets to "column detected" (0: none).
int launch_verify(abft_ws* ws, const float* dC, int64_t ldc, int f, double tau, int injected, int it,
                  cudaStream_t st, int plan_it = -1, float add_delta = 0.f, int log_inj = 0,
                  double* calib_out = nullptr, unsigned long long cond = 0);
int launch_localize(abft_ws* ws, float* dC, int64_t ldc, int f, double tau, int injected, const float* dG,
                    int64_t ldg, int it, int correct_mode, cudaStream_t st, int plan_it = -1);
int launch_drain(abft_ws* ws, float* dC0, float* dC1, int64_t ldc, const float* dG, int64_t ldg, int repeats,
                 cudaStream_t st);
int launch_inject(float* dC, int64_t ldc, int row, int col, int mode, float delta, int bit, InjectLog* log,
                  int frag, cudaStream_t st);
// Selects the verify body (ABFT_VERIFY_*); returns the previous setting or -1.
int set_verify_kernel(int which);
// The current selection (ABFT_VERIFY_*).
int verify_kernel();
// Polls each wait of the TMA verify body makes before it gives up; returns the
// previous limit, or -1 for a negative one.
int set_wait_limit(int polls);
int launch_verify_static(const float* Cf, int64_t ldc, int M, int N, const double* expv, double tau, int injected,
                         int* errcol, double* rowdiff, int* cm, cudaStream_t st);

}  // namespace abft
