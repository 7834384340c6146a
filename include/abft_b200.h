/*
 * abft_b200.h - C ABI of the B200-native asynchronous ABFT layer around SGEMM.
 *
 * Every function returns an int status (ABFT_OK == 0, negative on error; the
 * message is in abft_last_error()) unless it returns a value, and never aborts
 * the process. Device pointers are plain pointers, streams are cudaStream_t
 * passed as void*. Nothing in this header depends on torch or MPI.
 *
 * The reference (FaridRojas/Asynchronous_ABFT_for_MPI-CUDA_Architectures) has
 * no FFI: its operator surface is the set of header-inline, enqueue-only launch
 * helpers in kernels/abft_stepwise.cuh and kernels/swifi.cuh, the pass
 * functions in pipeline/passes.cuh and the host helpers in core/ and
 * distribution/. Each declaration below names the reference interface it
 * replaces (path:line within the reference project).
 *
 * Matrices are row-major (the reference's layout: main.cu:113-115); a rank
 * tile is A (M_b x K, lda), B (K x N_b, ldb), C (M_b x N_b, ldc). C is split
 * into F column fragments [offsets[f], offsets[f] + counts[f]).
 */
#ifndef ABFT_B200_H
#define ABFT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ABFT_OK 0
#define ABFT_ERR_ARG (-1)    /* bad argument (sizes, pointers, modes)            */
#define ABFT_ERR_CUDA (-2)   /* a CUDA runtime call or kernel launch failed      */
#define ABFT_ERR_CUBLAS (-3) /* a cuBLAS call failed                             */
#define ABFT_ERR_STATE (-4)  /* call out of order (e.g. online before encode)    */

#define ABFT_INJECT_NONE 0
#define ABFT_INJECT_ADD 1
#define ABFT_INJECT_SWIFI 2

#define ABFT_SEED_REFERENCE 0 /* injection draws of the reference (per rank, per iteration) */
#define ABFT_SEED_TILE 1      /* abft_injection_plan_tile with seed = base_seed + iteration  */

#define ABFT_CORRECT_INLOOP 0 /* correct inside the loop (reference behaviour) */
#define ABFT_CORRECT_DRAIN 1  /* locate in the loop, correct after it          */

/* Additive fault size of the reference (kernels/swifi.cuh:53). */
#define ABFT_ADD_FAULT_DELTA 1.0e6f

/* Last error message of the calling thread ("" when none). */
const char* abft_last_error(void);
/* ABI version: major * 10000 + minor * 100 + patch. */
int abft_version(void);

/* ------------------------------------------------------------------------
 * Host helpers (CPU only, bit-identical to the reference's host code).
 * ---------------------------------------------------------------------- */

/* fill_random, core/common.cuh:57-61 (dist 0). dist 1 = normal(0,1)
 * (std::normal_distribution<float>), an extension for non-square workloads. */
int abft_fill_random(float* host_out, int64_t n, uint64_t seed, int dist);
/* choose_grid, distribution/grid.cuh:7-12 */
int abft_choose_grid(int world, int* Pr, int* Pc);
/* split_dim, distribution/grid.cuh:15-28 */
int abft_split_dim(int total, int parts, int* counts, int* offsets);
/* Fragments per rank, main.cu:55-69 (small-matrix rule and --frag-cap). */
int abft_frag_count(int M, int K, int N, int M_b, int N_b, int frags_per_rank, int64_t frag_cap);
/* Row pitch (floats) for the pipeline's M_b x n row-major C buffers. The
 * reference allocates C densely (ld = N_b, pipeline/buffers.cuh); here n gets
 * 32 floats (128 B) more when n * 4 bytes is a multiple of 64 KB. With a 64 KB
 * pitch every row of a fragment that is a quarter of the row starts at the
 * same offset modulo 64 KB, and the verify kernel streams such a fragment
 * about 9 % slower on B200 (59 us against 53.5 us for 16384 x 4096 of a
 * 16384-wide C); the SGEMM's speed does not change. Any ldc >= n is valid
 * for every entry point; this is only the layout the sessions and the driver
 * allocate. Returns n unchanged otherwise; -1 for n < 1. */
int64_t abft_c_pitch(int n);
/* matrix_inf_norm, core/common.cuh:64-74 */
double abft_matrix_inf_norm(const float* host_M, int rows, int cols, int64_t ld);
/* compute_threshold_formula, core/common.cuh:77-83 */
double abft_threshold_formula(int k, double norm_A_inf, double norm_B_inf);
/* Per-fragment thresholds of regen_inputs, main.cu:147-164 (override > 0 wins). */
int abft_frag_thresholds(const float* host_A, int M_b, int K, int64_t lda, const float* host_B, int64_t ldb,
                         int F, const int* counts, const int* offsets, double override_tau, double* tau_out);
/* swifi_zone_range, kernels/swifi.cuh:25-31 ("any" and unknown -> [0,31]). */
int abft_swifi_zone_range(const char* zone, int* lo, int* hi);
/* Injection plan of one (rank, iteration): the inject_frag draw of
 * pass_online_loop (pipeline/passes.cuh:148-156) and the row/col(/bit) draws
 * of inject_add_constant / inject_single_bitflip (kernels/swifi.cuh:67-71,
 * :91-98). mode ABFT_INJECT_*; outputs -1 when nothing is injected. */
int abft_injection_plan(uint64_t base_seed, int rank, int it, int F, int M_b, const int* counts, int mode,
                        int zone_lo, int zone_hi, int* frag, int* row, int* col, int* bit);
/* Tile-uniform injection scheme (no counterpart in the reference, whose
 * injector cannot express it; the 1024^3 workload describes faults this way):
 * mt19937_64(seed) draws row uniform over [0, M_b) and column j uniform over
 * the whole tile [0, N_b), then the bit in [zone_lo, zone_hi] for SWIFI; the
 * fragment is the one holding j and col = j - offsets[frag]. */
int abft_injection_plan_tile(uint64_t seed, int M_b, int F, const int* counts, const int* offsets, int mode,
                             int zone_lo, int zone_hi, int* frag, int* row, int* col, int* bit);

/* ------------------------------------------------------------------------
 * Workspace: the device-side state of pipeline/buffers.cuh:7-46
 * (PipelineBuffers: dColSumA, dExpectedRow[F], dErrCol, dRowDiff, dRowSumB,
 * dExpectedCol, dActualCol, dCM, dNRestored) plus the verify kernels' scratch.
 * ---------------------------------------------------------------------- */
typedef struct abft_ws abft_ws;

/* Bytes of device memory a workspace needs. max_iters bounds the per-iteration
 * decision log and the post-loop drain list (0 = no log, no drain). */
size_t abft_ws_bytes(int M_b, int N_b, int K, int F, const int* counts, int max_iters);
/* buffers_init, pipeline/buffers.cuh:48-83 (device part). With dev_mem == NULL
 * the workspace allocates its own memory; otherwise dev_mem must hold
 * abft_ws_bytes(...) bytes, 256-byte aligned, and stays owned by the caller. */
int abft_ws_create(int M_b, int N_b, int K, int F, const int* counts, const int* offsets, int max_iters,
                   void* dev_mem, size_t dev_bytes, abft_ws** out);
/* buffers_free, pipeline/buffers.cuh:85-104 */
int abft_ws_destroy(abft_ws* ws);
/* Zero the confusion matrix, restore counter and drain list (the memsets of
 * pass_online_loop, pipeline/passes.cuh:126-127). */
int abft_ws_reset_counters(abft_ws* ws, void* stream);
/* Device address of the int32[5] counters {TP, TN, FP, FN, n_restored}. */
int* abft_ws_counters_device(abft_ws* ws);
/* Synchronous read of {TP, TN, FP, FN} and n_restored. */
int abft_ws_read_counters(abft_ws* ws, int cm[4], int* n_restored);
/* Synchronous read of the decision log: it_count iterations x F entries of
 * errcol (-1 clean), errrow (-1 none) and rowdiff. */
int abft_ws_read_log(abft_ws* ws, int it_count, int* errcol, int* errrow, double* rowdiff);
/* Synchronous read of the encode checksums (any pointer may be NULL):
 * colSumA[K], expRow[N_b], rowSumB[F*K], expCol[F*M_b]. */
int abft_ws_read_checksums(abft_ws* ws, double* colSumA, double* expRow, double* rowSumB, double* expCol);

/* ------------------------------------------------------------------------
 * Kernels (enqueue only, on the caller's stream).
 *
 * Calls that share a workspace must run one after another on the GPU (one
 * stream, or streams ordered by events): verify and localise keep their
 * per-column / per-row accumulators and arrival counters in the workspace and
 * leave them cleared for the next launch, as the reference's single verify
 * stream does with its shared scratch (pipeline/buffers.cuh:24-27). Separate
 * workspaces are independent.
 * ---------------------------------------------------------------------- */

/* Checksum encoding of one rank tile, all fragments:
 *   colSumA[k] = sum_i A[i,k]                    launch_col_checksum_A, kernels/abft_stepwise.cuh:243-248
 *   expRow[j]  = sum_k colSumA[k] * B[k,j]       launch_expected_row,   kernels/abft_stepwise.cuh:250-256
 *   rowSumB_f[k] = sum_{j in f} B[k,j]           k_row_checksum_B_g,    kernels/abft_stepwise.cuh:121-132
 *   expCol_f[i]  = sum_k A[i,k] * rowSumB_f[k]   k_expected_col_g,      kernels/abft_stepwise.cuh:134-146
 * The last two are the reference's per-fault localisation checksums, hoisted
 * to encode time (they depend only on A and B). Results are bit-identical to
 * the reference's kernels. */
int abft_encode(abft_ws* ws, const float* dA, int64_t lda, const float* dB, int64_t ldb, void* stream);

/* Verify fragment f of C: actualRow = column sums of the fragment, then the
 * detection arg-max and the confusion-matrix update. Replaces launch_actual_row
 * (kernels/abft_stepwise.cuh:258-263) + launch_detect_row (:208-216). dC is the
 * rank tile's base pointer. `it` indexes the decision log (-1 = no log). */
int abft_verify(abft_ws* ws, const float* dC, int64_t ldc, int f, double tau, int injected, int it, void* stream);

/* Calibration of fragment f (pass_calibrate, pipeline/passes.cuh:66-84):
 * writes |actualRow[j] - expectedRow[j]| for every column j of the fragment
 * into the device array dDiff[counts[f]], bit-identical to the reference's
 * host loop; no detection, no counter update. */
int abft_calibrate(abft_ws* ws, const float* dC, int64_t ldc, int f, double* dDiff, void* stream);

/* Verify one fragment without allocating anything. No counterpart in the
 * reference: it exists for callers that must not allocate device memory while
 * they run - a fault-tolerance hook called from inside another library's hot
 * loop, or a service whose device memory is fixed at start-up - because
 * cudaMalloc/cudaFree can synchronise the whole device and can fail under
 * memory pressure. Same computation and decision as abft_verify, but the
 * caller passes everything: the fragment dC_frag (M x N, leading dimension
 * ldc), its expected row dExpRow[N] (e.g. from abft_encode), and the outputs
 * dErrCol (int), dRowDiff (double) and dCM (int[4], TP TN FP FN, incremented).
 * Scratch is a static device array inside this library (about 161 KB), held
 * by every GPU that loads it until the process exits, limited to N <= 4096
 * columns (larger N returns ABFT_ERR_ARG). The array exists once per CUDA
 * context - normally once per device, in the runtime's primary context; a
 * second context on a device, or the one that follows cudaDeviceReset, has
 * its own copy. The first call in a context sets that context's copy up (it
 * looks up the array's device address and clears it on `stream`); make that
 * first call before any stream capture. All calls in a context share the
 * array: calls whose work overlaps on the GPU race; calls ordered one after
 * another (same stream, or synchronised) are safe. No cudaMalloc, cudaFree or
 * allocating library routine is called. */
int abft_verify_noalloc(const float* dC_frag, int64_t ldc, int M, int N, const double* dExpRow, double tau,
                        int injected, int* dErrCol, double* dRowDiff, int* dCM, void* stream);

/* Which body abft_verify (and the pipeline) uses for the column sums:
 * ABFT_VERIFY_AUTO picks the body that is faster inside the protected loop
 * (on B200: 128-bit loads at every size), ABFT_VERIFY_LDG streams the tile
 * with 128-bit loads, ABFT_VERIFY_TMA stages it through shared memory with
 * bulk tensor copies (falls back to LDG where a tensor map cannot describe
 * the fragment: unaligned base or pitch, fewer than 128 columns or 32 rows).
 * Decisions are identical for all three. Process-wide; returns the previous
 * setting, or ABFT_ERR_ARG. */
#define ABFT_VERIFY_AUTO 0
#define ABFT_VERIFY_LDG 1
#define ABFT_VERIFY_TMA 2
int abft_set_verify_kernel(int which);

/* Polls each wait of the TMA verify body makes for one bulk tensor copy
 * before it gives up (default 1048576). No counterpart in the reference, whose
 * kernels never wait on a copy. A wait that gives up marks the launch void:
 * the kernel waits (with the default limit) for the copies it issued, adds
 * nothing, finishes its arrival protocol and returns, and the next
 * abft_ws_read_counters returns ABFT_ERR_CUDA with a message that names the
 * wait; the context stays usable. Meant for tests of that failure path (0
 * makes every such wait give up at once). Process-wide; returns the previous
 * limit, or ABFT_ERR_ARG for a negative one. */
int abft_set_wait_limit(int polls);

/* Localise and correct fragment f, gated on the device by the verify result:
 * replaces launch_localize_correct (kernels/abft_stepwise.cuh:218-239).
 * dGolden (may be NULL) is the fault-free tile with leading dimension ldg,
 * used for the restore count exactly as k_locate_correct (:198-203).
 * correct_mode ABFT_CORRECT_DRAIN queues the fix for abft_drain instead. */
int abft_localize_correct(abft_ws* ws, float* dC, int64_t ldc, int f, double tau, int injected,
                          const float* dGolden, int64_t ldg, int it, int correct_mode, void* stream);

/* Post-loop drain of queued corrections (the correction drain described in the
 * reference README "Cross-iteration pipelining"): applies each queued fix to
 * the buffer that still holds its iteration (the last two iterations of a
 * double-buffered loop of `repeats` iterations) and counts restores against
 * dGolden. dC0/dC1 are the two buffers. */
int abft_drain(abft_ws* ws, float* dC0, float* dC1, int64_t ldc, const float* dGolden, int64_t ldg, int repeats,
               void* stream);

/* k_inject_add + inject_add_constant, kernels/swifi.cuh:55-76: C[row,col] += delta. */
int abft_inject_add(float* dC, int64_t ldc, int row, int col, float delta, void* stream);
/* k_inject_bitflip + inject_single_bitflip, kernels/swifi.cuh:33-40, :78-114:
 * C[row,col] bits ^= 1 << bit. Asynchronous: no host synchronisation. */
int abft_inject_bitflip(float* dC, int64_t ldc, int row, int col, int bit, void* stream);

/* Row-major SGEMM through cuBLAS with the reference's operand swap
 * (gemm_cublas, kernels/gemm_cublas.cuh:7-22): C = A * B, A M x K, B K x N. */
int abft_sgemm(void* cublas_handle, const float* dA, int lda, const float* dB, int ldb, float* dC, int ldc, int M,
               int N, int K);

/* ------------------------------------------------------------------------
 * Session: one rank's online pipeline (pipeline/passes.cuh, buffers.cuh).
 * Two streams (compute at high priority, verify at low priority), one cuBLAS
 * handle on the compute stream, per-fragment compute_done events and one
 * OnlineSlot per dC buffer (buffer, verify_done event, decision records).
 * ---------------------------------------------------------------------- */
typedef struct abft_session abft_session;

typedef struct abft_session_cfg {
    int M_b, N_b, K, F;
    const int* counts;  /* F fragment widths   (split_dim of N_b)   */
    const int* offsets; /* F fragment offsets                       */
    const float* dA;
    int64_t lda;
    const float* dB;
    int64_t ldb;
    float* dC0; /* OnlineSlot 0 buffer */
    float* dC1; /* OnlineSlot 1 buffer */
    int64_t ldc;
    int verify_priority; /* -1 lowest (default), 0 default, 1 highest      */
    int max_iters;       /* decision-log / drain capacity in iterations    */
} abft_session_cfg;

typedef struct abft_online_args {
    int mode;         /* ABFT_INJECT_NONE / ADD / SWIFI                     */
    int zone_lo;      /* SWIFI bit range, inclusive                         */
    int zone_hi;
    float add_delta;  /* additive fault size (ABFT_ADD_FAULT_DELTA)         */
    uint64_t base_seed;
    int rank;
    int repeats;
    int correct_mode; /* ABFT_CORRECT_INLOOP / ABFT_CORRECT_DRAIN           */
    int log;          /* 1: fill the decision + injection logs              */
    int profile;      /* 1: time every verify launch with CUDA events       */
    int graph;        /* 1: run the loop as a CUDA graph captured once per
                         (repeats, mode, correction, log, add_delta) and
                         replayed; the injection plan goes to a device table
                         and the verify kernel applies the fault. Needs
                         repeats <= max_iters; ignores profile.            */
    int seed_scheme;  /* ABFT_SEED_REFERENCE (default) or ABFT_SEED_TILE    */
} abft_online_args;

typedef struct abft_online_result {
    double device_ms; /* CUDA-event time of the whole loop                  */
    double host_ms;   /* host wall time of the loop (reference method)      */
    int cm[4];        /* TP, TN, FP, FN of this call                        */
    int n_restored;
    int kernel_launches;   /* our kernels launched inside the loop          */
    int verify_launches;   /* of which fused verify kernels                 */
    double verify_ms_sum;  /* sum of per-launch verify times (profile = 1)  */
    double verify_ms_max;
} abft_online_result;

/* buffers_init (pipeline/buffers.cuh:48-83) + gemm_warmup (kernels/gemm_cublas.cuh:25-42). */
int abft_session_create(const abft_session_cfg* cfg, abft_session** out);
int abft_session_destroy(abft_session* s);
abft_ws* abft_session_ws(abft_session* s);
/* Thresholds tau[F] used by the next online calls. */
int abft_session_set_tau(abft_session* s, const double* tau);
/* Golden (fault-free) tile for the restore count; NULL disables it. */
int abft_session_set_golden(abft_session* s, const float* dGolden, int64_t ldg);
/* The untimed encode of pass_online_loop (pipeline/passes.cuh:118-128). */
int abft_session_encode(abft_session* s, double* encode_ms);
/* pass_baseline, pipeline/passes.cuh:14-35: repeats x F SGEMMs into dC0.
 * graph = 1 replays them as a CUDA graph (captured once per repeats), the
 * unprotected counterpart of abft_online_args.graph. */
int abft_session_baseline(abft_session* s, int repeats, int graph, double* device_ms, double* host_ms);
/* A stricter unprotected baseline with no counterpart in the reference:
 * repeats x ONE SGEMM of the whole M_b x N_b tile (gemm_cublas,
 * kernels/gemm_cublas.cuh:7-22, called once instead of F times), so that the
 * cost of splitting C into fragments shows apart from the ABFT kernels. */
int abft_session_baseline_monolithic(abft_session* s, int repeats, int graph, double* device_ms, double* host_ms);
/* pass_online_loop, pipeline/passes.cuh:90-227 (timed part). */
int abft_session_online(abft_session* s, const abft_online_args* args, abft_online_result* res);
/* Injection log of the last online call: it_count x {frag, row, col, bit}
 * and the element's value before/after (may be NULL). */
int abft_session_read_injections(abft_session* s, int it_count, int* inj4, float* before_after);
/* End-to-end call from HOST memory: copies hA, hB into the session's A and B
 * (which must be device buffers it may overwrite), encodes, runs `repeats`
 * protected iterations and copies the final C buffer and the counters back.
 * The copies overlap the work: B arrives one fragment at a time and
 * iteration 0's SGEMM of a fragment starts once A and that fragment are in;
 * with in-loop correction each fragment of the final buffer goes back to the
 * host as soon as its last check finished. Always enqueued eagerly
 * (args->graph is ignored). Timed with CUDA events around the copies
 * (e2e_ms). hA, hB, hC should be pinned for the copies to be asynchronous. */
int abft_session_run_host(abft_session* s, const float* hA, const float* hB, float* hC,
                          const abft_online_args* args, abft_online_result* res, double* e2e_ms);
/* n_steps end-to-end calls back to back, one per input pair: step k copies
 * hA[k], hB[k] from HOST memory, encodes, runs `repeats` protected iterations
 * with base_seeds[k] (args->base_seed is ignored) and copies its final C to
 * hC[k] (entries may alias; copies into one buffer land in step order). Each
 * step's results are the same as abft_session_run_host's on the same inputs;
 * res[k] receives step k's counters and launch counts (device_ms = e2e_ms /
 * n_steps). Unlike n separate calls, the steps overlap: step k+1's inputs
 * are copied while step k computes, into a second device copy of A and B that
 * the session allocates on the first call (as large as A and B, freed with
 * the session; the session's own A and B are overwritten too), and step k's
 * result is copied back on its own stream while step k+1's SGEMMs run. No
 * counterpart in the reference, which generates its inputs on the host once
 * per trial; it is the same loop (pipeline/passes.cuh:90-227) fed from host
 * memory step after step. Enqueued eagerly (args->graph, log and profile are
 * ignored); hA, hB, hC should be pinned. e2e_ms: CUDA-event time of all steps,
 * copies included. */
int abft_session_run_host_steps(abft_session* s, int n_steps, const float* const* hA, const float* const* hB,
                                float* const* hC, const abft_online_args* args, const uint64_t* base_seeds,
                                abft_online_result* res, double* e2e_ms);

/* ------------------------------------------------------------------------
 * Metrics (metrics/metrics.cuh, core/common.cuh:86-106): the confusion
 * matrix, derived rates, GFLOPS, overhead, the stdout report and the
 * 41-column append-mode CSV, formatted exactly like the reference.
 * ---------------------------------------------------------------------- */
typedef struct abft_timing {
    double min_ms, median_ms, mean_ms, max_ms;
    int n_samples;
} abft_timing;

typedef struct abft_metrics {
    char scheme[16];     /* "baseline", "online", "calibrate"   */
    char inject[16];     /* "none", "add", "swifi"              */
    char swifi_zone[16];
    int baseline_only, calibrate;
    int M, K, N, Pr, Pc, frags_per_rank, num_fragments_total, repeats;
    double threshold_used;
    abft_timing baseline, protected_;
    int cm[4]; /* TP, TN, FP, FN */
    int n_restored;
    double calib_max_diff, calib_safety_factor, calib_suggested_tau;
    /* filled by abft_metrics_finalize */
    double overhead_pct, recall, precision, correction_precision_pct;
    double baseline_gflops_min, baseline_gflops_median, baseline_gflops_mean, baseline_gflops_max;
    double protected_gflops_min, protected_gflops_median, protected_gflops_mean, protected_gflops_max;
} abft_metrics;

/* stats_of, core/common.cuh:86-106 (median = sorted[n/2]). */
int abft_stats_of(const double* samples, int n, abft_timing* out);
/* finalize_metrics, metrics/metrics.cuh:132-149 (with compute_* :105-130). */
int abft_metrics_finalize(abft_metrics* m);
/* print_metrics, metrics/metrics.cuh:152-211, written into buf (NUL-terminated).
 * Returns the full length; truncates to cap - 1 characters. */
int abft_metrics_report(const abft_metrics* m, char* buf, size_t cap);
/* log_metrics_csv, metrics/metrics.cuh:214-254: appends one row, writing the
 * header first when the file does not exist. extra_header / extra_values
 * (both or neither) append further comma-separated columns after the
 * reference's 41. */
int abft_metrics_csv_append(const abft_metrics* m, const char* path, const char* extra_header,
                            const char* extra_values);

#ifdef __cplusplus
}
#endif

#endif /* ABFT_B200_H */
