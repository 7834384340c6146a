// One rank's online ABFT pipeline: the host scheduler of pass_baseline and
// pass_online_loop (pipeline/passes.cuh:14-35, :90-227) on B200.
//
// Streams: the protected SGEMMs run on a high-priority compute stream, every
// ABFT kernel on a low-priority verify stream, so verification fills the SMs
// the SGEMM leaves idle (wave tails, gaps between fragments) instead of
// competing with it. Per iteration it:
//   compute: [wait slot's verify_done] SGEMM f -> (inject) -> record compute_done[f]   (f = 0..F-1)
//   verify : wait compute_done[f] -> fused verify f -> gated localise/correct f         (f = 0..F-1)
//            -> record slot's verify_done
// The two dC buffers are the two OnlineSlots: iteration k+2 reuses slot k%2
// only after iteration k's verification finished, so iteration k's checks
// overlap iteration k+1's SGEMMs. Injection positions come from the host RNG
// (the reference's draws) and are passed as kernel arguments: no host
// synchronisation inside the loop.

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <new>
#include <string>
#include <vector>

#include "abft_b200.h"
#include "abft_internal.h"

using namespace abft;

struct abft_session {
    int device = 0;
    int M_b = 0, N_b = 0, K = 0, F = 0;
    std::vector<int> counts, offsets;
    const float* dA = nullptr;
    int64_t lda = 0;
    const float* dB = nullptr;
    int64_t ldb = 0;
    float* dC[2] = {nullptr, nullptr};
    int64_t ldc = 0;
    cudaStream_t compute = nullptr, verify = nullptr;
    cublasHandle_t handle = nullptr;
    std::vector<cudaEvent_t> compute_done;
    cudaEvent_t buf_done[2] = {nullptr, nullptr};
    cudaEvent_t t0 = nullptr, t1 = nullptr, vjoin = nullptr, cjoin = nullptr;
    std::vector<cudaEvent_t> vprof;
    abft_ws* ws = nullptr;
    std::vector<double> tau;
    const float* dG = nullptr;
    int64_t ldg = 0;
    bool encoded = false;
    int profile = 0;
    int max_iters = 0;
    int last_launches = 0;
    // graph mode: one captured loop, replayed while its shape stays the same
    cudaGraphExec_t gexec = nullptr;
    int g_repeats = -1, g_mode = -1, g_correct = -1, g_log = -1, g_launches = 0, g_vlaunches = 0;
    int g_vkernel = -1;  // verify body selection the graph was captured with
    float g_delta = 0.f;
    InjectPlan* plan_host = nullptr;  // pinned, max_iters entries
    cudaGraphExec_t bexec = nullptr;  // graph of the baseline pass
    int b_repeats = -1;
    cudaGraphExec_t mexec = nullptr;  // graph of the monolithic baseline pass
    int m_repeats = -1;
    // run_host: copy stream, input arrivals (A, then B per fragment), final
    // fragments ready for the host
    cudaStream_t xfer = nullptr;
    cudaEvent_t a_in = nullptr, xjoin = nullptr;
    // graph mode: stream on which the bodies of the conditional localisation
    // nodes are captured
    cudaStream_t body = nullptr;
    std::vector<cudaEvent_t> b_in, c_out;
    // run_host_steps: a second device copy of A and B (inputs alternate
    // between the two), a stream for result copies, per input copy its
    // arrival and release events, per C buffer the end of its last result
    // copy, and pinned per-step counters
    float* dA2 = nullptr;
    float* dB2 = nullptr;
    cudaStream_t xout = nullptr;
    cudaEvent_t in_a[2] = {nullptr, nullptr};
    std::vector<cudaEvent_t> in_b[2];
    cudaEvent_t in_free_c[2] = {nullptr, nullptr}, in_free_v[2] = {nullptr, nullptr};
    std::vector<cudaEvent_t> d2h_frag[2];  // result copy of fragment f out of C buffer q done
    cudaEvent_t vstep = nullptr, ojoin = nullptr;
    Counters* ctr_host = nullptr;
    int ctr_host_n = 0;
};

namespace {

// A named range on the host timeline of a profiler (Nsight Systems, or ncu
// --nvtx filters); without an attached tool each call returns at once.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    // printf-style name with one integer field ("abft step %d")
    NvtxRange(const char* fmt, int v) {
        char buf[64];
        std::snprintf(buf, sizeof(buf), fmt, v);
        nvtxRangePushA(buf);
    }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

#define CK(call)                                                     \
    do {                                                             \
        cudaError_t e_ = (call);                                     \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);          \
    } while (0)

#define RC(call)                                                     \
    do {                                                             \
        int rc_ = (call);                                            \
        if (rc_ != ABFT_OK) return rc_;                              \
    } while (0)

int sgemm_frag(abft_session* s, float* dC, int f) {
    const int off = s->offsets[f];
    return abft_sgemm(s->handle, s->dA, (int)s->lda, s->dB + off, (int)s->ldb, dC + off, (int)s->ldc, s->M_b,
                      s->counts[f], s->K);
}

// gemm_warmup, kernels/gemm_cublas.cuh:25-42: three 64^3 SGEMMs so that
// library loading and heuristics happen before any timed region.
int gemm_warmup(abft_session* s) {
    constexpr int W = 64;
    float* buf = nullptr;
    CK(cudaMalloc(&buf, sizeof(float) * W * W * 3));
    CK(cudaMemsetAsync(buf, 0, sizeof(float) * W * W * 3, s->compute));
    for (int i = 0; i < 3; ++i) {
        int rc = abft_sgemm(s->handle, buf, W, buf + W * W, W, buf + 2 * W * W, W, W, W, W);
        if (rc != ABFT_OK) {
            cudaFree(buf);
            return rc;
        }
    }
    const cudaError_t e = cudaStreamSynchronize(s->compute);
    cudaFree(buf);
    if (e != cudaSuccess) return cuda_fail(e, "gemm warm-up");
    return ABFT_OK;
}

struct Plan {
    int frag, row, col, bit;
};

// Transfer points of run_host: iteration 0's SGEMM of fragment f waits for A
// and for B's fragment f to arrive; the last iteration's fragment f records
// out_ready[f] once its verification and correction are enqueued, so that its
// copy to the host overlaps the SGEMMs of the fragments after it.
struct IoHooks {
    cudaEvent_t a_ready;
    const cudaEvent_t* b_ready;
    const cudaEvent_t* out_ready;  // null: no per-fragment signal
    // run_host_steps: both C buffers were used by an earlier step, so their
    // first use here waits for that step's verification of them ...
    bool carry_used = false;
    // ... and, where slot_free[buffer] is not null, fragment f's first SGEMM
    // into that buffer waits for slot_free[buffer][f], the earlier step's copy
    // of that fragment to the host (not for the copies of the fragments after
    // it, which start only at the end of that step)
    const cudaEvent_t* const* slot_free = nullptr;
};

// Graph mode: a conditional handle of the graph being captured on st, reset
// to 0 at every launch of the instantiated graph.
int cond_handle(cudaStream_t st, cudaGraphConditionalHandle* h) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaGraph_t g = nullptr;
    CK(cudaStreamGetCaptureInfo(st, &cs, nullptr, &g, nullptr, nullptr));
    if (cs != cudaStreamCaptureStatusActive || g == nullptr) {
        set_error("conditional localisation: stream is not capturing");
        return ABFT_ERR_STATE;
    }
    CK(cudaGraphConditionalHandleCreate(h, g, 0, cudaGraphCondAssignDefault));
    return ABFT_OK;
}

// Appends to st's capture an IF node on h (after all st has captured so far),
// continues st's capture after it, and captures `fill` into its body on the
// session's body stream.
template <class Fill>
int capture_if(abft_session* s, cudaStream_t st, cudaGraphConditionalHandle h, Fill fill) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaGraph_t g = nullptr;
    const cudaGraphNode_t* deps = nullptr;
    size_t nd = 0;
    CK(cudaStreamGetCaptureInfo(st, &cs, nullptr, &g, &deps, &nd));
    cudaGraphNodeParams p{};
    p.type = cudaGraphNodeTypeConditional;
    p.conditional.handle = h;
    p.conditional.type = cudaGraphCondTypeIf;
    p.conditional.size = 1;
    cudaGraphNode_t node = nullptr;
    CK(cudaGraphAddNode(&node, g, deps, nd, &p));
    cudaGraph_t body = p.conditional.phGraph_out[0];
    CK(cudaStreamUpdateCaptureDependencies(st, &node, 1, cudaStreamSetCaptureDependencies));
    CK(cudaStreamBeginCaptureToGraph(s->body, body, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal));
    const int rc = fill(s->body);
    cudaGraph_t out = nullptr;
    const cudaError_t e = cudaStreamEndCapture(s->body, &out);
    if (rc != ABFT_OK) return rc;
    CK(e);
    return ABFT_OK;
}

// Enqueue `repeats` protected iterations on the two streams (no host sync).
// graph = true: the injection is read from the device plan table by the verify
// kernel (capturable, the same graph serves every trial).
int enqueue_loop(abft_session* s, const abft_online_args* a, const std::vector<Plan>& plan, int* launches,
                 int* vlaunches, bool graph = false, const IoHooks* io = nullptr) {
    const bool inject_on = (a->mode == ABFT_INJECT_ADD || a->mode == ABFT_INJECT_SWIFI);
    const bool do_localize = inject_on;
    bool used[2] = {false, false};
    if (io && io->carry_used) used[0] = used[1] = true;
    bool first[2] = {true, true};
    int nl = 0, nv = 0;
    for (int it = 0; it < a->repeats; ++it) {
        const NvtxRange range("abft iteration %d", it);
        const int bi = it & 1;
        float* dC = s->dC[bi];
        if (used[bi]) CK(cudaStreamWaitEvent(s->compute, s->buf_done[bi], 0));
        const cudaEvent_t* slot_free = (first[bi] && io && io->slot_free) ? io->slot_free[bi] : nullptr;
        first[bi] = false;
        const int log_it = (a->log && it < s->max_iters) ? it : -1;
        for (int f = 0; f < s->F; ++f) {
            if (io && it == 0) {
                if (f == 0) CK(cudaStreamWaitEvent(s->compute, io->a_ready, 0));
                CK(cudaStreamWaitEvent(s->compute, io->b_ready[f], 0));
            }
            if (slot_free) CK(cudaStreamWaitEvent(s->compute, slot_free[f], 0));
            RC(sgemm_frag(s, dC, f));
            if (!graph && f == plan[it].frag) {
                InjectLog* lg = (log_it >= 0) ? s->ws->d.ilog + log_it : nullptr;
                const int mode = (a->mode == ABFT_INJECT_ADD) ? ABFT_INJECT_ADD : ABFT_INJECT_SWIFI;
                RC(launch_inject(dC + s->offsets[f], s->ldc, plan[it].row, plan[it].col, mode, a->add_delta,
                                 plan[it].bit, lg, f, s->compute));
                ++nl;
            }
            CK(cudaEventRecord(s->compute_done[f], s->compute));
        }
        for (int f = 0; f < s->F; ++f) {
            const int injected = (f == plan[it].frag) ? 1 : 0;
            CK(cudaStreamWaitEvent(s->verify, s->compute_done[f], 0));
            const bool prof = !graph && s->profile && (size_t)(2 * nv + 1) < s->vprof.size();
            if (prof) CK(cudaEventRecord(s->vprof[2 * nv], s->verify));
            // Graph mode: fragment f's localisation sits in a conditional node
            // that the verify kernel opens only when it detected a column, so
            // clean fragments cost no launch (host-enqueued, the localisation
            // kernel is launched and returns at once when nothing was found).
            cudaGraphConditionalHandle h = 0;
            if (graph && do_localize) RC(cond_handle(s->verify, &h));
            if (graph)
                RC(launch_verify(s->ws, dC, s->ldc, f, s->tau[f], 0, log_it, s->verify, it, a->add_delta,
                                 (a->log && inject_on) ? 1 : 0, nullptr, h));
            else
                RC(launch_verify(s->ws, dC, s->ldc, f, s->tau[f], injected, log_it, s->verify));
            if (prof) CK(cudaEventRecord(s->vprof[2 * nv + 1], s->verify));
            ++nl;
            ++nv;
            if (do_localize && graph) {
                RC(capture_if(s, s->verify, h, [&](cudaStream_t bs) {
                    return launch_localize(s->ws, dC, s->ldc, f, s->tau[f], injected, s->dG, s->ldg, it,
                                           a->correct_mode, bs, it);
                }));
            } else if (do_localize) {
                RC(launch_localize(s->ws, dC, s->ldc, f, s->tau[f], injected, s->dG, s->ldg, it, a->correct_mode,
                                   s->verify, -1));
                ++nl;
            }
            if (io && io->out_ready && it == a->repeats - 1) CK(cudaEventRecord(io->out_ready[f], s->verify));
        }
        CK(cudaEventRecord(s->buf_done[bi], s->verify));
        used[bi] = true;
    }
    if (do_localize && a->correct_mode == ABFT_CORRECT_DRAIN) {
        RC(launch_drain(s->ws, s->dC[0], s->dC[1], s->ldc, s->dG, s->ldg, a->repeats, s->verify));
        ++nl;
    }
    *launches = nl;
    *vlaunches = nv;
    return ABFT_OK;
}

int make_plan(abft_session* s, const abft_online_args* a, std::vector<Plan>& plan) {
    plan.assign(a->repeats, Plan{-1, -1, -1, -1});
    for (int it = 0; it < a->repeats; ++it) {
        if (a->seed_scheme == ABFT_SEED_TILE)
            RC(abft_injection_plan_tile(a->base_seed + (uint64_t)it, s->M_b, s->F, s->counts.data(), s->offsets.data(),
                                        a->mode, a->zone_lo, a->zone_hi, &plan[it].frag, &plan[it].row,
                                        &plan[it].col, &plan[it].bit));
        else
            RC(abft_injection_plan(a->base_seed, a->rank, it, s->F, s->M_b, s->counts.data(), a->mode, a->zone_lo,
                                   a->zone_hi, &plan[it].frag, &plan[it].row, &plan[it].col, &plan[it].bit));
    }
    return ABFT_OK;
}

void drop_graph(abft_session* s) {
    if (s->gexec) cudaGraphExecDestroy(s->gexec);
    s->gexec = nullptr;
    s->g_repeats = -1;
}

// Capture the loop once for this shape (repeats, mode, correction, logging,
// fault size, verify body selection); thresholds and the golden pointer are
// baked in, so setting them drops the graph.
int build_graph(abft_session* s, const abft_online_args* a, const std::vector<Plan>& plan) {
    if (s->gexec && s->g_repeats == a->repeats && s->g_mode == a->mode && s->g_correct == a->correct_mode &&
        s->g_log == a->log && s->g_delta == a->add_delta && s->g_vkernel == verify_kernel())
        return ABFT_OK;
    drop_graph(s);
    CK(cudaStreamBeginCapture(s->compute, cudaStreamCaptureModeThreadLocal));
    int nl = 0, nv = 0;
    int rc = ABFT_OK;
    cudaError_t e = cudaEventRecord(s->cjoin, s->compute);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s->verify, s->cjoin, 0);
    if (e != cudaSuccess) rc = cuda_fail(e, "graph fork");
    if (rc == ABFT_OK) rc = enqueue_loop(s, a, plan, &nl, &nv, true);
    if (rc == ABFT_OK) {
        e = cudaEventRecord(s->vjoin, s->verify);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s->compute, s->vjoin, 0);
        if (e != cudaSuccess) rc = cuda_fail(e, "graph join");
    }
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(s->compute, &g);
    if (rc == ABFT_OK && e != cudaSuccess) rc = cuda_fail(e, "cudaStreamEndCapture");
    if (rc == ABFT_OK) {
        e = cudaGraphInstantiate(&s->gexec, g, 0);
        if (e != cudaSuccess) {
            s->gexec = nullptr;
            rc = cuda_fail(e, "cudaGraphInstantiate");
        }
    }
    if (g) cudaGraphDestroy(g);
    (void)cudaGetLastError();
    if (rc != ABFT_OK) return rc;
    s->g_repeats = a->repeats;
    s->g_mode = a->mode;
    s->g_correct = a->correct_mode;
    s->g_log = a->log;
    s->g_delta = a->add_delta;
    s->g_vkernel = verify_kernel();
    s->g_launches = nl;
    s->g_vlaunches = nv;
    return ABFT_OK;
}

int check_args(abft_session* s, const abft_online_args* a) {
    if (!a || a->repeats < 0 || (a->mode < ABFT_INJECT_NONE || a->mode > ABFT_INJECT_SWIFI) ||
        (a->correct_mode != ABFT_CORRECT_INLOOP && a->correct_mode != ABFT_CORRECT_DRAIN)) {
        set_error("online: bad arguments");
        return ABFT_ERR_ARG;
    }
    if ((int)s->tau.size() != s->F) {
        set_error("online: thresholds not set (abft_session_set_tau)");
        return ABFT_ERR_STATE;
    }
    if (a->correct_mode == ABFT_CORRECT_DRAIN && a->mode != ABFT_INJECT_NONE && a->repeats > s->max_iters) {
        set_error("online: drain correction needs repeats <= max_iters");
        return ABFT_ERR_ARG;
    }
    if (a->seed_scheme != ABFT_SEED_REFERENCE && a->seed_scheme != ABFT_SEED_TILE) {
        set_error("online: unknown seed scheme");
        return ABFT_ERR_ARG;
    }
    if (a->graph && a->repeats > s->max_iters) {
        set_error("online: graph mode needs repeats <= max_iters (the device injection plan table)");
        return ABFT_ERR_ARG;
    }
    return ABFT_OK;
}

int ensure_prof_events(abft_session* s, int n_verify) {
    if (!s->profile) return ABFT_OK;
    while ((int)s->vprof.size() < 2 * n_verify) {
        cudaEvent_t e;
        CK(cudaEventCreate(&e));
        s->vprof.push_back(e);
    }
    return ABFT_OK;
}

// Resources of run_host_steps, made on its first call: the second device
// copy of A and B (same leading dimensions as the session's), the result-copy
// stream, the input and result events, and n_steps pinned counter records.
int ensure_step_resources(abft_session* s, int n_steps) {
    // each resource is made only if missing, so a set-up that failed part way
    // is completed by the next call (destroy releases whatever exists)
    auto event = [](cudaEvent_t* e) { return *e ? cudaSuccess : cudaEventCreateWithFlags(e, cudaEventDisableTiming); };
    if (!s->dA2) CK(cudaMalloc(&s->dA2, sizeof(float) * (size_t)s->lda * s->M_b));
    if (!s->dB2) CK(cudaMalloc(&s->dB2, sizeof(float) * (size_t)s->ldb * s->K));
    if (!s->xout) CK(cudaStreamCreateWithFlags(&s->xout, cudaStreamNonBlocking));
    for (int q = 0; q < 2; ++q) {
        CK(event(&s->in_a[q]));
        CK(event(&s->in_free_c[q]));
        CK(event(&s->in_free_v[q]));
        if ((int)s->in_b[q].size() != s->F) s->in_b[q].assign(s->F, nullptr);
        for (int f = 0; f < s->F; ++f) CK(event(&s->in_b[q][f]));
        if ((int)s->d2h_frag[q].size() != s->F) s->d2h_frag[q].assign(s->F, nullptr);
        for (int f = 0; f < s->F; ++f) CK(event(&s->d2h_frag[q][f]));
    }
    CK(event(&s->vstep));
    CK(event(&s->ojoin));
    if (s->ctr_host_n < n_steps) {
        if (s->ctr_host) CK(cudaFreeHost(s->ctr_host));
        s->ctr_host = nullptr;
        s->ctr_host_n = 0;
        CK(cudaMallocHost(&s->ctr_host, sizeof(Counters) * (size_t)n_steps));
        s->ctr_host_n = n_steps;
    }
    return ABFT_OK;
}

void prof_stats(abft_session* s, int nv, abft_online_result* r) {
    r->verify_ms_sum = 0.0;
    r->verify_ms_max = 0.0;
    if (!s->profile) return;
    for (int k = 0; k < nv && 2 * k + 1 < (int)s->vprof.size(); ++k) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, s->vprof[2 * k], s->vprof[2 * k + 1]) == cudaSuccess) {
            r->verify_ms_sum += ms;
            if (ms > r->verify_ms_max) r->verify_ms_max = ms;
        }
    }
}

}  // namespace

extern "C" {

int abft_session_create(const abft_session_cfg* c, abft_session** out) {
    if (!out || !c) {
        set_error("abft_session_create: NULL argument");
        return ABFT_ERR_ARG;
    }
    *out = nullptr;
    if (c->M_b < 1 || c->N_b < 1 || c->K < 1 || c->F < 1 || !c->counts || !c->offsets || !c->dA || !c->dB ||
        !c->dC0 || !c->dC1 || c->lda < c->K || c->ldb < c->N_b || c->ldc < c->N_b || c->max_iters < 0 ||
        c->lda > 0x7fffffff || c->ldb > 0x7fffffff || c->ldc > 0x7fffffff) {
        set_error("abft_session_create: bad configuration");
        return ABFT_ERR_ARG;
    }
    abft_session* s = new (std::nothrow) abft_session();
    if (!s) {
        set_error("out of host memory");
        return ABFT_ERR_ARG;
    }
    s->M_b = c->M_b;
    s->N_b = c->N_b;
    s->K = c->K;
    s->F = c->F;
    s->counts.assign(c->counts, c->counts + c->F);
    s->offsets.assign(c->offsets, c->offsets + c->F);
    s->dA = c->dA;
    s->lda = c->lda;
    s->dB = c->dB;
    s->ldb = c->ldb;
    s->dC[0] = c->dC0;
    s->dC[1] = c->dC1;
    s->ldc = c->ldc;
    s->max_iters = c->max_iters;
    auto fail = [&](int rc) {
        abft_session_destroy(s);
        return rc;
    };
    cudaError_t e = cudaGetDevice(&s->device);
    if (e != cudaSuccess) return fail(cuda_fail(e, "cudaGetDevice"));
    int least = 0, greatest = 0;
    e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
    if (e != cudaSuccess) return fail(cuda_fail(e, "stream priority range"));
    const int vprio = (c->verify_priority < 0) ? least : (c->verify_priority > 0 ? greatest : 0);
    e = cudaStreamCreateWithPriority(&s->compute, cudaStreamNonBlocking, greatest);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&s->verify, cudaStreamNonBlocking, vprio);
    if (e != cudaSuccess) return fail(cuda_fail(e, "stream create"));
    if (cublasCreate(&s->handle) != CUBLAS_STATUS_SUCCESS ||
        cublasSetStream(s->handle, s->compute) != CUBLAS_STATUS_SUCCESS) {
        set_error("cublasCreate/cublasSetStream failed");
        return fail(ABFT_ERR_CUBLAS);
    }
    s->compute_done.assign(s->F, nullptr);
    for (int f = 0; f < s->F && e == cudaSuccess; ++f)
        e = cudaEventCreateWithFlags(&s->compute_done[f], cudaEventDisableTiming);
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&s->buf_done[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreate(&s->t0);
    if (e == cudaSuccess) e = cudaEventCreate(&s->t1);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->vjoin, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->cjoin, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->a_in, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->xjoin, cudaEventDisableTiming);
    s->b_in.assign(s->F, nullptr);
    s->c_out.assign(s->F, nullptr);
    for (int f = 0; f < s->F && e == cudaSuccess; ++f) {
        e = cudaEventCreateWithFlags(&s->b_in[f], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->c_out[f], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->xfer, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->body, cudaStreamNonBlocking);
    if (e != cudaSuccess) return fail(cuda_fail(e, "event create"));
    int rc = abft_ws_create(s->M_b, s->N_b, s->K, s->F, c->counts, c->offsets, c->max_iters, nullptr, 0, &s->ws);
    if (rc != ABFT_OK) return fail(rc);
    e = cudaMallocHost(&s->plan_host, sizeof(InjectPlan) * (size_t)std::max(c->max_iters, 1));
    if (e != cudaSuccess) return fail(cuda_fail(e, "pinned plan buffer"));
    rc = gemm_warmup(s);
    if (rc != ABFT_OK) return fail(rc);
    *out = s;
    return ABFT_OK;
}

int abft_session_destroy(abft_session* s) {
    if (!s) return ABFT_OK;
    if (s->compute) cudaStreamSynchronize(s->compute);
    if (s->verify) cudaStreamSynchronize(s->verify);
    if (s->xfer) cudaStreamSynchronize(s->xfer);
    if (s->xout) cudaStreamSynchronize(s->xout);
    drop_graph(s);
    if (s->bexec) cudaGraphExecDestroy(s->bexec);
    if (s->mexec) cudaGraphExecDestroy(s->mexec);
    if (s->plan_host) cudaFreeHost(s->plan_host);
    for (auto e : s->compute_done)
        if (e) cudaEventDestroy(e);
    for (auto e : s->vprof)
        if (e) cudaEventDestroy(e);
    for (auto e : {s->buf_done[0], s->buf_done[1], s->t0, s->t1, s->vjoin, s->cjoin, s->a_in, s->xjoin})
        if (e) cudaEventDestroy(e);
    for (auto e : s->b_in)
        if (e) cudaEventDestroy(e);
    for (auto e : s->c_out)
        if (e) cudaEventDestroy(e);
    if (s->xfer) cudaStreamDestroy(s->xfer);
    if (s->body) cudaStreamDestroy(s->body);
    if (s->xout) cudaStreamDestroy(s->xout);
    for (int q = 0; q < 2; ++q) {
        for (auto e : {s->in_a[q], s->in_free_c[q], s->in_free_v[q]})
            if (e) cudaEventDestroy(e);
        for (auto e : s->in_b[q])
            if (e) cudaEventDestroy(e);
        for (auto e : s->d2h_frag[q])
            if (e) cudaEventDestroy(e);
    }
    for (auto e : {s->vstep, s->ojoin})
        if (e) cudaEventDestroy(e);
    if (s->dA2) cudaFree(s->dA2);
    if (s->dB2) cudaFree(s->dB2);
    if (s->ctr_host) cudaFreeHost(s->ctr_host);
    if (s->handle) cublasDestroy(s->handle);
    if (s->compute) cudaStreamDestroy(s->compute);
    if (s->verify) cudaStreamDestroy(s->verify);
    abft_ws_destroy(s->ws);
    delete s;
    return ABFT_OK;
}

abft_ws* abft_session_ws(abft_session* s) { return s ? s->ws : nullptr; }

int abft_session_set_tau(abft_session* s, const double* tau) {
    if (!s || !tau) {
        set_error("abft_session_set_tau: NULL argument");
        return ABFT_ERR_ARG;
    }
    s->tau.assign(tau, tau + s->F);
    drop_graph(s);
    return ABFT_OK;
}

int abft_session_set_golden(abft_session* s, const float* dG, int64_t ldg) {
    if (!s || (dG && ldg < s->N_b)) {
        set_error("abft_session_set_golden: bad argument");
        return ABFT_ERR_ARG;
    }
    s->dG = dG;
    s->ldg = dG ? ldg : 0;
    drop_graph(s);
    return ABFT_OK;
}

int abft_session_encode(abft_session* s, double* encode_ms) {
    if (!s) {
        set_error("abft_session_encode: NULL session");
        return ABFT_ERR_ARG;
    }
    const NvtxRange range("abft encode");
    CK(cudaEventRecord(s->t0, s->verify));
    RC(launch_encode(s->ws, s->dA, s->lda, s->dB, s->ldb, s->verify, nullptr));
    CK(cudaEventRecord(s->t1, s->verify));
    CK(cudaStreamSynchronize(s->verify));
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, s->t0, s->t1));
    if (encode_ms) *encode_ms = ms;
    s->encoded = true;
    return ABFT_OK;
}

namespace {

// One unprotected pass into dC0 on the compute stream: repeats x (F fragment
// SGEMMs, or one SGEMM of the whole tile), optionally replayed as a CUDA graph
// captured once per repeats; device time by events on the compute stream.
int baseline_pass(abft_session* s, int repeats, int graph, bool monolithic, double* device_ms, double* host_ms) {
    CK(cudaStreamSynchronize(s->compute));
    cudaGraphExec_t& exec = monolithic ? s->mexec : s->bexec;
    int& captured = monolithic ? s->m_repeats : s->b_repeats;
    auto enqueue = [&]() -> int {
        int rc = ABFT_OK;
        for (int it = 0; it < repeats && rc == ABFT_OK; ++it) {
            if (monolithic)
                rc = abft_sgemm(s->handle, s->dA, (int)s->lda, s->dB, (int)s->ldb, s->dC[0], (int)s->ldc, s->M_b,
                                s->N_b, s->K);
            else
                for (int f = 0; f < s->F && rc == ABFT_OK; ++f) rc = sgemm_frag(s, s->dC[0], f);
        }
        return rc;
    };
    if (graph && (!exec || captured != repeats)) {
        if (exec) cudaGraphExecDestroy(exec);
        exec = nullptr;
        CK(cudaStreamBeginCapture(s->compute, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue();
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(s->compute, &g);
        if (rc == ABFT_OK && e != cudaSuccess) rc = cuda_fail(e, "cudaStreamEndCapture (baseline)");
        if (rc == ABFT_OK) {
            e = cudaGraphInstantiate(&exec, g, 0);
            if (e != cudaSuccess) {
                exec = nullptr;
                rc = cuda_fail(e, "cudaGraphInstantiate (baseline)");
            }
        }
        if (g) cudaGraphDestroy(g);
        (void)cudaGetLastError();
        if (rc != ABFT_OK) return rc;
        captured = repeats;
    }
    const auto h0 = std::chrono::high_resolution_clock::now();
    CK(cudaEventRecord(s->t0, s->compute));
    if (graph) {
        CK(cudaGraphLaunch(exec, s->compute));
    } else {
        RC(enqueue());
    }
    CK(cudaEventRecord(s->t1, s->compute));
    CK(cudaEventSynchronize(s->t1));
    const auto h1 = std::chrono::high_resolution_clock::now();
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, s->t0, s->t1));
    if (device_ms) *device_ms = ms;
    if (host_ms) *host_ms = std::chrono::duration<double, std::milli>(h1 - h0).count();
    return ABFT_OK;
}

}  // namespace

int abft_session_baseline(abft_session* s, int repeats, int graph, double* device_ms, double* host_ms) {
    if (!s || repeats < 0) {
        set_error("abft_session_baseline: bad argument");
        return ABFT_ERR_ARG;
    }
    const NvtxRange range(graph ? "abft baseline pass (graph)" : "abft baseline pass");
    return baseline_pass(s, repeats, graph, false, device_ms, host_ms);
}

int abft_session_baseline_monolithic(abft_session* s, int repeats, int graph, double* device_ms, double* host_ms) {
    if (!s || repeats < 0) {
        set_error("abft_session_baseline_monolithic: bad argument");
        return ABFT_ERR_ARG;
    }
    const NvtxRange range(graph ? "abft monolithic baseline (graph)" : "abft monolithic baseline");
    return baseline_pass(s, repeats, graph, true, device_ms, host_ms);
}

int abft_session_online(abft_session* s, const abft_online_args* a, abft_online_result* r) {
    if (!s || !r) {
        set_error("abft_session_online: NULL argument");
        return ABFT_ERR_ARG;
    }
    RC(check_args(s, a));
    const NvtxRange range(a->graph ? "abft online loop (graph)" : "abft online loop");
    s->profile = a->profile ? 1 : 0;
    if (!s->encoded) {
        double ms;
        RC(abft_session_encode(s, &ms));
    }
    std::vector<Plan> plan;
    RC(make_plan(s, a, plan));
    RC(ensure_prof_events(s, a->repeats * s->F));
    RC(abft_ws_reset_counters(s->ws, s->verify));
    CK(cudaStreamSynchronize(s->verify));
    CK(cudaStreamSynchronize(s->compute));

    int nl = 0, nv = 0;
    if (a->graph) {
        RC(build_graph(s, a, plan));
        for (int it = 0; it < a->repeats; ++it)
            s->plan_host[it] = InjectPlan{plan[it].frag, plan[it].row, plan[it].col, plan[it].bit};
        CK(cudaMemcpyAsync(s->ws->d.plan, s->plan_host, sizeof(InjectPlan) * a->repeats, cudaMemcpyHostToDevice,
                           s->compute));
        RC(abft_ws_reset_counters(s->ws, s->compute));
        nl = s->g_launches;
        nv = s->g_vlaunches;
    }
    const auto h0 = std::chrono::high_resolution_clock::now();
    CK(cudaEventRecord(s->t0, s->compute));
    if (a->graph) {
        CK(cudaGraphLaunch(s->gexec, s->compute));
    } else {
        CK(cudaStreamWaitEvent(s->verify, s->t0, 0));
        RC(enqueue_loop(s, a, plan, &nl, &nv));
        CK(cudaEventRecord(s->vjoin, s->verify));
        CK(cudaStreamWaitEvent(s->compute, s->vjoin, 0));
    }
    CK(cudaEventRecord(s->t1, s->compute));
    CK(cudaEventSynchronize(s->t1));
    const auto h1 = std::chrono::high_resolution_clock::now();
    CK(cudaGetLastError());

    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, s->t0, s->t1));
    r->device_ms = ms;
    r->host_ms = std::chrono::duration<double, std::milli>(h1 - h0).count();
    RC(abft_ws_read_counters(s->ws, r->cm, &r->n_restored));
    // graph mode: one localisation kernel ran per detected fragment (TP + FP)
    if (a->graph && (a->mode == ABFT_INJECT_ADD || a->mode == ABFT_INJECT_SWIFI)) nl += r->cm[0] + r->cm[2];
    r->kernel_launches = nl;
    r->verify_launches = nv;
    prof_stats(s, nv, r);
    s->last_launches = nl;
    return ABFT_OK;
}

int abft_session_read_injections(abft_session* s, int it_count, int* inj4, float* before_after) {
    if (!s || it_count < 0 || it_count > s->max_iters) {
        set_error("abft_session_read_injections: range outside max_iters");
        return ABFT_ERR_ARG;
    }
    if (it_count == 0) return ABFT_OK;
    std::vector<InjectLog> h(it_count);
    CK(cudaMemcpy(h.data(), s->ws->d.ilog, sizeof(InjectLog) * it_count, cudaMemcpyDeviceToHost));
    for (int i = 0; i < it_count; ++i) {
        if (inj4) {
            inj4[4 * i + 0] = h[i].frag;
            inj4[4 * i + 1] = h[i].row;
            inj4[4 * i + 2] = h[i].col;
            inj4[4 * i + 3] = h[i].bit;
        }
        if (before_after) {
            before_after[2 * i] = h[i].before;
            before_after[2 * i + 1] = h[i].after;
        }
    }
    return ABFT_OK;
}

int abft_session_run_host(abft_session* s, const float* hA, const float* hB, float* hC, const abft_online_args* a,
                          abft_online_result* r, double* e2e_ms) {
    if (!s || !hA || !hB || !hC || !r) {
        set_error("abft_session_run_host: NULL argument");
        return ABFT_ERR_ARG;
    }
    RC(check_args(s, a));
    const NvtxRange range("abft run_host");
    s->profile = a->profile ? 1 : 0;
    if (a->repeats < 1) {
        set_error("abft_session_run_host: repeats must be >= 1");
        return ABFT_ERR_ARG;
    }
    std::vector<Plan> plan;
    RC(make_plan(s, a, plan));
    RC(ensure_prof_events(s, a->repeats * s->F));
    CK(cudaStreamSynchronize(s->verify));
    CK(cudaStreamSynchronize(s->compute));
    // Enqueue and wait; on an error part of the work may still be queued, and
    // copies into the caller's host buffers must not outlive this call.
    auto run = [&]() -> int {
        const auto h0 = std::chrono::high_resolution_clock::now();
        CK(cudaEventRecord(s->t0, s->compute));
        CK(cudaStreamWaitEvent(s->xfer, s->t0, 0));
        // inputs: host -> device on the copy stream, A first, then B one fragment
        // (column block) at a time; iteration 0's SGEMM of fragment f starts as
        // soon as A and B's fragment f are in.
        CK(cudaMemcpy2DAsync(const_cast<float*>(s->dA), sizeof(float) * s->lda, hA, sizeof(float) * s->K,
                             sizeof(float) * s->K, s->M_b, cudaMemcpyHostToDevice, s->xfer));
        CK(cudaEventRecord(s->a_in, s->xfer));
        for (int f = 0; f < s->F; ++f) {
            const int off = s->offsets[f];
            CK(cudaMemcpy2DAsync(const_cast<float*>(s->dB) + off, sizeof(float) * s->ldb, hB + off,
                                 sizeof(float) * s->N_b, sizeof(float) * s->counts[f], s->K, cudaMemcpyHostToDevice,
                                 s->xfer));
            CK(cudaEventRecord(s->b_in[f], s->xfer));
        }
        // the checksums need all of B: encoded on the verify stream while the
        // first SGEMMs run
        CK(cudaStreamWaitEvent(s->verify, s->b_in[s->F - 1], 0));
        int nl = 0, nv = 0;
        RC(abft_ws_reset_counters(s->ws, s->verify));
        RC(launch_encode(s->ws, s->dA, s->lda, s->dB, s->ldb, s->verify, &nl));
        s->encoded = true;
        // result: device -> host. With in-loop correction each fragment of the
        // final buffer is final once its last verification and correction ran,
        // and is copied then; drain correction rewrites the buffer after the loop.
        const bool drain = (a->mode == ABFT_INJECT_ADD || a->mode == ABFT_INJECT_SWIFI) &&
                           a->correct_mode == ABFT_CORRECT_DRAIN;
        const IoHooks io{s->a_in, s->b_in.data(), drain ? nullptr : s->c_out.data()};
        int nl2 = 0;
        RC(enqueue_loop(s, a, plan, &nl2, &nv, false, &io));
        CK(cudaEventRecord(s->vjoin, s->verify));
        const float* last = s->dC[(a->repeats - 1) & 1];
        if (drain) CK(cudaStreamWaitEvent(s->xfer, s->vjoin, 0));
        for (int f = 0; f < s->F; ++f) {
            const int off = s->offsets[f];
            if (!drain) CK(cudaStreamWaitEvent(s->xfer, s->c_out[f], 0));
            CK(cudaMemcpy2DAsync(hC + off, sizeof(float) * s->N_b, last + off, sizeof(float) * s->ldc,
                                 sizeof(float) * s->counts[f], s->M_b, cudaMemcpyDeviceToHost, s->xfer));
        }
        CK(cudaEventRecord(s->xjoin, s->xfer));
        CK(cudaStreamWaitEvent(s->compute, s->vjoin, 0));
        CK(cudaStreamWaitEvent(s->compute, s->xjoin, 0));
        Counters hc{};
        CK(cudaMemcpyAsync(&hc, s->ws->d.ctr, sizeof(hc), cudaMemcpyDeviceToHost, s->compute));
        CK(cudaEventRecord(s->t1, s->compute));
        CK(cudaEventSynchronize(s->t1));
        const auto h1 = std::chrono::high_resolution_clock::now();
        CK(cudaGetLastError());
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, s->t0, s->t1));
        if (e2e_ms) *e2e_ms = ms;
        r->device_ms = ms;
        r->host_ms = std::chrono::duration<double, std::milli>(h1 - h0).count();
        for (int i = 0; i < 4; ++i) r->cm[i] = hc.cm[i];
        r->n_restored = hc.n_restored;
        if (hc.fault) {
            set_error("verify: a bulk tensor copy did not complete within the wait limit; the decisions are void");
            return ABFT_ERR_CUDA;
        }
        r->kernel_launches = nl + nl2;
        r->verify_launches = nv;
        prof_stats(s, nv, r);
        s->last_launches = nl + nl2;
        return ABFT_OK;
    };
    const int rc = run();
    if (rc != ABFT_OK) {
        cudaStreamSynchronize(s->xfer);
        cudaStreamSynchronize(s->verify);
        cudaStreamSynchronize(s->compute);
    }
    return rc;
}

int abft_session_run_host_steps(abft_session* s, int n_steps, const float* const* hA, const float* const* hB,
                                float* const* hC, const abft_online_args* a, const uint64_t* base_seeds,
                                abft_online_result* res, double* e2e_ms) {
    if (!s || n_steps < 1 || !hA || !hB || !hC || !base_seeds || !res) {
        set_error("abft_session_run_host_steps: NULL argument or n_steps < 1");
        return ABFT_ERR_ARG;
    }
    for (int k = 0; k < n_steps; ++k) {
        if (!hA[k] || !hB[k] || !hC[k]) {
            set_error("abft_session_run_host_steps: NULL host buffer for step " + std::to_string(k));
            return ABFT_ERR_ARG;
        }
    }
    if (!a) {
        set_error("abft_session_run_host_steps: NULL args");
        return ABFT_ERR_ARG;
    }
    abft_online_args ak = *a;
    ak.log = 0;
    ak.profile = 0;
    ak.graph = 0;
    RC(check_args(s, &ak));
    if (ak.repeats < 1) {
        set_error("abft_session_run_host_steps: repeats must be >= 1");
        return ABFT_ERR_ARG;
    }
    RC(ensure_step_resources(s, n_steps));
    const NvtxRange range("abft run_host_steps (%d steps)", n_steps);
    s->profile = 0;
    std::vector<std::vector<Plan>> plans(n_steps);
    for (int k = 0; k < n_steps; ++k) {
        ak.base_seed = base_seeds[k];
        RC(make_plan(s, &ak, plans[k]));
    }
    CK(cudaStreamSynchronize(s->verify));
    CK(cudaStreamSynchronize(s->compute));
    const bool drain = (a->mode == ABFT_INJECT_ADD || a->mode == ABFT_INJECT_SWIFI) &&
                       a->correct_mode == ABFT_CORRECT_DRAIN;
    const int fin = (a->repeats - 1) & 1;  // the C buffer that holds a step's result
    float* const inA[2] = {const_cast<float*>(s->dA), s->dA2};
    float* const inB[2] = {const_cast<float*>(s->dB), s->dB2};
    const float* const origA = s->dA;
    const float* const origB = s->dB;

    auto run = [&]() -> int {
        CK(cudaEventRecord(s->t0, s->compute));
        CK(cudaStreamWaitEvent(s->xfer, s->t0, 0));
        CK(cudaStreamWaitEvent(s->xout, s->t0, 0));
        CK(cudaStreamWaitEvent(s->verify, s->t0, 0));
        RC(abft_ws_reset_counters(s->ws, s->verify));
        // inputs of step k into copy k % 2, once step k - 2 no longer reads it
        // (its SGEMMs on the compute stream, its encode on the verify stream);
        // B goes one fragment at a time, as in run_host
        auto upload = [&](int k) -> int {
            const int q = k & 1;
            if (k >= 2) {
                CK(cudaStreamWaitEvent(s->xfer, s->in_free_c[q], 0));
                CK(cudaStreamWaitEvent(s->xfer, s->in_free_v[q], 0));
            }
            CK(cudaMemcpy2DAsync(inA[q], sizeof(float) * s->lda, hA[k], sizeof(float) * s->K, sizeof(float) * s->K,
                                 s->M_b, cudaMemcpyHostToDevice, s->xfer));
            CK(cudaEventRecord(s->in_a[q], s->xfer));
            for (int f = 0; f < s->F; ++f) {
                const int off = s->offsets[f];
                CK(cudaMemcpy2DAsync(inB[q] + off, sizeof(float) * s->ldb, hB[k] + off, sizeof(float) * s->N_b,
                                     sizeof(float) * s->counts[f], s->K, cudaMemcpyHostToDevice, s->xfer));
                CK(cudaEventRecord(s->in_b[q][f], s->xfer));
            }
            return ABFT_OK;
        };
        RC(upload(0));
        bool pending[2] = {false, false};  // a result copy read this C buffer in the previous step
        for (int k = 0; k < n_steps; ++k) {
            const NvtxRange step_range("abft step %d", k);
            const int q = k & 1;
            // the SGEMMs of this step read copy q (sgemm_frag uses s->dA / s->dB)
            s->dA = inA[q];
            s->dB = inB[q];
            int nl = 0, nl2 = 0, nv = 0;
            CK(cudaStreamWaitEvent(s->verify, s->in_b[q][s->F - 1], 0));
            RC(launch_encode(s->ws, inA[q], s->lda, inB[q], s->ldb, s->verify, &nl));
            CK(cudaEventRecord(s->in_free_v[q], s->verify));
            const cudaEvent_t* const slot_free[2] = {pending[0] ? s->d2h_frag[0].data() : nullptr,
                                                     pending[1] ? s->d2h_frag[1].data() : nullptr};
            IoHooks io{s->in_a[q], s->in_b[q].data(), drain ? nullptr : s->c_out.data(), k > 0, slot_free};
            ak.base_seed = base_seeds[k];
            RC(enqueue_loop(s, &ak, plans[k], &nl2, &nv, false, &io));
            CK(cudaEventRecord(s->in_free_c[q], s->compute));
            // this step's counters, then cleared for the next step
            CK(cudaMemcpyAsync(&s->ctr_host[k], s->ws->d.ctr, sizeof(Counters), cudaMemcpyDeviceToHost, s->verify));
            CK(cudaMemsetAsync(s->ws->d.ctr, 0, sizeof(Counters), s->verify));
            CK(cudaEventRecord(s->vstep, s->verify));
            res[k] = abft_online_result{};
            res[k].kernel_launches = nl + nl2;
            res[k].verify_launches = nv;
            // the next step's inputs travel while this step computes
            if (k + 1 < n_steps) RC(upload(k + 1));
            // this step's result: each fragment once its last check ran (after
            // the whole step with drain correction)
            if (drain) CK(cudaStreamWaitEvent(s->xout, s->vstep, 0));
            const float* last = s->dC[fin];
            for (int f = 0; f < s->F; ++f) {
                const int off = s->offsets[f];
                if (!drain) CK(cudaStreamWaitEvent(s->xout, s->c_out[f], 0));
                CK(cudaMemcpy2DAsync(hC[k] + off, sizeof(float) * s->N_b, last + off, sizeof(float) * s->ldc,
                                     sizeof(float) * s->counts[f], s->M_b, cudaMemcpyDeviceToHost, s->xout));
                CK(cudaEventRecord(s->d2h_frag[fin][f], s->xout));
            }
            pending[fin] = true;
            pending[1 - fin] = false;
        }
        CK(cudaEventRecord(s->ojoin, s->xout));
        CK(cudaEventRecord(s->xjoin, s->xfer));
        CK(cudaStreamWaitEvent(s->compute, s->vstep, 0));
        CK(cudaStreamWaitEvent(s->compute, s->ojoin, 0));
        CK(cudaStreamWaitEvent(s->compute, s->xjoin, 0));
        CK(cudaEventRecord(s->t1, s->compute));
        CK(cudaEventSynchronize(s->t1));
        CK(cudaGetLastError());
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, s->t0, s->t1));
        if (e2e_ms) *e2e_ms = ms;
        int fault = 0;
        for (int k = 0; k < n_steps; ++k) {
            const Counters& c = s->ctr_host[k];
            for (int i = 0; i < 4; ++i) res[k].cm[i] = c.cm[i];
            res[k].n_restored = c.n_restored;
            res[k].device_ms = ms / n_steps;
            res[k].host_ms = 0.0;
            fault |= c.fault;
        }
        if (fault) {
            set_error("verify: a bulk tensor copy did not complete within the wait limit; the decisions are void");
            return ABFT_ERR_CUDA;
        }
        return ABFT_OK;
    };
    const int rc = run();
    s->dA = origA;
    s->dB = origB;
    if (rc != ABFT_OK) {
        cudaStreamSynchronize(s->xfer);
        cudaStreamSynchronize(s->xout);
        cudaStreamSynchronize(s->verify);
        cudaStreamSynchronize(s->compute);
    }
    // the checksums in the workspace belong to the last step's inputs, which
    // may sit in the second copy: a later online call must encode again
    s->encoded = false;
    return rc;
}

}  // extern "C"
