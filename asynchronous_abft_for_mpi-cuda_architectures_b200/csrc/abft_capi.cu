// C ABI: workspace management and the kernel-level entry points.

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>

#include "abft_b200.h"
#include "abft_internal.h"

namespace abft {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int cuda_fail(cudaError_t e, const char* what) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return ABFT_ERR_CUDA;
}

static size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

WsLayout ws_layout(int M_b, int N_b, int K, int F, int nfmax, int max_iters) {
    WsLayout L{};
    const size_t nacc = (size_t)acc_columns(nfmax);
    const size_t groups = nacc / kGroupCols;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t at = o;
        o += up256(bytes);
        return at;
    };
    L.colSumA = take(sizeof(double) * K);
    L.expRow = take(sizeof(double) * N_b);
    L.rowSumB = take(sizeof(double) * (size_t)F * K);
    L.expCol = take(sizeof(double) * (size_t)F * M_b);
    L.rec = take(sizeof(FragRecord) * F);
    L.ctr = take(sizeof(Counters));
    L.vacc_s = take(sizeof(double) * nacc);
    L.vacc_t = take(sizeof(float) * nacc);
    L.vacc_m = take(sizeof(uint32_t) * nacc);
    L.vact = take(sizeof(double) * nacc);
    L.vd = take(sizeof(double) * nacc);
    L.vw = take(sizeof(double) * nacc);
    L.vcnt = take(sizeof(int) * vcnt_ints((int)groups));
    L.lbd = take(sizeof(double) * M_b);
    L.lbr = take(sizeof(int) * M_b);
    L.lcnt = take(sizeof(int) * 4);
    L.dlog = take(sizeof(DecisionLog) * (size_t)std::max(max_iters, 1) * F);
    L.ilog = take(sizeof(InjectLog) * (size_t)std::max(max_iters, 1));
    L.pend = take(sizeof(PendingFix) * (size_t)std::max(max_iters, 1) * F);
    L.plan = take(sizeof(InjectPlan) * (size_t)std::max(max_iters, 1));
    L.total = o;
    return L;
}

}  // namespace abft

using namespace abft;

static int check_frags(int N_b, int F, const int* counts, const int* offsets) {
    if (F < 1 || !counts || !offsets) {
        set_error("fragment table missing");
        return ABFT_ERR_ARG;
    }
    for (int f = 0; f < F; ++f) {
        if (counts[f] < 1 || offsets[f] < 0 || (long long)offsets[f] + counts[f] > N_b) {
            set_error("fragment " + std::to_string(f) + " outside the tile");
            return ABFT_ERR_ARG;
        }
    }
    return ABFT_OK;
}

extern "C" {

const char* abft_last_error(void) { return g_last_error.c_str(); }

int abft_version(void) { return 10000; }

size_t abft_ws_bytes(int M_b, int N_b, int K, int F, const int* counts, int max_iters) {
    if (M_b < 1 || N_b < 1 || K < 1 || F < 1 || !counts) return 0;
    int nfmax = 0;
    for (int f = 0; f < F; ++f) nfmax = std::max(nfmax, counts[f]);
    return ws_layout(M_b, N_b, K, F, nfmax, std::max(max_iters, 0)).total;
}

int abft_ws_create(int M_b, int N_b, int K, int F, const int* counts, const int* offsets, int max_iters,
                   void* dev_mem, size_t dev_bytes, abft_ws** out) {
    if (!out) {
        set_error("out is NULL");
        return ABFT_ERR_ARG;
    }
    *out = nullptr;
    if (M_b < 1 || N_b < 1 || K < 1 || max_iters < 0) {
        set_error("tile sizes must be positive (M_b, N_b, K >= 1)");
        return ABFT_ERR_ARG;
    }
    if (int rc = check_frags(N_b, F, counts, offsets)) return rc;
    abft_ws* ws = new (std::nothrow) abft_ws();
    if (!ws) {
        set_error("out of host memory");
        return ABFT_ERR_ARG;
    }
    ws->M_b = M_b;
    ws->N_b = N_b;
    ws->K = K;
    ws->F = F;
    ws->max_iters = max_iters;
    ws->counts.assign(counts, counts + F);
    ws->offsets.assign(offsets, offsets + F);
    ws->nfmax = *std::max_element(ws->counts.begin(), ws->counts.end());
    ws->nacc = acc_columns(ws->nfmax);
    cudaError_t e = cudaGetDevice(&ws->device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ws->sms, cudaDevAttrMultiProcessorCount, ws->device);
    if (e != cudaSuccess) {
        delete ws;
        return cuda_fail(e, "device query");
    }
    WsLayout L = ws_layout(M_b, N_b, K, F, ws->nfmax, max_iters);
    ws->bytes = L.total;
    if (dev_mem) {
        if (dev_bytes < L.total || ((uintptr_t)dev_mem & 255u)) {
            delete ws;
            set_error("caller workspace too small or not 256-byte aligned (need " + std::to_string(L.total) +
                      " bytes)");
            return ABFT_ERR_ARG;
        }
        ws->base = dev_mem;
        ws->owns = false;
    } else {
        e = cudaMalloc(&ws->base, L.total);
        if (e != cudaSuccess) {
            delete ws;
            return cuda_fail(e, "workspace cudaMalloc");
        }
        ws->owns = true;
    }
    e = cudaMemset(ws->base, 0, L.total);
    if (e != cudaSuccess) {
        if (ws->owns) cudaFree(ws->base);
        delete ws;
        return cuda_fail(e, "workspace memset");
    }
    char* b = static_cast<char*>(ws->base);
    e = cudaMemset(b + L.vacc_m, 0xff, sizeof(uint32_t) * ws->nacc);
    // The clears run on the legacy default stream and do not block the host;
    // callers launch on their own (possibly non-blocking) streams, which are
    // not ordered after them, so they must be complete before returning.
    if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
    if (e != cudaSuccess) {
        if (ws->owns) cudaFree(ws->base);
        delete ws;
        return cuda_fail(e, "workspace memset");
    }
    WsDev& d = ws->d;
    d.colSumA = reinterpret_cast<double*>(b + L.colSumA);
    d.expRow = reinterpret_cast<double*>(b + L.expRow);
    d.rowSumB = reinterpret_cast<double*>(b + L.rowSumB);
    d.expCol = reinterpret_cast<double*>(b + L.expCol);
    d.rec = reinterpret_cast<FragRecord*>(b + L.rec);
    d.ctr = reinterpret_cast<Counters*>(b + L.ctr);
    d.vacc_s = reinterpret_cast<double*>(b + L.vacc_s);
    d.vacc_t = reinterpret_cast<float*>(b + L.vacc_t);
    d.vacc_m = reinterpret_cast<uint32_t*>(b + L.vacc_m);
    d.vact = reinterpret_cast<double*>(b + L.vact);
    d.vd = reinterpret_cast<double*>(b + L.vd);
    d.vw = reinterpret_cast<double*>(b + L.vw);
    d.vcnt = reinterpret_cast<int*>(b + L.vcnt);
    d.lbd = reinterpret_cast<double*>(b + L.lbd);
    d.lbr = reinterpret_cast<int*>(b + L.lbr);
    d.lcnt = reinterpret_cast<int*>(b + L.lcnt);
    d.dlog = reinterpret_cast<DecisionLog*>(b + L.dlog);
    d.ilog = reinterpret_cast<InjectLog*>(b + L.ilog);
    d.pend = reinterpret_cast<PendingFix*>(b + L.pend);
    d.plan = reinterpret_cast<InjectPlan*>(b + L.plan);
    *out = ws;
    return ABFT_OK;
}

int abft_ws_destroy(abft_ws* ws) {
    if (!ws) return ABFT_OK;
    int rc = ABFT_OK;
    if (ws->owns && ws->base) {
        cudaError_t e = cudaFree(ws->base);
        if (e != cudaSuccess) rc = cuda_fail(e, "workspace cudaFree");
    }
    delete ws;
    return rc;
}

int abft_ws_reset_counters(abft_ws* ws, void* stream) {
    if (!ws) {
        set_error("ws is NULL");
        return ABFT_ERR_ARG;
    }
    cudaError_t e = cudaMemsetAsync(ws->d.ctr, 0, sizeof(Counters), (cudaStream_t)stream);
    return e == cudaSuccess ? ABFT_OK : cuda_fail(e, "reset counters");
}

int* abft_ws_counters_device(abft_ws* ws) { return ws ? reinterpret_cast<int*>(ws->d.ctr) : nullptr; }

int abft_ws_read_counters(abft_ws* ws, int cm[4], int* n_restored) {
    if (!ws || !cm) {
        set_error("bad argument");
        return ABFT_ERR_ARG;
    }
    Counters c{};
    cudaError_t e = cudaMemcpy(&c, ws->d.ctr, sizeof(c), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "read counters");
    for (int i = 0; i < 4; ++i) cm[i] = c.cm[i];
    if (n_restored) *n_restored = c.n_restored;
    if (c.fault) {
        set_error("verify: a bulk tensor copy did not complete within the wait limit; the decisions are void");
        return ABFT_ERR_CUDA;
    }
    return ABFT_OK;
}

int abft_ws_read_log(abft_ws* ws, int it_count, int* errcol, int* errrow, double* rowdiff) {
    if (!ws || it_count < 0 || it_count > ws->max_iters) {
        set_error("log range outside the workspace's max_iters");
        return ABFT_ERR_ARG;
    }
    const size_t n = (size_t)it_count * ws->F;
    if (n == 0) return ABFT_OK;
    DecisionLog* h = new (std::nothrow) DecisionLog[n];
    if (!h) {
        set_error("out of host memory");
        return ABFT_ERR_ARG;
    }
    cudaError_t e = cudaMemcpy(h, ws->d.dlog, sizeof(DecisionLog) * n, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        delete[] h;
        return cuda_fail(e, "read log");
    }
    for (size_t i = 0; i < n; ++i) {
        if (errcol) errcol[i] = h[i].errcol;
        if (errrow) errrow[i] = h[i].errrow;
        if (rowdiff) rowdiff[i] = h[i].rowdiff;
    }
    delete[] h;
    return ABFT_OK;
}

int abft_ws_read_checksums(abft_ws* ws, double* colSumA, double* expRow, double* rowSumB, double* expCol) {
    if (!ws) {
        set_error("ws is NULL");
        return ABFT_ERR_ARG;
    }
    cudaError_t e = cudaSuccess;
    if (colSumA && e == cudaSuccess)
        e = cudaMemcpy(colSumA, ws->d.colSumA, sizeof(double) * ws->K, cudaMemcpyDeviceToHost);
    if (expRow && e == cudaSuccess)
        e = cudaMemcpy(expRow, ws->d.expRow, sizeof(double) * ws->N_b, cudaMemcpyDeviceToHost);
    if (rowSumB && e == cudaSuccess)
        e = cudaMemcpy(rowSumB, ws->d.rowSumB, sizeof(double) * (size_t)ws->F * ws->K, cudaMemcpyDeviceToHost);
    if (expCol && e == cudaSuccess)
        e = cudaMemcpy(expCol, ws->d.expCol, sizeof(double) * (size_t)ws->F * ws->M_b, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? ABFT_OK : cuda_fail(e, "read checksums");
}

int abft_encode(abft_ws* ws, const float* dA, int64_t lda, const float* dB, int64_t ldb, void* stream) {
    if (!ws || !dA || !dB || lda < ws->K || ldb < ws->N_b) {
        set_error("abft_encode: bad argument (need lda >= K, ldb >= N_b)");
        return ABFT_ERR_ARG;
    }
    return launch_encode(ws, dA, lda, dB, ldb, (cudaStream_t)stream, nullptr);
}

int abft_verify(abft_ws* ws, const float* dC, int64_t ldc, int f, double tau, int injected, int it, void* stream) {
    if (!ws || !dC || f < 0 || f >= ws->F || ldc < ws->N_b) {
        set_error("abft_verify: bad argument (fragment index, pointer or ldc < N_b)");
        return ABFT_ERR_ARG;
    }
    return launch_verify(ws, dC, ldc, f, tau, injected ? 1 : 0, it, (cudaStream_t)stream);
}

int abft_calibrate(abft_ws* ws, const float* dC, int64_t ldc, int f, double* dDiff, void* stream) {
    if (!ws || !dC || !dDiff || f < 0 || f >= ws->F || ldc < ws->N_b) {
        set_error("abft_calibrate: bad argument (fragment index, pointers or ldc < N_b)");
        return ABFT_ERR_ARG;
    }
    return launch_verify(ws, dC, ldc, f, INFINITY, 0, -1, (cudaStream_t)stream, -1, 0.f, 0, dDiff);
}

int abft_set_verify_kernel(int which) {
    const int prev = set_verify_kernel(which);
    if (prev < 0) {
        set_error("abft_set_verify_kernel: which must be ABFT_VERIFY_AUTO, _LDG or _TMA");
        return ABFT_ERR_ARG;
    }
    return prev;
}

int abft_set_wait_limit(int polls) {
    const int prev = set_wait_limit(polls);
    if (prev < 0) {
        set_error("abft_set_wait_limit: polls must be >= 0");
        return ABFT_ERR_ARG;
    }
    return prev;
}

int abft_verify_noalloc(const float* dC_frag, int64_t ldc, int M, int N, const double* dExpRow, double tau,
                        int injected, int* dErrCol, double* dRowDiff, int* dCM, void* stream) {
    if (!dC_frag || !dExpRow || !dErrCol || !dRowDiff || !dCM || M < 1 || N < 1 || ldc < N) {
        set_error("abft_verify_noalloc: bad argument (pointers, M >= 1, N >= 1, ldc >= N)");
        return ABFT_ERR_ARG;
    }
    return launch_verify_static(dC_frag, ldc, M, N, dExpRow, tau, injected ? 1 : 0, dErrCol, dRowDiff, dCM,
                                (cudaStream_t)stream);
}

int abft_localize_correct(abft_ws* ws, float* dC, int64_t ldc, int f, double tau, int injected, const float* dGolden,
                          int64_t ldg, int it, int correct_mode, void* stream) {
    if (!ws || !dC || f < 0 || f >= ws->F || ldc < ws->N_b || (dGolden && ldg < ws->N_b) ||
        (correct_mode != ABFT_CORRECT_INLOOP && correct_mode != ABFT_CORRECT_DRAIN)) {
        set_error("abft_localize_correct: bad argument");
        return ABFT_ERR_ARG;
    }
    return launch_localize(ws, dC, ldc, f, tau, injected ? 1 : 0, dGolden, ldg, it, correct_mode,
                           (cudaStream_t)stream);
}

int abft_drain(abft_ws* ws, float* dC0, float* dC1, int64_t ldc, const float* dGolden, int64_t ldg, int repeats,
               void* stream) {
    if (!ws || !dC0 || !dC1 || ldc < ws->N_b || repeats < 0 || (dGolden && ldg < ws->N_b)) {
        set_error("abft_drain: bad argument");
        return ABFT_ERR_ARG;
    }
    return launch_drain(ws, dC0, dC1, ldc, dGolden, ldg, repeats, (cudaStream_t)stream);
}

int abft_inject_add(float* dC, int64_t ldc, int row, int col, float delta, void* stream) {
    if (!dC || row < 0 || col < 0 || col >= ldc) {
        set_error("abft_inject_add: bad argument");
        return ABFT_ERR_ARG;
    }
    return launch_inject(dC, ldc, row, col, ABFT_INJECT_ADD, delta, 0, nullptr, -1, (cudaStream_t)stream);
}

int abft_inject_bitflip(float* dC, int64_t ldc, int row, int col, int bit, void* stream) {
    if (!dC || row < 0 || col < 0 || col >= ldc || bit < 0 || bit > 31) {
        set_error("abft_inject_bitflip: bad argument");
        return ABFT_ERR_ARG;
    }
    return launch_inject(dC, ldc, row, col, ABFT_INJECT_SWIFI, 0.f, bit, nullptr, -1, (cudaStream_t)stream);
}

int abft_sgemm(void* cublas_handle, const float* dA, int lda, const float* dB, int ldb, float* dC, int ldc, int M,
               int N, int K) {
    if (!cublas_handle || !dA || !dB || !dC) {
        set_error("abft_sgemm: bad argument");
        return ABFT_ERR_ARG;
    }
    const float alpha = 1.0f, beta = 0.0f;
    cublasStatus_t st = cublasSgemm((cublasHandle_t)cublas_handle, CUBLAS_OP_N, CUBLAS_OP_N, N, M, K, &alpha, dB,
                                    ldb, dA, lda, &beta, dC, ldc);
    if (st != CUBLAS_STATUS_SUCCESS) {
        set_error("cublasSgemm failed with status " + std::to_string((int)st));
        return ABFT_ERR_CUBLAS;
    }
    return ABFT_OK;
}

}  // extern "C"
