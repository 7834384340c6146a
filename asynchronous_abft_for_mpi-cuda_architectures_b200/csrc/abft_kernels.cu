// sm_100a kernels of the asynchronous ABFT layer.
//
// Checksum arithmetic follows the reference's kernels
// (kernels/abft_stepwise.cuh:9-206, kernels/swifi.cuh:33-59): FP64 sums of
// FP32 data. The decisions (detected column, located row, corrected value)
// are bit-identical to the reference's, whose sums run sequentially, one
// thread per column. The fast path does not run sequentially; it is made exact
// as follows.
//
// Certified fast sums. A verify CTA streams a tile of C with 128-bit loads
// (all SMs, HBM bound) and keeps, per column, the double sum S, the float sum
// T of |x| and the smallest nonzero |x|. Every x is an integer multiple of
// 2^p, p = ulp exponent of the smallest nonzero |x|; when T <= 2^(p+53) every
// partial sum of every order is a multiple of 2^p below 2^(p+53) and hence
// exactly representable, so S equals the reference's sequential sum bit for
// bit ("certified"). Otherwise S differs from it by at most 2*gamma_n*T and
// the decision logic carries that window: a column whose window cannot reach
// the threshold or the current maximum is decided without it; the few that
// can are re-summed in the reference's order (exact_chain, which proves runs
// of terms exact or absorbed and steps through the rest). The arg-max is then
// the reference's own 256-slot strided scan and tree on exact values. A
// second verify body (k_verify_tma) stages the tile through shared memory
// with bulk tensor copies; the localisation kernel certifies row sums alike.
//
// Encode kernels (colSumA, expectedRow, rowSumB_f, expectedCol_f) are
// sequential chains by definition; they run one chain per thread fed from
// shared memory by a deep cp.async pipeline so that the chain latency, not
// memory latency, bounds them.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <tuple>
#include <string>

#include "abft_b200.h"
#include "abft_internal.h"

namespace abft {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kListCap = 256;
constexpr int kBatch = 8;   // rows in flight per warp in the verify body
constexpr int kLocNarrow = 512;  // localise: rows of at most this many floats are summed 4 per warp at a time
// TMA-staged verify: 32-row x 128-column boxes (16 KB) through a 6-stage ring.
constexpr int kTmaRows = 32;
constexpr int kTmaStages = 6;
constexpr int kStageBytes = kTmaRows * kGroupCols * 4;
constexpr int kTmaSmem = kTmaStages * kStageBytes;
constexpr int kTmaAlign = 1024;  // alignment of the ring (bulk tensor copy destinations)
// The automatic choice never takes the TMA body. Timed alone on B200 it is
// 0.1-0.9 us ahead below 17 MB and behind from 33.6 MB up (2.5 us at 268 MB,
// 17 us at 1 GiB), but inside the protected loop, where verify runs beside
// the SGEMM, its ~97 KB of shared memory per CTA keeps it off the SMs the
// SGEMM occupies: the loop's overhead was higher with it at every measured
// workload (1024^3 to 16384^3, graph mode), while the 16 KB CTAs of the
// 128-bit-load body fit beside the SGEMM's.
constexpr long long kTmaMaxBytes = 0;
// Bound of every mbarrier wait (try_wait polls); a wait that runs out records a
// fault in the counters instead of spinning on.
constexpr int kSpinLimit = 1 << 20;

// ------------------------------------------------------------- helpers ----

// Release/acquire fence at device scope: orders this thread's earlier global
// writes (and atomics) before its later ones as seen by other CTAs; used around
// the arrival counters of the last-CTA-finalises pattern.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;\n" ::: "memory"); }

// Hint: bring the 128-byte line holding p into L2 (no register result, no fault).
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p)); }

// --- mbarrier + bulk tensor copy (TMA) primitives, shared::cta addresses ---
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete (at most
// `limit` polls).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int limit = kSpinLimit) {
    for (int i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// One 2-D box of the tensor map (x = column, y = row) into shared memory,
// completing on bar. No multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];\n" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Window w >= 0 with |d_reference - d| <= w for a sum S of n float terms with
// float |x|-sum T and smallest (|x| bits - 1) mbm1; w == 0 means S (and so d)
// is exactly the reference's value.
__device__ __forceinline__ double cert_window(double S, float T, uint32_t mbm1, int n, double d) {
    if (!isfinite(S)) return 0.0;  // NaN/Inf data: every order gives the same class
    const uint32_t nz = mbm1 + 1u;
    if (nz == 0u) return 0.0;  // all terms are +-0
    if (n > (1 << 21)) return INFINITY;
    int e = (int)(nz >> 23);
    if (e < 1) e = 1;
    const double tb = (double)T * (1.0 + 4.0 * (double)n * 0x1p-24);  // upper bound of sum |x|
    // 2^(p+53) with p = e - 150, built from its bits (e - 97 >= -96: always a normal double)
    const double limit = __longlong_as_double((long long)(e - 97 + 1023) << 52);
    if (tb <= limit) return 0.0;
    const double E = 2.0 * (double)n * 0x1p-53 * tb * (1.0 + 0x1p-30);
    const double w = E * (1.0 + 0x1p-40) + d * 0x1p-51 + 0x1p-1000;
    return (w > 0.0) ? w : INFINITY;
}

__device__ __forceinline__ void acc1(float x, double& s, float& t, uint32_t& m) {
    s = __dadd_rn(s, (double)x);
    t += fabsf(x);
    m = min(m, (__float_as_uint(x) & 0x7fffffffu) - 1u);
}

// 2^k for -1022 <= k <= 1023, built from its bits.
__device__ __forceinline__ double pow2i(int k) { return __longlong_as_double((long long)(k + 1023) << 52); }

// Exponent q of the lowest set bit of a finite nonzero double (s = odd * 2^q).
__device__ __forceinline__ int dbl_lowbit_exp(double s) {
    const unsigned long long b = (unsigned long long)__double_as_longlong(s);
    const int e = (int)((b >> 52) & 0x7ff);
    unsigned long long m = b & ((1ull << 52) - 1);
    if (e == 0) return -1074 + (__ffsll((long long)m) - 1);
    m |= 1ull << 52;
    return (e - 1075) + (__ffsll((long long)m) - 1);
}

// Adds a run of terms to the sequential sum s when the result is known
// without running the sequence: S = their sum (any order), T = their
// |x|-sum, amax = largest |x| bits, mbm1 = smallest (|x| bits - 1) (zeros
// excluded). Two cases are decided exactly:
//  * no rounding: s and every term are multiples of 2^p and |s| + T <= 2^(p+53),
//    so every sequential partial sum is representable, and so are S and s + S;
//  * absorption: every |x| < ulp(s) / 4, so each sequential add rounds back to s.
// Returns false (s unchanged) when neither applies or a term is Inf / NaN.
__device__ __forceinline__ bool run_shortcut(double& s, double S, double T, uint32_t amax, uint32_t mbm1) {
    if (amax >= 0x7f800000u || !isfinite(s)) return false;
    constexpr int kNone = 1 << 30;
    int p = (mbm1 == kFull) ? kNone : max((int)((mbm1 + 1u) >> 23), 1) - 150;
    if (s != 0.0) p = min(p, dbl_lowbit_exp(s));
    if (p == kNone) return true;  // s == +0 and every term is +-0: s stays +0
    if (p + 53 <= 1023 && (fabs(s) + T) * (1.0 + 0x1p-40) <= pow2i(p + 53)) {
        s = s + S;
        return true;
    }
    if (s != 0.0) {
        const int es = (int)(((unsigned long long)__double_as_longlong(s) >> 52) & 0x7ff);
        if (es >= 55 && (double)__uint_as_float(amax) < pow2i(es - 1077)) return true;
    }
    return false;
}

// s += lane 0's value, then lane 1's, ... lane m-1's, one rounding each
// (m is warp-uniform).
__device__ __forceinline__ void seq_run(double& s, float v, int m) {
    if (m >= 32) {
#pragma unroll
        for (int r = 0; r < 32; ++r) s = __dadd_rn(s, (double)__shfl_sync(kFull, v, r));
    } else {
        for (int r = 0; r < m; ++r) s = __dadd_rn(s, (double)__shfl_sync(kFull, v, r));
    }
}

// Warp-wide statistics of one value per lane, folded into a block's.
__device__ __forceinline__ void warp_stats(double& S, double& T, uint32_t& amax, uint32_t& mbm1) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        S += __shfl_xor_sync(kFull, S, o);
        T += __shfl_xor_sync(kFull, T, o);
    }
    amax = __reduce_max_sync(kFull, amax);
    mbm1 = __reduce_min_sync(kFull, mbm1);
}

// Sequential double sum x[0] + x[stride] + ... (n terms) in ascending order,
// starting from 0.0: the reference's per-thread loop, bit for bit.
// Warp-cooperative: lane l holds terms l, l + 32, ... of a 128-term block
// (loaded through L2, one block ahead: the verify kernel may have written one
// of them in graph mode). A block, else each of its 32-term runs, is added in
// one step when run_shortcut proves the sequential result; only the remaining
// runs execute their 32 dependent adds (all runs, once two consecutive blocks
// offered no shortcut, so that hard columns cost no more than the plain chain).
__device__ __forceinline__ double exact_chain(const float* __restrict__ x, long long stride, int n) {
    constexpr int U = 4;
    const int lane = threadIdx.x & 31;
    double s = 0.0;
    int hard = 0;  // consecutive blocks in which no run could be shortcut
    int b0 = 0;
    {
        float v[U], vn[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = u * 32 + lane;
            v[u] = (i < n) ? __ldcg(x + (long long)i * stride) : 0.f;
        }
        for (; b0 < n && hard < 2; b0 += 32 * U) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = b0 + 32 * U + u * 32 + lane;
                vn[u] = (i < n) ? __ldcg(x + (long long)i * stride) : 0.f;
            }
            double S = 0.0, T = 0.0;
            uint32_t amax = 0u, mbm1 = kFull;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t a = __float_as_uint(v[u]) & 0x7fffffffu;
                S += (double)v[u];
                T += (double)__uint_as_float(a);
                amax = max(amax, a);
                mbm1 = min(mbm1, a - 1u);
            }
            warp_stats(S, T, amax, mbm1);
            if (run_shortcut(s, S, T, amax, mbm1)) {
                hard = 0;
            } else {
                bool any = false;
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int c0 = b0 + u * 32;
                    if (c0 >= n) break;
                    const uint32_t a = __float_as_uint(v[u]) & 0x7fffffffu;
                    double Sc = (double)v[u], Tc = (double)__uint_as_float(a);
                    uint32_t ac = a, mc = a - 1u;
                    warp_stats(Sc, Tc, ac, mc);
                    if (run_shortcut(s, Sc, Tc, ac, mc)) {
                        any = true;
                        continue;
                    }
                    seq_run(s, v[u], min(32, n - c0));
                }
                hard = any ? 0 : hard + 1;
            }
#pragma unroll
            for (int u = 0; u < U; ++u) v[u] = vn[u];
        }
    }
    // Two blocks in a row offered no shortcut: the column is hard and the
    // statistics would only add cost. The rest runs as the plain chain, 32
    // terms prefetched ahead.
    if (b0 < n) {
        float v = (b0 + lane < n) ? __ldcg(x + (long long)(b0 + lane) * stride) : 0.f;
        for (int i0 = b0; i0 < n; i0 += 32) {
            const int nx = i0 + 32 + lane;
            const float vn = (nx < n) ? __ldcg(x + (long long)nx * stride) : 0.f;
            seq_run(s, v, min(32, n - i0));
            v = vn;
        }
    }
    return s;
}

struct SelectSmem {
    double d[kThreads];
    int j[kThreads];
    int list[kListCap];
    int cnt;
    int flag;
};

// The order in which the reference's arg-max (k_detect_row / k_locate_correct,
// kernels/abft_stepwise.cuh:85-110, :174-187) picks among entries above tau:
// a strided scan keeps, per slot j % 256, the first strictly larger entry, and
// a tree then lets the right operand (slot t + s against slot t) win only when
// strictly larger. Among equal values the winner is the entry whose slot has
// the smallest bit-reversed index (the tree's last level puts even slots before
// odd ones, the one before it slots 0 mod 4 before 2 mod 4, ...), and within a
// slot the smallest j. better() is that order as a comparison, so a reduction
// in any order and grouping returns the reference's winner; j < 0 is "none".
__device__ __forceinline__ bool sel_better(double da, int ja, double db, int jb) {
    if (ja < 0) return false;
    if (jb < 0) return true;
    if (da != db) return da > db;
    const unsigned ka = __brev((unsigned)ja & (kThreads - 1u)), kb = __brev((unsigned)jb & (kThreads - 1u));
    if (ka != kb) return ka < kb;
    return ja < jb;
}

// Loads of the arg-max inputs: CG = written by other CTAs of this grid (read
// through L2), otherwise written by this CTA (shared or global memory).
template <bool CG>
__device__ __forceinline__ double ld_sel(const double* p) {
    if (CG) return __ldcg(p);
    return *p;
}

// Arg-max of k_detect_row / k_locate_correct (kernels/abft_stepwise.cuh:85-110,
// :174-187) over n entries, run by one 256-thread CTA. act/dd/ww hold the fast
// sum, its |act - exp| and window; entries that could change the outcome are
// first re-summed exactly by `exact(j)` (warp-cooperative). Entries with
// live(j) false are known to be at most tau and are not read. Returns the
// reference's winner or -1.
template <bool CG, class Exact, class Live>
__device__ int final_select(int n, double tau, const double* __restrict__ expv, double* act, double* dd, double* ww,
                            Exact exact, Live live, SelectSmem& sm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // Pass 1: largest certified candidate; is there any candidate at all, any uncertified one?
    double bc = -INFINITY;
    int anyc = 0, anyu = 0;
#pragma unroll 4
    for (int j = tid; j < n; j += kThreads) {
        if (!live(j)) continue;
        const double wv = ld_sel<CG>(ww + j), dv = ld_sel<CG>(dd + j);
        if (wv == 0.0 && dv > tau && dv > bc) bc = dv;
        if (dv + wv > tau) {
            anyc = 1;
            if (wv != 0.0) anyu = 1;
        }
    }
    if (!__syncthreads_or(anyc)) return -1;  // every |actual - expected| <= tau
    anyu = __syncthreads_or(anyu);

    if (anyu) {
        // the maximum is order independent: warp shuffles, then across warps
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bc = fmax(bc, __shfl_xor_sync(kFull, bc, o));
        if (lane == 0) sm.d[warp] = bc;
        __syncthreads();
        double best_cert = sm.d[0];
        for (int k = 1; k < kWarps; ++k) best_cert = fmax(best_cert, sm.d[k]);
        __syncthreads();
        for (;;) {
            if (tid == 0) sm.cnt = 0;
            __syncthreads();
#pragma unroll 4
            for (int j = tid; j < n; j += kThreads) {
                if (!live(j)) continue;
                const double wv = ld_sel<CG>(ww + j);
                if (wv != 0.0) {
                    const double hi = ld_sel<CG>(dd + j) + wv;
                    if (hi > tau && hi >= best_cert) {
                        const int k = atomicAdd(&sm.cnt, 1);
                        if (k < kListCap) sm.list[k] = j;
                    }
                }
            }
            __syncthreads();
            const int cnt = sm.cnt;
            const int todo = min(cnt, kListCap);
            for (int k = warp; k < todo; k += kWarps) {
                const int j = sm.list[k];
                const double S = exact(j);
                if (lane == 0) {
                    act[j] = S;
                    dd[j] = fabs(S - expv[j]);
                    ww[j] = 0.0;
                }
            }
            __syncthreads();
            if (cnt <= kListCap) break;
        }
    }

    // Pass 3: the reference's 256-slot strided scan and shared-memory tree
    // (strictly larger right operand wins); the last five tree levels run as
    // warp shuffles inside warp 0, pairing the same slots.
    double best = 0.0;
    int bj = -1;
#pragma unroll 4
    for (int j = tid; j < n; j += kThreads) {
        if (live(j) && ld_sel<CG>(ww + j) == 0.0) {
            const double dv = ld_sel<CG>(dd + j);
            if (dv > tau && dv > best) {
                best = dv;
                bj = j;
            }
        }
    }
    sm.d[tid] = best;
    sm.j[tid] = bj;
    __syncthreads();
    for (int s = kThreads / 2; s >= 32; s >>= 1) {
        if (tid < s && sm.d[tid + s] > sm.d[tid]) {
            sm.d[tid] = sm.d[tid + s];
            sm.j[tid] = sm.j[tid + s];
        }
        __syncthreads();
    }
    if (warp == 0) {
        double v = sm.d[lane];
        int vj = sm.j[lane];
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) {
            const double ov = __shfl_down_sync(kFull, v, s);
            const int oj = __shfl_down_sync(kFull, vj, s);
            if (lane < s && ov > v) {
                v = ov;
                vj = oj;
            }
        }
        if (lane == 0) sm.j[0] = vj;
    }
    __syncthreads();
    const int w = sm.j[0];
    __syncthreads();
    return w;
}

// ------------------------------------------------------------- verify -----

// Second half of the verify kernels. Every CTA of column group g = blockIdx.x
// folds its per-column partials (S, |x|-sum, smallest |x| bits - 1 of columns
// c0..c0+3 in each thread) into the group's accumulators (skipped with fold =
// false: a CTA whose copies did not all land adds nothing, and its launch is
// void). The last of the group's gridDim.y CTAs certifies the group's 128
// columns (in parallel with the other groups' streaming) and votes whether any
// may exceed tau; the last group to finish runs the reference's arg-max only
// when some group voted yes (or, calibrating, each group writes its own
// columns' exact differences). Shared memory touched: dsm (kWarps * kGroupCols
// * 16 bytes, for the fold only) and sel.
__device__ __forceinline__ void verify_tail(unsigned char* dsm, SelectSmem& sel, bool fold, double s0, double s1,
                                            double s2, double s3, float t0, float t1, float t2, float t3,
                                            uint32_t m0, uint32_t m1, uint32_t m2, uint32_t m3,
                                            const float* __restrict__ C, long long ldc, int M, int N,
                                            const double* __restrict__ expv, double tau, int injected, int f, int F,
                                            int it, const WsDev& w, double* calib_out,
                                            cudaGraphConditionalHandle cond) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = blockIdx.x;
    const int col = g * kGroupCols + tid;  // the column this thread finishes (tid < kGroupCols)
    if (fold) {
        double(*s_s)[kGroupCols] = reinterpret_cast<double(*)[kGroupCols]>(dsm);
        float(*s_t)[kGroupCols] = reinterpret_cast<float(*)[kGroupCols]>(dsm + kWarps * kGroupCols * 8);
        uint32_t(*s_m)[kGroupCols] = reinterpret_cast<uint32_t(*)[kGroupCols]>(dsm + kWarps * kGroupCols * 12);
        const int cl = lane * 4;
        s_s[warp][cl + 0] = s0; s_s[warp][cl + 1] = s1; s_s[warp][cl + 2] = s2; s_s[warp][cl + 3] = s3;
        s_t[warp][cl + 0] = t0; s_t[warp][cl + 1] = t1; s_t[warp][cl + 2] = t2; s_t[warp][cl + 3] = t3;
        s_m[warp][cl + 0] = m0; s_m[warp][cl + 1] = m1; s_m[warp][cl + 2] = m2; s_m[warp][cl + 3] = m3;
        __syncthreads();
        if (tid < kGroupCols && col < N) {
            double S = 0.0;
            float T = 0.f;
            uint32_t mb = kFull;
#pragma unroll
            for (int k = 0; k < kWarps; ++k) {
                S = __dadd_rn(S, s_s[k][tid]);
                T += s_t[k][tid];
                mb = min(mb, s_m[k][tid]);
            }
            atomicAdd(w.vacc_s + col, S);
            atomicAdd(w.vacc_t + col, T);
            atomicMin(w.vacc_m + col, mb);
        }
    }
    fence_acq_rel_gpu();
    __syncthreads();
    if (tid == 0) sel.flag = (atomicAdd(w.vcnt + kArriveGroup + g, 1) == (int)gridDim.y - 1);
    __syncthreads();
    if (!sel.flag) return;
    fence_acq_rel_gpu();

    // Last CTA of the group: certify its columns, reset their accumulators.
    double S = 0.0, d = 0.0, wv = 0.0;
    int cand = 0;
    if (tid < kGroupCols && col < N) {
        S = __ldcg(w.vacc_s + col);
        const float T = __ldcg(w.vacc_t + col);
        const uint32_t mb = __ldcg(w.vacc_m + col);
        const double E = expv[col];
        w.vacc_s[col] = 0.0;
        w.vacc_t[col] = 0.f;
        w.vacc_m[col] = kFull;
        d = fabs(S - E);
        wv = cert_window(S, T, mb, M, d);
        w.vact[col] = S;
        w.vd[col] = d;
        w.vw[col] = wv;
        cand = (d + wv > tau) ? 1 : 0;
    }
    if (calib_out != nullptr) {
        // Calibration (pass_calibrate, pipeline/passes.cuh:66-84): every
        // |actualRow - expectedRow| exactly, the group's uncertified columns
        // re-summed in the reference's order (one warp per column); no
        // detection, no counters.
        if (tid < kGroupCols) sel.d[tid] = (col < N) ? wv : 0.0;
        __syncthreads();
        for (int c = warp; c < kGroupCols; c += kWarps) {
            const int j = g * kGroupCols + c;
            if (j < N && sel.d[c] != 0.0) {
                const double Sx = exact_chain(C + j, ldc, M);
                if (lane == 0) calib_out[j] = fabs(Sx - expv[j]);
            }
        }
        if (tid < kGroupCols && col < N && wv == 0.0) calib_out[col] = d;
        cand = 0;
    }
    // With at most 32 groups the final word's high half is a mask of the
    // groups that voted yes, and only those are read by the decision: a group
    // that votes no needs no fence before its arrival (the common case). With
    // more groups it holds a count, and every group fences.
    const bool mask_mode = gridDim.x <= 32u;
    cand = __syncthreads_or(cand);
    if (cand || !mask_mode) {
        fence_acq_rel_gpu();  // this group's act / d / w before its arrival
        __syncthreads();
    }
    if (tid == 0) {
        // every CTA of the group has arrived: its counters go back to zero
        w.vcnt[kArriveGroup + g] = 0;
        w.vcnt[kArriveGroup + gridDim.x + g] = 0;
        unsigned long long vote = 0ull;
        if (cand) vote = mask_mode ? (1ull << (32 + g)) : (1ull << 32);
        // one atomic both counts this group and carries its vote
        unsigned long long* fin = reinterpret_cast<unsigned long long*>(w.vcnt);
        const unsigned long long old = atomicAdd(fin, 1ull + vote);
        sel.flag = ((unsigned)old == gridDim.x - 1u);
        sel.cnt = (int)((old + vote) >> 32);  // vote mask (or count), this group included
    }
    __syncthreads();
    if (!sel.flag) return;
    fence_acq_rel_gpu();

    // Last group: the fragment's decision.
    const unsigned votes = (unsigned)sel.cnt;
    __syncthreads();
    if (calib_out != nullptr) {
        if (tid == 0) *reinterpret_cast<unsigned long long*>(w.vcnt) = 0ull;
        return;
    }
    // The reference's detection (k_detect_row) on exact values; a fragment in
    // which no column can exceed tau has no winner.
    int ec = -1;
    if (votes != 0u)
        ec = final_select<true>(
            N, tau, expv, w.vact, w.vd, w.vw, [&](int j) { return exact_chain(C + j, ldc, M); },
            [&](int j) { return !mask_mode || ((votes >> (j / kGroupCols)) & 1u) != 0u; }, sel);
    if (tid == 0) {
        const double rd = (ec >= 0) ? (__ldcg(w.vact + ec) - expv[ec]) : 0.0;
        w.rec[f].errcol = ec;
        w.rec[f].errrow = -1;
        w.rec[f].rowdiff = rd;
        const int det = ec >= 0;
        const int idx = injected ? (det ? 0 : 3) : (det ? 2 : 1);
        atomicAdd(&w.ctr->cm[idx], 1);
        // graph mode: the localisation node of this fragment runs only if a
        // column was detected
        if (cond != 0) cudaGraphSetConditional(cond, det ? 1u : 0u);
        if (it >= 0) {
            DecisionLog& L = w.dlog[(long long)it * F + f];
            L.errcol = ec;
            L.errrow = -1;
            L.rowdiff = rd;
        }
        *reinterpret_cast<unsigned long long*>(w.vcnt) = 0ull;
    }
}


// Fused actualRow + detect for one fragment (M x N, leading dimension ldc).
// grid = (groups of 128 columns, CTAs per group). A column group's rows are
// cut into n_large units of unit_rows rows (a multiple of kBatch * kWarps),
// then units of kBatch * kWarps rows up to M: CTA y of
// the group takes unit y first, then one thread fetches the index of the CTA's
// next unit from the group's counter while the current unit streams, so CTAs
// that get less bandwidth take fewer units and the group's CTAs finish within
// about one unit of each other (a CTA-level grab keeps the counter at a few
// atomics per microsecond). Each thread streams 4 columns with 128-bit loads
// and keeps per-column (sum, |x|-sum, smallest |x|); the CTA adds those into
// per-column accumulators with device atomics (any order: certified sums are
// exact in every order, uncertified ones carry a window valid for every
// order); the tail finishes the columns and the decision. Shared memory:
// 16 KB for the CTA's fold.
template <bool VEC>
__global__ void __launch_bounds__(kThreads, 4)
    k_verify(const float* __restrict__ C, long long ldc, int M, int N, int unit_rows, int n_large,
             const double* __restrict__ expv,
             double tau, int injected, int f, int F, int it, WsDev w, float* Cw, const InjectPlan* __restrict__ plan,
             int plan_it, float add_delta, int log_inj, double* calib_out, cudaGraphConditionalHandle cond) {
    extern __shared__ __align__(16) unsigned char dsm[];
    __shared__ SelectSmem sel;
    __shared__ int s_next[2];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = blockIdx.x;
    const int c0 = g * kGroupCols + lane * 4;
    // units 0 .. n_large - 1 hold unit_rows rows each from row 0, the rest
    // one batch per warp (kBatch * kWarps rows) each
    constexpr int kSmall = kBatch * kWarps;
    const int tail0 = n_large * unit_rows;
    const int nunits = (tail0 >= M) ? (M + unit_rows - 1) / unit_rows : n_large + (M - tail0 + kSmall - 1) / kSmall;
    int* const next_unit = w.vcnt + kArriveGroup + gridDim.x + g;

    // The expected checksums of this group's columns (1 KB) are read only by
    // the group's last CTA; the group's first CTA pulls them into L2 meanwhile.
    if (blockIdx.y == 0 && tid < kGroupCols / 16 && g * kGroupCols + tid * 16 < N)
        prefetch_l2(expv + g * kGroupCols + tid * 16);

    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
    uint32_t m0 = kFull, m1 = kFull, m2 = kFull, m3 = kFull;

    // Graph mode: this iteration's planned fault is applied here, by the
    // thread whose loads cover the element: warp (row mod kWarps) of whichever
    // CTA takes the row's unit (nothing reads C between the SGEMM and this
    // kernel, so the result equals injecting on the compute stream).
    int inj_row = -1, inj_k = 0, inj_bit = -1;
    if (plan != nullptr) {
        const InjectPlan p = plan[plan_it];
        injected = (p.frag == f) ? 1 : 0;
        if (injected && p.row >= 0 && p.row < M && (p.row % kWarps) == warp && p.col >= c0 && p.col < c0 + 4 &&
            p.col < N) {
            inj_row = p.row;
            inj_k = p.col - c0;
            inj_bit = p.bit;
        }
    }

    auto load = [&](int r) -> float4 {
        const float* p = C + (long long)r * ldc + c0;
        if (VEC) {
            if (c0 < N) return __ldg(reinterpret_cast<const float4*>(p));
            return make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            float4 v;
            v.x = (c0 + 0 < N) ? __ldg(p + 0) : 0.f;
            v.y = (c0 + 1 < N) ? __ldg(p + 1) : 0.f;
            v.z = (c0 + 2 < N) ? __ldg(p + 2) : 0.f;
            v.w = (c0 + 3 < N) ? __ldg(p + 3) : 0.f;
            return v;
        }
    };
    auto acc = [&](float4 v) {
        acc1(v.x, s0, t0, m0);
        acc1(v.y, s1, t1, m1);
        acc1(v.z, s2, t2, m2);
        acc1(v.w, s3, t3, m3);
    };

    int u = blockIdx.y;
    int nxt = 0;
    if (tid == 0 && u < nunits) nxt = (int)gridDim.y + atomicAdd(next_unit, 1);
    for (int i = 0; u < nunits; ++i) {
        const int r0 = (u < n_large) ? u * unit_rows : tail0 + (u - n_large) * kSmall;
        const int r1 = min(M, r0 + ((u < n_large) ? unit_rows : kSmall));
        // Batches of kBatch rows per warp (rows warp, warp + kWarps, ...),
        // predicated, so that every load of a batch is in flight at once.
        for (int r = r0 + warp; r < r1; r += kBatch * kWarps) {
            float4 v[kBatch];
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const int rr = r + k * kWarps;
                v[k] = (rr < r1) ? load(rr) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (inj_row >= 0) {
#pragma unroll
                for (int k = 0; k < kBatch; ++k) {
                    if (r + k * kWarps == inj_row) {
                        const float before = inj_k == 0 ? v[k].x : inj_k == 1 ? v[k].y : inj_k == 2 ? v[k].z : v[k].w;
                        const float after = (inj_bit < 0)
                                                ? __fadd_rn(before, add_delta)
                                                : __uint_as_float(__float_as_uint(before) ^ (1u << inj_bit));
                        if (inj_k == 0) v[k].x = after;
                        else if (inj_k == 1) v[k].y = after;
                        else if (inj_k == 2) v[k].z = after;
                        else v[k].w = after;
                        Cw[(long long)inj_row * ldc + c0 + inj_k] = after;
                        if (log_inj) {
                            InjectLog& L = w.ilog[plan_it];
                            L.frag = f;
                            L.row = inj_row;
                            L.col = c0 + inj_k;
                            L.bit = inj_bit;
                            L.before = before;
                            L.after = after;
                        }
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < kBatch; ++k) acc(v[k]);
        }
        // the next unit (fetched during this one) for every thread; slot i & 1
        // is written again only after the next barrier
        if (tid == 0) s_next[i & 1] = nxt;
        __syncthreads();
        u = s_next[i & 1];
        if (tid == 0 && u < nunits) nxt = (int)gridDim.y + atomicAdd(next_unit, 1);
    }

    verify_tail(dsm, sel, true, s0, s1, s2, s3, t0, t1, t2, t3, m0, m1, m2, m3, C, ldc, M, N, expv, tau, injected, f,
                F, it, w, calib_out, cond);
}

// The same fused verify with the tile staged by the Tensor Memory Accelerator:
// one thread keeps up to kTmaStages 32 x 128 boxes of this CTA's column strip
// in flight (cp.async.bulk.tensor, completion on an mbarrier per stage) while
// the eight warps accumulate from shared memory, so the HBM stream never waits
// for the FP64 add chains. Boxes past row M or column N are zero-filled by the
// copy engine; zeros leave S, the |x|-sum and the smallest nonzero |x| as they
// are. rows_per is a multiple of kTmaRows, so no box crosses into the next
// chunk. Requires a 16-byte aligned fragment and ldc % 4 == 0 (tensor map).
__global__ void __launch_bounds__(kThreads, 2)
    k_verify_tma(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ C, long long ldc, int M, int N,
                 int rows_per, const double* __restrict__ expv, double tau, int injected, int f, int F, int it,
                 WsDev w, float* Cw, const InjectPlan* __restrict__ plan, int plan_it, float add_delta, int log_inj,
                 double* calib_out, cudaGraphConditionalHandle cond, int wait_limit) {
    // The dynamic shared memory is launched kTmaAlign bytes larger than the
    // ring and the ring starts at the first kTmaAlign boundary in it: where
    // the dynamic area begins depends on the static shared memory before it
    // and on how the kernel was compiled, and the copies need the alignment.
    extern __shared__ __align__(16) unsigned char ring_raw[];
    __shared__ SelectSmem sel;
    __shared__ __align__(8) uint64_t full[kTmaStages];
    unsigned char* const ring = ring_raw + ((kTmaAlign - (smem_addr(ring_raw) & (kTmaAlign - 1))) & (kTmaAlign - 1));

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = blockIdx.x, chunk = blockIdx.y;
    const int gc0 = g * kGroupCols;
    const int c0 = gc0 + lane * 4;
    const int r0 = chunk * rows_per;
    const int r1 = min(M, r0 + rows_per);
    // (cannot fail: keeps a misplaced ring from ever reaching a copy)
    const bool ring_ok = (smem_addr(ring) & (kTmaAlign - 1)) == 0;
    const int nst = ring_ok ? (r1 - r0 + kTmaRows - 1) / kTmaRows : 0;
    if (!ring_ok && tid == 0) atomicOr(&w.ctr->fault, 1);

    if (tid == 0) {
#pragma unroll
        for (int k = 0; k < kTmaStages; ++k) mbar_init(&full[k], 1);
        mbar_init_fence();
    }
    __syncthreads();
    if (tid == 0) {
        const int first = min(nst, kTmaStages);
        for (int k = 0; k < first; ++k) {
            mbar_expect_tx(&full[k], kStageBytes);
            tma_load_2d(ring + k * kStageBytes, &tmap, &full[k], gc0, r0 + k * kTmaRows);
        }
    }
    if (chunk == 0 && tid < kGroupCols / 16 && gc0 + tid * 16 < N) prefetch_l2(expv + gc0 + tid * 16);

    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
    uint32_t m0 = kFull, m1 = kFull, m2 = kFull, m3 = kFull;

    // Graph mode: the planned fault is applied by the thread that reads the
    // element (as in k_verify): it changes its register copy and writes C.
    int inj_row = -1, inj_k = 0, inj_bit = -1;
    if (plan != nullptr) {
        const InjectPlan p = plan[plan_it];
        injected = (p.frag == f) ? 1 : 0;
        if (injected && p.row >= r0 && p.row < r1 && ((p.row - r0) % kWarps) == warp && p.col >= c0 &&
            p.col < c0 + 4 && p.col < N) {
            inj_row = p.row;
            inj_k = p.col - c0;
            inj_bit = p.bit;
        }
    }

    int fault = 0, k = 0;
    for (; k < nst; ++k) {
        const int st = k % kTmaStages;
        const bool got = mbar_wait(&full[st], (uint32_t)(k / kTmaStages) & 1u, wait_limit);
        if (got) {
            const float* tile = reinterpret_cast<const float*>(ring + st * kStageBytes);
            const int rb = r0 + k * kTmaRows;
#pragma unroll
            for (int u = 0; u < kTmaRows / kWarps; ++u) {
                const int rs = warp + u * kWarps;
                const int row = rb + rs;
                float4 v = *reinterpret_cast<const float4*>(tile + rs * kGroupCols + lane * 4);
                if (row < r1) {
                    if (row == inj_row) {
                        const float before = inj_k == 0 ? v.x : inj_k == 1 ? v.y : inj_k == 2 ? v.z : v.w;
                        const float after = (inj_bit < 0) ? __fadd_rn(before, add_delta)
                                                          : __uint_as_float(__float_as_uint(before) ^ (1u << inj_bit));
                        if (inj_k == 0) v.x = after;
                        else if (inj_k == 1) v.y = after;
                        else if (inj_k == 2) v.z = after;
                        else v.w = after;
                        Cw[(long long)inj_row * ldc + c0 + inj_k] = after;
                        if (log_inj) {
                            InjectLog& L = w.ilog[plan_it];
                            L.frag = f;
                            L.row = inj_row;
                            L.col = c0 + inj_k;
                            L.bit = inj_bit;
                            L.before = before;
                            L.after = after;
                        }
                    }
                    acc1(v.x, s0, t0, m0);
                    acc1(v.y, s1, t1, m1);
                    acc1(v.z, s2, t2, m2);
                    acc1(v.w, s3, t3, m3);
                }
            }
        }
        // every warp is done with stage st (or a wait ran out): refill it
        if (__syncthreads_or(!got)) {
            fault = 1;
            break;
        }
        if (tid == 0 && k + kTmaStages < nst) {
            mbar_expect_tx(&full[st], kStageBytes);
            tma_load_2d(ring + st * kStageBytes, &tmap, &full[st], gc0, r0 + (k + kTmaStages) * kTmaRows);
        }
    }
    if (fault) {
        // A copy did not land in time: record it, give the copies still in
        // flight a bounded chance to land, then finish the arrival protocol
        // (the counters carry the fault; the decisions of this launch are void).
        if (tid == 0) {
            atomicExch(&w.ctr->fault, 1);
            for (int j = k; j < min(nst, k + kTmaStages); ++j)
                (void)mbar_wait(&full[j % kTmaStages], (uint32_t)(j / kTmaStages) & 1u);
        }
        __syncthreads();
    }

    // After a fault the ring may still receive a late copy: the tail then
    // leaves shared memory other than `sel` alone and adds nothing.
    verify_tail(ring, sel, !fault, s0, s1, s2, s3, t0, t1, t2, t3, m0, m1, m2, m3, C, ldc, M, N, expv, tau, injected,
                f, F, it, w, calib_out, cond);
}

// ----------------------------------------------------------- localise -----

// Statistics of ROWS rows of X (rows rb, rb + kWarps, ...; those at or past
// r1 give zeros) over columns [0, N), one warp: per row the double sum S,
// the float |x|-sum and the smallest (|x| bits - 1), reduced across the warp so
// that every lane holds them. ROWS rows side by side overlap their loads and
// add chains (narrow rows); a single row keeps 8 loads of 16 bytes per lane in
// flight along the row (wide rows; 4 measured 2-3 % slower on B200).
template <bool VEC, int ROWS>
__device__ __forceinline__ void row_stats(const float* __restrict__ X, long long ld, int N, int rb, int r1,
                                          double (&s)[ROWS], float (&t)[ROWS], uint32_t (&m)[ROWS]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
        s[u] = 0.0;
        t[u] = 0.f;
        m[u] = kFull;
    }
    if (VEC) {
#pragma unroll(ROWS == 1 ? 8 : 2)
        for (int c = lane * 4; c < N; c += 128) {
            float4 v[ROWS];
#pragma unroll
            for (int u = 0; u < ROWS; ++u) {
                const int r = rb + u * kWarps;
                v[u] = (r < r1) ? __ldg(reinterpret_cast<const float4*>(X + (long long)r * ld + c))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < ROWS; ++u) {
                acc1(v[u].x, s[u], t[u], m[u]);
                acc1(v[u].y, s[u], t[u], m[u]);
                acc1(v[u].z, s[u], t[u], m[u]);
                acc1(v[u].w, s[u], t[u], m[u]);
            }
        }
    } else {
#pragma unroll(ROWS == 1 ? 4 : 2)
        for (int c = lane; c < N; c += 32) {
            float v[ROWS];
#pragma unroll
            for (int u = 0; u < ROWS; ++u) {
                const int r = rb + u * kWarps;
                v[u] = (r < r1) ? __ldg(X + (long long)r * ld + c) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < ROWS; ++u) acc1(v[u], s[u], t[u], m[u]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int u = 0; u < ROWS; ++u) {
            s[u] = __dadd_rn(s[u], __shfl_xor_sync(kFull, s[u], o));
            t[u] += __shfl_xor_sync(kFull, t[u], o);
            m[u] = min(m[u], __shfl_xor_sync(kFull, m[u], o));
        }
    }
}

// |sum of a row in the reference's order - E|, for the rare uncertified
// candidate row: kept out of line so that the streaming loop of the
// localisation keeps its registers.
__device__ __noinline__ double exact_row_diff(const float* __restrict__ row, int n, double E) {
    return fabs(exact_chain(row, 1, n) - E);
}

// Gated localisation + correction for one fragment: row sums of the fragment
// (a warp sums ROWS rows side by side), certified like the column sums, then
// the reference's row arg-max (k_locate_correct) and the correction C =
// float(double(C) - rowdiff). The arg-max is split across the grid: a row
// whose fast sum could exceed tau but is not certified is re-summed in the
// reference's order by the warp that summed it (its data is still in cache),
// so every candidate value is exact; each CTA keeps its best row under the
// reference's order (sel_better) and the last CTA reduces the per-CTA bests
// (one entry per row block instead of one per row).
template <bool VEC, int ROWS>
__global__ void __launch_bounds__(kThreads)
    k_localize(float* C, long long ldc, int M, int N, int rows_per, int nblocks, const double* __restrict__ expc,
               double tau, int injected, const float* __restrict__ G, long long ldg, int frag_off, int f, int F,
               int it, int drain, int pend_cap, WsDev w, const InjectPlan* __restrict__ plan, int plan_it) {
    __shared__ double s_bd[kThreads];
    __shared__ int s_bj[kThreads];
    __shared__ int s_last;
    const int ec = __ldcg(&w.rec[f].errcol);
    if (ec < 0) return;
    if (plan != nullptr) injected = (plan[plan_it].frag == f) ? 1 : 0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r0 = blockIdx.x * rows_per;
    const int r1 = min(M, r0 + rows_per);
    // this warp's best row so far, in shared memory (written by lane 0, read
    // by the whole warp; rows above tau are rare)
    if (lane == 0) {
        s_bd[warp] = 0.0;
        s_bj[warp] = -1;
    }
    __syncwarp();
    // ROWS rows per warp at a time, independent accumulators: their loads and
    // add chains overlap instead of paying one latency per row (narrow rows);
    // a single row keeps 8 loads per lane in flight along the row instead.
    for (int rb = r0 + warp; rb < r1; rb += ROWS * kWarps) {
        // the expected sums first: their loads overlap the row's
        double E[ROWS];
#pragma unroll
        for (int u = 0; u < ROWS; ++u) E[u] = (rb + u * kWarps < r1) ? expc[rb + u * kWarps] : 0.0;
        double s[ROWS];
        float t[ROWS];
        uint32_t m[ROWS];
        row_stats<VEC, ROWS>(C, ldc, N, rb, r1, s, t, m);
#pragma unroll
        for (int u = 0; u < ROWS; ++u) {
            const int r = rb + u * kWarps;
            if (r < r1) {  // every lane holds the same statistics: warp-uniform branches
                double d = fabs(s[u] - E[u]);
                const double wv = cert_window(s[u], t[u], m[u], N, d);
                if (wv != 0.0 && d + wv > tau) d = exact_row_diff(C + (long long)r * ldc, N, E[u]);
                // the reference's scan takes entries above tau and above its
                // initial 0
                if (d > tau && d > 0.0 && sel_better(d, r, s_bd[warp], s_bj[warp])) {
                    __syncwarp();
                    if (lane == 0) {
                        s_bd[warp] = d;
                        s_bj[warp] = r;
                    }
                    __syncwarp();
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        double bd = s_bd[0];
        int bj = s_bj[0];
        for (int k = 1; k < kWarps; ++k)
            if (sel_better(s_bd[k], s_bj[k], bd, bj)) {
                bd = s_bd[k];
                bj = s_bj[k];
            }
        w.lbd[blockIdx.x] = bd;
        w.lbr[blockIdx.x] = bj;
        fence_acq_rel_gpu();  // this block's best before its arrival
        s_last = (atomicAdd(w.lcnt, 1) == nblocks - 1);
    }
    __syncthreads();
    if (!s_last) return;
    fence_acq_rel_gpu();

    // Last CTA: the best of the per-block bests.
    double bd = 0.0;
    int bj = -1;
    for (int b = tid; b < nblocks; b += kThreads) {
        const int j = __ldcg(w.lbr + b);
        if (j >= 0) {
            const double d = __ldcg(w.lbd + b);
            if (sel_better(d, j, bd, bj)) {
                bd = d;
                bj = j;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const double od = __shfl_xor_sync(kFull, bd, o);
        const int oj = __shfl_xor_sync(kFull, bj, o);
        if (sel_better(od, oj, bd, bj)) {
            bd = od;
            bj = oj;
        }
    }
    if (lane == 0) {
        s_bd[warp] = bd;
        s_bj[warp] = bj;
    }
    __syncthreads();
    if (tid == 0) {
        int er = -1;
        double be = 0.0;
        for (int k = 0; k < kWarps; ++k)
            if (sel_better(s_bd[k], s_bj[k], be, er)) {
                be = s_bd[k];
                er = s_bj[k];
            }
        *w.lcnt = 0;
        const double rd = __ldcg(&w.rec[f].rowdiff);
        if (er >= 0) {
            float* p = C + (long long)er * ldc + ec;
            const float cf = __ldcg(p);
            const float c = static_cast<float>(static_cast<double>(cf) - rd);
            if (drain) {
                const int k = atomicAdd(&w.ctr->n_pending, 1);
                if (k < pend_cap) {
                    PendingFix& q = w.pend[k];
                    q.it = it; q.f = f; q.er = er; q.ec = ec; q.injected = injected; q.off = frag_off;
                    q.rowdiff = rd; q.tau = tau; q.c_fault = cf; q.pad = 0.f;
                }
            } else {
                *p = c;
                if (injected && G != nullptr) {
                    const float gv = G[(long long)er * ldg + frag_off + ec];
                    if (fabs(static_cast<double>(c) - static_cast<double>(gv)) <= tau) atomicAdd(&w.ctr->n_restored, 1);
                }
            }
        }
        w.rec[f].errrow = er;
        if (it >= 0) w.dlog[(long long)it * F + f].errrow = er;
    }
}

// Row sums in the reference's order (k_row_checksum_B_g,
// kernels/abft_stepwise.cuh:121-132: out[r] = sum over c < N of X[r, c],
// sequential double adds), bit for bit: a warp sums ROWS rows side by side
// (or one wide row) in any order with the certificate of the verify kernel,
// and a row whose sum is not certified is re-summed in the reference's order
// by the whole warp (exact_chain). Encode-time; no gate.
template <bool VEC, int ROWS>
__global__ void __launch_bounds__(kThreads)
    k_rowsum(const float* __restrict__ X, long long ld, int R, int N, int rows_per, double* __restrict__ out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = blockIdx.x * rows_per;
    const int r1 = min(R, r0 + rows_per);
    for (int rb = r0 + warp; rb < r1; rb += ROWS * kWarps) {
        double s[ROWS];
        float t[ROWS];
        uint32_t m[ROWS];
        row_stats<VEC, ROWS>(X, ld, N, rb, r1, s, t, m);
#pragma unroll
        for (int u = 0; u < ROWS; ++u) {
            const int r = rb + u * kWarps;
            if (r < r1) {  // every lane holds the same statistics: warp-uniform branches
                double S = s[u];
                if (cert_window(S, t[u], m[u], N, fabs(S)) != 0.0) S = exact_chain(X + (long long)r * ld, 1, N);
                if (lane == 0) out[r] = S;
            }
        }
    }
}

// Post-loop drain: one thread per queued fix.
__global__ void k_drain(float* C0, float* C1, long long ldc, const float* G, long long ldg, int repeats, int cap,
                        WsDev w) {
    const int n = min(__ldcg(&w.ctr->n_pending), cap);
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < n; k += gridDim.x * blockDim.x) {
        const PendingFix q = w.pend[k];
        const int off = q.off;
        const float c = static_cast<float>(static_cast<double>(q.c_fault) - q.rowdiff);
        if (q.it >= repeats - 2) {
            float* C = (q.it % 2 == 0) ? C0 : C1;
            C[(long long)q.er * ldc + off + q.ec] = c;
        }
        if (q.injected && G != nullptr) {
            const float gv = G[(long long)q.er * ldg + off + q.ec];
            if (fabs(static_cast<double>(c) - static_cast<double>(gv)) <= q.tau) atomicAdd(&w.ctr->n_restored, 1);
        }
    }
}

// ----------------------------------------------------------- injectors ----

__global__ void k_inject(float* C, long long ldc, int row, int col, int mode, float delta, int bit, InjectLog* log,
                         int frag) {
    float* p = C + (long long)row * ldc + col;
    const float before = *p;
    const float after = (mode == ABFT_INJECT_ADD) ? __fadd_rn(before, delta)
                                                  : __uint_as_float(__float_as_uint(before) ^ (1u << bit));
    *p = after;
    if (log != nullptr) {
        log->frag = frag;
        log->row = row;
        log->col = col;
        log->bit = (mode == ABFT_INJECT_ADD) ? -1 : bit;
        log->before = before;
        log->after = after;
    }
}

// ------------------------------------------------------------- encode -----

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Column chains stage 32-row x 32-column tiles (4 KB) through shared memory:
// 16 stages (64 KB per one-warp CTA) keep a chain fed best, 6 stages (24 KB)
// let up to 9 CTAs share an SM, so that many columns still run as one wave
// (a second wave would double the time of the whole launch).
constexpr int kColStagesDeep = 16;
constexpr int kColStagesShallow = 6;
constexpr int col_smem(int stages) { return stages * 32 * 32 * 4; }

// Column chains in row order, one warp = 32 columns: out[c] = sum over rows r
// of X[r, c] (sequential double adds; replaces k_col_checksum_A,
// abft_stepwise.cuh:9-18) or, WEIGHTED, the fused multiply-add chain of
// wrow[r] * X[r, c] (nvcc contracts the reference's s += a * b; replaces
// k_expected_row, :31-41).
template <bool WEIGHTED, bool VEC, int kColStages>
__global__ void __launch_bounds__(32)
    k_colchain(const float* __restrict__ X, long long ld, int R, int ncols, const double* __restrict__ wrow,
               double* __restrict__ out) {
    extern __shared__ __align__(16) float tile[];
    const int lane = threadIdx.x;
    const int cbase = blockIdx.x * 32;
    const int ncv = min(32, ncols - cbase);
    const int nblk = (R + 31) / 32;
    auto issue = [&](int blk) {
        if (blk < nblk) {
            float* t = tile + (blk % kColStages) * 32 * 32;
            const int rb0 = blk * 32;
            if (VEC) {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int q = lane + 32 * u;
                    const int rr = q >> 3, cc = (q & 7) * 4;
                    const int r = rb0 + rr;
                    const bool ok = (r < R) && (cc < ncv);
                    const float* src = ok ? (X + (long long)r * ld + cbase + cc) : X;
                    cp_async16(t + rr * 32 + cc, src, ok ? 4 * min(4, ncv - cc) : 0);
                }
            } else {
                for (int rr = 0; rr < 32; ++rr) {
                    const int r = rb0 + rr;
                    const bool ok = (r < R) && (lane < ncv);
                    const float* src = ok ? (X + (long long)r * ld + cbase + lane) : X;
                    cp_async4(t + rr * 32 + lane, src, ok ? 4 : 0);
                }
            }
        }
        cp_async_commit();
    };
    for (int b = 0; b < kColStages - 1; ++b) issue(b);
    double s = 0.0;
    for (int blk = 0; blk < nblk; ++blk) {
        cp_async_wait<kColStages - 2>();
        __syncwarp();
        const float* t = tile + (blk % kColStages) * 32 * 32;
        const int rb0 = blk * 32;
        const int nr = min(32, R - rb0);
        double wv = 0.0;
        if (WEIGHTED) wv = (rb0 + lane < R) ? __ldg(wrow + rb0 + lane) : 0.0;
        if (nr == 32) {
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) {
                const double x = (double)t[rr * 32 + lane];
                if (WEIGHTED) s = __fma_rn(__shfl_sync(kFull, wv, rr), x, s);
                else s = __dadd_rn(s, x);
            }
        } else {
            for (int rr = 0; rr < 32; ++rr) {
                const double x = (double)t[rr * 32 + lane];
                const double wr = WEIGHTED ? __shfl_sync(kFull, wv, rr) : 0.0;
                if (rr < nr) s = WEIGHTED ? __fma_rn(wr, x, s) : __dadd_rn(s, x);
            }
        }
        __syncwarp();
        issue(blk + kColStages - 1);
    }
    cp_async_wait<0>();
    if (lane < ncv) out[cbase + lane] = s;
}

constexpr int kRowStages = 8;
constexpr int kRowAcc = 4;

// Row chains: for a in [0, nacc): out[a*ostride + r] = fused multiply-add
// chain over columns c of X[r, c] * W[a*wstride + c] in column order, four
// weight vectors per pass. One warp = 32 rows; tiles of 32 x 32 staged
// through padded shared memory. Replaces k_expected_col_g
// (abft_stepwise.cuh:134-146).
__global__ void __launch_bounds__(32)
    k_rowchain(const float* __restrict__ X, long long ld, int R, int L, const double* __restrict__ W,
               long long wstride, int nacc, double* __restrict__ out, long long ostride) {
    __shared__ float tile[kRowStages][32][33];
    __shared__ __align__(16) double wsm[kRowStages][kRowAcc][32];
    const int lane = threadIdx.x;
    const int rbase = blockIdx.x * 32;
    const int nrv = min(32, R - rbase);
    const int nblk = (L + 31) / 32;
    const double* Wg = W + (long long)blockIdx.y * kRowAcc * wstride;
    const int na = min(kRowAcc, nacc - (int)blockIdx.y * kRowAcc);
    auto issue = [&](int blk) {
        if (blk < nblk) {
            const int slot = blk % kRowStages;
            const int c = blk * 32 + lane;
            for (int rr = 0; rr < 32; ++rr) {
                const bool ok = (rr < nrv) && (c < L);
                const float* src = ok ? (X + (long long)(rbase + rr) * ld + c) : X;
                cp_async4(&tile[slot][rr][lane], src, ok ? 4 : 0);
            }
            for (int a = 0; a < kRowAcc; ++a) {
                const bool ok = (a < na) && (c < L);
                const double* src = ok ? (Wg + (long long)a * wstride + c) : W;
                cp_async8(&wsm[slot][a][lane], src, ok ? 8 : 0);
            }
        }
        cp_async_commit();
    };
    for (int b = 0; b < kRowStages - 1; ++b) issue(b);
    double s[kRowAcc] = {0.0, 0.0, 0.0, 0.0};
    for (int blk = 0; blk < nblk; ++blk) {
        cp_async_wait<kRowStages - 2>();
        __syncwarp();
        const int slot = blk % kRowStages;
        const int nc = min(32, L - blk * 32);
        if (nc == 32) {
#pragma unroll 8
            for (int c = 0; c < 32; ++c) {
                const double x = (double)tile[slot][lane][c];
#pragma unroll
                for (int a = 0; a < kRowAcc; ++a) s[a] = __fma_rn(x, wsm[slot][a][c], s[a]);
            }
        } else {
            for (int c = 0; c < nc; ++c) {
                const double x = (double)tile[slot][lane][c];
#pragma unroll
                for (int a = 0; a < kRowAcc; ++a) s[a] = __fma_rn(x, wsm[slot][a][c], s[a]);
            }
        }
        __syncwarp();
        issue(blk + kRowStages - 1);
    }
    cp_async_wait<0>();
    if (lane < nrv) {
        for (int a = 0; a < na; ++a) out[((long long)blockIdx.y * kRowAcc + a) * ostride + rbase + lane] = s[a];
    }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, what);
    return ABFT_OK;
}

// Verify geometry: column groups x CTAs per group, sized to one full wave of
// resident CTAs (target = resident CTAs per SM x SMs; a second, mostly empty
// wave would double the launch time). A unit of rows is at least two batches
// per warp (2 * kBatch * kWarps = 128 rows: measured on B200, one-batch units
// lose more to the per-unit barrier than they gain in balance) and about
// 1/kUnitsPerCta of a CTA's share; a group has no more CTAs than units (this
// bounds the atomics per accumulator to M / 128). n_large: the units of
// unit_rows rows; the rows after them form one-batch units. When every CTA
// has at least four units, the last ~2 per CTA are one-batch units, so that
// the group's CTAs finish closer together (16384 x 4096 at pitch 16416:
// 54.1 -> 53.3 us; no change on fragments with fewer units per CTA).
constexpr int kUnitsPerCta = 16;
void verify_geometry(int target, int M, int N, int& groups, int& chunks, int& unit_rows, int& n_large) {
    constexpr int kUnit = kBatch * kWarps;
    groups = (N + kGroupCols - 1) / kGroupCols;
    chunks = std::min(std::max(target / groups, 1), kMaxChunks);
    unit_rows = kUnit * std::max(2, M / (chunks * kUnit * kUnitsPerCta));
    const int units = (M + unit_rows - 1) / unit_rows;
    chunks = std::min(chunks, units);
    n_large = units;
    if (M >= 4 * chunks * unit_rows) n_large = (M - 2 * chunks * kUnit) / unit_rows;
}

// Geometry of the TMA-staged verify: as above, with row chunks a multiple of
// the box height (no box crosses into the next chunk) and at least two boxes.
void verify_geometry_tma(int target, int M, int N, int& groups, int& chunks, int& rows_per) {
    groups = (N + kGroupCols - 1) / kGroupCols;
    chunks = target / groups;
    if (chunks < 1) chunks = 1;
    if (chunks > kMaxChunks) chunks = kMaxChunks;
    rows_per = (M + chunks - 1) / chunks;
    rows_per = ((rows_per + kTmaRows - 1) / kTmaRows) * kTmaRows;
    rows_per = std::max(rows_per, 2 * kTmaRows);
    chunks = (M + rows_per - 1) / rows_per;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda); null when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        (void)cudaGetLastError();
    });
    return fn;
}

// Tensor map of one fragment (M rows of N floats, row pitch ldc floats) with
// kTmaRows x kGroupCols boxes, zero fill outside. False if it cannot be made.
bool fragment_tensor_map(CUtensorMap* map, const float* Cf, int64_t ldc, int M, int N) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)ldc * sizeof(float)};
    const cuuint32_t box[2] = {(cuuint32_t)kGroupCols, (cuuint32_t)kTmaRows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(Cf), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Which verify body launch_verify uses: 0 = by size, 1 = 128-bit loads, 2 = TMA.
std::atomic<int> g_verify_kernel{0};
// Polls each wait of the TMA verify body makes for a bulk copy before it gives
// up (records a fault); lowered only by tests of that failure path.
std::atomic<int> g_wait_limit{kSpinLimit};

// Resident CTAs per SM of a kernel at a dynamic shared memory size (cached).
int resident_per_sm(const void* fn, int smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, const void*, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_tuple(dev, fn, smem);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, smem) != cudaSuccess || n < 1) {
        (void)cudaGetLastError();
        n = 1;
    }
    cache[key] = n;
    return n;
}

}  // namespace

// ------------------------------------------------------------ launchers ---

// Large dynamic shared memory must be enabled once per device and kernel.
int ensure_kernel_attrs(int device) {
    static std::mutex mu;
    static std::set<int> done;
    std::lock_guard<std::mutex> lock(mu);
    if (done.count(device)) return ABFT_OK;
    cudaError_t e = cudaSuccess;
    auto set = [&](const void* fn, int bytes) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    };
    set((const void*)k_colchain<false, true, kColStagesDeep>, col_smem(kColStagesDeep));
    set((const void*)k_colchain<false, false, kColStagesDeep>, col_smem(kColStagesDeep));
    set((const void*)k_colchain<false, true, kColStagesShallow>, col_smem(kColStagesShallow));
    set((const void*)k_colchain<false, false, kColStagesShallow>, col_smem(kColStagesShallow));
    set((const void*)k_colchain<true, true, kColStagesDeep>, col_smem(kColStagesDeep));
    set((const void*)k_colchain<true, false, kColStagesDeep>, col_smem(kColStagesDeep));
    set((const void*)k_colchain<true, true, kColStagesShallow>, col_smem(kColStagesShallow));
    set((const void*)k_colchain<true, false, kColStagesShallow>, col_smem(kColStagesShallow));
    set((const void*)k_verify<true>, kVerifySmemMax);
    set((const void*)k_verify<false>, kVerifySmemMax);
    set((const void*)k_verify_tma, kTmaSmem + kTmaAlign);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    done.insert(device);
    return ABFT_OK;
}

// Rows per CTA of the row-sum kernels (localise, encode): about 64 KB of the
// matrix per CTA, but no more rows than give two CTAs per SM (whole warps of
// rows, 8 to 256 rows).
int row_block(int R, int N, int sms) {
    long long rows = 65536 / ((long long)N * 4);
    rows = std::min(rows, (long long)((R + 2 * sms - 1) / (2 * sms)));
    if (rows < kWarps) rows = kWarps;
    if (rows > 256) rows = 256;
    return (int)((rows + kWarps - 1) / kWarps) * kWarps;
}

int launch_encode(abft_ws* ws, const float* dA, int64_t lda, const float* dB, int64_t ldb, cudaStream_t st,
                  int* launches) {
    if (int rc = ensure_kernel_attrs(ws->device)) return rc;
    const int M = ws->M_b, K = ws->K, N = ws->N_b, F = ws->F;
    int n = 0;
    // Column chains of K columns over R rows, as one wave of one-warp CTAs.
    auto colchain = [&](bool weighted, const float* X, int64_t ld, int R, int ncols, const double* wrow,
                        double* out) {
        const bool vec = aligned16(X) && (ld % 4 == 0);
        const int ctas = (ncols + 31) / 32;
        const bool deep = ctas <= ws->sms * (227 * 1024 / col_smem(kColStagesDeep));
        const dim3 grid(ctas);
#define ABFT_COLCHAIN(W, V, S) k_colchain<W, V, S><<<grid, 32, col_smem(S), st>>>(X, ld, R, ncols, wrow, out)
#define ABFT_COLCHAIN_STAGES(W, V) \
    do {                           \
        if (deep)                  \
            ABFT_COLCHAIN(W, V, kColStagesDeep); \
        else                       \
            ABFT_COLCHAIN(W, V, kColStagesShallow); \
    } while (0)
        if (weighted && vec) ABFT_COLCHAIN_STAGES(true, true);
        else if (weighted) ABFT_COLCHAIN_STAGES(true, false);
        else if (vec) ABFT_COLCHAIN_STAGES(false, true);
        else ABFT_COLCHAIN_STAGES(false, false);
#undef ABFT_COLCHAIN_STAGES
#undef ABFT_COLCHAIN
    };
    // colSumA[K]: sequential chains over the M rows of A. (A certified
    // parallel sum, as verify uses, loses here at large M: one tiny element
    // among M uniform terms sets the certificate's exponent, and at M = 16384
    // about 12 % of columns fail it and need the sequential re-sum anyway.)
    colchain(false, dA, lda, M, K, nullptr, ws->d.colSumA);
    ++n;
    if (int rc = check_launch("encode colSumA")) return rc;
    // expRow[N_b]: fused multiply-add chains over the K rows of B.
    colchain(true, dB, ldb, K, N, ws->d.colSumA, ws->d.expRow);
    ++n;
    if (int rc = check_launch("encode expectedRow")) return rc;
    // rowSumB_f[K] per fragment: certified row sums over the fragment's columns of each B row.
    for (int f = 0; f < F; ++f) {
        const float* Bf = dB + ws->offsets[f];
        const int Nf = ws->counts[f];
        const int rows_per = row_block(K, Nf, ws->sms);
        const int nblocks = (K + rows_per - 1) / rows_per;
        const bool vec = aligned16(Bf) && (ldb % 4 == 0) && (Nf % 4 == 0);
        double* out = ws->d.rowSumB + (long long)f * K;
        if (vec && Nf <= kLocNarrow) k_rowsum<true, 4><<<nblocks, kThreads, 0, st>>>(Bf, ldb, K, Nf, rows_per, out);
        else if (vec) k_rowsum<true, 1><<<nblocks, kThreads, 0, st>>>(Bf, ldb, K, Nf, rows_per, out);
        else if (Nf <= kLocNarrow) k_rowsum<false, 4><<<nblocks, kThreads, 0, st>>>(Bf, ldb, K, Nf, rows_per, out);
        else k_rowsum<false, 1><<<nblocks, kThreads, 0, st>>>(Bf, ldb, K, Nf, rows_per, out);
        ++n;
        if (int rc = check_launch("encode rowSumB")) return rc;
    }
    // expCol_f[M_b]: fused multiply-add chains over each A row, four fragments per pass.
    {
        dim3 grid((M + 31) / 32, (F + kRowAcc - 1) / kRowAcc);
        k_rowchain<<<grid, 32, 0, st>>>(dA, lda, M, K, ws->d.rowSumB, K, F, ws->d.expCol, M);
        ++n;
        if (int rc = check_launch("encode expectedCol")) return rc;
    }
    if (launches) *launches += n;
    return ABFT_OK;
}

int launch_verify(abft_ws* ws, const float* dC, int64_t ldc, int f, double tau, int injected, int it,
                  cudaStream_t st, int plan_it, float add_delta, int log_inj, double* calib_out,
                  unsigned long long cond) {
    const int M = ws->M_b, N = ws->counts[f];
    const float* Cf = dC + ws->offsets[f];
    if (int rc = ensure_kernel_attrs(ws->device)) return rc;
    const double* expv = ws->d.expRow + ws->offsets[f];
    if (it >= ws->max_iters) it = -1;
    const InjectPlan* plan = (plan_it >= 0) ? ws->d.plan : nullptr;
    float* Cw = const_cast<float*>(Cf);
    int groups, chunks;

    // TMA-staged body: 16-byte aligned fragment, pitch a multiple of 4 floats,
    // at least one full box; when selected explicitly.
    const int choice = g_verify_kernel.load(std::memory_order_relaxed);
    const bool tma_ok = aligned16(Cf) && (ldc % 4 == 0) && N >= kGroupCols && M >= kTmaRows;
    const bool want_tma = (choice == 2) || (choice == 0 && 4LL * M * N < kTmaMaxBytes);
    CUtensorMap map;
    if (tma_ok && want_tma && fragment_tensor_map(&map, Cf, ldc, M, N)) {
        const int per_sm = resident_per_sm((const void*)k_verify_tma, kTmaSmem + kTmaAlign);
        int rows_per;
        verify_geometry_tma(per_sm * ws->sms, M, N, groups, chunks, rows_per);
        k_verify_tma<<<dim3(groups, chunks), kThreads, kTmaSmem + kTmaAlign, st>>>(
            map, Cf, ldc, M, N, rows_per, expv, tau, injected, f, ws->F, it, ws->d, Cw, plan, plan_it, add_delta,
            log_inj, calib_out, cond, g_wait_limit.load(std::memory_order_relaxed));
        return check_launch("verify (tma)");
    }

    const bool vec = aligned16(Cf) && (ldc % 4 == 0) && (N % 4 == 0);
    // 16 KB of shared memory per CTA: the fold of its eight warps' partials
    const int smem = kWarps * kGroupCols * 16;
    const int per_sm = resident_per_sm(vec ? (const void*)k_verify<true> : (const void*)k_verify<false>, smem);
    int unit_rows, n_large;
    verify_geometry(per_sm * ws->sms, M, N, groups, chunks, unit_rows, n_large);
    dim3 grid(groups, chunks);
    if (vec)
        k_verify<true><<<grid, kThreads, smem, st>>>(Cf, ldc, M, N, unit_rows, n_large, expv, tau, injected, f, ws->F, it,
                                                     ws->d, Cw, plan, plan_it, add_delta, log_inj, calib_out, cond);
    else
        k_verify<false><<<grid, kThreads, smem, st>>>(Cf, ldc, M, N, unit_rows, n_large, expv, tau, injected, f, ws->F, it,
                                                      ws->d, Cw, plan, plan_it, add_delta, log_inj, calib_out, cond);
    return check_launch("verify");
}

int launch_localize(abft_ws* ws, float* dC, int64_t ldc, int f, double tau, int injected, const float* dG,
                    int64_t ldg, int it, int correct_mode, cudaStream_t st, int plan_it) {
    const int M = ws->M_b, N = ws->counts[f];
    float* Cf = dC + ws->offsets[f];
    // A short fragment (up to 4096 rows) is localised while the next
    // fragment's small split-K SGEMM runs: blocks of a full 64 KB, rather
    // than two CTAs on every SM, leave that SGEMM more of the machine
    // (1024^3 in 16 fragments: pipeline overhead 5.8 -> 5.2 % with graphs,
    // 6.4 -> 6.2 % eager; 4096^3 unchanged).
    int rows_per = row_block(M, N, ws->sms);
    if (M <= 4096) rows_per = std::max(rows_per, row_block(1 << 30, N, ws->sms));
    const int nblocks = (M + rows_per - 1) / rows_per;
    const bool vec = aligned16(Cf) && (ldc % 4 == 0) && (N % 4 == 0);
    const double* expc = ws->d.expCol + (long long)f * M;
    if (it >= ws->max_iters) it = -1;
    const int drain = (correct_mode == ABFT_CORRECT_DRAIN) ? 1 : 0;
    const int cap = ws->max_iters * ws->F;
    if (drain && (cap <= 0 || it < 0)) {
        set_error("drain correction needs a workspace with max_iters > iteration index");
        return ABFT_ERR_ARG;
    }
    const InjectPlan* plan = plan_it >= 0 ? ws->d.plan : nullptr;
#define ABFT_LOCALIZE_LAUNCH(V, R)                                                                               \
    k_localize<V, R><<<nblocks, kThreads, 0, st>>>(Cf, ldc, M, N, rows_per, nblocks, expc, tau, injected, dG, ldg, \
                                                   ws->offsets[f], f, ws->F, it, drain, cap, ws->d, plan, plan_it)
    const bool narrow = N <= kLocNarrow;
    if (vec && narrow) ABFT_LOCALIZE_LAUNCH(true, 4);
    else if (vec) ABFT_LOCALIZE_LAUNCH(true, 1);
    else if (narrow) ABFT_LOCALIZE_LAUNCH(false, 4);
    else ABFT_LOCALIZE_LAUNCH(false, 1);
#undef ABFT_LOCALIZE_LAUNCH
    return check_launch("localize");
}

int launch_drain(abft_ws* ws, float* dC0, float* dC1, int64_t ldc, const float* dG, int64_t ldg, int repeats,
                 cudaStream_t st) {
    const int cap = ws->max_iters * ws->F;
    k_drain<<<1, kThreads, 0, st>>>(dC0, dC1, ldc, dG, ldg, repeats, cap, ws->d);
    return check_launch("drain");
}

int launch_inject(float* dC, int64_t ldc, int row, int col, int mode, float delta, int bit, InjectLog* log,
                  int frag, cudaStream_t st) {
    k_inject<<<1, 1, 0, st>>>(dC, ldc, row, col, mode, delta, bit, log, frag);
    return check_launch("inject");
}

}  // namespace abft

// ------------------------------------------------ verify without allocation --
//
// abft_verify_noalloc runs the fused verify kernel above on scratch that lives
// in a static device array of this library instead of a workspace, for callers
// that may not allocate device memory (see include/abft_b200.h). The array is
// at most kStaticMaxCols columns wide:
//   [0, 32 KiB)         per-column double sums         (double[4096])
//   [32 KiB, 48 KiB)    per-column float |x| sums      (float[4096])
//   [48 KiB, 64 KiB)    per-column smallest |x| bits-1 (uint32[4096], starts at 0xffffffff)
//   [64 KiB, 96 KiB)    per-column final sums          (double[4096])
//   [96 KiB, 128 KiB)   per-column |actual - expected| (double[4096])
//   [128 KiB, 160 KiB)  per-column windows             (double[4096])
//   then the arrival and work counters (2 + 2 x 32 ints, 512 bytes), one
//   decision record and one counter block (256 bytes each).
// Every call in a CUDA context shares that context's copy of the array. The
// kernel's last CTAs put the accumulators and the arrival counters back to
// their start values, and the copy-out kernel zeroes the counter block, so
// each call starts clean; two calls whose kernels overlap on the GPU race on
// the array.
namespace abft {
namespace {

constexpr int kStaticMaxCols = 4096;
constexpr size_t kStaticColBytes = 160 * 1024;
constexpr size_t kStaticCounterBytes = 512;
constexpr size_t kStaticScratchBytes = kStaticColBytes + kStaticCounterBytes + 2 * 256;
static_assert(sizeof(int) * vcnt_ints(kStaticMaxCols / kGroupCols) <= kStaticCounterBytes, "verify counters");
static __device__ __align__(256) unsigned char g_verify_scratch[kStaticScratchBytes];

struct StaticScratchState {
    unsigned char* base = nullptr;  // device address of g_verify_scratch in this context
    int sms = 0;
};
std::mutex g_static_mu;
// Set-up state per CUDA context: a module's static device array exists once
// per context, at an address of that context (a second context on a device,
// or the context that follows cudaDeviceReset, has its own, uncleared copy).
// Keyed by the driver's context id, which is never reused within a process;
// where the driver does not offer it, by device and array address.
std::map<std::pair<unsigned long long, uintptr_t>, StaticScratchState> g_static;

// Unique id of the calling thread's current context (0 when unavailable).
unsigned long long current_context_id() {
    static std::once_flag once;
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
        (void)cudaGetLastError();
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr &&
        get_id(ctx, &id) == CUDA_SUCCESS)
        return id;
    return 0;
}

// Set-up once per context, with the caller's device current: resolve the
// device address of the static array (host code may not use the symbol
// itself; cudaGetSymbolAddress also makes the runtime's context current) and
// bring the array to its start values on the caller's stream.
int static_scratch(int device, cudaStream_t st, StaticScratchState* out) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_verify_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(verify scratch)");
    const unsigned long long ctx = current_context_id();
    const auto key = std::make_pair(ctx != 0 ? ctx : (unsigned long long)device | (1ull << 63),
                                    reinterpret_cast<uintptr_t>(p));
    std::lock_guard<std::mutex> lock(g_static_mu);
    auto it = g_static.find(key);
    if (it == g_static.end()) {
        StaticScratchState s;
        e = cudaMemsetAsync(p, 0, kStaticScratchBytes, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(static_cast<unsigned char*>(p) + 48 * 1024, 0xff, 16 * 1024, st);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess) return cuda_fail(e, "verify scratch set-up");
        s.base = static_cast<unsigned char*>(p);
        it = g_static.emplace(key, s).first;
    }
    *out = it->second;
    return ABFT_OK;
}

__global__ void k_static_copyout(const FragRecord* rec, Counters* ctr, int* errcol, double* rowdiff, int* cm) {
    if (threadIdx.x == 0) {
        *errcol = rec->errcol;
        *rowdiff = rec->rowdiff;
        for (int i = 0; i < 4; ++i) {
            const int v = ctr->cm[i];
            if (v != 0) atomicAdd(cm + i, v);
            ctr->cm[i] = 0;
        }
    }
}

}  // namespace

int set_verify_kernel(int which) {
    if (which < ABFT_VERIFY_AUTO || which > ABFT_VERIFY_TMA) return -1;
    return g_verify_kernel.exchange(which);
}

int verify_kernel() { return g_verify_kernel.load(std::memory_order_relaxed); }

int set_wait_limit(int polls) {
    if (polls < 0) return -1;
    return g_wait_limit.exchange(polls);
}

int launch_verify_static(const float* Cf, int64_t ldc, int M, int N, const double* expv, double tau, int injected,
                         int* errcol, double* rowdiff, int* cm, cudaStream_t st) {
    if (N > kStaticMaxCols) {
        set_error("abft_verify_noalloc: fragment has " + std::to_string(N) + " columns; the static scratch holds " +
                  std::to_string(kStaticMaxCols));
        return ABFT_ERR_ARG;
    }
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    StaticScratchState s;
    if (int rc = static_scratch(device, st, &s)) return rc;
    if (int rc = ensure_kernel_attrs(device)) return rc;
    WsDev w{};
    w.vacc_s = reinterpret_cast<double*>(s.base);
    w.vacc_t = reinterpret_cast<float*>(s.base + 32 * 1024);
    w.vacc_m = reinterpret_cast<uint32_t*>(s.base + 48 * 1024);
    w.vact = reinterpret_cast<double*>(s.base + 64 * 1024);
    w.vd = reinterpret_cast<double*>(s.base + 96 * 1024);
    w.vw = reinterpret_cast<double*>(s.base + 128 * 1024);
    w.vcnt = reinterpret_cast<int*>(s.base + kStaticColBytes);
    w.rec = reinterpret_cast<FragRecord*>(s.base + kStaticColBytes + kStaticCounterBytes);
    w.ctr = reinterpret_cast<Counters*>(s.base + kStaticColBytes + kStaticCounterBytes + 256);
    const bool vec = aligned16(Cf) && (ldc % 4 == 0) && (N % 4 == 0);
    const int smem = kWarps * kGroupCols * 16;
    const int per_sm = resident_per_sm(vec ? (const void*)k_verify<true> : (const void*)k_verify<false>, smem);
    int groups, chunks, unit_rows, n_large;
    verify_geometry(per_sm * s.sms, M, N, groups, chunks, unit_rows, n_large);
    dim3 grid(groups, chunks);
    if (vec)
        k_verify<true><<<grid, kThreads, smem, st>>>(Cf, ldc, M, N, unit_rows, n_large, expv, tau, injected, 0, 1, -1, w,
                                                     nullptr, nullptr, 0, 0.f, 0, nullptr, 0);
    else
        k_verify<false><<<grid, kThreads, smem, st>>>(Cf, ldc, M, N, unit_rows, n_large, expv, tau, injected, 0, 1, -1, w,
                                                      nullptr, nullptr, 0, 0.f, 0, nullptr, 0);
    if (int rc = check_launch("verify (static scratch)")) return rc;
    k_static_copyout<<<1, 32, 0, st>>>(w.rec, w.ctr, errcol, rowdiff, cm);
    return check_launch("verify copy-out");
}

}  // namespace abft
