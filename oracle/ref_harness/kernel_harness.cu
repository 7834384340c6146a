// GPU harness around the reference's own ABFT kernels and injectors.
//
// TEST INFRASTRUCTURE ONLY. Compiled by oracle/Makefile from the reference
// sources where they lie into oracle/_ref/kernel_harness (sm_100a). The GPU
// tests use it to run the reference's launch helpers on exactly the inputs
// that the new kernels and the CPU oracle see:
//   launch_col_checksum_A   kernels/abft_stepwise.cuh:243-248
//   launch_expected_row     kernels/abft_stepwise.cuh:250-256
//   launch_actual_row       kernels/abft_stepwise.cuh:258-263
//   launch_detect_row       kernels/abft_stepwise.cuh:208-216
//   launch_localize_correct kernels/abft_stepwise.cuh:218-239
//   inject_add_constant     kernels/swifi.cuh:61-76
//   inject_single_bitflip   kernels/swifi.cuh:78-114
// The per-fragment order follows the verify half of pass_online_loop
// (pipeline/passes.cuh:180-198) with do_localize on.
//
// File format (little endian), written by tests/refharness.py:
//   verify mode input : int32 M K N F has_golden, int32 injected[F], float64 tau[F],
//                       float32 A[M*K], B[K*N], C[M*N], golden[M*N] (if has_golden)
//   verify mode output: float64 colSumA[K], expRow[N], actRow[N], int32 errcol[F],
//                       float64 rowdiff[F], float64 rowSumB[F*K], expCol[F*M], actCol[F*M],
//                       float32 C[M*N], int32 cm[4], int32 n_restored
//   inject mode input : int32 M N F frag ldc_unused, uint64 seed, int32 mode(0 add,1 swifi),
//                       int32 zone_len, char zone[zone_len], float32 C[M*N]
//   inject mode output: int32 row col bit, float32 before after, float32 C[M*N]

#include "core/common.cuh"
#include "core/types.cuh"
#include "distribution/grid.cuh"
#include "kernels/abft_stepwise.cuh"
#include "kernels/swifi.cuh"

#include <cstdio>

#define HCHECK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { \
    std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
    std::exit(5); } } while (0)

template <class T> static void rd(FILE* f, T* p, size_t n) {
    if (n && std::fread(p, sizeof(T), n, f) != n) { std::fprintf(stderr, "short read\n"); std::exit(6); }
}
template <class T> static void wr(FILE* f, const T* p, size_t n) {
    if (n && std::fwrite(p, sizeof(T), n, f) != n) { std::fprintf(stderr, "short write\n"); std::exit(6); }
}

static int run_verify(const char* in_path, const char* out_path) {
    FILE* fi = std::fopen(in_path, "rb");
    if (!fi) return 7;
    int hdr[5];
    rd(fi, hdr, 5);
    int M = hdr[0], K = hdr[1], N = hdr[2], F = hdr[3], has_golden = hdr[4];
    if (M <= 0 || K <= 0 || N <= 0 || F <= 0 || F > N || (size_t)M * K > (1u << 26) ||
        (size_t)K * N > (1u << 26) || (size_t)M * N > (1u << 26)) {
        std::fprintf(stderr, "bad sizes\n");
        return 8;
    }
    std::vector<int> injected(F);
    std::vector<double> tau(F);
    rd(fi, injected.data(), F);
    rd(fi, tau.data(), F);
    std::vector<float> A((size_t)M * K), B((size_t)K * N), C((size_t)M * N), G;
    rd(fi, A.data(), A.size());
    rd(fi, B.data(), B.size());
    rd(fi, C.data(), C.size());
    if (has_golden) { G.resize((size_t)M * N); rd(fi, G.data(), G.size()); }
    std::fclose(fi);

    // Fragment geometry exactly as buffers_init (pipeline/buffers.cuh:56-57).
    std::vector<int> cc, co;
    split_dim(N, F, cc, co);
    int nfmax = *std::max_element(cc.begin(), cc.end());

    float *dA, *dB, *dC, *dG = nullptr;
    double *dColSumA, *dExpRow, *dActRow, *dRowDiff, *dRowSumB, *dExpCol, *dActCol;
    int *dErrCol, *dCM, *dNR;
    HCHECK(cudaMalloc(&dA, A.size() * 4));
    HCHECK(cudaMalloc(&dB, B.size() * 4));
    HCHECK(cudaMalloc(&dC, C.size() * 4));
    if (has_golden) HCHECK(cudaMalloc(&dG, G.size() * 4));
    HCHECK(cudaMalloc(&dColSumA, sizeof(double) * K));
    HCHECK(cudaMalloc(&dExpRow, sizeof(double) * (size_t)F * nfmax));
    HCHECK(cudaMalloc(&dActRow, sizeof(double) * (size_t)F * nfmax));
    HCHECK(cudaMalloc(&dRowDiff, sizeof(double) * F));
    HCHECK(cudaMalloc(&dErrCol, sizeof(int) * F));
    HCHECK(cudaMalloc(&dRowSumB, sizeof(double) * K));
    HCHECK(cudaMalloc(&dExpCol, sizeof(double) * M));
    HCHECK(cudaMalloc(&dActCol, sizeof(double) * M));
    HCHECK(cudaMalloc(&dCM, sizeof(int) * 4));
    HCHECK(cudaMalloc(&dNR, sizeof(int)));
    HCHECK(cudaMemcpy(dA, A.data(), A.size() * 4, cudaMemcpyHostToDevice));
    HCHECK(cudaMemcpy(dB, B.data(), B.size() * 4, cudaMemcpyHostToDevice));
    HCHECK(cudaMemcpy(dC, C.data(), C.size() * 4, cudaMemcpyHostToDevice));
    if (has_golden) HCHECK(cudaMemcpy(dG, G.data(), G.size() * 4, cudaMemcpyHostToDevice));
    HCHECK(cudaMemset(dCM, 0, sizeof(int) * 4));
    HCHECK(cudaMemset(dNR, 0, sizeof(int)));
    cudaStream_t s;
    HCHECK(cudaStreamCreate(&s));

    launch_col_checksum_A(dA, K, dColSumA, M, K, s);
    for (int f = 0; f < F; ++f)
        launch_expected_row(dColSumA, dB + co[f], N, dExpRow + (size_t)f * nfmax, K, cc[f], s);
    HCHECK(cudaGetLastError());

    std::vector<double> colSumA(K), expRow(N), actRow(N), rowdiff(F), rowSumB((size_t)F * K, 0.0),
        expCol((size_t)F * M, 0.0), actCol((size_t)F * M, 0.0);
    std::vector<int> errcol(F);
    for (int f = 0; f < F; ++f) {
        launch_actual_row(dC + co[f], N, dActRow + (size_t)f * nfmax, M, cc[f], s);
        launch_detect_row(dExpRow + (size_t)f * nfmax, dActRow + (size_t)f * nfmax, cc[f], tau[f],
                          dErrCol + f, dRowDiff + f, injected[f], dCM, s);
        launch_localize_correct(dA, K, dB + co[f], N, dC + co[f], N, dRowSumB, dExpCol, dActCol, M, K,
                                cc[f], tau[f], dErrCol + f, dRowDiff + f, dG, N, co[f], injected[f],
                                dNR, s);
        HCHECK(cudaGetLastError());
        HCHECK(cudaStreamSynchronize(s));
        int ec = 0;
        HCHECK(cudaMemcpy(&ec, dErrCol + f, sizeof(int), cudaMemcpyDeviceToHost));
        if (ec >= 0) {
            HCHECK(cudaMemcpy(rowSumB.data() + (size_t)f * K, dRowSumB, sizeof(double) * K, cudaMemcpyDeviceToHost));
            HCHECK(cudaMemcpy(expCol.data() + (size_t)f * M, dExpCol, sizeof(double) * M, cudaMemcpyDeviceToHost));
            HCHECK(cudaMemcpy(actCol.data() + (size_t)f * M, dActCol, sizeof(double) * M, cudaMemcpyDeviceToHost));
        }
    }
    HCHECK(cudaStreamSynchronize(s));
    HCHECK(cudaMemcpy(colSumA.data(), dColSumA, sizeof(double) * K, cudaMemcpyDeviceToHost));
    for (int f = 0; f < F; ++f) {
        HCHECK(cudaMemcpy(expRow.data() + co[f], dExpRow + (size_t)f * nfmax, sizeof(double) * cc[f], cudaMemcpyDeviceToHost));
        HCHECK(cudaMemcpy(actRow.data() + co[f], dActRow + (size_t)f * nfmax, sizeof(double) * cc[f], cudaMemcpyDeviceToHost));
    }
    HCHECK(cudaMemcpy(errcol.data(), dErrCol, sizeof(int) * F, cudaMemcpyDeviceToHost));
    HCHECK(cudaMemcpy(rowdiff.data(), dRowDiff, sizeof(double) * F, cudaMemcpyDeviceToHost));
    HCHECK(cudaMemcpy(C.data(), dC, C.size() * 4, cudaMemcpyDeviceToHost));
    int cm[4], nr;
    HCHECK(cudaMemcpy(cm, dCM, sizeof(cm), cudaMemcpyDeviceToHost));
    HCHECK(cudaMemcpy(&nr, dNR, sizeof(int), cudaMemcpyDeviceToHost));

    FILE* fo = std::fopen(out_path, "wb");
    if (!fo) return 9;
    wr(fo, colSumA.data(), K);
    wr(fo, expRow.data(), N);
    wr(fo, actRow.data(), N);
    wr(fo, errcol.data(), F);
    wr(fo, rowdiff.data(), F);
    wr(fo, rowSumB.data(), rowSumB.size());
    wr(fo, expCol.data(), expCol.size());
    wr(fo, actCol.data(), actCol.size());
    wr(fo, C.data(), C.size());
    wr(fo, cm, 4);
    wr(fo, &nr, 1);
    std::fclose(fo);
    cudaStreamDestroy(s);
    return 0;
}

static int run_inject(const char* in_path, const char* out_path) {
    FILE* fi = std::fopen(in_path, "rb");
    if (!fi) return 7;
    int hdr[5];
    rd(fi, hdr, 5);
    int M = hdr[0], N = hdr[1], F = hdr[2], frag = hdr[3];
    uint64_t seed;
    rd(fi, &seed, 1);
    int mode, zl;
    rd(fi, &mode, 1);
    rd(fi, &zl, 1);
    if (M <= 0 || N <= 0 || F <= 0 || F > N || frag < 0 || frag >= F || zl < 0 || zl > 64 ||
        (size_t)M * N > (1u << 26)) {
        std::fprintf(stderr, "bad sizes\n");
        return 8;
    }
    std::string zone(zl, ' ');
    rd(fi, &zone[0], zl);
    std::vector<float> C((size_t)M * N);
    rd(fi, C.data(), C.size());
    std::fclose(fi);
    std::vector<int> cc, co;
    split_dim(N, F, cc, co);
    float* dC;
    HCHECK(cudaMalloc(&dC, C.size() * 4));
    HCHECK(cudaMemcpy(dC, C.data(), C.size() * 4, cudaMemcpyHostToDevice));
    cudaStream_t s;
    HCHECK(cudaStreamCreate(&s));
    InjectionInfo info = (mode == 0)
        ? inject_add_constant(dC + co[frag], N, M, cc[frag], frag, seed, s)
        : inject_single_bitflip(dC + co[frag], N, M, cc[frag], frag, seed, s, zone);
    HCHECK(cudaGetLastError());
    HCHECK(cudaStreamSynchronize(s));
    HCHECK(cudaMemcpy(C.data(), dC, C.size() * 4, cudaMemcpyDeviceToHost));
    FILE* fo = std::fopen(out_path, "wb");
    if (!fo) return 9;
    int rcb[3] = {info.row, info.col, info.bit_position};
    float ba[2] = {info.value_before, info.value_after};
    wr(fo, rcb, 3);
    wr(fo, ba, 2);
    wr(fo, C.data(), C.size());
    std::fclose(fo);
    cudaStreamDestroy(s);
    cudaFree(dC);
    return 0;
}

int main(int argc, char** argv) {
    if (argc != 4) { std::fprintf(stderr, "kernel_harness {verify|inject} IN OUT\n"); return 2; }
    std::string mode = argv[1];
    if (mode == "verify") return run_verify(argv[2], argv[3]);
    if (mode == "inject") return run_inject(argv[2], argv[3]);
    return 2;
}
