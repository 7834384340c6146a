// Self-test of the multi-process MPI stand-in (oracle/mpi_stub_tcp/mpi.h),
// run as WORLD_SIZE processes by tests/test_mpi_stub_cpu.py. It follows the
// reference driver's patterns (main.cu:32-37, distribution/grid.cuh:31-91,
// metrics/metrics.cuh:67-102, main.cu:279-308) and checks every result;
// prints "ok <rank>" and exits 0, or prints the failed check and exits 1.
//
// TEST INFRASTRUCTURE ONLY.
#include <cmath>
#include <cstdio>
#include <vector>

#include "mpi.h"

#define CHECK(c)                                                                  \
    do {                                                                          \
        if (!(c)) {                                                               \
            std::fprintf(stderr, "rank %d: check failed: %s (line %d)\n", rank, #c, __LINE__); \
            return 1;                                                             \
        }                                                                         \
    } while (0)

static float value_of(int stripe, size_t i) { return (float)(stripe * 1000003u + i % 9973u) * 0.5f; }

int main(int argc, char** argv) {
    MPI_Init(&argc, &argv);
    int rank = -1, size = -1;
    MPI_Comm_rank(MPI_COMM_WORLD, &rank);
    MPI_Comm_size(MPI_COMM_WORLD, &size);

    // near-square grid as choose_grid (distribution/grid.cuh:7-12)
    int Pr = 1;
    for (int p = 1; p * p <= size; ++p)
        if (size % p == 0) Pr = p;
    const int Pc = size / Pr, pr = rank / Pc, pc = rank % Pc;
    MPI_Comm row = 0, col = 0;
    MPI_Comm_split(MPI_COMM_WORLD, pr, pc, &row);
    MPI_Comm_split(MPI_COMM_WORLD, pc, pr, &col);
    int rr = -1, rs = -1, cr = -1, cs = -1;
    MPI_Comm_rank(row, &rr);
    MPI_Comm_size(row, &rs);
    MPI_Comm_rank(col, &cr);
    MPI_Comm_size(col, &cs);
    CHECK(rr == pc && rs == Pc && cr == pr && cs == Pr);

    // panels: rank 0 sends stripe pr to (pr, 0) with tag 100 and stripe pc to
    // (0, pc) with tag 200 (large messages), then row / column broadcasts.
    // Rank 0 sends all the tag-200 messages FIRST, so a rank that receives
    // both must queue the tag-200 message while it waits for tag 100.
    const size_t n = (size_t)3 * 1024 * 1024 + 7;  // ~12 MB
    std::vector<float> a(n, -1.f), b(n, -1.f);
    if (rank == 0) {
        for (int q = 1; q < Pc; ++q) {
            std::vector<float> s(n);
            for (size_t i = 0; i < n; ++i) s[i] = value_of(500 + q, i);
            MPI_Send(s.data(), (int)n, MPI_FLOAT, q, 200, MPI_COMM_WORLD);
        }
        for (int p = 1; p < Pr; ++p) {
            std::vector<float> s(n);
            for (size_t i = 0; i < n; ++i) s[i] = value_of(p, i);
            MPI_Send(s.data(), (int)n, MPI_FLOAT, p * Pc, 100, MPI_COMM_WORLD);
        }
        for (size_t i = 0; i < n; ++i) a[i] = value_of(0, i), b[i] = value_of(500, i);
    } else {
        if (pc == 0) MPI_Recv(a.data(), (int)n, MPI_FLOAT, 0, 100, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
        if (pr == 0) MPI_Recv(b.data(), (int)n, MPI_FLOAT, 0, 200, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
    }
    MPI_Bcast(a.data(), (int)n, MPI_FLOAT, 0, row);
    MPI_Bcast(b.data(), (int)n, MPI_FLOAT, 0, col);
    for (size_t i = 0; i < n; i += 997) CHECK(a[i] == value_of(pr, i) && b[i] == value_of(500 + pc, i));
    CHECK(a[n - 1] == value_of(pr, n - 1) && b[n - 1] == value_of(500 + pc, n - 1));

    // matching by tag: rank 0 sends tag 7 then tag 8 to the last rank, which
    // receives tag 8 first (the tag-7 message waits in the queue)
    if (size > 1) {
        int x7 = 70 + size, x8 = 80 + size;
        if (rank == 0) {
            MPI_Send(&x7, 1, MPI_INT, size - 1, 7, MPI_COMM_WORLD);
            MPI_Send(&x8, 1, MPI_INT, size - 1, 8, MPI_COMM_WORLD);
        } else if (rank == size - 1) {
            int y7 = 0, y8 = 0;
            MPI_Recv(&y8, 1, MPI_INT, 0, 8, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
            MPI_Recv(&y7, 1, MPI_INT, 0, 7, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
            CHECK(y7 == x7 && y8 == x8);
        }
    }

    // reductions onto rank 0 (metrics/metrics.cuh:67-102)
    int cm[4] = {rank, 1, 2 * rank, 3}, cm_sum[4] = {0, 0, 0, 0};
    MPI_Reduce(cm, cm_sum, 4, MPI_INT, MPI_SUM, 0, MPI_COMM_WORLD);
    double t[4] = {1.0 * rank, -2.0 * rank, 0.5, rank == size - 1 ? 9.0 : 1.0}, t_max[4] = {0, 0, 0, 0};
    MPI_Reduce(t, t_max, 4, MPI_DOUBLE, MPI_MAX, 0, MPI_COMM_WORLD);
    float f = 0.25f * (float)rank, f_sum = -1.f;
    MPI_Reduce(&f, &f_sum, 1, MPI_FLOAT, MPI_SUM, 0, MPI_COMM_WORLD);
    if (rank == 0) {
        const int s = size * (size - 1) / 2;
        CHECK(cm_sum[0] == s && cm_sum[1] == size && cm_sum[2] == 2 * s && cm_sum[3] == 3 * size);
        CHECK(t_max[0] == size - 1.0 && t_max[1] == 0.0 && t_max[2] == 0.5 && t_max[3] == 9.0);
        float want = 0.f;
        for (int r = 0; r < size; ++r) want += 0.25f * (float)r;  // rank order
        CHECK(f_sum == want);
    }
    // a row reduction too (communicator other than the world)
    int one = 1, row_sum = 0;
    MPI_Reduce(&one, &row_sum, 1, MPI_INT, MPI_SUM, 0, row);
    if (rr == 0) CHECK(row_sum == Pc);

    // calibration gather (main.cu:279-308): counts, then ragged doubles
    const int mine = rank + 1;
    std::vector<int> counts(size, 0), displs(size, 0);
    MPI_Gather(&mine, 1, MPI_INT, counts.data(), 1, MPI_INT, 0, MPI_COMM_WORLD);
    std::vector<double> vals(mine);
    for (int i = 0; i < mine; ++i) vals[i] = rank + 0.125 * i;
    std::vector<double> all;
    if (rank == 0) {
        int total = 0;
        for (int r = 0; r < size; ++r) {
            CHECK(counts[r] == r + 1);
            displs[r] = total;
            total += counts[r];
        }
        all.resize(total);
    }
    MPI_Gatherv(vals.data(), mine, MPI_DOUBLE, rank == 0 ? all.data() : nullptr, counts.data(), displs.data(),
                MPI_DOUBLE, 0, MPI_COMM_WORLD);
    if (rank == 0) {
        size_t k = 0;
        for (int r = 0; r < size; ++r)
            for (int i = 0; i <= r; ++i) CHECK(all[k++] == r + 0.125 * i);
    }

    // barriers on every communicator, repeatedly
    for (int i = 0; i < 3; ++i) {
        MPI_Barrier(MPI_COMM_WORLD);
        MPI_Barrier(row);
        MPI_Barrier(col);
    }
    MPI_Comm_free(&row);
    MPI_Comm_free(&col);
    std::printf("ok %d\n", rank);
    std::fflush(stdout);
    MPI_Finalize();
    return 0;
}
