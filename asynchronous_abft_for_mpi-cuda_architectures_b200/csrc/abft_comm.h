// Rank plumbing of the abft_gemm driver: NCCL over NVLink for every payload,
// a small TCP rendezvous only to hand out the NCCL unique id.
//
// Replaces the reference's MPI layer (main.cu:15-37, distribution/grid.cuh,
// metrics/metrics.cuh:67-102). Launch with torchrun (--no-python) or any
// launcher that sets RANK / WORLD_SIZE / LOCAL_RANK / MASTER_ADDR /
// MASTER_PORT; the rendezvous listens on ABFT_BOOTSTRAP_PORT (default
// MASTER_PORT + 1, or 29511).
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <string>

struct RankEnv {
    int rank = 0, world = 1, local_rank = 0;
    std::string master_addr = "127.0.0.1";
    int port = 29511;
};

RankEnv rank_env_from_environment();

struct Comm {
    int rank = 0, world = 1;
    ncclComm_t world_comm = nullptr, row_comm = nullptr, col_comm = nullptr;
    cudaStream_t stream = nullptr;
    void* scratch = nullptr;  // small device buffer for barriers and reductions
};

// Creates the world communicator and the row / column communicators of a
// Pr x Pc grid (colour pr keyed by pc, and colour pc keyed by pr, like
// MPI_Comm_split in main.cu:36-37). With world == 1 nothing is created.
// Returns an empty string on success, else an error message.
std::string comm_init(Comm& c, const RankEnv& env, int pr, int pc, int timeout_s);
void comm_destroy(Comm& c);

// Device-side collectives on c.stream, synchronised before returning.
std::string comm_barrier(Comm& c);
std::string comm_allreduce_int_sum(Comm& c, int* host_vals, int n);
std::string comm_allreduce_double_max(Comm& c, double* host_vals, int n);
// Broadcast of a device buffer within a communicator from `root`.
std::string comm_bcast(Comm& c, ncclComm_t comm, void* dev, size_t count_floats, int root);
// Point-to-point float transfer on the world communicator.
std::string comm_send(Comm& c, const void* dev, size_t count_floats, int peer);
std::string comm_recv(Comm& c, void* dev, size_t count_floats, int peer);
// Byte transfers of HOST buffers, staged through device memory (end-of-run
// payloads such as the calibration diffs).
std::string comm_send_host(Comm& c, const void* host, size_t bytes, int peer);
std::string comm_recv_host(Comm& c, void* host, size_t bytes, int peer);
