// NCCL communicators for the abft_gemm driver (see abft_comm.h).

#include "abft_comm.h"

#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <sys/socket.h>
#include <unistd.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

namespace {

int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : dflt;
}

bool send_all(int fd, const void* p, size_t n) {
    const char* b = static_cast<const char*>(p);
    while (n) {
        ssize_t k = ::send(fd, b, n, MSG_NOSIGNAL);
        if (k <= 0) return false;
        b += k;
        n -= (size_t)k;
    }
    return true;
}

bool recv_all(int fd, void* p, size_t n) {
    char* b = static_cast<char*>(p);
    while (n) {
        ssize_t k = ::recv(fd, b, n, 0);
        if (k <= 0) return false;
        b += k;
        n -= (size_t)k;
    }
    return true;
}

// Rank 0 serves the NCCL unique id to world - 1 peers; others fetch it.
std::string exchange_id(const RankEnv& env, ncclUniqueId& id, int timeout_s) {
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(timeout_s);
    if (env.rank == 0) {
        int fd = ::socket(AF_INET, SOCK_STREAM, 0);
        if (fd < 0) return "socket() failed";
        int one = 1;
        ::setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
        sockaddr_in a{};
        a.sin_family = AF_INET;
        a.sin_addr.s_addr = htonl(INADDR_ANY);
        a.sin_port = htons((uint16_t)env.port);
        if (::bind(fd, (sockaddr*)&a, sizeof(a)) != 0 || ::listen(fd, 64) != 0) {
            ::close(fd);
            return "bind/listen on bootstrap port " + std::to_string(env.port) + " failed";
        }
        timeval tv{timeout_s, 0};
        ::setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
        for (int served = 0; served < env.world - 1; ++served) {
            int cfd = ::accept(fd, nullptr, nullptr);
            if (cfd < 0) {
                ::close(fd);
                return "bootstrap accept timed out";
            }
            bool ok = send_all(cfd, &id, sizeof(id));
            ::close(cfd);
            if (!ok) {
                ::close(fd);
                return "bootstrap send failed";
            }
        }
        ::close(fd);
        return "";
    }
    while (std::chrono::steady_clock::now() < deadline) {
        addrinfo hints{}, *res = nullptr;
        hints.ai_family = AF_INET;
        hints.ai_socktype = SOCK_STREAM;
        if (::getaddrinfo(env.master_addr.c_str(), std::to_string(env.port).c_str(), &hints, &res) == 0 && res) {
            int fd = ::socket(AF_INET, SOCK_STREAM, 0);
            if (fd >= 0 && ::connect(fd, res->ai_addr, res->ai_addrlen) == 0) {
                bool ok = recv_all(fd, &id, sizeof(id));
                ::close(fd);
                ::freeaddrinfo(res);
                return ok ? "" : "bootstrap receive failed";
            }
            if (fd >= 0) ::close(fd);
            ::freeaddrinfo(res);
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(100));
    }
    return "could not reach the bootstrap server at " + env.master_addr + ":" + std::to_string(env.port);
}

std::string nccl_msg(ncclResult_t r, const char* what) {
    return std::string(what) + ": " + ncclGetErrorString(r);
}

std::string sync(Comm& c) {
    cudaError_t e = cudaStreamSynchronize(c.stream);
    return e == cudaSuccess ? "" : std::string("stream sync: ") + cudaGetErrorString(e);
}

}  // namespace

RankEnv rank_env_from_environment() {
    RankEnv e;
    e.rank = env_int("RANK", env_int("OMPI_COMM_WORLD_RANK", env_int("PMI_RANK", 0)));
    e.world = env_int("WORLD_SIZE", env_int("OMPI_COMM_WORLD_SIZE", env_int("PMI_SIZE", 1)));
    e.local_rank = env_int("LOCAL_RANK", env_int("SLURM_LOCALID", env_int("OMPI_COMM_WORLD_LOCAL_RANK", 0)));
    if (const char* a = std::getenv("MASTER_ADDR")) e.master_addr = a;
    const int mp = env_int("MASTER_PORT", 0);
    e.port = env_int("ABFT_BOOTSTRAP_PORT", mp > 0 ? mp + 1 : 29511);
    return e;
}

std::string comm_init(Comm& c, const RankEnv& env, int pr, int pc, int timeout_s) {
    c.rank = env.rank;
    c.world = env.world;
    cudaError_t ce = cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking);
    if (ce == cudaSuccess) ce = cudaMalloc(&c.scratch, 4096);
    if (ce != cudaSuccess) return std::string("comm buffers: ") + cudaGetErrorString(ce);
    if (env.world == 1) return "";
    ncclUniqueId id{};
    if (env.rank == 0) {
        ncclResult_t r = ncclGetUniqueId(&id);
        if (r != ncclSuccess) return nccl_msg(r, "ncclGetUniqueId");
    }
    std::string err = exchange_id(env, id, timeout_s);
    if (!err.empty()) return err;
    ncclResult_t r = ncclCommInitRank(&c.world_comm, env.world, id, env.rank);
    if (r != ncclSuccess) return nccl_msg(r, "ncclCommInitRank");
    r = ncclCommSplit(c.world_comm, pr, pc, &c.row_comm, nullptr);
    if (r != ncclSuccess) return nccl_msg(r, "ncclCommSplit(row)");
    r = ncclCommSplit(c.world_comm, pc, pr, &c.col_comm, nullptr);
    if (r != ncclSuccess) return nccl_msg(r, "ncclCommSplit(col)");
    return "";
}

void comm_destroy(Comm& c) {
    if (c.stream) cudaStreamSynchronize(c.stream);
    for (ncclComm_t* p : {&c.row_comm, &c.col_comm, &c.world_comm})
        if (*p) {
            ncclCommDestroy(*p);
            *p = nullptr;
        }
    if (c.scratch) cudaFree(c.scratch);
    if (c.stream) cudaStreamDestroy(c.stream);
    c.scratch = nullptr;
    c.stream = nullptr;
}

std::string comm_barrier(Comm& c) {
    if (c.world == 1) return "";
    ncclResult_t r = ncclAllReduce(c.scratch, c.scratch, 1, ncclInt32, ncclSum, c.world_comm, c.stream);
    if (r != ncclSuccess) return nccl_msg(r, "barrier");
    return sync(c);
}

std::string comm_allreduce_int_sum(Comm& c, int* v, int n) {
    if (c.world == 1) return "";
    if ((size_t)n * sizeof(int) > 4096) return "allreduce payload too large";
    cudaMemcpyAsync(c.scratch, v, sizeof(int) * n, cudaMemcpyHostToDevice, c.stream);
    ncclResult_t r = ncclAllReduce(c.scratch, c.scratch, n, ncclInt32, ncclSum, c.world_comm, c.stream);
    if (r != ncclSuccess) return nccl_msg(r, "allreduce(int, sum)");
    cudaMemcpyAsync(v, c.scratch, sizeof(int) * n, cudaMemcpyDeviceToHost, c.stream);
    return sync(c);
}

std::string comm_allreduce_double_max(Comm& c, double* v, int n) {
    if (c.world == 1) return "";
    if ((size_t)n * sizeof(double) > 4096) return "allreduce payload too large";
    cudaMemcpyAsync(c.scratch, v, sizeof(double) * n, cudaMemcpyHostToDevice, c.stream);
    ncclResult_t r = ncclAllReduce(c.scratch, c.scratch, n, ncclFloat64, ncclMax, c.world_comm, c.stream);
    if (r != ncclSuccess) return nccl_msg(r, "allreduce(double, max)");
    cudaMemcpyAsync(v, c.scratch, sizeof(double) * n, cudaMemcpyDeviceToHost, c.stream);
    return sync(c);
}

std::string comm_bcast(Comm& c, ncclComm_t comm, void* dev, size_t count, int root) {
    if (c.world == 1) return "";
    ncclResult_t r = ncclBroadcast(dev, dev, count, ncclFloat32, root, comm, c.stream);
    if (r != ncclSuccess) return nccl_msg(r, "broadcast");
    return sync(c);
}

std::string comm_send(Comm& c, const void* dev, size_t count, int peer) {
    ncclResult_t r = ncclSend(dev, count, ncclFloat32, peer, c.world_comm, c.stream);
    if (r != ncclSuccess) return nccl_msg(r, "send");
    return sync(c);
}

std::string comm_recv(Comm& c, void* dev, size_t count, int peer) {
    ncclResult_t r = ncclRecv(dev, count, ncclFloat32, peer, c.world_comm, c.stream);
    if (r != ncclSuccess) return nccl_msg(r, "recv");
    return sync(c);
}

std::string comm_send_host(Comm& c, const void* host, size_t bytes, int peer) {
    if (bytes == 0) return "";
    void* dev = nullptr;
    cudaError_t e = cudaMalloc(&dev, bytes);
    if (e == cudaSuccess) e = cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return std::string("staging: ") + cudaGetErrorString(e);
    ncclResult_t r = ncclSend(dev, bytes, ncclChar, peer, c.world_comm, c.stream);
    std::string err = (r != ncclSuccess) ? nccl_msg(r, "send") : sync(c);
    cudaFree(dev);
    return err;
}

std::string comm_recv_host(Comm& c, void* host, size_t bytes, int peer) {
    if (bytes == 0) return "";
    void* dev = nullptr;
    cudaError_t e = cudaMalloc(&dev, bytes);
    if (e != cudaSuccess) return std::string("staging: ") + cudaGetErrorString(e);
    ncclResult_t r = ncclRecv(dev, bytes, ncclChar, peer, c.world_comm, c.stream);
    std::string err = (r != ncclSuccess) ? nccl_msg(r, "recv") : sync(c);
    if (err.empty()) {
        e = cudaMemcpy(host, dev, bytes, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) err = std::string("staging: ") + cudaGetErrorString(e);
    }
    cudaFree(dev);
    return err;
}
