/*
 * Multi-process stand-in for the MPI calls the reference driver makes, over
 * loopback TCP between the processes of one machine.
 *
 * TEST INFRASTRUCTURE ONLY. This image has no MPI; with this header the
 * reference's own sources (main.cu and the headers it includes) compile
 * unmodified into a driver that runs as several ranks, launched like this
 * project's driver by torchrun (RANK, WORLD_SIZE and MASTER_ADDR from the
 * environment; the sockets use ports ABFT_MPI_STUB_PORT + rank, default
 * MASTER_PORT + 100 + rank). It is compiled only by oracle/Makefile into
 * oracle/_ref/ and by the tests, and is never part of the shipped library.
 *
 * Covered, with the MPI semantics the reference relies on: Init, Finalize,
 * Comm_rank, Comm_size, Comm_split (collective over the parent, members
 * ordered by (key, parent rank)), Comm_free, Barrier, Abort, Error_string,
 * Send / Recv (blocking, matched by communicator, source and tag, messages
 * from one source in order), Bcast, Reduce (MPI_SUM, MPI_MAX over MPI_INT /
 * MPI_FLOAT / MPI_DOUBLE, combined in rank order at the root), Gather and
 * Gatherv. Collectives are built from point-to-point messages (linear, root
 * first). A peer that closes its socket, a rank that does not connect within
 * min(ABFT_MPI_STUB_TIMEOUT, 120) seconds, or a wait for data longer than
 * ABFT_MPI_STUB_TIMEOUT seconds (default 600) ends the process with an error
 * instead of hanging.
 */
#ifndef ABFT_ORACLE_MPI_STUB_TCP_H
#define ABFT_ORACLE_MPI_STUB_TCP_H

#include <arpa/inet.h>
#include <errno.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <unistd.h>

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <string>
#include <thread>
#include <vector>

typedef int MPI_Comm;
typedef int MPI_Datatype;
typedef int MPI_Op;
typedef struct { int source, tag, error; } MPI_Status;

#define MPI_SUCCESS 0
#define MPI_MAX_ERROR_STRING 64
#define MPI_COMM_WORLD ((MPI_Comm)1)
#define MPI_INT ((MPI_Datatype)4)
#define MPI_FLOAT ((MPI_Datatype)(0x100 | 4))
#define MPI_DOUBLE ((MPI_Datatype)8)
#define MPI_SUM ((MPI_Op)1)
#define MPI_MAX ((MPI_Op)2)
#define MPI_STATUS_IGNORE ((MPI_Status*)0)

namespace mpi_stub {

struct Comm {
    std::vector<int> members;  // world ranks, in communicator rank order
    int me = -1;               // this process's rank in the communicator
};

struct Msg {
    int comm, tag;
    std::vector<char> data;
};

struct State {
    int rank = 0, size = 1;
    int timeout_s = 600;
    std::vector<int> fd;                   // socket to each world rank (-1: self)
    std::vector<std::deque<Msg>> pending;  // received but not yet matched, per source
    std::vector<Comm> comms;               // index = MPI_Comm handle (0 unused)
};

inline State& st() {
    static State s;
    return s;
}

[[noreturn]] inline void die(const std::string& what) {
    std::fprintf(stderr, "[mpi stub rank %d] %s\n", st().rank, what.c_str());
    std::fflush(stderr);
    std::_Exit(3);
}

inline size_t dsize(MPI_Datatype t) { return (size_t)(t & 0xff); }

inline int env_int(const char* name, int dflt) {
    const char* e = std::getenv(name);
    return e ? std::atoi(e) : dflt;
}

inline void write_all(int fd, const void* p, size_t n) {
    const char* c = static_cast<const char*>(p);
    while (n > 0) {
        ssize_t k = ::send(fd, c, n, MSG_NOSIGNAL);
        if (k < 0 && errno == EINTR) continue;
        if (k <= 0) die(std::string("send failed: ") + std::strerror(errno));
        c += k;
        n -= (size_t)k;
    }
}

inline void read_all(int fd, void* p, size_t n) {
    char* c = static_cast<char*>(p);
    while (n > 0) {
        ssize_t k = ::recv(fd, c, n, 0);
        if (k < 0 && errno == EINTR) continue;
        if (k == 0) die("a peer closed its connection (it exited or aborted)");
        if (k < 0) die(std::string("receive failed or timed out: ") + std::strerror(errno));
        c += k;
        n -= (size_t)k;
    }
}

struct Header {
    int32_t comm, tag;
    int64_t bytes;
};

inline void send_raw(int dst, int comm, int tag, const void* data, size_t bytes) {
    State& s = st();
    if (dst == s.rank) {  // to self: queued locally
        Msg m{comm, tag, std::vector<char>(static_cast<const char*>(data), static_cast<const char*>(data) + bytes)};
        s.pending[dst].push_back(std::move(m));
        return;
    }
    Header h{comm, tag, (int64_t)bytes};
    write_all(s.fd[dst], &h, sizeof(h));
    if (bytes) write_all(s.fd[dst], data, bytes);
}

// Receives the next message from world rank src on (comm, tag) into data
// (at most cap bytes); messages that arrive first on other (comm, tag) pairs
// are queued. Returns the payload size.
inline size_t recv_raw(int src, int comm, int tag, void* data, size_t cap) {
    State& s = st();
    auto& q = s.pending[src];
    for (auto it = q.begin(); it != q.end(); ++it) {
        if (it->comm == comm && it->tag == tag) {
            if (it->data.size() > cap) die("message longer than the receive buffer");
            if (!it->data.empty()) std::memcpy(data, it->data.data(), it->data.size());
            const size_t n = it->data.size();
            q.erase(it);
            return n;
        }
    }
    if (src == s.rank) die("receive from self with no matching send");
    for (;;) {
        Header h{};
        read_all(s.fd[src], &h, sizeof(h));
        if (h.comm == comm && h.tag == tag) {
            if ((size_t)h.bytes > cap) die("message longer than the receive buffer");
            if (h.bytes) read_all(s.fd[src], data, (size_t)h.bytes);
            return (size_t)h.bytes;
        }
        Msg m{h.comm, h.tag, std::vector<char>((size_t)h.bytes)};
        if (h.bytes) read_all(s.fd[src], m.data.data(), (size_t)h.bytes);
        q.push_back(std::move(m));
    }
}

inline const Comm& comm_of(MPI_Comm c) {
    State& s = st();
    if (c < 1 || c >= (int)s.comms.size() || s.comms[c].me < 0) die("invalid communicator");
    return s.comms[c];
}

// internal tags of the collectives (user tags are >= 0)
constexpr int kTagBcast = -1, kTagReduce = -2, kTagGather = -3, kTagBarrier = -4, kTagSplit = -5;

inline void set_timeout(int fd, int seconds) {
    timeval tv{seconds, 0};
    setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
    setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &tv, sizeof(tv));
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
}

// Full mesh of loopback connections: rank r listens on base + r, connects to
// every lower rank and accepts every higher one; a connecting rank first sends
// its rank number.
inline void connect_mesh() {
    State& s = st();
    const int base = env_int("ABFT_MPI_STUB_PORT", env_int("MASTER_PORT", 29500) + 100);
    const char* addr = std::getenv("MASTER_ADDR");
    const std::string host = addr ? addr : "127.0.0.1";
    const int setup_s = s.timeout_s < 120 ? s.timeout_s : 120;  // every rank should start within this
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(setup_s);
    int lfd = ::socket(AF_INET, SOCK_STREAM, 0);
    if (lfd < 0) die("socket");
    int one = 1;
    setsockopt(lfd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in me{};
    me.sin_family = AF_INET;
    me.sin_port = htons((uint16_t)(base + s.rank));
    if (inet_pton(AF_INET, host.c_str(), &me.sin_addr) != 1) die("MASTER_ADDR must be an IPv4 address");
    if (::bind(lfd, reinterpret_cast<sockaddr*>(&me), sizeof(me)) != 0)
        die("bind to port " + std::to_string(base + s.rank) + ": " + std::strerror(errno));
    if (::listen(lfd, s.size) != 0) die("listen");
    for (int q = 0; q < s.rank; ++q) {
        sockaddr_in to{};
        to.sin_family = AF_INET;
        to.sin_port = htons((uint16_t)(base + q));
        if (inet_pton(AF_INET, host.c_str(), &to.sin_addr) != 1) die("MASTER_ADDR must be an IPv4 address");
        for (;;) {
            int fd = ::socket(AF_INET, SOCK_STREAM, 0);
            if (fd < 0) die("socket");
            if (::connect(fd, reinterpret_cast<sockaddr*>(&to), sizeof(to)) == 0) {
                set_timeout(fd, s.timeout_s);
                int32_t r = s.rank;
                write_all(fd, &r, sizeof(r));
                s.fd[q] = fd;
                break;
            }
            ::close(fd);
            if (std::chrono::steady_clock::now() > deadline) die("could not connect to rank " + std::to_string(q));
            std::this_thread::sleep_for(std::chrono::milliseconds(50));
        }
    }
    for (int n = s.rank + 1; n < s.size; ++n) {
        pollfd p{lfd, POLLIN, 0};
        const auto left = std::chrono::duration_cast<std::chrono::milliseconds>(
                              deadline - std::chrono::steady_clock::now()).count();
        if (left <= 0 || ::poll(&p, 1, (int)left) <= 0) die("timed out waiting for higher ranks to connect");
        int fd = ::accept(lfd, nullptr, nullptr);
        if (fd < 0) die("accept");
        set_timeout(fd, s.timeout_s);
        int32_t r = -1;
        read_all(fd, &r, sizeof(r));
        if (r <= s.rank || r >= s.size || s.fd[r] >= 0) die("unexpected peer rank " + std::to_string(r));
        s.fd[r] = fd;
    }
    ::close(lfd);
}

template <class T>
inline void combine(T* acc, const T* in, int n, MPI_Op op) {
    for (int i = 0; i < n; ++i) acc[i] = (op == MPI_SUM) ? acc[i] + in[i] : (in[i] > acc[i] ? in[i] : acc[i]);
}

}  // namespace mpi_stub

inline int MPI_Init(int*, char***) {
    using namespace mpi_stub;
    State& s = st();
    s.size = env_int("WORLD_SIZE", 1);
    s.rank = env_int("RANK", 0);
    s.timeout_s = env_int("ABFT_MPI_STUB_TIMEOUT", 600);
    if (s.size < 1 || s.rank < 0 || s.rank >= s.size) die("bad RANK / WORLD_SIZE");
    s.fd.assign(s.size, -1);
    s.pending.assign(s.size, {});
    s.comms.assign(2, Comm{});
    for (int r = 0; r < s.size; ++r) s.comms[1].members.push_back(r);
    s.comms[1].me = s.rank;
    if (s.size > 1) connect_mesh();
    return MPI_SUCCESS;
}

inline int MPI_Finalize() {
    using namespace mpi_stub;
    for (int& fd : st().fd)
        if (fd >= 0) {
            ::close(fd);
            fd = -1;
        }
    return MPI_SUCCESS;
}

inline int MPI_Comm_rank(MPI_Comm c, int* r) {
    *r = mpi_stub::comm_of(c).me;
    return MPI_SUCCESS;
}

inline int MPI_Comm_size(MPI_Comm c, int* n) {
    *n = (int)mpi_stub::comm_of(c).members.size();
    return MPI_SUCCESS;
}

inline int MPI_Abort(MPI_Comm, int code) {
    std::fprintf(stderr, "MPI_Abort(%d) [mpi stub rank %d]\n", code, mpi_stub::st().rank);
    std::fflush(stderr);
    std::_Exit(code == 0 ? 1 : (code & 0xff ? code & 0xff : 1));
}

inline int MPI_Error_string(int, char* s, int* len) {
    std::snprintf(s, MPI_MAX_ERROR_STRING, "mpi stub error");
    *len = (int)std::strlen(s);
    return MPI_SUCCESS;
}

inline int MPI_Send(const void* buf, int count, MPI_Datatype t, int dest, int tag, MPI_Comm c) {
    const auto& cm = mpi_stub::comm_of(c);
    if (dest < 0 || dest >= (int)cm.members.size() || tag < 0) mpi_stub::die("MPI_Send: bad destination or tag");
    mpi_stub::send_raw(cm.members[dest], c, tag, buf, (size_t)count * mpi_stub::dsize(t));
    return MPI_SUCCESS;
}

inline int MPI_Recv(void* buf, int count, MPI_Datatype t, int source, int tag, MPI_Comm c, MPI_Status* status) {
    const auto& cm = mpi_stub::comm_of(c);
    if (source < 0 || source >= (int)cm.members.size() || tag < 0) mpi_stub::die("MPI_Recv: bad source or tag");
    mpi_stub::recv_raw(cm.members[source], c, tag, buf, (size_t)count * mpi_stub::dsize(t));
    if (status) *status = MPI_Status{source, tag, MPI_SUCCESS};
    return MPI_SUCCESS;
}

inline int MPI_Bcast(void* buf, int count, MPI_Datatype t, int root, MPI_Comm c) {
    const auto& cm = mpi_stub::comm_of(c);
    const size_t bytes = (size_t)count * mpi_stub::dsize(t);
    if (cm.me == root) {
        for (int i = 0; i < (int)cm.members.size(); ++i)
            if (i != root) mpi_stub::send_raw(cm.members[i], c, mpi_stub::kTagBcast, buf, bytes);
    } else {
        mpi_stub::recv_raw(cm.members[root], c, mpi_stub::kTagBcast, buf, bytes);
    }
    return MPI_SUCCESS;
}

inline int MPI_Reduce(const void* in, void* out, int n, MPI_Datatype t, MPI_Op op, int root, MPI_Comm c) {
    using namespace mpi_stub;
    const auto& cm = comm_of(c);
    const size_t bytes = (size_t)n * dsize(t);
    if (op != MPI_SUM && op != MPI_MAX) die("MPI_Reduce: only MPI_SUM and MPI_MAX");
    if (cm.me != root) {
        send_raw(cm.members[root], c, kTagReduce, in, bytes);
        return MPI_SUCCESS;
    }
    // rank order: start from rank 0's contribution, fold in 1, 2, ...
    std::vector<char> acc(bytes), part(bytes);
    for (int i = 0; i < (int)cm.members.size(); ++i) {
        if (i == root) std::memcpy(part.data(), in, bytes);
        else recv_raw(cm.members[i], c, kTagReduce, part.data(), bytes);
        if (i == 0) {
            acc = part;
            continue;
        }
        if (t == MPI_INT) combine(reinterpret_cast<int*>(acc.data()), reinterpret_cast<const int*>(part.data()), n, op);
        else if (t == MPI_FLOAT)
            combine(reinterpret_cast<float*>(acc.data()), reinterpret_cast<const float*>(part.data()), n, op);
        else if (t == MPI_DOUBLE)
            combine(reinterpret_cast<double*>(acc.data()), reinterpret_cast<const double*>(part.data()), n, op);
        else die("MPI_Reduce: unsupported datatype");
    }
    if (bytes) std::memcpy(out, acc.data(), bytes);
    return MPI_SUCCESS;
}

inline int MPI_Gatherv(const void* in, int n, MPI_Datatype t, void* out, const int* counts, const int* displs,
                       MPI_Datatype, int root, MPI_Comm c) {
    using namespace mpi_stub;
    const auto& cm = comm_of(c);
    const size_t es = dsize(t);
    if (cm.me != root) {
        send_raw(cm.members[root], c, kTagGather, in, (size_t)n * es);
        return MPI_SUCCESS;
    }
    for (int i = 0; i < (int)cm.members.size(); ++i) {
        char* dst = static_cast<char*>(out) + (size_t)displs[i] * es;
        if (i == root) {
            if (n) std::memcpy(dst, in, (size_t)n * es);
        } else {
            recv_raw(cm.members[i], c, kTagGather, dst, (size_t)counts[i] * es);
        }
    }
    return MPI_SUCCESS;
}

inline int MPI_Gather(const void* in, int n, MPI_Datatype t, void* out, int rn, MPI_Datatype rt, int root,
                      MPI_Comm c) {
    const int size = (int)mpi_stub::comm_of(c).members.size();
    std::vector<int> counts(size, rn), displs(size);
    for (int i = 0; i < size; ++i) displs[i] = i * rn;
    return MPI_Gatherv(in, n, t, out, counts.data(), displs.data(), rt, root, c);
}

inline int MPI_Barrier(MPI_Comm c) {
    using namespace mpi_stub;
    const auto& cm = comm_of(c);
    char token = 0;
    if (cm.me == 0) {
        for (int i = 1; i < (int)cm.members.size(); ++i) recv_raw(cm.members[i], c, kTagBarrier, &token, 1);
        for (int i = 1; i < (int)cm.members.size(); ++i) send_raw(cm.members[i], c, kTagBarrier, &token, 1);
    } else {
        send_raw(cm.members[0], c, kTagBarrier, &token, 1);
        recv_raw(cm.members[0], c, kTagBarrier, &token, 1);
    }
    return MPI_SUCCESS;
}

// Collective over the parent: every member sends (color, key) to the
// parent's rank 0, which answers each with the world ranks of its new
// communicator in (key, parent rank) order. The new handle is the next free
// index, the same in every process because splits are called collectively in
// the same order.
inline int MPI_Comm_split(MPI_Comm parent, int color, int key, MPI_Comm* out) {
    using namespace mpi_stub;
    State& s = st();
    const Comm pc = comm_of(parent);
    const int handle = (int)s.comms.size();
    s.comms.push_back(Comm{});
    const int np = (int)pc.members.size();
    int32_t ck[2] = {color, key};
    std::vector<int32_t> mine;
    if (pc.me == 0) {
        std::vector<int32_t> all(2 * (size_t)np);
        for (int i = 0; i < np; ++i) {
            if (i == 0) std::memcpy(&all[0], ck, sizeof(ck));
            else recv_raw(pc.members[i], parent, kTagSplit, &all[2 * (size_t)i], sizeof(ck));
        }
        for (int i = 0; i < np; ++i) {
            std::vector<int> same;
            for (int j = 0; j < np; ++j)
                if (all[2 * (size_t)j] == all[2 * (size_t)i]) same.push_back(j);
            // stable order by key, ties by parent rank
            for (size_t a = 1; a < same.size(); ++a)
                for (size_t b = a; b > 0 && all[2 * (size_t)same[b] + 1] < all[2 * (size_t)same[b - 1] + 1]; --b)
                    std::swap(same[b], same[b - 1]);
            std::vector<int32_t> world(same.size());
            for (size_t k = 0; k < same.size(); ++k) world[k] = pc.members[same[k]];
            if (i == 0) mine = world;
            else send_raw(pc.members[i], parent, kTagSplit, world.data(), world.size() * sizeof(int32_t));
        }
    } else {
        send_raw(pc.members[0], parent, kTagSplit, ck, sizeof(ck));
        std::vector<int32_t> buf((size_t)np);
        const size_t got = recv_raw(pc.members[0], parent, kTagSplit, buf.data(), buf.size() * sizeof(int32_t));
        mine.assign(buf.begin(), buf.begin() + (long)(got / sizeof(int32_t)));
    }
    Comm& nc = s.comms[handle];
    nc.members.assign(mine.begin(), mine.end());
    for (size_t k = 0; k < nc.members.size(); ++k)
        if (nc.members[k] == s.rank) nc.me = (int)k;
    if (nc.me < 0) die("MPI_Comm_split: this rank is missing from its new communicator");
    *out = handle;
    return MPI_SUCCESS;
}

inline int MPI_Comm_free(MPI_Comm* c) {
    *c = 0;
    return MPI_SUCCESS;
}

#endif
