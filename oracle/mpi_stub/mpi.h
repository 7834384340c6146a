/*
 * Single-rank stand-in for the few MPI calls the reference driver makes.
 *
 * TEST INFRASTRUCTURE ONLY. This header exists so that the reference's own
 * sources (main.cu, core/, distribution/, kernels/, pipeline/, metrics/) can be
 * compiled unmodified for sm_100a in an image that has no MPI installation.
 * The result is a ONE-rank build: MPI_COMM_WORLD has size 1, collectives copy
 * their send buffer to the receive buffer, point-to-point calls abort (the
 * reference never issues them with one rank: distribution/grid.cuh:31-58 and
 * :61-91 only Send/Recv between distinct ranks).
 *
 * It is compiled only by oracle/Makefile into oracle/_ref/ and is never part of
 * the shipped library.
 */
#ifndef ABFT_ORACLE_MPI_STUB_H
#define ABFT_ORACLE_MPI_STUB_H

#include <cstdio>
#include <cstdlib>
#include <cstring>

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

static inline size_t mpi_stub_size(MPI_Datatype t) { return (size_t)(t & 0xff); }

static inline int MPI_Init(int*, char***) { return MPI_SUCCESS; }
static inline int MPI_Finalize() { return MPI_SUCCESS; }
static inline int MPI_Comm_rank(MPI_Comm, int* r) { *r = 0; return MPI_SUCCESS; }
static inline int MPI_Comm_size(MPI_Comm, int* s) { *s = 1; return MPI_SUCCESS; }
static inline int MPI_Comm_split(MPI_Comm, int, int, MPI_Comm* out) { *out = 2; return MPI_SUCCESS; }
static inline int MPI_Comm_free(MPI_Comm*) { return MPI_SUCCESS; }
static inline int MPI_Barrier(MPI_Comm) { return MPI_SUCCESS; }
static inline int MPI_Abort(MPI_Comm, int code) {
    std::fprintf(stderr, "MPI_Abort(%d) [single-rank stub]\n", code);
    std::exit(code == 0 ? 1 : (code & 0xff ? code & 0xff : 1));
}
static inline int MPI_Error_string(int, char* s, int* len) {
    std::snprintf(s, MPI_MAX_ERROR_STRING, "mpi stub error");
    *len = (int)std::strlen(s);
    return MPI_SUCCESS;
}
static inline int MPI_Bcast(void*, int, MPI_Datatype, int, MPI_Comm) { return MPI_SUCCESS; }
static inline int MPI_Reduce(const void* in, void* out, int n, MPI_Datatype t, MPI_Op, int, MPI_Comm) {
    std::memcpy(out, in, (size_t)n * mpi_stub_size(t));
    return MPI_SUCCESS;
}
static inline int MPI_Gather(const void* in, int n, MPI_Datatype t, void* out, int, MPI_Datatype, int, MPI_Comm) {
    std::memcpy(out, in, (size_t)n * mpi_stub_size(t));
    return MPI_SUCCESS;
}
static inline int MPI_Gatherv(const void* in, int n, MPI_Datatype t, void* out, const int*, const int*,
                              MPI_Datatype, int, MPI_Comm) {
    if (out && n > 0) std::memcpy(out, in, (size_t)n * mpi_stub_size(t));
    return MPI_SUCCESS;
}
static inline int MPI_Send(const void*, int, MPI_Datatype, int, int, MPI_Comm) {
    std::fprintf(stderr, "MPI_Send is not available in the single-rank stub\n");
    std::exit(3);
}
static inline int MPI_Recv(void*, int, MPI_Datatype, int, int, MPI_Comm, MPI_Status*) {
    std::fprintf(stderr, "MPI_Recv is not available in the single-rank stub\n");
    std::exit(3);
}

#endif
