// Candidate sharding across GPUs: one NCCL communicator per context, one process per GPU.
//
// The planners' candidates are independent rows, so a level's solve runs rank-locally on a contiguous
// slice of them; only these small exchanges cross NVLink per level (none inside the Adam loop unless
// early stopping needs the global minimum cost):
//   min_f32        the global minimum of one float (early stopping)
//   argmin_global  (cost, global index) of every rank -> the lowest cost, lowest index on ties, and
//                  the rank that holds it (one ncclAllGather of 8 bytes per rank)
//   bcast_host     the winning plan from its owner to every rank
//   allgather_f32  every rank's per-candidate values (the CEM energies)
//
// Failure handling. The communicator is created non-blocking (ncclCommInitRankConfig, blocking = 0), and
// every NCCL call and every wait for a collective to finish is bounded on the host by `timeout_ms`
// (JEPA_B200_NCCL_TIMEOUT_MS, default 120 s). A rank that never joins, a peer that died, or an NCCL
// error ends the wait: the communicator is aborted (ncclCommAbort, which also ends collectives still in
// flight on this GPU), the call logs the reason and returns false, and the planner returns -1. Every
// later collective on an aborted shard fails at once, so ranks never wait on a communicator that is gone.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <cstddef>

namespace jb {

struct Shard {
    int rank = 0, world = 1, device = 0;
    ncclComm_t comm = nullptr;
    int * dbuf = nullptr;     // 2 + 2 * world ints of device scratch for the small collectives
    long long timeout_ms = 120000;
    bool aborted = false;

    ~Shard();
    // creates the communicator (rank `rank` of `world`) and waits, bounded, until every rank has joined
    bool init(const void * nccl_id128);
    bool min_f32(float v, float * out, cudaStream_t st);
    bool argmin_global(float cost, int gidx, float * cost_out, int * gidx_out, int * owner, cudaStream_t st);
    bool bcast_host(float * host, size_t n, int root, cudaStream_t st);
    // every rank's n device floats, in rank order, into recv [world * n] on every rank; enqueued on st
    // (the caller's later kernels on st consume it; finish() bounds the wait for it)
    bool allgather_f32(const float * send, float * recv, size_t n, cudaStream_t st);
    // waits (bounded) until the work enqueued on st, collectives included, has finished
    bool finish(cudaStream_t st, const char * what);

  private:
    bool settle(ncclResult_t r, const char * what);   // an NCCL call's result, waited out when in progress
    void abort(const char * why);
};

}  // namespace jb
