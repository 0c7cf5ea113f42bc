// Candidate sharding across GPUs: one NCCL communicator per context, one process per GPU.
//
// The planners' candidates are independent rows, so a level's solve runs rank-locally on a contiguous
// slice of them; only these small exchanges cross NVLink per level (none inside the Adam loop unless
// early stopping needs the global minimum cost):
//   min_f32        the global minimum of one float (early stopping)
//   argmin_global  (cost, global index) of every rank -> the lowest cost, lowest index on ties, and
//                  the rank that holds it (one ncclAllGather of 8 bytes per rank)
//   bcast_host     the winning plan from its owner to every rank
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <cstddef>

namespace jb {

struct Shard {
    int rank = 0, world = 1, device = 0;
    ncclComm_t comm = nullptr;
    int * dbuf = nullptr;     // 2 * world ints of device scratch for the small collectives
    ~Shard();
    float min_f32(float v, cudaStream_t st);
    void argmin_global(float cost, int gidx, float * cost_out, int * gidx_out, int * owner, cudaStream_t st);
    bool bcast_host(float * host, size_t n, int root, cudaStream_t st);
    // every rank's n device floats, in rank order, into recv [world * n] on every rank (CEM energies)
    bool allgather_f32(const float * send, float * recv, size_t n, cudaStream_t st);
};

}  // namespace jb
