// NCCL plumbing of the candidate sharding (see shard.h) and the jepa_b200_* sharding entry points.
#include "shard.h"
#include "common.h"
#include "model.h"
#include "hplan.h"
#include "ac.h"

#include "../../include/jepa_b200.h"

#include <cmath>
#include <cstring>
#include <vector>

namespace jb {

namespace {
bool nccl_ok(ncclResult_t r, const char * what) {
    if (r == ncclSuccess) return true;
    log("jepa: NCCL error in %s: %s\n", what, ncclGetErrorString(r));
    return false;
}
}  // namespace

Shard::~Shard() {
    if (comm) ncclCommDestroy(comm);
    if (dbuf) cudaFree(dbuf);
}

float Shard::min_f32(float v, cudaStream_t st) {
    float * d = (float *) dbuf;
    cudaMemcpyAsync(d, &v, 4, cudaMemcpyHostToDevice, st);
    nccl_ok(ncclAllReduce(d, d, 1, ncclFloat, ncclMin, comm, st), "ncclAllReduce(min)");
    float out = v;
    cudaMemcpyAsync(&out, d, 4, cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    return out;
}

void Shard::argmin_global(float cost, int gidx, float * cost_out, int * gidx_out, int * owner, cudaStream_t st) {
    int mine[2];
    memcpy(&mine[0], &cost, 4);
    mine[1] = gidx;
    std::vector<int> all((size_t) 2 * world);
    cudaMemcpyAsync(dbuf, mine, 8, cudaMemcpyHostToDevice, st);
    nccl_ok(ncclAllGather(dbuf, dbuf + 2, 2, ncclInt32, comm, st), "ncclAllGather(argmin)");
    cudaMemcpyAsync(all.data(), dbuf + 2, (size_t) 8 * world, cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    float best = INFINITY;
    int bi = -1, br = 0;
    for (int r = 0; r < world; r++) {
        float c;
        memcpy(&c, &all[(size_t) 2 * r], 4);
        const int i = all[(size_t) 2 * r + 1];
        if (bi < 0 || c < best || (c == best && i < bi)) { best = c; bi = i; br = r; }
    }
    *cost_out = best;
    *gidx_out = bi;
    *owner = br;
}

bool Shard::bcast_host(float * host, size_t n, int root, cudaStream_t st) {
    float * d = nullptr;
    if (!cuda_ok(cudaMalloc(&d, n * 4), "broadcast buffer")) return false;
    bool ok = cuda_ok(cudaMemcpyAsync(d, host, n * 4, cudaMemcpyHostToDevice, st), "broadcast") &&
              nccl_ok(ncclBroadcast(d, d, n, ncclFloat, root, comm, st), "ncclBroadcast") &&
              cuda_ok(cudaMemcpyAsync(host, d, n * 4, cudaMemcpyDeviceToHost, st), "broadcast") &&
              cuda_ok(cudaStreamSynchronize(st), "broadcast");
    cudaFree(d);
    return ok;
}

bool Shard::allgather_f32(const float * send, float * recv, size_t n, cudaStream_t st) {
    return nccl_ok(ncclAllGather(send, recv, n, ncclFloat, comm, st), "ncclAllGather(energy)");
}

}  // namespace jb

extern "C" int jepa_b200_nccl_unique_id(void * out128) {
    if (!out128) return -1;
    ncclUniqueId id;
    if (!jb::nccl_ok(ncclGetUniqueId(&id), "ncclGetUniqueId")) return -1;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out128, &id, sizeof(id));
    return 0;
}

extern "C" int jepa_b200_context_set_shard(jepa_context * ctx, int rank, int world, const void * nccl_id) {
    if (!ctx || world < 1 || rank < 0 || rank >= world) return -1;
    ctx->shard.reset();
    ctx->hplan.reset();   // workspaces are sized for the rank's slice
    ctx->ac.reset();
    if (world == 1) return 0;
    if (!nccl_id) return -1;
    cudaSetDevice(ctx->device);
    auto sh = std::make_unique<jb::Shard>();
    sh->rank = rank;
    sh->world = world;
    sh->device = ctx->device;
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    if (!jb::nccl_ok(ncclCommInitRank(&sh->comm, world, id, rank), "ncclCommInitRank")) return -1;
    if (!jb::cuda_ok(cudaMalloc(&sh->dbuf, sizeof(int) * (size_t) (2 + 2 * world)), "shard buffer")) return -1;
    ctx->shard = std::move(sh);
    return 0;
}
