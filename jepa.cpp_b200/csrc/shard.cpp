// NCCL plumbing of the candidate sharding (see shard.h) and the jepa_b200_* sharding entry points.
#include "shard.h"
#include "common.h"
#include "model.h"
#include "hplan.h"
#include "ac.h"

#include "../../include/jepa_b200.h"

#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

namespace jb {

namespace {
bool nccl_ok(ncclResult_t r, const char * what) {
    if (r == ncclSuccess) return true;
    log("jepa: NCCL error in %s: %s\n", what, ncclGetErrorString(r));
    return false;
}

using Clock = std::chrono::steady_clock;

long long env_timeout_ms() {
    const char * v = getenv("JEPA_B200_NCCL_TIMEOUT_MS");
    if (!v || !*v) return 120000;
    const long long t = atoll(v);
    return t > 0 ? t : 120000;
}
}  // namespace

Shard::~Shard() {
    if (comm) {
        if (aborted || ncclCommDestroy(comm) != ncclSuccess) ncclCommAbort(comm);
    }
    if (dbuf) cudaFree(dbuf);
}

void Shard::abort(const char * why) {
    log("jepa: shard rank %d of %d: %s; aborting the NCCL communicator\n", rank, world, why);
    if (comm && !aborted) ncclCommAbort(comm);
    comm = nullptr;
    aborted = true;
}

bool Shard::settle(ncclResult_t r, const char * what) {
    if (aborted || !comm) { log("jepa: %s: the NCCL communicator was aborted earlier\n", what); return false; }
    if (r != ncclSuccess && r != ncclInProgress) {
        log("jepa: NCCL error in %s: %s\n", what, ncclGetErrorString(r));
        abort(what);
        return false;
    }
    const auto t0 = Clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) st = ncclSystemError;
        if (st == ncclSuccess) return true;
        if (st != ncclInProgress) {
            log("jepa: NCCL error in %s: %s\n", what, ncclGetErrorString(st));
            abort(what);
            return false;
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > timeout_ms) {
            log("jepa: %s did not complete within %lld ms (a rank that never joined or stopped?)\n", what, timeout_ms);
            abort(what);
            return false;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

bool Shard::finish(cudaStream_t st, const char * what) {
    if (aborted || !comm) { log("jepa: %s: the NCCL communicator was aborted earlier\n", what); return false; }
    const auto t0 = Clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return true;
        if (q != cudaErrorNotReady) { cuda_ok(q, what); abort(what); return false; }
        ncclResult_t ae = ncclSuccess;
        if (ncclCommGetAsyncError(comm, &ae) == ncclSuccess && ae != ncclSuccess && ae != ncclInProgress) {
            log("jepa: NCCL error in %s: %s\n", what, ncclGetErrorString(ae));
            abort(what);
            return false;
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > timeout_ms) {
            log("jepa: %s did not finish within %lld ms (a peer that stopped?)\n", what, timeout_ms);
            abort(what);
            return false;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

bool Shard::init(const void * nccl_id128) {
    timeout_ms = env_timeout_ms();
    ncclUniqueId id;
    memcpy(&id, nccl_id128, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        log("jepa: NCCL error in ncclCommInitRankConfig: %s\n", ncclGetErrorString(r));
        if (comm) ncclCommAbort(comm);
        comm = nullptr;
        aborted = true;
        return false;
    }
    if (!comm) { log("jepa: ncclCommInitRankConfig returned no communicator\n"); aborted = true; return false; }
    if (!settle(ncclSuccess, "joining the NCCL communicator")) return false;
    return cuda_ok(cudaMalloc(&dbuf, sizeof(int) * (size_t) (2 + 2 * world)), "shard buffer");
}

bool Shard::min_f32(float v, float * out, cudaStream_t st) {
    float * d = (float *) dbuf;
    *out = v;
    if (!cuda_ok(cudaMemcpyAsync(d, &v, 4, cudaMemcpyHostToDevice, st), "min_f32")) return false;
    if (!settle(ncclAllReduce(d, d, 1, ncclFloat, ncclMin, comm, st), "ncclAllReduce(min)")) return false;
    if (!cuda_ok(cudaMemcpyAsync(out, d, 4, cudaMemcpyDeviceToHost, st), "min_f32")) return false;
    return finish(st, "ncclAllReduce(min)");
}

bool Shard::argmin_global(float cost, int gidx, float * cost_out, int * gidx_out, int * owner, cudaStream_t st) {
    int mine[2];
    memcpy(&mine[0], &cost, 4);
    mine[1] = gidx;
    std::vector<int> all((size_t) 2 * world);
    if (!cuda_ok(cudaMemcpyAsync(dbuf, mine, 8, cudaMemcpyHostToDevice, st), "argmin")) return false;
    if (!settle(ncclAllGather(dbuf, dbuf + 2, 2, ncclInt32, comm, st), "ncclAllGather(argmin)")) return false;
    if (!cuda_ok(cudaMemcpyAsync(all.data(), dbuf + 2, (size_t) 8 * world, cudaMemcpyDeviceToHost, st), "argmin")) return false;
    if (!finish(st, "ncclAllGather(argmin)")) return false;
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
    return true;
}

bool Shard::bcast_host(float * host, size_t n, int root, cudaStream_t st) {
    float * d = nullptr;
    if (!cuda_ok(cudaMalloc(&d, n * 4), "broadcast buffer")) return false;
    bool ok = cuda_ok(cudaMemcpyAsync(d, host, n * 4, cudaMemcpyHostToDevice, st), "broadcast") &&
              settle(ncclBroadcast(d, d, n, ncclFloat, root, comm, st), "ncclBroadcast") &&
              cuda_ok(cudaMemcpyAsync(host, d, n * 4, cudaMemcpyDeviceToHost, st), "broadcast") &&
              finish(st, "ncclBroadcast");
    if (ok) cudaFree(d);   // an aborted exchange may leave the buffer in use: kept then
    return ok;
}

bool Shard::allgather_f32(const float * send, float * recv, size_t n, cudaStream_t st) {
    return settle(ncclAllGather(send, recv, n, ncclFloat, comm, st), "ncclAllGather(energy)");
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
    if (!sh->init(nccl_id)) return -1;
    ctx->shard = std::move(sh);
    return 0;
}
