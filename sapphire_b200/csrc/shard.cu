// shard.cu - row sharding of weights across GPUs (one process per GPU).
//
// The reference is single-process CPU code with no communication backend; the
// design here splits the output rows of every weight over `world` ranks and
// gathers the row slices with an NCCL all-gather over NVLink.
//
// NCCL is opened with dlopen on first use, not linked: an unsharded process
// never loads it, and a process that already loaded an NCCL (e.g. the one
// bundled with PyTorch) reuses that copy instead of pinning a second one.
#include <cstring>
#include <dlfcn.h>
#include <mutex>
#include <nccl.h>

#include "internal.cuh"

namespace {
struct NcclApi {
    bool ok = false;
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    const char *(*getErrorString)(ncclResult_t) = nullptr;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            LOG_ERROR("cannot load NCCL: %s", dlerror());
            return;
        }
        api.getUniqueId = (decltype(api.getUniqueId))dlsym(h, "ncclGetUniqueId");
        api.commInitRank = (decltype(api.commInitRank))dlsym(h, "ncclCommInitRank");
        api.allGather = (decltype(api.allGather))dlsym(h, "ncclAllGather");
        api.commDestroy = (decltype(api.commDestroy))dlsym(h, "ncclCommDestroy");
        api.getErrorString = (decltype(api.getErrorString))dlsym(h, "ncclGetErrorString");
        api.ok = api.getUniqueId && api.commInitRank && api.allGather && api.commDestroy && api.getErrorString;
        if (!api.ok) LOG_ERROR("NCCL library lacks an expected entry point");
    });
    return api;
}
}  // namespace

extern "C" SAPPHIRE_API int kernel_shard_unique_id(void *id_out) {
    if (!id_out) return -1;
    const NcclApi &api = nccl();
    if (!api.ok) return -1;
    ncclUniqueId id;
    ncclResult_t r = api.getUniqueId(&id);
    if (r != ncclSuccess) {
        LOG_ERROR("kernel_shard_unique_id: ncclGetUniqueId failed: %s", api.getErrorString(r));
        return -1;
    }
    static_assert(sizeof(ncclUniqueId) == SAPPHIRE_UNIQUE_ID_BYTES, "NCCL unique id size");
    memcpy(id_out, &id, sizeof id);
    return 0;
}

extern "C" SAPPHIRE_API int kernel_ctx_init_sharded(kernel_context_t *ctx, int rank, int world_size,
                                                    const void *unique_id) {
    if (!ctx || world_size < 1 || rank < 0 || rank >= world_size) {
        LOG_ERROR("kernel_ctx_init_sharded: bad arguments (rank %d, world %d)", rank, world_size);
        return -1;
    }
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (!ctx->initialized) {
        ctx_fail(ctx, "kernel_ctx_init_sharded", "context not initialized");
        return -1;
    }
    if (!ctx->weights.empty()) {
        ctx_fail(ctx, "kernel_ctx_init_sharded", "shard before uploading any weight");
        return -1;
    }
    if (ctx->nccl_comm) {
        ctx_fail(ctx, "kernel_ctx_init_sharded", "context is already sharded");
        return -1;
    }
    if (world_size == 1) {
        ctx->rank = 0;
        ctx->world = 1;
        return 0;
    }
    if (!unique_id) {
        ctx_fail(ctx, "kernel_ctx_init_sharded", "unique id is NULL");
        return -1;
    }
    const NcclApi &api = nccl();
    if (!api.ok) {
        ctx_fail(ctx, "kernel_ctx_init_sharded", "NCCL is not available");
        return -1;
    }
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof id);
    ncclComm_t comm = nullptr;
    ncclResult_t r = api.commInitRank(&comm, world_size, id, rank);
    if (prev >= 0) cudaSetDevice(prev);
    if (r != ncclSuccess) {
        ctx_fail(ctx, "kernel_ctx_init_sharded", "ncclCommInitRank failed: %s", api.getErrorString(r));
        return -1;
    }
    ctx->nccl_comm = comm;
    ctx->rank = rank;
    ctx->world = world_size;
    return 0;
}

extern "C" SAPPHIRE_API int kernel_ctx_shard_info(kernel_context_t *ctx, int *rank, int *world_size) {
    if (!ctx) return -1;
    if (rank) *rank = ctx->rank;
    if (world_size) *world_size = ctx->world;
    return 0;
}

extern "C" SAPPHIRE_API int sapphire_shard_rows(int rows, int rank, int world_size, int *row0, int *nrows) {
    if (rows < 0 || world_size < 1 || rank < 0 || rank >= world_size || !row0 || !nrows) return -1;
    shard_rows(rows, rank, world_size, row0, nrows);
    return 0;
}

int shard_allgather(kernel_context_t *ctx, const float *send, float *recv, size_t count, cudaStream_t stream) {
    if (!ctx->nccl_comm) {
        ctx_fail(ctx, "shard_allgather", "context has no communicator");
        return -1;
    }
    const NcclApi &api = nccl();
    ncclResult_t r = api.allGather(send, recv, count, ncclFloat, (ncclComm_t)ctx->nccl_comm, stream);
    if (r != ncclSuccess) {
        ctx_fail(ctx, "shard_allgather", "ncclAllGather failed: %s", api.getErrorString(r));
        return -1;
    }
    return 0;
}

void shard_destroy(kernel_context_t *ctx) {
    if (ctx->nccl_comm) {
        nccl().commDestroy((ncclComm_t)ctx->nccl_comm);
        ctx->nccl_comm = nullptr;
    }
    ctx->rank = 0;
    ctx->world = 1;
}
