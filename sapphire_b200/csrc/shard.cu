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
#include <vector>
#include <mutex>
#include <nccl.h>

#include "internal.cuh"

namespace {
struct NcclApi {
    bool ok = false;
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
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
        api.allReduce = (decltype(api.allReduce))dlsym(h, "ncclAllReduce");
        api.commDestroy = (decltype(api.commDestroy))dlsym(h, "ncclCommDestroy");
        api.getErrorString = (decltype(api.getErrorString))dlsym(h, "ncclGetErrorString");
        api.ok = api.getUniqueId && api.commInitRank && api.allGather && api.allReduce && api.commDestroy &&
                  api.getErrorString;
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

// ---------------------------------------------------- peer-memory gather --
// A row-sharded batch-1 product gathered without NCCL, in the manner of a
// low-latency protocol: the GEMV of every rank sends each finished row to all
// ranks as one 8-byte word (value | epoch << 32) over NVLink; an aligned
// 8-byte store arrives whole, so a word carrying the current epoch holds the
// current value and no fence or barrier is needed.  ll_pull_kernel then waits
// for each word of the rank's own buffer to carry the epoch (bounded by time;
// one that expires sets bit 3 of *err and leaves NaN) and writes the values to
// y.  Two buffers alternate by epoch parity: a rank writes the buffer of epoch
// e + 2 only after its pull of e + 1, which waited for every rank's GEMV of
// e + 1, which each rank started after its own pull of epoch e had finished.
namespace {
constexpr unsigned long long kPeerWaitNs = 2000000000ull;
constexpr int kPullThreads = 256;

// Waits are bounded by time (wait_ns per word, restarted while words keep
// arriving); the first expiry in a block sets bit 3 of *err and a block-wide
// flag, after which the block's threads stop waiting and store NaN for every
// word that is still stale.
__global__ void __launch_bounds__(kPullThreads) ll_pull_kernel(const unsigned long long *ll, long long rows,
                                                               unsigned epoch, float *y, int *err,
                                                               unsigned long long wait_ns) {
    __shared__ int s_expired;
    if (threadIdx.x == 0) s_expired = 0;
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < rows; i += stride) {
        unsigned long long w;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(ll + i) : "memory");
        if ((unsigned)(w >> 32) != epoch) {
            uint64_t t0;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
            for (;;) {
                if (*reinterpret_cast<volatile int *>(&s_expired)) {
                    w = 0x7FC00000ull;   // NaN
                    break;
                }
                __nanosleep(64);
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(ll + i) : "memory");
                if ((unsigned)(w >> 32) == epoch) break;
                uint64_t t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (t - t0 > wait_ns) {
                    atomicOr(err, 8);
                    s_expired = 1;
                    w = 0x7FC00000ull;   // NaN
                    break;
                }
            }
        }
        y[i] = __uint_as_float((unsigned)(w & 0xFFFFFFFFull));
    }
}

int nccl_allgather_bytes(kernel_context_t *ctx, const void *mine, void *all, size_t bytes) {
    uint8_t *d = nullptr;
    CUDA_TRY(ctx, cudaMalloc(&d, bytes * (ctx->world + 1)));
    int rc = -1;
    do {
        if (cudaMemcpy(d, mine, bytes, cudaMemcpyHostToDevice) != cudaSuccess) break;
        if (nccl().allGather(d, d + bytes, bytes, ncclUint8, (ncclComm_t)ctx->nccl_comm, ctx->stream) != ncclSuccess)
            break;
        if (cudaMemcpyAsync(all, d + bytes, bytes * ctx->world, cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess)
            break;
        if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) break;
        rc = 0;
    } while (false);
    cudaFree(d);
    cudaGetLastError();
    return rc;
}

// Collective mapping of one device allocation per rank into every rank.
int map_buffers(kernel_context_t *ctx, size_t bytes, void **local, void **peers) {
    for (int k = 0; k < kMaxPeers; ++k) peers[k] = nullptr;
    *local = nullptr;
    if (ctx->world > kMaxPeers) return -1;
    int ok = 1;
    cudaIpcMemHandle_t mine{};
    if (cudaMalloc(local, bytes) != cudaSuccess || cudaMemset(*local, 0, bytes) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&mine, *local) != cudaSuccess)
        ok = 0;
    cudaGetLastError();
    std::vector<cudaIpcMemHandle_t> all(ctx->world);
    if (nccl_allgather_bytes(ctx, &mine, all.data(), sizeof mine)) return -1;
    for (int k = 0; k < ctx->world && ok; ++k) {
        if (k == ctx->rank) {
            peers[k] = *local;
        } else if (cudaIpcOpenMemHandle(&peers[k], all[k], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            peers[k] = nullptr;
            ok = 0;
        }
    }
    cudaGetLastError();
    std::vector<int> oks(ctx->world, 0);
    if (nccl_allgather_bytes(ctx, &ok, oks.data(), sizeof ok)) return -1;
    for (int v : oks)
        if (v != 1) return -1;
    return 0;
}

// Collective: every rank of the group calls it at the same product.  The
// gather is used only if every rank mapped every peer (agreed over NCCL).
void peer_gather_setup(kernel_context_t *ctx) {
    PeerGather *g = new PeerGather();
    ctx->pg = g;
    g->tried = true;
    if (ctx->world > kMaxPeers) return;
    g->cap_rows = (size_t)4 << 20;   // y of up to 4M rows; 2 x 32 MB per rank
    const size_t bytes = 2 * g->cap_rows * sizeof(unsigned long long);
    int ok = 1;
    cudaIpcMemHandle_t mine{};
    if (cudaMalloc(&g->local, bytes) != cudaSuccess || cudaMemset(g->local, 0, bytes) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&mine, g->local) != cudaSuccess)
        ok = 0;
    cudaGetLastError();
    std::vector<cudaIpcMemHandle_t> all(ctx->world);
    if (nccl_allgather_bytes(ctx, &mine, all.data(), sizeof mine)) return;   // no agreement possible: NCCL path
    for (int k = 0; k < ctx->world && ok; ++k) {
        if (k == ctx->rank) {
            g->peer[k] = g->local;
        } else if (cudaIpcOpenMemHandle(reinterpret_cast<void **>(&g->peer[k]), all[k],
                                        cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            g->peer[k] = nullptr;
            ok = 0;
        }
    }
    cudaGetLastError();
    // Every rank must agree (a mixed decision would leave ranks waiting on
    // each other): AND of the ranks' results.
    std::vector<int> oks(ctx->world, 0);
    if (nccl_allgather_bytes(ctx, &ok, oks.data(), sizeof ok)) return;
    bool all_ok = true;
    for (int v : oks) all_ok = all_ok && v == 1;
    g->ready = all_ok;
    if (!all_ok) LOG_WARN("peer-memory gather unavailable; sharded products use NCCL");
}
}  // namespace

bool shard_peer_product(kernel_context_t *ctx, const DevWeight &w, const float *x, float *Y, int rows, int per,
                        bool y_on_dev, int *rc) {
    *rc = 0;
    // The decision depends only on arguments every rank shares (the pipelined
    // kernel is used on every rank, whatever its local row count).
    if (ctx->world > kMaxPeers || (size_t)per * ctx->world > ((size_t)4 << 20) || !pipe_supported(ctx, w)) return false;
    if (!ctx->pg) peer_gather_setup(ctx);
    PeerGather &g = *ctx->pg;
    if (!g.ready || (size_t)per * ctx->world > g.cap_rows) return false;
    *rc = -1;
    cudaStream_t st = ctx->stream;
    const unsigned epoch = ++g.epoch;
    const size_t buf = (size_t)(epoch & 1u) * g.cap_rows;
    float *yd = Y;
    if (!y_on_dev) {
        if (ensure_scratch(ctx, &ctx->d_y, &ctx->d_y_cap, (size_t)rows * sizeof(float))) return true;
        yd = ctx->d_y;
    }
    GatherArgs ga{};
    for (int k = 0; k < ctx->world; ++k) ga.targets[k] = g.peer[k] + buf;
    ga.n = ctx->world;
    ga.row_off = w.row0;
    ga.epoch = epoch;
    ga.self = g.local + buf;
    ga.y_full = yd;
    ga.rows_full = rows;
    ga.wait_ns = kPeerWaitNs;
    size_t pf = 0, ci = 0;
    pipe_scratch_size(ctx, w, &pf, &ci);
    if (ensure_pipe_scratch(ctx, pf, ci)) return true;
    // The streaming kernel gathers y itself once its warps are done; a rank
    // with no rows, or the dense kernel, leaves the gather to a pull kernel.
    bool gathered = false;
    if (w.ntiles > 0 && launch_gemv_pipe_ll(ctx, w, x, nullptr, ctx->d_part, ctx->d_cnt, ctx->d_err, &ga, &gathered,
                                            st))
        return true;
    if (!gathered) {
        const int grid =
            (int)std::max<long long>(1, std::min<long long>(4 * 148, ((long long)rows + kPullThreads - 1) / kPullThreads));
        cudaError_t e = launch_pdl(ll_pull_kernel, dim3(grid), dim3(kPullThreads), 0, st,
                                   (const unsigned long long *)(g.local + buf), (long long)rows, epoch, yd, ctx->d_err,
                                   kPeerWaitNs);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) {
            ctx_fail(ctx, "kernel_gemv", "gather launch failed: %s", cudaGetErrorString(e));
            return true;
        }
    }
    cudaError_t e = cudaSuccess;
    if (!y_on_dev) {
        e = cudaMemcpyAsync(Y, yd, (size_t)rows * sizeof(float), cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "kernel_gemv", "gather copy-out failed: %s", cudaGetErrorString(e));
            return true;
        }
    }
    *rc = 0;
    return true;
}

void shard_destroy(kernel_context_t *ctx) {
    if (ctx->pg) {
        cudaDeviceSynchronize();
        for (int k = 0; k < kMaxPeers; ++k)
            if (ctx->pg->peer[k] && k != ctx->rank) cudaIpcCloseMemHandle(ctx->pg->peer[k]);
        if (ctx->pg->local) cudaFree(ctx->pg->local);
        cudaGetLastError();
        delete ctx->pg;
        ctx->pg = nullptr;
    }
    if (ctx->nccl_comm) {
        nccl().commDestroy((ncclComm_t)ctx->nccl_comm);
        ctx->nccl_comm = nullptr;
    }
    ctx->rank = 0;
    ctx->world = 1;
}

// Test-only: runs the peer-gather pull on a local buffer of `rows` words that
// no rank writes (epoch 0, the pull waits for epoch 1), with a wait limit of
// wait_ns, on the context's GPU.  The bounded wait runs out: y (device,
// `rows` floats) receives NaN, bit 3 of the error word is set and the call
// returns -1 after its synchronisation.  No GPU fault is involved.
extern "C" SAPPHIRE_API int sapphire_test_pull_expiry(kernel_context_t *ctx, float *y, long long rows,
                                                      unsigned long long wait_ns) {
    if (!ctx || !y || rows <= 0) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (!ctx->initialized || ensure_err_word(ctx)) return -1;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    unsigned long long *buf = nullptr;
    int rc = -1;
    if (cudaMalloc(&buf, (size_t)rows * sizeof(unsigned long long)) == cudaSuccess &&
        cudaMemsetAsync(buf, 0, (size_t)rows * sizeof(unsigned long long), ctx->stream) == cudaSuccess) {
        const int grid = (int)std::max<long long>(1, std::min<long long>(4 * 148, (rows + kPullThreads - 1) / kPullThreads));
        cudaError_t e = launch_pdl(ll_pull_kernel, dim3(grid), dim3(kPullThreads), 0, ctx->stream,
                                   (const unsigned long long *)buf, rows, 1u, y, ctx->d_err, wait_ns);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "sapphire_test_pull_expiry", "%s", cudaGetErrorString(e));
        } else {
            rc = check_kernel_error(ctx, "sapphire_test_pull_expiry");
        }
    }
    if (buf) cudaFree(buf);
    cudaGetLastError();
    if (prev >= 0) cudaSetDevice(prev);
    return rc;
}

int shard_map_buffers(kernel_context_t *ctx, size_t bytes, void **local, void **peers) {
    if (!ctx->nccl_comm) {
        ctx_fail(ctx, "shard_map_buffers", "context has no communicator");
        return -1;
    }
    if (map_buffers(ctx, bytes, local, peers)) {
        shard_unmap_buffers(ctx, *local, peers);
        *local = nullptr;
        ctx_fail(ctx, "shard_map_buffers", "not every rank could map every peer's memory");
        return -1;
    }
    return 0;
}

void shard_unmap_buffers(kernel_context_t *ctx, void *local, void **peers) {
    for (int k = 0; k < kMaxPeers; ++k) {
        if (peers[k] && k != ctx->rank) cudaIpcCloseMemHandle(peers[k]);
        peers[k] = nullptr;
    }
    if (local) cudaFree(local);
    cudaGetLastError();
}
