// internal.cuh - context, device-weight and launcher declarations shared by
// the .cu sources of libsapphire_cuda.so.
#pragma once

#include <cuda_runtime.h>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>
#include <thread>
#include <condition_variable>
#include <atomic>
#include <utility>

#include "common.h"

// Rows per tile of the GEMV device layout: one warp lane owns one row.
constexpr int kTileRows = 32;
// Most ranks a peer-memory gather serves.
constexpr int kMaxPeers = 8;

// Peer-memory gather of row-sharded batch-1 products (shard.cu): each rank's
// allocation holds two buffers of cap_rows 8-byte words (value | epoch << 32),
// used alternately by epoch parity; peer[k] maps rank k's allocation.
struct PeerGather {
    bool tried = false, ready = false;
    size_t cap_rows = 0;
    unsigned long long *local = nullptr;
    unsigned long long *peer[kMaxPeers] = {};
    unsigned epoch = 0;
};


// Device copy of one weight tensor, re-laid out for the GEMV kernels.
//
// Tile layout ("lane = row"): rows are grouped in tiles of 32; inside a tile
// the packed row data is cut into 16-byte chunks and stored chunk-major,
//     codes[((tile * kchunks) + chunk) * 32 + lane]   (uint4, lane = row % 32)
// so one warp-wide 16-byte load reads chunk `chunk` of 32 consecutive rows as
// one contiguous 512-byte segment.  Scales are stored the same way,
//     scales[((tile * nscale) + s) * 32 + lane]        (fp32)
// Chunk contents per dtype (weights in column order):
//     Q8_0 : 16 int8 codes, two chunks per block, nscale = nb
//     Q4_0 : the block's 16 code bytes (32 weights, interleaved nibbles), nscale = nb
//     TQ2_0: 64 columns (two trit blocks) of 32 rows per 512-byte chunk group,
//            interleaved as 2-bit planes (repack.cu), nscale = 1 (row scale)
//     F32  : 4 floats;  BF16: 8 bf16 values; nscale = 0
// Padding rows (past the tensor's last row) hold zero codes and zero scales.
struct DevWeight {
    uint64_t uid = 0;
    const void *src = nullptr;     // tensor data pointer at upload time
    tensor_dtype_t dtype = DTYPE_F32;
    int rows = 0, cols = 0;        // logical shape of the full tensor
    int row0 = 0, nrows = 0;       // rows held by this context (row shard)
    int nb = 0;                    // 32-wide blocks per row (quantized dtypes)
    int ntiles = 0;                // ceil(nrows / 32)
    int kchunks = 0;               // 16-byte chunks per row
    int nscale = 0;                // scales per row in the tile layout
    uint4 *codes = nullptr;
    float *scales = nullptr;
    size_t bytes = 0;              // device bytes held
};

// Weights covered by one 16-byte chunk of the tile layout.
inline int chunk_weights(tensor_dtype_t dt) {
    switch (dt) {
        case DTYPE_Q8_0: return 16;
        case DTYPE_Q4_0: return 32;
        case DTYPE_TQ2_0: return 64;
        case DTYPE_F32: return 4;
        case DTYPE_BF16: return 8;
        default: return 0;
    }
}

// Simple host worker pool for kernel_parallel_for (host callbacks only).
struct HostPool {
    std::vector<std::thread> threads;
    std::mutex m;
    std::condition_variable cv_work, cv_done;
    uint64_t task_seq = 0;
    int busy = 0;
    bool stop = false;
    parallel_for_fn_t fn = nullptr;
    void *arg = nullptr;
    int n = 0;
    std::atomic<int> next{0};
};

struct sapphire_context {
    int num_threads = 0;
    int chunk_size = 16;
    bool initialized = false;
    bool fp32_products = false;    // batched Q4_0 products keep fp32 activations (kernel_ctx_set_fp32_products)
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    std::recursive_mutex exec_mutex;

    std::unordered_map<uint64_t, DevWeight> weights;

    // Device scratch: activations in, results out, gather buffer.
    float *d_x = nullptr;  size_t d_x_cap = 0;
    float *d_y = nullptr;  size_t d_y_cap = 0;
    float *d_g = nullptr;  size_t d_g_cap = 0;
    float *d_t = nullptr;  size_t d_t_cap = 0;
    // Scratch of the pipelined GEMV: split-tile partials and arrival
    // counters (kept at zero between launches), and an error word in mapped
    // host memory that kernels set when a bounded wait gives up.
    float *d_part = nullptr; size_t d_part_cap = 0;
    int *d_cnt = nullptr;    size_t d_cnt_cap = 0;
    int *h_err = nullptr;    int *d_err = nullptr;
    // bf16 copy of the activations for the tensor-core batched product.
    float *d_xb = nullptr;   size_t d_xb_cap = 0;

    HostPool *pool = nullptr;

    // Row sharding (NCCL); world == 1 means unsharded.
    int rank = 0, world = 1;
    void *nccl_comm = nullptr;   // ncclComm_t
    PeerGather *pg = nullptr;    // peer-memory gather, set up on first use

    std::string last_error;
};

// ------------------------------------------------ programmatic dependent launch
// Kernels launched with launch_pdl may start while the previous kernel on the
// stream is still running.  Each such kernel calls pdl_trigger() early (its
// own dependents may then be scheduled) and pdl_wait() before it reads what an
// earlier kernel wrote or writes what one may still read; pdl_wait returns
// once the previous grid has completed and its memory is visible.  Every
// kernel launched this way calls pdl_wait (so completion is transitive).
// Outside such a launch both are no-ops.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
#endif

// ------------------------------------------------------------------ helpers
// Record an error on the context (if any) and log it.
void ctx_fail(kernel_context_t *ctx, const char *where, const char *fmt, ...)
    __attribute__((format(printf, 3, 4)));

#define CUDA_TRY(ctx, call)                                                       \
    do {                                                                          \
        cudaError_t _e = (call);                                                  \
        if (_e != cudaSuccess) {                                                  \
            ctx_fail((ctx), __func__, "%s failed: %s", #call, cudaGetErrorString(_e)); \
            return -1;                                                            \
        }                                                                         \
    } while (0)

// True if p is device (or managed) memory; *dev receives its ordinal.
bool ptr_is_device(const void *p, int *dev);
// Device address of page-locked host memory (registered or cudaHostAlloc'ed
// while `device` was current) as that device sees it through its mapping;
// nullptr for any other pointer.
float *host_mapped(float *p, int device);

// Process-wide context used for NULL-context dense GEMV and the row ABI.
kernel_context_t *default_context();

// Grow a device scratch buffer (on ctx's device) to at least `bytes`.
int ensure_scratch(kernel_context_t *ctx, float **buf, size_t *cap, size_t bytes);

// Device copy of A for ctx (uploads on first use).  On a sharded context the
// copy holds the rank's rows, or every row when `whole` (weights a decoder
// replicates on every rank).  nullptr on error.
const DevWeight *ctx_weight(kernel_context_t *ctx, const tensor_t *A, bool whole = false);

// Logical (rows, cols) of a 2-D tensor; false if not a usable 2-D tensor.
bool weight_shape(const tensor_t *A, int *rows, int *cols);

// --------------------------------------------------------------- launchers
// y[b*y_stride + r] = sum_k W[r,k] * x[b*x_stride + k] for r < w.nrows,
// b < batch.  x, y are device pointers.  Enqueued on `stream`.
int launch_gemv(kernel_context_t *ctx, const DevWeight &w, const float *x, int x_stride,
                float *y, int y_stride, int batch, cudaStream_t stream);

// Re-lay out `nrows` packed host-format rows (device pointer `src`, the
// reference block layout) into tiles starting at tile `tile0` of w.
int launch_repack(kernel_context_t *ctx, const DevWeight &w, const void *src, int nrows,
                  int tile0, cudaStream_t stream);

// Quantizers / unpack on device buffers.
int launch_quantize(kernel_context_t *ctx, tensor_dtype_t dt, void *dst, const float *src,
                    int rows, int cols, cudaStream_t stream);
int launch_pack_tq2(kernel_context_t *ctx, void *dst, const int8_t *trits, const float *scales,
                    int rows, int cols, int *d_err, cudaStream_t stream);
int launch_dequantize(kernel_context_t *ctx, tensor_dtype_t dt, float *dst, const void *src,
                      int rows, int cols, cudaStream_t stream);
// One packed row (reference layout, device pointer) dotted with x -> out[0].
int launch_row_dot(kernel_context_t *ctx, tensor_dtype_t dt, const void *row, const float *x,
                   int nb, int cols, float *out, cudaStream_t stream);
// y[i] += alpha * t[i] on device.
int launch_axpy(kernel_context_t *ctx, float *y, const float *t, float alpha, size_t n,
                cudaStream_t stream);

// The context's error word (mapped host memory; created at kernel_ctx_init).
int ensure_err_word(kernel_context_t *ctx);
// Error word (mapped host memory) plus split-tile scratch of the pipelined
// GEMV, grown to at least the given sizes.
int ensure_pipe_scratch(kernel_context_t *ctx, size_t part_floats, size_t cnt_ints);

// SMs of a device (cached; 148 when the query fails).
int sm_count(int dev);

// Pipelined batch-1 GEMV (gemv_pipe.cu): quantized formats are served by
// gemv_stream (gemv_stream.cu), dense F32 / BF16 by gemv_pipe.
bool pipe_supported(kernel_context_t *ctx, const DevWeight &w);
void pipe_scratch_size(kernel_context_t *ctx, const DevWeight &w, size_t *part_floats, size_t *cnt_ints);
int launch_gemv_pipe(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, float *part,
                     int *cnt, int *err, cudaStream_t stream);
int pipe_kmax(long long T, long long W, int nseg);
// Peer-memory gather of a row-sharded batch-1 product (shard.cu): each row r
// goes to every rank k as the 8-byte word (epoch << 32 | value bits) at
// targets[k][row_off + r]; `self` is this rank's own buffer of the epoch,
// from which y_full[0, rows_full) is gathered.
struct GatherArgs {
    unsigned long long *targets[kMaxPeers];
    int n, row_off;
    unsigned epoch;
    const unsigned long long *self;
    float *y_full;
    long long rows_full;
    unsigned long long wait_ns;
};
// The pipelined GEMV with its rows sent to a peer-memory gather (g != nullptr)
// instead of y.  *gathered = true when the kernel also gathered y_full (the
// streaming kernel does; the dense kernel leaves it to a pull kernel).
int launch_gemv_pipe_ll(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, float *part, int *cnt,
                        int *err, const GatherArgs *g, bool *gathered, cudaStream_t stream);
// Streaming batch-1 GEMV of the quantized formats (gemv_stream.cu).
bool stream_dtype(tensor_dtype_t dt);
bool stream_supported(kernel_context_t *ctx, const DevWeight &w);
void stream_scratch_size(kernel_context_t *ctx, const DevWeight &w, size_t *part_floats, size_t *cnt_ints);
int launch_gemv_stream(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, float *part, int *cnt,
                       int *err, const GatherArgs *g, cudaStream_t stream);
// Latency-bound GEMV of a small Q8_0 / Q4_0 weight (gemv_pipe.cu): one CTA per
// 32-row tile, no scratch.
bool direct_supported(const DevWeight &w);
int launch_gemv_direct(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, cudaStream_t stream);
// The same with x produced inside the kernel (decode fusion): the residual
// update h_out = h_in + rmsnorm_delta(t, w_post) (stored by block 0) and
// x = rmsnorm_delta(h_out, w_next); or x = gelu(gu[:cols]) * gu[cols:].
int launch_gemv_direct_resnorm(kernel_context_t *ctx, const DevWeight &w, const float *t, const float *w_post,
                               const float *h_in, const float *w_next, float *h_out, float eps, float *y,
                               cudaStream_t stream);
int launch_gemv_direct_geglu(kernel_context_t *ctx, const DevWeight &w, const float *gu, float *y,
                             cudaStream_t stream);
// Weights of at most this many 32-row tiles take the direct kernel.
constexpr int kDirectMaxTiles = 512;
// Batch-1 product through the pipelined kernel when it applies, else the
// tile kernel; checks nothing on the host (asynchronous).
int launch_gemv_best(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, cudaStream_t stream);
// Y[b*y_stride + r] for b < batch with whichever kernel serves the format.
int launch_product(kernel_context_t *ctx, const DevWeight &w, const float *x, int x_stride, float *y, int y_stride,
                   int batch, cudaStream_t stream);
// Reads and clears the error word after a synchronisation; -1 if a kernel
// reported a failed wait (the split-tile counters are then cleared too).
// Bits: 1 GEMV copy wait, 2/4 prefill-product waits, 8 peer-gather wait.
int check_kernel_error(kernel_context_t *ctx, const char *who);

// Tensor-core batched product of a Q4_0 weight (gemm_tc.cu), used for
// batch >= kGemmTcMinBatch: activations rounded to bf16, weights dequantised
// exactly (hi + lo bf16 halves), fp32 accumulation.  err: error word.
constexpr int kGemmTcMinBatch = 16;
bool gemm_tc_supported(const DevWeight &w, int batch);
int launch_gemm_tc(kernel_context_t *ctx, const DevWeight &w, const float *x, int ldx, float *y, int ldy, int batch,
                   int *err, cudaStream_t stream);
// Same product from bf16 activations already on the device: xb [batch][ldxb],
// ldxb >= 32 * nb and a multiple of 8, 16-byte aligned, zero past the columns.
int launch_gemm_tc_bf16(kernel_context_t *ctx, const DevWeight &w, const void *xb, int ldxb, float *y, int ldy,
                        int batch, int *err, cudaStream_t stream);

// Sharded all-gather of per-rank slices (NCCL).  Defined in shard.cu.
int shard_allgather(kernel_context_t *ctx, const float *send, float *recv, size_t count,
                    cudaStream_t stream);
void shard_destroy(kernel_context_t *ctx);
// Collective over the ranks of a sharded context: allocates `bytes` of zeroed
// device memory on this rank and maps every rank's allocation (CUDA IPC,
// handles exchanged over NCCL); peers[k] is rank k's (peers[rank] = *local).
// 0 when every rank mapped every peer, else -1 on every rank.
int shard_map_buffers(kernel_context_t *ctx, size_t bytes, void **local, void **peers);
void shard_unmap_buffers(kernel_context_t *ctx, void *local, void **peers);
// Batch-1 sharded product gathered over peer memory into y[0, rows): true if
// it ran (every rank decides the same from the arguments); false means use the
// NCCL path.  -1 through *rc on error.
bool shard_peer_product(kernel_context_t *ctx, const DevWeight &w, const float *x, float *Y, int rows, int per,
                        bool y_on_dev, int *rc);

// Rows owned by `rank` of `world` for a tensor of `rows` rows.
inline void shard_rows(int rows, int rank, int world, int *row0, int *nrows) {
    int per = (rows + world - 1) / world;
    int b = rank * per;
    int e = b + per;
    if (b > rows) b = rows;
    if (e > rows) e = rows;
    *row0 = b;
    *nrows = e - b;
}
