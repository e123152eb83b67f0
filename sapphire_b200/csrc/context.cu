// context.cu - kernel_context_t lifecycle, device-weight cache and upload,
// scratch buffers, host worker pool.
//
// Replaces the reference's thread-pool context (src/kernels/pool.c:12-268):
// kernel_ctx_create / kernel_ctx_init / kernel_ctx_destroy keep their
// signatures and return codes, but the context now owns a GPU stream and the
// device copies of weights; the host workers only serve kernel_parallel_for.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <unistd.h>

#include "internal.cuh"

// ------------------------------------------------------------- registry ---
// Live contexts, so tensor_release can drop device copies everywhere.
namespace {
std::mutex g_registry_mu;
std::vector<kernel_context_t *> g_registry;
std::mutex g_default_mu;
kernel_context_t *g_default[64] = {nullptr};

void free_weight(DevWeight &w) {
    if (w.codes) cudaFree(w.codes);
    if (w.scales) cudaFree(w.scales);
    w.codes = nullptr;
    w.scales = nullptr;
    w.bytes = 0;
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

void pool_worker(HostPool *p) {
    uint64_t seen = 0;
    for (;;) {
        parallel_for_fn_t fn;
        void *arg;
        int n;
        {
            std::unique_lock<std::mutex> lk(p->m);
            p->cv_work.wait(lk, [&] { return p->stop || p->task_seq != seen; });
            if (p->stop) return;
            seen = p->task_seq;
            fn = p->fn;
            arg = p->arg;
            n = p->n;
        }
        for (;;) {
            int i = p->next.fetch_add(1);
            if (i >= n) break;
            fn(arg, i);
        }
        {
            std::lock_guard<std::mutex> lk(p->m);
            if (--p->busy == 0) p->cv_done.notify_all();
        }
    }
}
}  // namespace

void ctx_fail(kernel_context_t *ctx, const char *where, const char *fmt, ...) {
    char msg[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    sapphire_log(SAPPHIRE_LOG_ERROR, "context.cu", 0, where, "%s", msg);
    if (ctx) ctx->last_error = std::string(where) + ": " + msg;
}

bool ptr_is_device(const void *p, int *dev) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // clear the sticky-free error state
        return false;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
        if (dev) *dev = a.device;
        return true;
    }
    return false;
}

float *host_mapped(float *p, int device) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    // Only memory page-locked for this device's context: memory pinned by
    // another device's context without the portable flag is not mapped here.
    return (a.type == cudaMemoryTypeHost && a.device == device) ? static_cast<float *>(a.devicePointer) : nullptr;
}

bool weight_shape(const tensor_t *A, int *rows, int *cols) {
    if (!A || tensor_ndim(A) != 2) return false;
    const int *s = tensor_shape(A);
    if (!s || s[0] <= 0 || s[1] <= 0) return false;
    *rows = s[0];
    *cols = s[1];
    return true;
}

int sm_count(int dev) {
    static int cached[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

size_t sapphire_row_bytes_internal(tensor_dtype_t dt, int cols) {
    if (cols <= 0) return 0;
    const size_t nb = ((size_t)cols + 31) / 32;
    switch (dt) {
        case DTYPE_Q4_0: return nb * 20;
        case DTYPE_Q8_0: return nb * 36;
        case DTYPE_TQ2_0: return 4 + nb * 8;
        case DTYPE_F32: return (size_t)cols * 4;
        case DTYPE_BF16:
        case DTYPE_F16: return (size_t)cols * 2;
        default: return 0;
    }
}

extern "C" SAPPHIRE_API size_t sapphire_row_bytes(tensor_dtype_t dtype, int cols) {
    return sapphire_row_bytes_internal(dtype, cols);
}

// ------------------------------------------------------------ lifecycle ---
extern "C" SAPPHIRE_API kernel_context_t *kernel_ctx_create(int num_threads, int chunk_size) {
    if (num_threads <= 0) {
        long n = sysconf(_SC_NPROCESSORS_ONLN);
        num_threads = n > 0 ? (int)n : 1;
    }
    if (chunk_size <= 0) chunk_size = 16;
    kernel_context_t *ctx = new (std::nothrow) sapphire_context();
    if (!ctx) return nullptr;
    ctx->num_threads = num_threads;
    ctx->chunk_size = chunk_size;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = 0;
    }
    ctx->device = dev;
    {
        std::lock_guard<std::mutex> lk(g_registry_mu);
        g_registry.push_back(ctx);
    }
    return ctx;
}

extern "C" SAPPHIRE_API int kernel_ctx_init(kernel_context_t *ctx) {
    if (!ctx) {
        LOG_ERROR("kernel_ctx_init: NULL context");
        return -1;
    }
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (ctx->initialized) return 0;
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess || ndev == 0) {
        ctx_fail(ctx, "kernel_ctx_init", "no CUDA device available (%s)",
                 e == cudaSuccess ? "0 devices" : cudaGetErrorString(e));
        cudaGetLastError();
        return -1;
    }
    if (ctx->device >= ndev) ctx->device = 0;
    DeviceGuard g(ctx->device);
    if (!ctx->stream) {
        CUDA_TRY(ctx, cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
        ctx->own_stream = true;
    }
    if (ensure_err_word(ctx)) return -1;
    if (!ctx->pool) {
        HostPool *p = new HostPool();
        try {
            for (int i = 0; i < ctx->num_threads; ++i) p->threads.emplace_back(pool_worker, p);
        } catch (...) {
            {
                std::lock_guard<std::mutex> l2(p->m);
                p->stop = true;
            }
            p->cv_work.notify_all();
            for (auto &t : p->threads) t.join();
            delete p;
            ctx_fail(ctx, "kernel_ctx_init", "failed to start %d host workers", ctx->num_threads);
            return -1;
        }
        ctx->pool = p;
    }
    ctx->initialized = true;
    return 0;
}

extern "C" SAPPHIRE_API void kernel_ctx_destroy(kernel_context_t *ctx) {
    if (!ctx) return;
    {
        std::lock_guard<std::mutex> lk(g_registry_mu);
        g_registry.erase(std::remove(g_registry.begin(), g_registry.end(), ctx), g_registry.end());
    }
    {
        std::lock_guard<std::mutex> lk(g_default_mu);
        for (auto &d : g_default)
            if (d == ctx) d = nullptr;
    }
    {
        std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
        if (ctx->initialized || !ctx->weights.empty()) {
            DeviceGuard g(ctx->device);
            if (ctx->stream) cudaStreamSynchronize(ctx->stream);
            for (auto &kv : ctx->weights) free_weight(kv.second);
            ctx->weights.clear();
            if (ctx->d_x) cudaFree(ctx->d_x);
            if (ctx->d_y) cudaFree(ctx->d_y);
            if (ctx->d_g) cudaFree(ctx->d_g);
            if (ctx->d_t) cudaFree(ctx->d_t);
            if (ctx->d_part) cudaFree(ctx->d_part);
            if (ctx->d_cnt) cudaFree(ctx->d_cnt);
            if (ctx->d_xb) cudaFree(ctx->d_xb);
            if (ctx->h_err) cudaFreeHost(ctx->h_err);
            shard_destroy(ctx);
            if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
        }
        if (ctx->pool) {
            HostPool *p = ctx->pool;
            {
                std::lock_guard<std::mutex> l2(p->m);
                p->stop = true;
            }
            p->cv_work.notify_all();
            for (auto &t : p->threads) t.join();
            delete p;
            ctx->pool = nullptr;
        }
    }
    delete ctx;
}

kernel_context_t *default_context() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = 0;
    }
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_default_mu);
    if (!g_default[dev]) {
        kernel_context_t *c = kernel_ctx_create(1, 16);
        if (!c) return nullptr;
        if (kernel_ctx_init(c) != 0) {
            kernel_ctx_destroy(c);
            return nullptr;
        }
        g_default[dev] = c;
    }
    return g_default[dev];
}

// -------------------------------------------------------- parallel_for ----
extern "C" SAPPHIRE_API int kernel_parallel_for(kernel_context_t *ctx, parallel_for_fn_t fn, void *arg, int n) {
    if (!ctx || !fn || n <= 0) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    HostPool *p = ctx->pool;
    if (!p || p->threads.empty()) {
        // Not initialised: run on the calling thread (the reference would wait
        // forever for workers that were never started).
        for (int i = 0; i < n; ++i) fn(arg, i);
        return 0;
    }
    std::unique_lock<std::mutex> l2(p->m);
    p->fn = fn;
    p->arg = arg;
    p->n = n;
    p->next.store(0);
    p->busy = (int)p->threads.size();
    p->task_seq++;
    p->cv_work.notify_all();
    p->cv_done.wait(l2, [&] { return p->busy == 0; });
    return 0;
}

// ------------------------------------------------------------- scratch ----
int ensure_scratch(kernel_context_t *ctx, float **buf, size_t *cap, size_t bytes) {
    if (*cap >= bytes && *buf) return 0;
    size_t want = std::max(bytes, (size_t)1 << 16);
    want = (want + 4095) & ~(size_t)4095;
    if (*buf) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(*buf);
        *buf = nullptr;
        *cap = 0;
    }
    CUDA_TRY(ctx, cudaMalloc((void **)buf, want));
    *cap = want;
    // New scratch starts zeroed: the split-tile partial words of the
    // streaming GEMV are valid only when tagged with the current launch's
    // epoch, and zero is never an epoch.
    CUDA_TRY(ctx, cudaMemsetAsync(*buf, 0, want, ctx->stream));
    return 0;
}

// ------------------------------------------------ pipelined GEMV scratch ---
// The error word lives in mapped pinned host memory: a kernel writes it only
// on failure and the host reads it after a sync.  Created at kernel_ctx_init
// (so entry points that must not allocate can still report errors).
int ensure_err_word(kernel_context_t *ctx) {
    if (ctx->h_err) return 0;
    int *h = nullptr;
    CUDA_TRY(ctx, cudaHostAlloc((void **)&h, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable));
    *h = 0;
    int *d = nullptr;
    if (cudaHostGetDevicePointer((void **)&d, h, 0) != cudaSuccess) {
        cudaGetLastError();
        cudaFreeHost(h);
        ctx_fail(ctx, "ensure_err_word", "no device alias for the mapped error word");
        return -1;
    }
    ctx->h_err = h;
    ctx->d_err = d;
    return 0;
}

// Partial sums and zeroed arrival counters for the pipelined kernel, grown on
// demand; the counters return to zero at the end of every launch, so only new
// memory needs clearing (check_kernel_error clears them after a launch that
// gave up, since a warp that bails out leaves its tiles' counts behind).
int ensure_pipe_scratch(kernel_context_t *ctx, size_t part_floats, size_t cnt_ints) {
    if (ensure_err_word(ctx)) return -1;
    if (ensure_scratch(ctx, &ctx->d_part, &ctx->d_part_cap, part_floats * sizeof(float))) return -1;
    if (ctx->d_cnt_cap < cnt_ints * sizeof(int) || !ctx->d_cnt) {
        float *buf = reinterpret_cast<float *>(ctx->d_cnt);
        size_t cap = ctx->d_cnt_cap;
        if (ensure_scratch(ctx, &buf, &cap, cnt_ints * sizeof(int))) return -1;
        ctx->d_cnt = reinterpret_cast<int *>(buf);
        ctx->d_cnt_cap = cap;
        CUDA_TRY(ctx, cudaMemsetAsync(ctx->d_cnt, 0, cap, ctx->stream));
    }
    return 0;
}

int launch_gemv_best(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, cudaStream_t st) {
    if (w.ntiles <= kDirectMaxTiles && direct_supported(w)) return launch_gemv_direct(ctx, w, x, y, st);
    if (pipe_supported(ctx, w)) {
        size_t pf = 0, ci = 0;
        pipe_scratch_size(ctx, w, &pf, &ci);
        if (ensure_pipe_scratch(ctx, pf, ci)) return -1;
        return launch_gemv_pipe(ctx, w, x, y, ctx->d_part, ctx->d_cnt, ctx->d_err, st);
    }
    if (w.dtype == DTYPE_F32 || w.dtype == DTYPE_BF16) return launch_gemv(ctx, w, x, w.cols, y, w.nrows, 1, st);
    ctx_fail(ctx, "kernel_gemv", "%s weight with %d columns exceeds the kernel's shared-memory budget",
             dtype_name(w.dtype), w.cols);
    return -1;
}

int launch_product(kernel_context_t *ctx, const DevWeight &w, const float *x, int x_stride, float *y, int y_stride,
                   int batch, cudaStream_t st) {
    if (batch == 1) return launch_gemv_best(ctx, w, x, y, st);
    if (w.dtype == DTYPE_F32 || w.dtype == DTYPE_BF16) return launch_gemv(ctx, w, x, x_stride, y, y_stride, batch, st);
    if (!ctx->fp32_products && gemm_tc_supported(w, batch)) {
        if (ensure_pipe_scratch(ctx, 0, 0)) return -1;
        return launch_gemm_tc(ctx, w, x, x_stride, y, y_stride, batch, ctx->d_err, st);
    }
    // Other quantized products: one pipelined pass per activation row.
    for (int b = 0; b < batch; ++b)
        if (launch_gemv_best(ctx, w, x + (size_t)b * x_stride, y + (size_t)b * y_stride, st)) return -1;
    return 0;
}

int check_kernel_error(kernel_context_t *ctx, const char *who) {
    const int bits = ctx->h_err ? *reinterpret_cast<volatile int *>(ctx->h_err) : 0;
    if (!bits) return 0;
    *ctx->h_err = 0;
    // A GEMV warp that gave up left the arrival counts of the tiles it had
    // joined behind; later launches sharing the counters would miscount.
    if (ctx->d_cnt && ctx->d_cnt_cap) cudaMemsetAsync(ctx->d_cnt, 0, ctx->d_cnt_cap, ctx->stream);
    if (bits & 8)
        ctx_fail(ctx, who, "a peer-memory gather gave up waiting for another rank's rows (bounded wait expired)");
    else if (bits & 16)
        ctx_fail(ctx, who, "a persistent decode step gave up waiting for another block's output (bounded wait expired)");
    else if (bits == 4)
        ctx_fail(ctx, who, "a token id outside the vocabulary reached the embedding");
    else
        ctx_fail(ctx, who, "a kernel gave up waiting for its asynchronous copies (bounded wait expired)");
    return -1;
}

// ------------------------------------------------------- weight upload ----
static int fill_layout(kernel_context_t *ctx, DevWeight &w) {
    w.nb = (w.cols + 31) / 32;
    w.ntiles = (w.nrows + kTileRows - 1) / kTileRows;
    switch (w.dtype) {
        case DTYPE_Q8_0: w.kchunks = 2 * w.nb; w.nscale = w.nb; break;
        case DTYPE_Q4_0: w.kchunks = w.nb; w.nscale = w.nb; break;
        case DTYPE_TQ2_0: w.kchunks = (w.nb + 1) / 2; w.nscale = 1; break;
        case DTYPE_F32: w.kchunks = (w.cols + 3) / 4; w.nscale = 0; break;
        case DTYPE_BF16: w.kchunks = (w.cols + 7) / 8; w.nscale = 0; break;
        default:
            ctx_fail(ctx, "kernel_tensor_upload", "dtype %s has no GEMV path", dtype_name(w.dtype));
            return -1;
    }
    return 0;
}

static int upload(kernel_context_t *ctx, const tensor_t *A, DevWeight &w, bool whole) {
    const void *data = tensor_data(A);
    if (!data) {
        ctx_fail(ctx, "kernel_tensor_upload", "tensor has no data");
        return -1;
    }
    w.uid = sapphire_tensor_uid(A);
    w.src = data;
    w.dtype = tensor_dtype(A);
    if (!weight_shape(A, &w.rows, &w.cols)) {
        ctx_fail(ctx, "kernel_tensor_upload", "weight must be 2-D with positive shape");
        return -1;
    }
    if (whole) {
        w.row0 = 0;
        w.nrows = w.rows;
    } else {
        shard_rows(w.rows, ctx->rank, ctx->world, &w.row0, &w.nrows);
    }
    if (fill_layout(ctx, w)) return -1;
    const size_t code_bytes = (size_t)w.ntiles * w.kchunks * 32 * 16;
    const size_t scale_bytes = (size_t)w.ntiles * w.nscale * 32 * sizeof(float);
    if (w.ntiles > 0) {
        CUDA_TRY(ctx, cudaMalloc((void **)&w.codes, code_bytes));
        if (scale_bytes) {
            if (cudaMalloc((void **)&w.scales, scale_bytes) != cudaSuccess) {
                cudaGetLastError();
                free_weight(w);
                ctx_fail(ctx, "kernel_tensor_upload", "cudaMalloc of %zu scale bytes failed", scale_bytes);
                return -1;
            }
        }
    }
    w.bytes = code_bytes + scale_bytes;
    if (w.nrows == 0) return 0;

    const size_t row_bytes = sapphire_row_bytes_internal(w.dtype, w.cols);
    const uint8_t *src = static_cast<const uint8_t *>(data) + (size_t)w.row0 * row_bytes;
    int dev = -1;
    int rc = 0;
    if (ptr_is_device(data, &dev)) {
        if (dev != ctx->device) {
            free_weight(w);
            ctx_fail(ctx, "kernel_tensor_upload", "weight lives on device %d, context on %d", dev, ctx->device);
            return -1;
        }
        rc = launch_repack(ctx, w, src, w.nrows, 0, ctx->stream);
    } else {
        // Stage host rows through a bounded device buffer, 32-row aligned.
        const size_t budget = (size_t)128 << 20;
        size_t rows_per = std::max<size_t>(kTileRows, (budget / std::max<size_t>(row_bytes, 1)) / kTileRows * kTileRows);
        if (rows_per > (size_t)w.nrows) rows_per = (size_t)w.nrows;
        void *stage = nullptr;
        if (cudaMalloc(&stage, rows_per * row_bytes) != cudaSuccess) {
            cudaGetLastError();
            free_weight(w);
            ctx_fail(ctx, "kernel_tensor_upload", "cudaMalloc of %zu staging bytes failed", rows_per * row_bytes);
            return -1;
        }
        for (size_t r = 0; r < (size_t)w.nrows && rc == 0; r += rows_per) {
            const size_t nr = std::min(rows_per, (size_t)w.nrows - r);
            cudaError_t e = cudaMemcpyAsync(stage, src + r * row_bytes, nr * row_bytes, cudaMemcpyHostToDevice,
                                            ctx->stream);
            if (e != cudaSuccess) {
                ctx_fail(ctx, "kernel_tensor_upload", "host-to-device copy failed: %s", cudaGetErrorString(e));
                rc = -1;
                break;
            }
            rc = launch_repack(ctx, w, stage, (int)nr, (int)(r / kTileRows), ctx->stream);
            if (rc == 0 && cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
                ctx_fail(ctx, "kernel_tensor_upload", "repack failed: %s", cudaGetErrorString(cudaGetLastError()));
                rc = -1;
            }
        }
        cudaFree(stage);
    }
    if (rc == 0) {
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "kernel_tensor_upload", "upload failed: %s", cudaGetErrorString(e));
            rc = -1;
        }
    }
    if (rc) free_weight(w);
    return rc;
}

const DevWeight *ctx_weight(kernel_context_t *ctx, const tensor_t *A, bool whole) {
    const uint64_t uid = sapphire_tensor_uid(A);
    auto it = ctx->weights.find(uid);
    if (it != ctx->weights.end()) {
        const DevWeight &w = it->second;
        int r = 0, c = 0;
        if (w.src == tensor_data(A) && w.dtype == tensor_dtype(A) && weight_shape(A, &r, &c) && r == w.rows &&
            c == w.cols && (whole ? w.nrows == w.rows : true))
            return &w;
        cudaStreamSynchronize(ctx->stream);
        free_weight(it->second);
        ctx->weights.erase(it);
    }
    DevWeight w;
    if (upload(ctx, A, w, whole)) return nullptr;
    auto res = ctx->weights.emplace(uid, w);
    return &res.first->second;
}

extern "C" SAPPHIRE_API int kernel_tensor_upload(kernel_context_t *ctx, const tensor_t *A) {
    if (!ctx || !A) {
        LOG_ERROR("kernel_tensor_upload: NULL argument");
        return -1;
    }
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (!ctx->initialized) {
        ctx_fail(ctx, "kernel_tensor_upload", "context not initialized");
        return -1;
    }
    DeviceGuard g(ctx->device);
    return ctx_weight(ctx, A) ? 0 : -1;
}

extern "C" SAPPHIRE_API int kernel_tensor_evict(kernel_context_t *ctx, const tensor_t *A) {
    if (!ctx || !A) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    auto it = ctx->weights.find(sapphire_tensor_uid(A));
    if (it == ctx->weights.end()) return 0;
    DeviceGuard g(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    free_weight(it->second);
    ctx->weights.erase(it);
    return 0;
}

extern "C" SAPPHIRE_API size_t kernel_ctx_resident_bytes(kernel_context_t *ctx) {
    if (!ctx) return 0;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    size_t n = 0;
    for (auto &kv : ctx->weights) n += kv.second.bytes;
    return n;
}

void sapphire_on_tensor_release(uint64_t uid) {
    std::lock_guard<std::mutex> lk(g_registry_mu);
    for (kernel_context_t *ctx : g_registry) {
        std::lock_guard<std::recursive_mutex> l2(ctx->exec_mutex);
        auto it = ctx->weights.find(uid);
        if (it == ctx->weights.end()) continue;
        DeviceGuard g(ctx->device);
        if (ctx->stream) cudaStreamSynchronize(ctx->stream);
        free_weight(it->second);
        ctx->weights.erase(it);
    }
}

// -------------------------------------------------------------- streams ---
extern "C" SAPPHIRE_API int kernel_ctx_synchronize(kernel_context_t *ctx) {
    if (!ctx) return -1;
    if (!ctx->stream) return 0;
    DeviceGuard g(ctx->device);
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    // Errors of asynchronous calls (kernel_gemv_device and the like) surface
    // here: a kernel whose bounded wait expired set the error word.
    return check_kernel_error(ctx, "kernel_ctx_synchronize");
}

extern "C" SAPPHIRE_API void *kernel_ctx_get_stream(kernel_context_t *ctx) {
    return ctx ? (void *)ctx->stream : nullptr;
}

extern "C" SAPPHIRE_API int kernel_ctx_set_stream(kernel_context_t *ctx, void *stream) {
    if (!ctx) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    DeviceGuard g(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    ctx->stream = (cudaStream_t)stream;
    ctx->own_stream = false;
    return 0;
}

extern "C" SAPPHIRE_API int kernel_ctx_get_device(kernel_context_t *ctx) { return ctx ? ctx->device : -1; }

extern "C" SAPPHIRE_API int kernel_ctx_set_fp32_products(kernel_context_t *ctx, int on) {
    if (!ctx) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    ctx->fp32_products = on != 0;
    return 0;
}

extern "C" SAPPHIRE_API int kernel_ctx_set_device(kernel_context_t *ctx, int device) {
    if (!ctx) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (ctx->initialized) {
        ctx_fail(ctx, "kernel_ctx_set_device", "context already initialized on device %d", ctx->device);
        return -1;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess) {
        cudaGetLastError();
        ndev = 0;
    }
    if (device < 0 || device >= ndev) {
        ctx_fail(ctx, "kernel_ctx_set_device", "no device %d (%d visible)", device, ndev);
        return -1;
    }
    ctx->device = device;
    return 0;
}

extern "C" SAPPHIRE_API const char *kernel_ctx_last_error(kernel_context_t *ctx) {
    return ctx ? ctx->last_error.c_str() : "";
}

extern "C" SAPPHIRE_API void *kernel_host_alloc(size_t bytes) {
    void *p = nullptr;
    if (cudaHostAlloc(&p, bytes ? bytes : 1, cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        LOG_ERROR("kernel_host_alloc: cudaHostAlloc(%zu) failed", bytes);
        return nullptr;
    }
    return p;
}

extern "C" SAPPHIRE_API void kernel_host_free(void *p) {
    if (p) cudaFreeHost(p);
}
