// dispatch.cu - public GEMV entry points (include/kernels.h, sapphire_cuda.h).
//
// Argument checks, error codes and NULL-context rules follow the reference
// dispatcher (src/kernels/dispatch.c:87-266) and backend
// (src/kernels/pool.c:270-362).  Every product goes to the GPU kernels in
// gemv.cu; nothing on this path computes on the CPU.
#include <cstring>
#include <algorithm>

#include "internal.cuh"

namespace {

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

bool gemv_dtype(tensor_dtype_t dt) {
    return dt == DTYPE_F32 || dt == DTYPE_BF16 || dt == DTYPE_Q4_0 || dt == DTYPE_Q8_0 || dt == DTYPE_TQ2_0;
}

bool quantized(tensor_dtype_t dt) { return dt == DTYPE_Q4_0 || dt == DTYPE_Q8_0 || dt == DTYPE_TQ2_0; }

// Y[b*rows + r] = A[r,:] . X[b*cols ..], b < batch.  X and Y host or device.
// sync: wait for completion before returning (required when Y is host memory).
int run_product(kernel_context_t *ctx, float *Y, const tensor_t *A, const float *X, int batch, bool sync,
                bool device_only) {
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (!ctx->initialized) {
        ctx_fail(ctx, "kernel_gemv", "context not initialized");
        return -1;
    }
    DeviceGuard g(ctx->device);
    int rows = 0, cols = 0;
    if (!weight_shape(A, &rows, &cols)) {
        ctx_fail(ctx, "kernel_gemv", "weight must be 2-D with positive shape");
        return -1;
    }
    const DevWeight *w = ctx_weight(ctx, A);
    if (!w) return -1;
    cudaStream_t st = ctx->stream;

    int xdev = -1, ydev = -1;
    const bool x_on_dev = ptr_is_device(X, &xdev);
    const bool y_on_dev = ptr_is_device(Y, &ydev);
    if ((x_on_dev && xdev != ctx->device) || (y_on_dev && ydev != ctx->device)) {
        ctx_fail(ctx, "kernel_gemv", "x/y live on another GPU than the context (%d)", ctx->device);
        return -1;
    }
    if (device_only && (!x_on_dev || !y_on_dev)) {
        ctx_fail(ctx, "kernel_gemv_device", "x and y must be device pointers on the context's GPU");
        return -1;
    }

    const float *xd = X;
    if (!x_on_dev) {
        if (ensure_scratch(ctx, &ctx->d_x, &ctx->d_x_cap, (size_t)batch * cols * sizeof(float))) return -1;
        CUDA_TRY(ctx, cudaMemcpyAsync(ctx->d_x, X, (size_t)batch * cols * sizeof(float), cudaMemcpyHostToDevice, st));
        xd = ctx->d_x;
    }

    if (ctx->world <= 1) {
        float *yd = Y;
        bool copy_out = false;
        if (!y_on_dev) {
            // A batch-1 result for page-locked host memory is written by the
            // kernel itself through the memory's device mapping: its rows
            // cross PCIe while the product runs instead of in a copy after it
            // (y is valid once the stream has synchronised, as before).
            float *mapped = batch == 1 ? host_mapped(Y, ctx->device) : nullptr;
            if (mapped) {
                yd = mapped;
            } else {
                if (ensure_scratch(ctx, &ctx->d_y, &ctx->d_y_cap, (size_t)batch * rows * sizeof(float))) return -1;
                yd = ctx->d_y;
                copy_out = true;
            }
        }
        if (launch_product(ctx, *w, xd, cols, yd, rows, batch, st)) return -1;
        if (copy_out)
            CUDA_TRY(ctx, cudaMemcpyAsync(Y, yd, (size_t)batch * rows * sizeof(float), cudaMemcpyDeviceToHost, st));
    } else {
        // Row-sharded: each rank computes Y_local[b][per] for its rows, then an
        // all-gather yields [world][b][per], copied out as Y[b][rows].
        const int per = (rows + ctx->world - 1) / ctx->world;
        const size_t slice = (size_t)batch * per;
        if (ensure_scratch(ctx, &ctx->d_g, &ctx->d_g_cap, (slice * (ctx->world + 1)) * sizeof(float))) return -1;
        float *send = ctx->d_g;
        float *recv = ctx->d_g + slice;
        int prc = 0;
        const cudaMemcpyKind kind = y_on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
        if (batch == 1 && shard_peer_product(ctx, *w, xd, Y, rows, per, y_on_dev, &prc)) {
            // gathered over peer memory by the GEMV itself
            if (prc) return -1;
        } else {
            if (w->nrows < per) CUDA_TRY(ctx, cudaMemsetAsync(send, 0, slice * sizeof(float), st));
            if (launch_product(ctx, *w, xd, cols, send, per, batch, st)) return -1;
            if (batch == 1) {
                // Rank r's rows start at r * per, its slot in the gathered
                // buffer: gather straight into y when it holds world * per
                // rows, else copy the first `rows` values once.
                const bool direct = y_on_dev && (size_t)per * ctx->world == (size_t)rows;
                if (shard_allgather(ctx, send, direct ? Y : recv, slice, st)) return -1;
                if (!direct) CUDA_TRY(ctx, cudaMemcpyAsync(Y, recv, (size_t)rows * sizeof(float), kind, st));
            } else {
                if (shard_allgather(ctx, send, recv, slice, st)) return -1;
                for (int r = 0; r < ctx->world; ++r) {
                    int row0 = 0, nr = 0;
                    shard_rows(rows, r, ctx->world, &row0, &nr);
                    if (nr == 0) continue;
                    CUDA_TRY(ctx, cudaMemcpy2DAsync(Y + row0, (size_t)rows * sizeof(float), recv + (size_t)r * slice,
                                                    (size_t)per * sizeof(float), (size_t)nr * sizeof(float), batch,
                                                    kind, st));
                }
            }
        }
    }
    if (sync) {
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "kernel_gemv", "GPU execution failed: %s", cudaGetErrorString(e));
            return -1;
        }
        if (check_kernel_error(ctx, "kernel_gemv")) return -1;
    }
    return 0;
}

// Common validation of kernel_gemv (src/kernels/dispatch.c:101-156).
int check_gemv_args(const char *who, float *y, const tensor_t *A, const float *x) {
    if (!y || !A || !x) {
        LOG_ERROR("%s: NULL y, A or x", who);
        return -1;
    }
    if (tensor_ndim(A) != 2) {
        LOG_ERROR("%s: A has to be two-dimensional", who);
        return -1;
    }
    const int *shape = tensor_shape(A);
    if (!shape) {
        LOG_ERROR("%s: A has no shape", who);
        return -1;
    }
    if (shape[0] <= 0 || shape[1] <= 0) {
        LOG_ERROR("%s: A has a non-positive dimension (%d x %d)", who, shape[0], shape[1]);
        return -1;
    }
    if (!gemv_dtype(tensor_dtype(A))) {
        LOG_ERROR("%s: no product for dtype %d", who, (int)tensor_dtype(A));
        return -1;
    }
    return 0;
}

}  // namespace

extern "C" SAPPHIRE_API int kernel_gemv(kernel_context_t *ctx, float *y, const tensor_t *A, const float *x) {
    if (check_gemv_args("kernel_gemv", y, A, x)) return -1;
    if (!ctx) {
        if (quantized(tensor_dtype(A))) {
            LOG_ERROR("a quantized weight needs a context (got NULL)");
            return -1;
        }
        ctx = default_context();
        if (!ctx) {
            LOG_ERROR("no GPU context available");
            return -1;
        }
    }
    return run_product(ctx, y, A, x, 1, true, false);
}

extern "C" SAPPHIRE_API int kernel_gemm(kernel_context_t *ctx, float *Y, const tensor_t *A, const float *X,
                                        int batch_size, int out_stride) {
    if (!Y || !A || !X || batch_size <= 0) {
        LOG_ERROR("NULL buffer or batch_size <= 0");
        return -1;
    }
    if (!ctx) {
        LOG_ERROR("a context is required (got NULL)");
        return -1;
    }
    if (check_gemv_args("kernel_gemm", Y, A, X)) return -1;
    // out_stride == 0 is the reference's non-batched path (is_gemm = 0).
    return run_product(ctx, Y, A, X, out_stride ? batch_size : 1, true, false);
}

extern "C" SAPPHIRE_API int kernel_gemv_tensor(kernel_context_t *ctx, const tensor_t *y, const tensor_t *A,
                                               const tensor_t *x) {
    if (!y || !A || !x) {
        LOG_ERROR("NULL tensor argument");
        return -1;
    }
    if (tensor_ndim(y) != 1 || tensor_dtype(y) != DTYPE_F32) {
        LOG_ERROR("y has to be a one-dimensional F32 tensor");
        return -1;
    }
    if (tensor_ndim(x) != 1 || tensor_dtype(x) != DTYPE_F32) {
        LOG_ERROR("x has to be a one-dimensional F32 tensor");
        return -1;
    }
    const int *sa = tensor_shape(A), *sx = tensor_shape(x), *sy = tensor_shape(y);
    if (!sa || !sx || !sy) {
        LOG_ERROR("a tensor has no shape");
        return -1;
    }
    if (sa[1] != sx[0]) {
        LOG_ERROR("A has %d columns but x has %d elements", sa[1], sx[0]);
        return -1;
    }
    if (sy[0] != sa[0]) {
        LOG_ERROR("y has %d elements but A has %d rows", sy[0], sa[0]);
        return -1;
    }
    return kernel_gemv(ctx, tensor_data_f32(y), A, (const float *)tensor_data(x));
}

extern "C" SAPPHIRE_API int kernel_gemv_add(kernel_context_t *ctx, float *y, const tensor_t *A, const float *x,
                                            float alpha) {
    if (!y || !A || !x) {
        LOG_ERROR("NULL buffer or tensor");
        return -1;
    }
    if (tensor_ndim(A) != 2) {
        LOG_ERROR("A has to be two-dimensional");
        return -1;
    }
    if (check_gemv_args("kernel_gemv_add", y, A, x)) return -1;
    if (!ctx) {
        if (quantized(tensor_dtype(A))) {
            LOG_ERROR("a quantized weight needs a context (got NULL)");
            return -1;
        }
        ctx = default_context();
        if (!ctx) return -1;
    }
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (!ctx->initialized) {
        ctx_fail(ctx, "kernel_gemv_add", "context not initialized");
        return -1;
    }
    DeviceGuard g(ctx->device);
    const int m = tensor_shape(A)[0];
    int ydev = -1;
    const bool y_on_dev = ptr_is_device(y, &ydev);
    // The product goes to a context-owned device temporary (no allocation per call).
    if (ensure_scratch(ctx, &ctx->d_t, &ctx->d_t_cap, 2 * (size_t)m * sizeof(float))) return -1;
    float *t = ctx->d_t, *yd = ctx->d_t + m;
    int rc = run_product(ctx, t, A, x, 1, false, false);
    if (rc == 0) {
        cudaStream_t st = ctx->stream;
        if (!y_on_dev) {
            if (cudaMemcpyAsync(yd, y, (size_t)m * sizeof(float), cudaMemcpyHostToDevice, st) != cudaSuccess) rc = -1;
        } else {
            yd = y;
        }
        if (rc == 0) rc = launch_axpy(ctx, yd, t, alpha, (size_t)m, st);
        if (rc == 0 && !y_on_dev &&
            cudaMemcpyAsync(y, yd, (size_t)m * sizeof(float), cudaMemcpyDeviceToHost, st) != cudaSuccess)
            rc = -1;
        if (cudaStreamSynchronize(st) != cudaSuccess) rc = -1;
        if (rc) ctx_fail(ctx, "kernel_gemv_add", "device step failed: %s", cudaGetErrorString(cudaGetLastError()));
    }
    return rc;
}

extern "C" SAPPHIRE_API int kernel_gemv_batch(kernel_context_t *ctx, float *Y, const tensor_t *A, const float *X,
                                              int batch_size) {
    if (!Y || !A || !X || batch_size <= 0) {
        LOG_ERROR("NULL buffer or batch size <= 0");
        return -1;
    }
    if (tensor_ndim(A) != 2) {
        LOG_ERROR("A has to be two-dimensional");
        return -1;
    }
    if (batch_size > 1 && ctx) {
        if (check_gemv_args("kernel_gemv_batch", Y, A, X)) return -1;
        return run_product(ctx, Y, A, X, batch_size, true, false);
    }
    const int m = tensor_shape(A)[0], n = tensor_shape(A)[1];
    for (int k = 0; k < batch_size; ++k)
        if (kernel_gemv(ctx, Y + (size_t)k * m, A, X + (size_t)k * n) != 0) return -1;
    return 0;
}

extern "C" SAPPHIRE_API int kernel_get_simd_lane_count(tensor_dtype_t dtype) {
    switch (dtype) {
        case DTYPE_F32:
        case DTYPE_BF16:
        case DTYPE_F16:
        case DTYPE_Q4_0:
        case DTYPE_Q8_0:
        case DTYPE_TQ2_0:
            return 8;
        default:
            return 1;
    }
}

extern "C" SAPPHIRE_API int kernel_gemv_device(kernel_context_t *ctx, float *y, const tensor_t *A, const float *x) {
    if (check_gemv_args("kernel_gemv_device", y, A, x)) return -1;
    if (!ctx) {
        LOG_ERROR("kernel_gemv_device requires a context");
        return -1;
    }
    return run_product(ctx, y, A, x, 1, false, true);
}

extern "C" SAPPHIRE_API int kernel_gemm_device(kernel_context_t *ctx, float *Y, const tensor_t *A, const float *X,
                                               int batch_size) {
    if (batch_size <= 0 || check_gemv_args("kernel_gemm_device", Y, A, X)) return -1;
    if (!ctx) {
        LOG_ERROR("kernel_gemm_device requires a context");
        return -1;
    }
    return run_product(ctx, Y, A, X, batch_size, false, true);
}

extern "C" SAPPHIRE_API int kernel_gemm_device_bf16(kernel_context_t *ctx, float *Y, const tensor_t *A,
                                                    const void *Xb, int batch_size, int x_stride) {
    if (!ctx || !Y || !A || !Xb || batch_size <= 0) {
        LOG_ERROR("kernel_gemm_device_bf16 invalid arguments");
        return -1;
    }
    if (tensor_dtype(A) != DTYPE_Q4_0) {
        LOG_ERROR("kernel_gemm_device_bf16 needs a Q4_0 weight");
        return -1;
    }
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (!ctx->initialized || ctx->world > 1) {
        ctx_fail(ctx, "kernel_gemm_device_bf16", "needs an initialized, unsharded context");
        return -1;
    }
    DeviceGuard g(ctx->device);
    int xdev = -1, ydev = -1;
    if (!ptr_is_device(Xb, &xdev) || !ptr_is_device(Y, &ydev) || xdev != ctx->device || ydev != ctx->device) {
        ctx_fail(ctx, "kernel_gemm_device_bf16", "Y and Xb must be device pointers on the context's GPU");
        return -1;
    }
    const DevWeight *w = ctx_weight(ctx, A);
    if (!w) return -1;
    if (ensure_pipe_scratch(ctx, 0, 0)) return -1;
    return launch_gemm_tc_bf16(ctx, *w, Xb, x_stride, Y, w->nrows, batch_size, ctx->d_err, ctx->stream);
}

// ------------------------------------------------------------ quantisers --
namespace {

// Run a device step over (possibly host) input/output buffers: device
// pointers are used in place, host ones are staged whole through temporaries.
struct Staged {
    void *dev = nullptr;
    bool owned = false;
};

int stage_in(kernel_context_t *ctx, const void *p, size_t bytes, Staged &s) {
    int dev = -1;
    if (ptr_is_device(p, &dev)) {
        if (dev != ctx->device) {
            ctx_fail(ctx, "stage_in", "buffer lives on device %d, context on %d", dev, ctx->device);
            return -1;
        }
        s.dev = const_cast<void *>(p);
        return 0;
    }
    CUDA_TRY(ctx, cudaMalloc(&s.dev, bytes ? bytes : 1));
    s.owned = true;
    CUDA_TRY(ctx, cudaMemcpyAsync(s.dev, p, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return 0;
}

int stage_out(kernel_context_t *ctx, void *p, size_t bytes, Staged &s) {
    int dev = -1;
    if (ptr_is_device(p, &dev)) {
        if (dev != ctx->device) {
            ctx_fail(ctx, "stage_out", "buffer lives on device %d, context on %d", dev, ctx->device);
            return -1;
        }
        s.dev = p;
        return 0;
    }
    CUDA_TRY(ctx, cudaMalloc(&s.dev, bytes ? bytes : 1));
    s.owned = true;
    return 0;
}

int finish_out(kernel_context_t *ctx, void *p, size_t bytes, Staged &s) {
    if (s.owned) CUDA_TRY(ctx, cudaMemcpyAsync(p, s.dev, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return 0;
}

void release(Staged &s) {
    if (s.owned && s.dev) cudaFree(s.dev);
    s.dev = nullptr;
}

kernel_context_t *ready_ctx(kernel_context_t *ctx, const char *who) {
    if (!ctx) ctx = default_context();
    if (!ctx) {
        LOG_ERROR("%s: no GPU context available", who);
        return nullptr;
    }
    if (!ctx->initialized) {
        ctx_fail(ctx, who, "context not initialized");
        return nullptr;
    }
    return ctx;
}

int quantize_common(kernel_context_t *ctx, tensor_dtype_t dt, void *dst, const float *src, int rows, int cols) {
    const char *who = dt == DTYPE_Q4_0 ? "kernel_quantize_q4_0" : "kernel_quantize_q8_0";
    if (!dst || !src || rows <= 0 || cols <= 0) {
        LOG_ERROR("%s invalid arguments", who);
        return -1;
    }
    ctx = ready_ctx(ctx, who);
    if (!ctx) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    DeviceGuard g(ctx->device);
    const size_t in_bytes = (size_t)rows * cols * sizeof(float);
    const size_t out_bytes = (size_t)rows * sapphire_row_bytes_internal(dt, cols);
    Staged si, so;
    int rc = stage_in(ctx, src, in_bytes, si);
    if (rc == 0) rc = stage_out(ctx, dst, out_bytes, so);
    if (rc == 0) rc = launch_quantize(ctx, dt, so.dev, (const float *)si.dev, rows, cols, ctx->stream);
    if (rc == 0) rc = finish_out(ctx, dst, out_bytes, so);
    cudaStreamSynchronize(ctx->stream);
    release(si);
    release(so);
    return rc;
}

}  // namespace

extern "C" SAPPHIRE_API int kernel_quantize_q4_0(kernel_context_t *ctx, void *dst, const float *src, int rows,
                                                 int cols) {
    return quantize_common(ctx, DTYPE_Q4_0, dst, src, rows, cols);
}

extern "C" SAPPHIRE_API int kernel_quantize_q8_0(kernel_context_t *ctx, void *dst, const float *src, int rows,
                                                 int cols) {
    return quantize_common(ctx, DTYPE_Q8_0, dst, src, rows, cols);
}

extern "C" SAPPHIRE_API int kernel_pack_tq2_0(kernel_context_t *ctx, void *dst, const int8_t *trits,
                                              const float *row_scales, int rows, int cols) {
    if (!dst || !trits || !row_scales || rows <= 0 || cols <= 0) {
        LOG_ERROR("kernel_pack_tq2_0 invalid arguments");
        return -1;
    }
    ctx = ready_ctx(ctx, "kernel_pack_tq2_0");
    if (!ctx) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    DeviceGuard g(ctx->device);
    const size_t out_bytes = (size_t)rows * sapphire_row_bytes_internal(DTYPE_TQ2_0, cols);
    Staged st, ss, so;
    int *d_err = nullptr;
    int rc = stage_in(ctx, trits, (size_t)rows * cols, st);
    if (rc == 0) rc = stage_in(ctx, row_scales, (size_t)rows * sizeof(float), ss);
    if (rc == 0) rc = stage_out(ctx, dst, out_bytes, so);
    if (rc == 0 && cudaMalloc((void **)&d_err, sizeof(int)) != cudaSuccess) rc = -1;
    if (rc == 0 && cudaMemsetAsync(d_err, 0, sizeof(int), ctx->stream) != cudaSuccess) rc = -1;
    if (rc == 0)
        rc = launch_pack_tq2(ctx, so.dev, (const int8_t *)st.dev, (const float *)ss.dev, rows, cols, d_err,
                             ctx->stream);
    if (rc == 0) rc = finish_out(ctx, dst, out_bytes, so);
    int h_err = 0;
    if (rc == 0 && cudaMemcpy(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) rc = -1;
    cudaStreamSynchronize(ctx->stream);
    if (d_err) cudaFree(d_err);
    release(st);
    release(ss);
    release(so);
    if (rc == 0 && h_err) {
        ctx_fail(ctx, "kernel_pack_tq2_0", "trit values must be -1, 0 or +1");
        return -1;
    }
    return rc;
}

extern "C" SAPPHIRE_API int kernel_dequantize(kernel_context_t *ctx, float *dst, const tensor_t *A) {
    int rows = 0, cols = 0;
    if (!dst || !A || !weight_shape(A, &rows, &cols) || !tensor_data(A)) {
        LOG_ERROR("kernel_dequantize invalid arguments");
        return -1;
    }
    const tensor_dtype_t dt = tensor_dtype(A);
    if (!gemv_dtype(dt)) {
        LOG_ERROR("kernel_dequantize unsupported dtype %d", (int)dt);
        return -1;
    }
    ctx = ready_ctx(ctx, "kernel_dequantize");
    if (!ctx) return -1;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    DeviceGuard g(ctx->device);
    const size_t in_bytes = (size_t)rows * sapphire_row_bytes_internal(dt, cols);
    const size_t out_bytes = (size_t)rows * cols * sizeof(float);
    Staged si, so;
    int rc = stage_in(ctx, tensor_data(A), in_bytes, si);
    if (rc == 0) rc = stage_out(ctx, dst, out_bytes, so);
    if (rc == 0) rc = launch_dequantize(ctx, dt, (float *)so.dev, si.dev, rows, cols, ctx->stream);
    if (rc == 0) rc = finish_out(ctx, dst, out_bytes, so);
    cudaStreamSynchronize(ctx->stream);
    release(si);
    release(so);
    return rc;
}

// ------------------------------------------------------------- row ABI ----
// The reference row kernels (src/kernels/q4_0_avx.c:102-148, q8_0_avx.c,
// bf16_avx.c, f32_avx.c) take one host row and return its dot product.  Here
// each call runs row_dot_kernel on the default context's GPU.
namespace {
float row_call(tensor_dtype_t dt, const void *W_row, const float *x, int block_count, int block_size) {
    if (!W_row || !x || block_count <= 0) return 0.0f;
    int nb = 0, cols = 0;
    if (quantized(dt)) {
        if (block_size != 32) return 0.0f;
        nb = block_count;
        cols = block_count * 32;
    } else {
        cols = (block_size == 1) ? block_count : block_count * block_size;
        nb = (cols + 31) / 32;
    }
    kernel_context_t *ctx = default_context();
    if (!ctx) {
        LOG_ERROR("row kernel: no GPU context available");
        return 0.0f;
    }
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    DeviceGuard g(ctx->device);
    const size_t wbytes = (dt == DTYPE_TQ2_0) ? 4 + (size_t)8 * nb : sapphire_row_bytes_internal(dt, cols);
    const size_t xbytes = (size_t)cols * sizeof(float);
    // Layout of d_g: [x | out | row bytes]
    const size_t need = xbytes + 16 + wbytes;
    if (ensure_scratch(ctx, &ctx->d_g, &ctx->d_g_cap, need + 64)) return 0.0f;
    float *dx = ctx->d_g;
    float *dout = reinterpret_cast<float *>(reinterpret_cast<char *>(ctx->d_g) + ((xbytes + 15) & ~(size_t)15));
    void *drow = reinterpret_cast<char *>(dout) + 16;
    cudaStream_t st = ctx->stream;
    float result = 0.0f;
    if (cudaMemcpyAsync(dx, x, xbytes, cudaMemcpyDefault, st) != cudaSuccess ||
        cudaMemcpyAsync(drow, W_row, wbytes, cudaMemcpyDefault, st) != cudaSuccess ||
        launch_row_dot(ctx, dt, drow, dx, nb, cols, dout, st) != 0 ||
        cudaMemcpyAsync(&result, dout, sizeof(float), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        ctx_fail(ctx, "row kernel", "device row product failed: %s", cudaGetErrorString(cudaGetLastError()));
        return 0.0f;
    }
    return result;
}

void gemm_rows_call(tensor_dtype_t dt, const gemm_args_t *a) {
    if (!a || !a->w_row || !a->X || !a->Y || a->batch_size <= 0) return;
    for (int i = 0; i < a->batch_size; ++i)
        a->Y[(size_t)i * a->out_stride] = row_call(dt, a->w_row, a->X + (size_t)i * a->d_model, a->d_model, 1);
}
}  // namespace

extern "C" SAPPHIRE_API float quantized_gemv_q4_0_aligned(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_Q4_0, W, x, n, bs);
}
extern "C" SAPPHIRE_API float quantized_gemv_q4_0_unaligned(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_Q4_0, W, x, n, bs);
}
extern "C" SAPPHIRE_API float quantized_gemv_q8_0_aligned(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_Q8_0, W, x, n, bs);
}
extern "C" SAPPHIRE_API float quantized_gemv_q8_0_unaligned(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_Q8_0, W, x, n, bs);
}
extern "C" SAPPHIRE_API float quantized_gemv_tq2_0(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_TQ2_0, W, x, n, bs);
}
extern "C" SAPPHIRE_API float quantized_gemv_bf16_avx2(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_BF16, W, x, n, bs);
}
extern "C" SAPPHIRE_API float quantized_gemv_bf16_scalar(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_BF16, W, x, n, bs);
}
extern "C" SAPPHIRE_API float quantized_gemv_f32_avx2(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_F32, W, x, n, bs);
}
extern "C" SAPPHIRE_API float quantized_gemv_f32_scalar(const void *W, const float *x, int n, int bs) {
    return row_call(DTYPE_F32, W, x, n, bs);
}
extern "C" SAPPHIRE_API void kernel_gemm_f32_avx2(const gemm_args_t *a) { gemm_rows_call(DTYPE_F32, a); }
extern "C" SAPPHIRE_API void kernel_gemm_bf16_avx2(const gemm_args_t *a) { gemm_rows_call(DTYPE_BF16, a); }
