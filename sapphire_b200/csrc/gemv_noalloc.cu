// gemv_noalloc.cu - kernel_gemv_device_noalloc: the batch-1 pipelined GEMV
// with its scratch in a fixed device array instead of memory the context
// allocates.
//
// Who needs it: code that must not call cudaMalloc / cudaFree at the moment
// it multiplies - for example a serving loop that owns a fixed memory budget
// or pool and forbids the runtime from growing it, or code on a path where an
// allocation (which may synchronise the device) would stall other streams.
// Such a caller uploads its weights while allocation is still allowed
// (kernel_tensor_upload at model load) and afterwards multiplies with this
// entry point, which allocates nothing.
//
// The scratch (split-tile partial sums and per-tile arrival counters) lives
// in g_noalloc_scratch below, kNoallocScratchBytes (4 MiB) per GPU, held by
// every GPU that loads this library until the process exits.  Host code
// cannot use the array's name as a device address; the device address is
// fetched once per device with cudaGetSymbolAddress.
//
// Errors: the kernel reports an expired bounded wait in the context's error
// word, a 4-byte mapped host word created by kernel_ctx_init (not here), so
// such an error surfaces as -1 from the next kernel_ctx_synchronize (or the
// next synchronous call) on the context.
#include "internal.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = (size_t)4 << 20;

// The scratch every call of kernel_gemv_device_noalloc shares.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_scratch on the current device (looked up once
// per device, with that device current).  nullptr on failure.
void *noalloc_scratch_ptr(kernel_context_t *ctx, int dev) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (dev < 0 || dev >= 64) return nullptr;
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            ctx_fail(ctx, "kernel_gemv_device_noalloc", "cudaGetSymbolAddress(scratch) failed: %s",
                     cudaGetErrorString(e));
            return nullptr;
        }
        g_noalloc_ptr[dev] = p;
    }
    return g_noalloc_ptr[dev];
}

}  // namespace

extern "C" SAPPHIRE_API int kernel_gemv_device_noalloc(kernel_context_t *ctx, float *y, const tensor_t *A,
                                                       const float *x) {
    if (!ctx || !y || !A || !x) {
        LOG_ERROR("kernel_gemv_device_noalloc: NULL argument");
        return -1;
    }
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (!ctx->initialized) {
        ctx_fail(ctx, "kernel_gemv_device_noalloc", "context not initialized");
        return -1;
    }
    if (ctx->world > 1) {
        ctx_fail(ctx, "kernel_gemv_device_noalloc", "not available on a sharded context");
        return -1;
    }
    // The weight must already be resident: uploading would allocate.
    auto it = ctx->weights.find(sapphire_tensor_uid(A));
    int rows = 0, cols = 0;
    if (it == ctx->weights.end() || !weight_shape(A, &rows, &cols) || it->second.src != tensor_data(A) ||
        it->second.rows != rows || it->second.cols != cols || it->second.dtype != tensor_dtype(A)) {
        ctx_fail(ctx, "kernel_gemv_device_noalloc",
                 "weight is not resident; call kernel_tensor_upload first (it allocates)");
        return -1;
    }
    const DevWeight &w = it->second;
    if (!pipe_supported(ctx, w)) {
        ctx_fail(ctx, "kernel_gemv_device_noalloc", "dtype %s / %d columns not supported by the pipelined kernel",
                 dtype_name(w.dtype), w.cols);
        return -1;
    }
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != ctx->device) cudaSetDevice(ctx->device);
    int xdev = -1, ydev = -1;
    int rc = 0;
    if (!ptr_is_device(x, &xdev) || !ptr_is_device(y, &ydev) || xdev != ctx->device || ydev != ctx->device) {
        ctx_fail(ctx, "kernel_gemv_device_noalloc", "x and y must be device memory of the context's GPU");
        rc = -1;
    }
    if (rc == 0 && !ctx->d_err) {
        ctx_fail(ctx, "kernel_gemv_device_noalloc", "context has no error word (kernel_ctx_init creates it)");
        rc = -1;
    }
    // Scratch layout: [counters (ntiles ints) | pad to 256 B | partial sums
    // (ntiles * kmax * 32 floats)].
    size_t part_floats = 0, cnt_ints = 0;
    if (rc == 0) pipe_scratch_size(ctx, w, &part_floats, &cnt_ints);
    const size_t cnt_off = 0;
    const size_t part_off = cnt_off + ((cnt_ints * sizeof(int) + 255) & ~(size_t)255);
    const size_t need = part_off + part_floats * sizeof(float);
    if (rc == 0 && need > kNoallocScratchBytes) {
        ctx_fail(ctx, "kernel_gemv_device_noalloc",
                 "weight needs %zu bytes of scratch, above the fixed %zu-byte maximum (%d rows x %d cols)", need,
                 kNoallocScratchBytes, w.rows, w.cols);
        rc = -1;
    }
    unsigned char *base = nullptr;
    if (rc == 0) {
        base = static_cast<unsigned char *>(noalloc_scratch_ptr(ctx, ctx->device));
        if (!base) rc = -1;
    }
    if (rc == 0) {
        // The array keeps the last call's contents: the arrival counters
        // must start at zero.
        cudaError_t e = cudaMemsetAsync(base, 0, part_off, ctx->stream);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "kernel_gemv_device_noalloc", "clearing scratch failed: %s", cudaGetErrorString(e));
            rc = -1;
        }
    }
    if (rc == 0)
        rc = launch_gemv_pipe(ctx, w, x, y, reinterpret_cast<float *>(base + part_off),
                              reinterpret_cast<int *>(base + cnt_off), ctx->d_err, ctx->stream);
    if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
    return rc;
}
