// gemv.cu - small-batch GEMV for dense F32 / BF16 weights (tile layout).
//
// Computes what the reference's dense row kernels compute for every row
// (src/kernels/f32_avx.c:44-135, bf16_avx.c:55-150, applied per row by
// src/kernels/pool.c:106-143), for up to 8 activation rows per launch.
// Quantized formats use the pipelined tensor-core kernel (gemv_pipe.cu).
//
// Mapping: one warp owns one 32-row tile, lane i owns row tile*32+i for the
// whole K range, so there is no cross-lane reduction.  Each lane streams its
// row's 16-byte chunks with coalesced warp-wide 512-byte loads (tile layout in
// internal.cuh) and reads x from shared memory at addresses that are uniform
// across the warp (broadcast, no bank conflicts).
#include "internal.cuh"

namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kThreads = kWarpsPerCta * 32;

template <tensor_dtype_t DT>
struct Step;

template <>
struct Step<DTYPE_F32> {
    static constexpr int kW = 4;
    template <int B>
    static __device__ __forceinline__ void chunk(uint4 c, const float *xs, int xstride, float (&part)[B]) {
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float4 v = *reinterpret_cast<const float4 *>(xs + b * xstride);
            float a = part[b];
            a = fmaf(__uint_as_float(c.x), v.x, a);
            a = fmaf(__uint_as_float(c.y), v.y, a);
            a = fmaf(__uint_as_float(c.z), v.z, a);
            a = fmaf(__uint_as_float(c.w), v.w, a);
            part[b] = a;
        }
    }
};

template <>
struct Step<DTYPE_BF16> {
    static constexpr int kW = 8;
    template <int B>
    static __device__ __forceinline__ void chunk(uint4 c, const float *xs, int xstride, float (&part)[B]) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        float f[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i + 0] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float4 *x4 = reinterpret_cast<const float4 *>(xs + b * xstride);
            const float4 v0 = x4[0], v1 = x4[1];
            float a = part[b];
            a = fmaf(f[0], v0.x, a);
            a = fmaf(f[1], v0.y, a);
            a = fmaf(f[2], v0.z, a);
            a = fmaf(f[3], v0.w, a);
            a = fmaf(f[4], v1.x, a);
            a = fmaf(f[5], v1.y, a);
            a = fmaf(f[6], v1.z, a);
            a = fmaf(f[7], v1.w, a);
            part[b] = a;
        }
    }
};

template <tensor_dtype_t DT, int B>
__global__ void __launch_bounds__(kThreads)
gemv_dense(const uint4 *__restrict__ codes, const float *__restrict__ x, int x_stride, float *__restrict__ y,
           int y_stride, int nrows, int cols, int kchunks, int ntiles) {
    extern __shared__ float4 smem4[];
    float *xs = reinterpret_cast<float *>(smem4);
    constexpr int W = Step<DT>::kW;
    const int xpad = kchunks * W;
    for (int b = 0; b < B; ++b)
        for (int i = threadIdx.x; i < xpad; i += blockDim.x)
            xs[b * xpad + i] = (i < cols) ? x[(size_t)b * x_stride + i] : 0.0f;
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int tile = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (tile >= ntiles) return;
    const uint4 *cp = codes + (size_t)tile * kchunks * 32 + lane;
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.0f;
    constexpr int G = 8;
    int kc = 0;
    for (; kc + G <= kchunks; kc += G) {
        uint4 c[G];
#pragma unroll
        for (int i = 0; i < G; ++i) c[i] = __ldg(cp + (size_t)(kc + i) * 32);
#pragma unroll
        for (int i = 0; i < G; ++i) Step<DT>::template chunk<B>(c[i], xs + (kc + i) * W, xpad, acc);
    }
    for (; kc < kchunks; ++kc) Step<DT>::template chunk<B>(__ldg(cp + (size_t)kc * 32), xs + kc * W, xpad, acc);
    const int row = tile * 32 + lane;
    if (row < nrows) {
#pragma unroll
        for (int b = 0; b < B; ++b) y[(size_t)b * y_stride + row] = acc[b];
    }
}

constexpr size_t kMaxSmem = 227 * 1024;

template <typename K>
int prepare(kernel_context_t *ctx, K kernel, size_t smem) {
    if (smem > kMaxSmem) {
        ctx_fail(ctx, "launch_gemv", "activation rows need %zu bytes of shared memory (max %zu)", smem, kMaxSmem);
        return -1;
    }
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "launch_gemv", "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return -1;
        }
    }
    return 0;
}

template <int B>
int launch_b(kernel_context_t *ctx, const DevWeight &w, const float *x, int xs, float *y, int ys, cudaStream_t st) {
    const int grid = (w.ntiles + kWarpsPerCta - 1) / kWarpsPerCta;
    if (grid == 0) return 0;
    const size_t xpad = (size_t)w.kchunks * chunk_weights(w.dtype);
    const size_t smem = (size_t)B * xpad * sizeof(float);
    if (w.dtype == DTYPE_F32) {
        auto k = gemv_dense<DTYPE_F32, B>;
        if (prepare(ctx, k, smem)) return -1;
        k<<<grid, kThreads, smem, st>>>(w.codes, x, xs, y, ys, w.nrows, w.cols, w.kchunks, w.ntiles);
    } else if (w.dtype == DTYPE_BF16) {
        auto k = gemv_dense<DTYPE_BF16, B>;
        if (prepare(ctx, k, smem)) return -1;
        k<<<grid, kThreads, smem, st>>>(w.codes, x, xs, y, ys, w.nrows, w.cols, w.kchunks, w.ntiles);
    } else {
        ctx_fail(ctx, "launch_gemv", "no batched tile kernel for dtype %s", dtype_name(w.dtype));
        return -1;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ctx_fail(ctx, "launch_gemv", "kernel launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

}  // namespace

int launch_gemv(kernel_context_t *ctx, const DevWeight &w, const float *x, int x_stride, float *y, int y_stride,
                int batch, cudaStream_t stream) {
    const size_t row_smem = (size_t)w.kchunks * chunk_weights(w.dtype) * sizeof(float);
    int done = 0;
    while (done < batch) {
        const int left = batch - done;
        int b = left >= 8 ? 8 : left >= 4 ? 4 : left >= 2 ? 2 : 1;
        while (b > 1 && (size_t)b * row_smem > kMaxSmem) b >>= 1;
        const float *xb = x + (size_t)done * x_stride;
        float *yb = y + (size_t)done * y_stride;
        int rc;
        switch (b) {
            case 8: rc = launch_b<8>(ctx, w, xb, x_stride, yb, y_stride, stream); break;
            case 4: rc = launch_b<4>(ctx, w, xb, x_stride, yb, y_stride, stream); break;
            case 2: rc = launch_b<2>(ctx, w, xb, x_stride, yb, y_stride, stream); break;
            default: rc = launch_b<1>(ctx, w, xb, x_stride, yb, y_stride, stream); break;
        }
        if (rc) return rc;
        done += b;
    }
    return 0;
}
