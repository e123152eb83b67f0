// gemv.cu - batch-1 (and small-batch) GEMV kernels over the tile layout.
//
// Computes what the reference row kernels compute for every row
// (src/kernels/q4_0_avx.c:102-148, q8_0_avx.c:16-136, f32_avx.c, bf16_avx.c,
// driven per row by the pool in src/kernels/pool.c:106-143), plus the ternary
// format of this library:
//     Q4_0 : y_r = sum_b scale_rb * sum_j (q_rbj - 8) * x_{32b+j}
//     Q8_0 : y_r = sum_b scale_rb * sum_j  q_rbj      * x_{32b+j}
//     TQ2_0: y_r = scale_r * sum_j (c_rj - 1) * x_j
//     F32 / BF16: plain dot products.
// The reference multiplies each code by its scale before the FMA; here the
// block's integer-weighted sum is formed first and scaled once per block.
// Both are fp32 with fp32 accumulation; results agree to rounding.
//
// Mapping: one warp owns one 32-row tile, lane i owns row tile*32+i for the
// whole K range, so there is no cross-lane reduction.  Each lane streams its
// row's 16-byte chunks with coalesced warp-wide 512-byte loads (see the tile
// layout in internal.cuh) and reads x from shared memory at addresses that are
// uniform across the warp (broadcast, no bank conflicts).
//
// Integer codes become floats without I2F: a code byte u placed in the low
// mantissa bits of 2^23 (bit pattern 0x4B0000uu) is the float 2^23 + u, and one
// FADD removes the offset exactly.
#include "internal.cuh"

namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kThreads = kWarpsPerCta * 32;
constexpr float kTwo23 = 8388608.0f;

// Float value 2^23 + (byte k of w).
__device__ __forceinline__ float byte_plus_2p23(uint32_t w, const int k) {
    return __int_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (unsigned)k));
}

template <tensor_dtype_t DT>
struct Step;

// ---------------------------------------------------------------- Q8_0 ----
template <>
struct Step<DTYPE_Q8_0> {
    // 16 int8 codes times x[0..16), added to part[] (no scale).
    template <int B>
    static __device__ __forceinline__ void chunk(uint4 c, const float *xs, int xstride, float (&part)[B]) {
        const uint32_t w[4] = {c.x ^ 0x80808080u, c.y ^ 0x80808080u, c.z ^ 0x80808080u,
                               c.w ^ 0x80808080u};
        float f[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[4 * i + 0] = byte_plus_2p23(w[i], 0) - (kTwo23 + 128.0f);
            f[4 * i + 1] = byte_plus_2p23(w[i], 1) - (kTwo23 + 128.0f);
            f[4 * i + 2] = byte_plus_2p23(w[i], 2) - (kTwo23 + 128.0f);
            f[4 * i + 3] = byte_plus_2p23(w[i], 3) - (kTwo23 + 128.0f);
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float4 *x4 = reinterpret_cast<const float4 *>(xs + b * xstride);
            float a0 = part[b], a1 = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 v = x4[i];
                a0 = fmaf(f[4 * i + 0], v.x, a0);
                a1 = fmaf(f[4 * i + 1], v.y, a1);
                a0 = fmaf(f[4 * i + 2], v.z, a0);
                a1 = fmaf(f[4 * i + 3], v.w, a1);
            }
            part[b] = a0 + a1;
        }
    }
};

// ---------------------------------------------------------------- Q4_0 ----
template <>
struct Step<DTYPE_Q4_0> {
    // One block: 32 nibbles (byte i = elements 2i | 2i+1 << 4) times x[0..32).
    template <int B>
    static __device__ __forceinline__ void chunk(uint4 c, const float *xs, int xstride, float (&part)[B]) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        float f[32];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = w[i] & 0x0F0F0F0Fu;
            const uint32_t hi = (w[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                f[8 * i + 2 * k + 0] = byte_plus_2p23(lo, k) - (kTwo23 + 8.0f);
                f[8 * i + 2 * k + 1] = byte_plus_2p23(hi, k) - (kTwo23 + 8.0f);
            }
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float4 *x4 = reinterpret_cast<const float4 *>(xs + b * xstride);
            float a0 = part[b], a1 = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 v = x4[i];
                a0 = fmaf(f[4 * i + 0], v.x, a0);
                a1 = fmaf(f[4 * i + 1], v.y, a1);
                a0 = fmaf(f[4 * i + 2], v.z, a0);
                a1 = fmaf(f[4 * i + 3], v.w, a1);
            }
            part[b] = a0 + a1;
        }
    }
};

// --------------------------------------------------------------- TQ2_0 ----
template <>
struct Step<DTYPE_TQ2_0> {
    // 64 trits (4 words x 4 bytes x 4 trits).  Trit p of a byte (bits 2p..2p+1)
    // is decoded in place as (c - 1) * 4^p by keeping the exponent byte and
    // its two bits; acc[p] collects those and the caller rescales by 4^-p.
    template <int B>
    static __device__ __forceinline__ void chunk(uint4 c, const float *xs, int xstride, float (&acc)[4][B]) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t bb = __byte_perm(w[i], 0x4B000000u, 0x7440u | (unsigned)k);
                const float f0 = __int_as_float(bb & 0x4B000003u) - (kTwo23 + 1.0f);
                const float f1 = __int_as_float(bb & 0x4B00000Cu) - (kTwo23 + 4.0f);
                const float f2 = __int_as_float(bb & 0x4B000030u) - (kTwo23 + 16.0f);
                const float f3 = __int_as_float(bb & 0x4B0000C0u) - (kTwo23 + 64.0f);
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float4 v = reinterpret_cast<const float4 *>(xs + b * xstride)[4 * i + k];
                    acc[0][b] = fmaf(f0, v.x, acc[0][b]);
                    acc[1][b] = fmaf(f1, v.y, acc[1][b]);
                    acc[2][b] = fmaf(f2, v.z, acc[2][b]);
                    acc[3][b] = fmaf(f3, v.w, acc[3][b]);
                }
            }
        }
    }
};

// ---------------------------------------------------------------- dense ---
template <>
struct Step<DTYPE_F32> {
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

__device__ __forceinline__ uint4 ld_chunk(const uint4 *p) { return __ldg(p); }

// Stage B rows of x (cols floats, row stride x_stride) into shared memory,
// zero-padded to xpad floats per row.
template <int B>
__device__ __forceinline__ void stage_x(float *xs, const float *__restrict__ x, int x_stride, int cols, int xpad) {
    for (int b = 0; b < B; ++b)
        for (int i = threadIdx.x; i < xpad; i += blockDim.x)
            xs[b * xpad + i] = (i < cols) ? x[(size_t)b * x_stride + i] : 0.0f;
    __syncthreads();
}

// ----------------------------------------------------------- kernels ------
// Per-block-scaled formats (Q8_0: 2 chunks per block, Q4_0: 1 chunk per block).
template <tensor_dtype_t DT, int CPB, int B>
__global__ void __launch_bounds__(kThreads)
gemv_blockscaled(const uint4 *__restrict__ codes, const float *__restrict__ scales,
                 const float *__restrict__ x, int x_stride, float *__restrict__ y, int y_stride,
                 int nrows, int cols, int nb, int ntiles) {
    extern __shared__ float4 smem4[];
    float *xs = reinterpret_cast<float *>(smem4);
    const int xpad = nb * 32;
    stage_x<B>(xs, x, x_stride, cols, xpad);

    const int lane = threadIdx.x & 31;
    const int tile = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (tile >= ntiles) return;
    const int kchunks = nb * CPB;
    const uint4 *cp = codes + (size_t)tile * kchunks * 32 + lane;
    const float *sp = scales + (size_t)tile * nb * 32 + lane;

    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.0f;

    constexpr int G = (CPB == 2) ? 4 : 8;   // blocks per unrolled group (8 x 16 B in flight)
    int blk = 0;
    for (; blk + G <= nb; blk += G) {
        uint4 c[G * CPB];
        float s[G];
#pragma unroll
        for (int i = 0; i < G * CPB; ++i) c[i] = ld_chunk(cp + (size_t)(blk * CPB + i) * 32);
#pragma unroll
        for (int i = 0; i < G; ++i) s[i] = __ldg(sp + (size_t)(blk + i) * 32);
#pragma unroll
        for (int i = 0; i < G; ++i) {
            float part[B];
#pragma unroll
            for (int b = 0; b < B; ++b) part[b] = 0.0f;
#pragma unroll
            for (int h = 0; h < CPB; ++h)
                Step<DT>::template chunk<B>(c[i * CPB + h], xs + (blk + i) * 32 + h * (32 / CPB), xpad, part);
#pragma unroll
            for (int b = 0; b < B; ++b) acc[b] = fmaf(s[i], part[b], acc[b]);
        }
    }
    for (; blk < nb; ++blk) {
        uint4 c[CPB];
#pragma unroll
        for (int h = 0; h < CPB; ++h) c[h] = ld_chunk(cp + (size_t)(blk * CPB + h) * 32);
        const float s = __ldg(sp + (size_t)blk * 32);
        float part[B];
#pragma unroll
        for (int b = 0; b < B; ++b) part[b] = 0.0f;
#pragma unroll
        for (int h = 0; h < CPB; ++h)
            Step<DT>::template chunk<B>(c[h], xs + blk * 32 + h * (32 / CPB), xpad, part);
#pragma unroll
        for (int b = 0; b < B; ++b) acc[b] = fmaf(s, part[b], acc[b]);
    }

    const int row = tile * 32 + lane;
    if (row < nrows) {
#pragma unroll
        for (int b = 0; b < B; ++b) y[(size_t)b * y_stride + row] = acc[b];
    }
}

// Ternary: one row scale, four position accumulators.
template <int B>
__global__ void __launch_bounds__(kThreads)
gemv_tq2(const uint4 *__restrict__ codes, const float *__restrict__ scales,
         const float *__restrict__ x, int x_stride, float *__restrict__ y, int y_stride,
         int nrows, int cols, int kchunks, int ntiles) {
    extern __shared__ float4 smem4[];
    float *xs = reinterpret_cast<float *>(smem4);
    const int xpad = kchunks * 64;
    stage_x<B>(xs, x, x_stride, cols, xpad);

    const int lane = threadIdx.x & 31;
    const int tile = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (tile >= ntiles) return;
    const uint4 *cp = codes + (size_t)tile * kchunks * 32 + lane;

    float acc[4][B];
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int b = 0; b < B; ++b) acc[p][b] = 0.0f;

    constexpr int G = 8;
    int kc = 0;
    for (; kc + G <= kchunks; kc += G) {
        uint4 c[G];
#pragma unroll
        for (int i = 0; i < G; ++i) c[i] = ld_chunk(cp + (size_t)(kc + i) * 32);
#pragma unroll
        for (int i = 0; i < G; ++i) Step<DTYPE_TQ2_0>::template chunk<B>(c[i], xs + (kc + i) * 64, xpad, acc);
    }
    for (; kc < kchunks; ++kc) {
        const uint4 c = ld_chunk(cp + (size_t)kc * 32);
        Step<DTYPE_TQ2_0>::template chunk<B>(c, xs + kc * 64, xpad, acc);
    }
    const int row = tile * 32 + lane;
    if (row < nrows) {
        const float s = __ldg(scales + (size_t)tile * 32 + lane);
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float d = acc[0][b] + 0.25f * acc[1][b] + 0.0625f * acc[2][b] + 0.015625f * acc[3][b];
            y[(size_t)b * y_stride + row] = s * d;
        }
    }
}

// Dense F32 / BF16 (no scales).
template <tensor_dtype_t DT, int B>
__global__ void __launch_bounds__(kThreads)
gemv_dense(const uint4 *__restrict__ codes, const float *__restrict__ x, int x_stride,
           float *__restrict__ y, int y_stride, int nrows, int cols, int kchunks, int ntiles) {
    extern __shared__ float4 smem4[];
    float *xs = reinterpret_cast<float *>(smem4);
    constexpr int W = (DT == DTYPE_F32) ? 4 : 8;
    const int xpad = kchunks * W;
    stage_x<B>(xs, x, x_stride, cols, xpad);

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
        for (int i = 0; i < G; ++i) c[i] = ld_chunk(cp + (size_t)(kc + i) * 32);
#pragma unroll
        for (int i = 0; i < G; ++i) Step<DT>::template chunk<B>(c[i], xs + (kc + i) * W, xpad, acc);
    }
    for (; kc < kchunks; ++kc) Step<DT>::template chunk<B>(ld_chunk(cp + (size_t)kc * 32), xs + kc * W, xpad, acc);
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
        ctx_fail(ctx, "launch_gemv", "activation rows need %zu bytes of shared memory (max %zu)",
                 smem, kMaxSmem);
        return -1;
    }
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kMaxSmem);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "launch_gemv", "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return -1;
        }
    }
    return 0;
}

template <int B>
int launch_b(kernel_context_t *ctx, const DevWeight &w, const float *x, int xs, float *y, int ys,
             cudaStream_t st) {
    const int grid = (w.ntiles + kWarpsPerCta - 1) / kWarpsPerCta;
    if (grid == 0) return 0;
    const size_t xpad = (size_t)w.kchunks * chunk_weights(w.dtype);
    const size_t smem = (size_t)B * xpad * sizeof(float);
    switch (w.dtype) {
        case DTYPE_Q8_0: {
            auto k = gemv_blockscaled<DTYPE_Q8_0, 2, B>;
            if (prepare(ctx, k, smem)) return -1;
            k<<<grid, kThreads, smem, st>>>(w.codes, w.scales, x, xs, y, ys, w.nrows, w.cols, w.nb, w.ntiles);
            break;
        }
        case DTYPE_Q4_0: {
            auto k = gemv_blockscaled<DTYPE_Q4_0, 1, B>;
            if (prepare(ctx, k, smem)) return -1;
            k<<<grid, kThreads, smem, st>>>(w.codes, w.scales, x, xs, y, ys, w.nrows, w.cols, w.nb, w.ntiles);
            break;
        }
        case DTYPE_TQ2_0: {
            auto k = gemv_tq2<B>;
            if (prepare(ctx, k, smem)) return -1;
            k<<<grid, kThreads, smem, st>>>(w.codes, w.scales, x, xs, y, ys, w.nrows, w.cols, w.kchunks, w.ntiles);
            break;
        }
        case DTYPE_F32: {
            auto k = gemv_dense<DTYPE_F32, B>;
            if (prepare(ctx, k, smem)) return -1;
            k<<<grid, kThreads, smem, st>>>(w.codes, x, xs, y, ys, w.nrows, w.cols, w.kchunks, w.ntiles);
            break;
        }
        case DTYPE_BF16: {
            auto k = gemv_dense<DTYPE_BF16, B>;
            if (prepare(ctx, k, smem)) return -1;
            k<<<grid, kThreads, smem, st>>>(w.codes, x, xs, y, ys, w.nrows, w.cols, w.kchunks, w.ntiles);
            break;
        }
        default:
            ctx_fail(ctx, "launch_gemv", "no GEMV kernel for dtype %s", dtype_name(w.dtype));
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

int launch_gemv(kernel_context_t *ctx, const DevWeight &w, const float *x, int x_stride, float *y,
                int y_stride, int batch, cudaStream_t stream) {
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
