// quant.cu - quantisers, ternary packer, unpackers and one-row kernels.
//
// The reference ships no quantiser (src/tensor/tensor.c:238-244 is a stub),
// so the block formulas below are this library's definition; they follow the
// published Q4_0 / Q8_0 recipe with the reference's block structs
// (include/kernels.h:28-38) and its interleaved nibble order
// (src/kernels/q4_0_avx.c:61-65).  Every float step is a single IEEE-rounded
// operation written with __fmul_rn / __fadd_rn / __fdiv_rn so no FMA
// contraction can change a code: the CPU restatement in the test oracle
// produces the same bytes.
#include "internal.cuh"

namespace {

__device__ __forceinline__ void st_u32(uint8_t *p, uint32_t v, bool aligned) {
    if (aligned) {
        *reinterpret_cast<uint32_t *>(p) = v;
    } else {
        p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
    }
}

__device__ __forceinline__ uint32_t ld_u32(const uint8_t *p, bool aligned) {
    if (aligned) return *reinterpret_cast<const uint32_t *>(p);
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// One thread per (row, block).
__global__ void quantize_q4_0_kernel(const float *__restrict__ src, int rows, int cols, int nb,
                                     uint8_t *__restrict__ dst, bool aligned) {
    const size_t n = (size_t)rows * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / nb;
        const int b = (int)(i % nb);
        float v[32];
        const float *s = src + r * cols + (size_t)b * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (b * 32 + j < cols) ? s[j] : 0.0f;
        float amax = 0.0f, m = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float a = fabsf(v[j]);
            if (a > amax) { amax = a; m = v[j]; }
        }
        const float d = __fdiv_rn(m, -8.0f);
        const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
        uint32_t q[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float t = __fadd_rn(__fmul_rn(v[j], id), 8.5f);
            q[j] = (t >= 15.0f) ? 15u : (t >= 1.0f ? (uint32_t)__float2int_rz(t) : 0u);
        }
        uint8_t *out = dst + i * 20;
        st_u32(out, __float_as_uint(d), aligned);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            uint32_t word = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int e = 8 * w + 2 * k;          // byte 4w+k holds elements e, e+1
                word |= (q[e] | (q[e + 1] << 4)) << (8 * k);
            }
            st_u32(out + 4 + 4 * w, word, aligned);
        }
    }
}

__global__ void quantize_q8_0_kernel(const float *__restrict__ src, int rows, int cols, int nb,
                                     uint8_t *__restrict__ dst, bool aligned) {
    const size_t n = (size_t)rows * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / nb;
        const int b = (int)(i % nb);
        float v[32];
        const float *s = src + r * cols + (size_t)b * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (b * 32 + j < cols) ? s[j] : 0.0f;
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
        uint8_t *out = dst + i * 36;
        st_u32(out, __float_as_uint(d), aligned);
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            uint32_t word = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float t = roundf(__fmul_rn(v[4 * w + k], id));
                int q = (t != t) ? 0 : (t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t));
                word |= ((uint32_t)(uint8_t)(int8_t)q) << (8 * k);
            }
            st_u32(out + 4 + 4 * w, word, aligned);
        }
    }
}

// One thread per (row, block); err receives 1 if a trit is outside {-1,0,1}.
__global__ void pack_tq2_kernel(const int8_t *__restrict__ trits, const float *__restrict__ scales, int rows,
                                int cols, int nb, uint8_t *__restrict__ dst, int *err) {
    const size_t n = (size_t)rows * nb;
    const size_t row_bytes = 4 + (size_t)8 * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / nb;
        const int b = (int)(i % nb);
        uint8_t *row = dst + r * row_bytes;
        if (b == 0) {
            const float s = scales[r];
            const uint32_t u = __float_as_uint(s);
            row[0] = (uint8_t)u; row[1] = (uint8_t)(u >> 8); row[2] = (uint8_t)(u >> 16); row[3] = (uint8_t)(u >> 24);
        }
        uint8_t *blk = row + 4 + (size_t)8 * b;
        bool bad = false;
        for (int byte = 0; byte < 8; ++byte) {
            uint32_t v = 0;
            for (int p = 0; p < 4; ++p) {
                const int c = b * 32 + byte * 4 + p;
                int t = 0;
                if (c < cols) {
                    t = trits[r * cols + c];
                    if (t < -1 || t > 1) { bad = true; t = 0; }
                }
                v |= (uint32_t)(t + 1) << (2 * p);
            }
            blk[byte] = (uint8_t)v;
        }
        if (bad) atomicOr(err, 1);
    }
}

// Unpack: one thread per (row, block), writes the block's columns < cols.
__global__ void dequant_kernel(tensor_dtype_t dt, const uint8_t *__restrict__ src, int rows, int cols, int nb,
                               float *__restrict__ dst, bool aligned) {
    const size_t n = (size_t)rows * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / nb;
        const int b = (int)(i % nb);
        float *o = dst + r * cols + (size_t)b * 32;
        const int lim = min(32, cols - b * 32);
        if (dt == DTYPE_Q4_0) {
            const uint8_t *p = src + i * 20;
            const float s = __uint_as_float(ld_u32(p, aligned));
            for (int j = 0; j < lim; ++j) {
                const uint8_t byte = p[4 + j / 2];
                const int q = (j & 1) ? (byte >> 4) : (byte & 15);
                o[j] = __fmul_rn((float)(q - 8), s);
            }
        } else if (dt == DTYPE_Q8_0) {
            const uint8_t *p = src + i * 36;
            const float s = __uint_as_float(ld_u32(p, aligned));
            for (int j = 0; j < lim; ++j) o[j] = __fmul_rn((float)(int8_t)p[4 + j], s);
        } else if (dt == DTYPE_TQ2_0) {
            const uint8_t *row = src + r * (4 + (size_t)8 * nb);
            const float s = __uint_as_float(ld_u32(row, aligned));
            const uint8_t *blk = row + 4 + (size_t)8 * b;
            for (int j = 0; j < lim; ++j) {
                const int c = (blk[j / 4] >> (2 * (j % 4))) & 3;
                o[j] = __fmul_rn((float)(c - 1), s);
            }
        } else if (dt == DTYPE_F32) {
            const uint8_t *p = src + (r * cols + (size_t)b * 32) * 4;
            for (int j = 0; j < lim; ++j) o[j] = __uint_as_float(ld_u32(p + 4 * j, aligned));
        } else if (dt == DTYPE_BF16) {
            const uint8_t *p = src + (r * cols + (size_t)b * 32) * 2;
            for (int j = 0; j < lim; ++j) o[j] = __uint_as_float(((uint32_t)p[2 * j] | ((uint32_t)p[2 * j + 1] << 8)) << 16);
        }
    }
}

int grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    if (g > 148 * 64) g = 148 * 64;
    if (g == 0) g = 1;
    return (int)g;
}

int check_launch(kernel_context_t *ctx, const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ctx_fail(ctx, what, "launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

}  // namespace

int launch_quantize(kernel_context_t *ctx, tensor_dtype_t dt, void *dst, const float *src, int rows, int cols,
                    cudaStream_t st) {
    const int nb = (cols + 31) / 32;
    const size_t n = (size_t)rows * nb;
    const bool aligned = ((uintptr_t)dst & 3) == 0;
    if (dt == DTYPE_Q4_0)
        quantize_q4_0_kernel<<<grid_for(n), 256, 0, st>>>(src, rows, cols, nb, (uint8_t *)dst, aligned);
    else if (dt == DTYPE_Q8_0)
        quantize_q8_0_kernel<<<grid_for(n), 256, 0, st>>>(src, rows, cols, nb, (uint8_t *)dst, aligned);
    else {
        ctx_fail(ctx, "launch_quantize", "no quantiser for %s", dtype_name(dt));
        return -1;
    }
    return check_launch(ctx, "launch_quantize");
}

int launch_pack_tq2(kernel_context_t *ctx, void *dst, const int8_t *trits, const float *scales, int rows, int cols,
                    int *d_err, cudaStream_t st) {
    const int nb = (cols + 31) / 32;
    pack_tq2_kernel<<<grid_for((size_t)rows * nb), 256, 0, st>>>(trits, scales, rows, cols, nb, (uint8_t *)dst, d_err);
    return check_launch(ctx, "launch_pack_tq2");
}

int launch_dequantize(kernel_context_t *ctx, tensor_dtype_t dt, float *dst, const void *src, int rows, int cols,
                      cudaStream_t st) {
    const int nb = (cols + 31) / 32;
    const bool aligned = ((uintptr_t)src & 3) == 0;
    dequant_kernel<<<grid_for((size_t)rows * nb), 256, 0, st>>>(dt, (const uint8_t *)src, rows, cols, nb, dst, aligned);
    return check_launch(ctx, "launch_dequantize");
}

// ------------------------------------------------------------- row ABI ----
// One packed row in the reference layout, dotted with x[0 .. nb*32) by one
// CTA; the result goes to out[0].
namespace {
__global__ void row_dot_kernel(tensor_dtype_t dt, const uint8_t *__restrict__ row, const float *__restrict__ x,
                               int nb, int cols, float *out) {
    float acc = 0.0f;
    if (dt == DTYPE_Q4_0 || dt == DTYPE_Q8_0) {
        const int bytes = dt == DTYPE_Q4_0 ? 20 : 36;
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            const uint8_t *p = row + (size_t)b * bytes;
            const float s = __uint_as_float(ld_u32(p, false));
            float part = 0.0f;
            for (int j = 0; j < 32; ++j) {
                int q;
                if (dt == DTYPE_Q4_0) {
                    const uint8_t byte = p[4 + j / 2];
                    q = ((j & 1) ? (byte >> 4) : (byte & 15)) - 8;
                } else {
                    q = (int8_t)p[4 + j];
                }
                part = fmaf((float)q, x[b * 32 + j], part);
            }
            acc = fmaf(s, part, acc);
        }
    } else if (dt == DTYPE_TQ2_0) {
        const float s = __uint_as_float(ld_u32(row, false));
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            const uint8_t *blk = row + 4 + (size_t)b * 8;
            float part = 0.0f;
            for (int j = 0; j < 32; ++j) part = fmaf((float)(((blk[j / 4] >> (2 * (j % 4))) & 3) - 1), x[b * 32 + j], part);
            acc += part;
        }
        acc *= s;
    } else {
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            float w;
            if (dt == DTYPE_F32) w = __uint_as_float(ld_u32(row + (size_t)c * 4, false));
            else w = __uint_as_float(((uint32_t)row[2 * c] | ((uint32_t)row[2 * c + 1] << 8)) << 16);
            acc = fmaf(w, x[c], acc);
        }
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    __shared__ float red[32];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
        out[0] = t;
    }
}

__global__ void axpy_kernel(float *y, const float *t, float alpha, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = fmaf(alpha, t[i], y[i]);
}
}  // namespace

int launch_row_dot(kernel_context_t *ctx, tensor_dtype_t dt, const void *row, const float *x, int nb, int cols,
                   float *out, cudaStream_t st) {
    row_dot_kernel<<<1, 256, 0, st>>>(dt, (const uint8_t *)row, x, nb, cols, out);
    return check_launch(ctx, "launch_row_dot");
}

int launch_axpy(kernel_context_t *ctx, float *y, const float *t, float alpha, size_t n, cudaStream_t st) {
    axpy_kernel<<<grid_for(n), 256, 0, st>>>(y, t, alpha, n);
    return check_launch(ctx, "launch_axpy");
}
