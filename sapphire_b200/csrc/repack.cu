// repack.cu - host block layout -> GEMV tile layout (see internal.cuh).
//
// Input rows are the reference's packed formats, rows back to back
// (row r starts at r * row_bytes, src/kernels/pool.c:297-301):
//   Q4_0 20-byte and Q8_0 36-byte blocks (include/kernels.h:28-38), TQ2_0 rows
//   (fp32 scale + 8-byte trit blocks), dense F32 / BF16 rows.
// The repack only moves bytes: codes and scales keep their exact bits.
#include "internal.cuh"

namespace {

// Load 4 bytes from a possibly unaligned address.
__device__ __forceinline__ uint32_t ld_u32(const uint8_t *p, bool aligned) {
    if (aligned) return *reinterpret_cast<const uint32_t *>(p);
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// One thread per (tile, block, lane).  Q8_0: two output chunks per block.
__global__ void repack_q8_0(const uint8_t *__restrict__ src, int nrows, int nb, int tile0, int ntile_in,
                            uint4 *__restrict__ codes, float *__restrict__ scales, bool aligned) {
    const size_t n = (size_t)ntile_in * nb * 32;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const size_t tb = i >> 5;                  // tile_local * nb + b
        const int b = (int)(tb % nb);
        const int tl = (int)(tb / nb);
        const int r = tl * 32 + lane;              // row within this upload chunk
        uint32_t w[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
        if (r < nrows) {
            const uint8_t *p = src + ((size_t)r * nb + b) * 36;
#pragma unroll
            for (int k = 0; k < 9; ++k) w[k] = ld_u32(p + 4 * k, aligned);
        }
        const size_t tile = (size_t)tile0 + tl;
        codes[(tile * 2 * nb + 2 * b + 0) * 32 + lane] = make_uint4(w[1], w[2], w[3], w[4]);
        codes[(tile * 2 * nb + 2 * b + 1) * 32 + lane] = make_uint4(w[5], w[6], w[7], w[8]);
        scales[(tile * nb + b) * 32 + lane] = __uint_as_float(w[0]);
    }
}

__global__ void repack_q4_0(const uint8_t *__restrict__ src, int nrows, int nb, int tile0, int ntile_in,
                            uint4 *__restrict__ codes, float *__restrict__ scales, bool aligned) {
    const size_t n = (size_t)ntile_in * nb * 32;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const size_t tb = i >> 5;
        const int b = (int)(tb % nb);
        const int tl = (int)(tb / nb);
        const int r = tl * 32 + lane;
        uint32_t w[5] = {0, 0, 0, 0, 0};
        if (r < nrows) {
            const uint8_t *p = src + ((size_t)r * nb + b) * 20;
#pragma unroll
            for (int k = 0; k < 5; ++k) w[k] = ld_u32(p + 4 * k, aligned);
        }
        const size_t tile = (size_t)tile0 + tl;
        codes[(tile * nb + b) * 32 + lane] = make_uint4(w[1], w[2], w[3], w[4]);
        scales[(tile * nb + b) * 32 + lane] = __uint_as_float(w[0]);
    }
}

// TQ2_0 row: 4-byte scale then nb 8-byte blocks; one output chunk = 2 blocks.
__global__ void repack_tq2_0(const uint8_t *__restrict__ src, int nrows, int nb, int kchunks, int tile0,
                             int ntile_in, uint4 *__restrict__ codes, float *__restrict__ scales, bool aligned) {
    const size_t row_bytes = 4 + (size_t)8 * nb;
    const size_t n = (size_t)ntile_in * kchunks * 32;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const size_t tk = i >> 5;
        const int kc = (int)(tk % kchunks);
        const int tl = (int)(tk / kchunks);
        const int r = tl * 32 + lane;
        // Padding trits decode to 0 (code 1) so padded columns stay inert even
        // if the staged activation were not zero there.
        uint32_t w[4] = {0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u};
        uint32_t s = 0;
        if (r < nrows) {
            const uint8_t *p = src + (size_t)r * row_bytes;
            if (kc == 0) s = ld_u32(p, aligned);
            const uint8_t *q = p + 4 + (size_t)16 * kc;
            w[0] = ld_u32(q, aligned);
            w[1] = ld_u32(q + 4, aligned);
            if (2 * kc + 1 < nb) {
                w[2] = ld_u32(q + 8, aligned);
                w[3] = ld_u32(q + 12, aligned);
            }
        }
        const size_t tile = (size_t)tile0 + tl;
        codes[(tile * kchunks + kc) * 32 + lane] = make_uint4(w[0], w[1], w[2], w[3]);
        if (kc == 0) scales[tile * 32 + lane] = __uint_as_float(s);
    }
}

// Dense rows: W elements of `esize` bytes per 16-byte chunk.
__global__ void repack_dense(const uint8_t *__restrict__ src, int nrows, int cols, int esize, int kchunks,
                             int tile0, int ntile_in, uint4 *__restrict__ codes) {
    const int per = 16 / esize;
    const size_t n = (size_t)ntile_in * kchunks * 32;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const size_t tk = i >> 5;
        const int kc = (int)(tk % kchunks);
        const int tl = (int)(tk / kchunks);
        const int r = tl * 32 + lane;
        uint8_t bytes[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) bytes[k] = 0;
        if (r < nrows) {
            const uint8_t *p = src + (size_t)r * cols * esize;
            for (int e = 0; e < per; ++e) {
                const int c = kc * per + e;
                if (c < cols)
                    for (int k = 0; k < esize; ++k) bytes[e * esize + k] = p[(size_t)c * esize + k];
            }
        }
        uint4 v;
        v.x = bytes[0] | (bytes[1] << 8) | (bytes[2] << 16) | ((uint32_t)bytes[3] << 24);
        v.y = bytes[4] | (bytes[5] << 8) | (bytes[6] << 16) | ((uint32_t)bytes[7] << 24);
        v.z = bytes[8] | (bytes[9] << 8) | (bytes[10] << 16) | ((uint32_t)bytes[11] << 24);
        v.w = bytes[12] | (bytes[13] << 8) | (bytes[14] << 16) | ((uint32_t)bytes[15] << 24);
        const size_t tile = (size_t)tile0 + tl;
        codes[(tile * kchunks + kc) * 32 + lane] = v;
    }
}

int grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    if (g > 148 * 64) g = 148 * 64;
    if (g == 0) g = 1;
    return (int)g;
}

}  // namespace

int launch_repack(kernel_context_t *ctx, const DevWeight &w, const void *src, int nrows, int tile0,
                  cudaStream_t st) {
    const int ntile_in = (nrows + 31) / 32;
    if (ntile_in == 0) return 0;
    const uint8_t *s = static_cast<const uint8_t *>(src);
    const bool aligned = ((uintptr_t)src & 3) == 0;
    switch (w.dtype) {
        case DTYPE_Q8_0: {
            size_t n = (size_t)ntile_in * w.nb * 32;
            repack_q8_0<<<grid_for(n), 256, 0, st>>>(s, nrows, w.nb, tile0, ntile_in, w.codes, w.scales, aligned);
            break;
        }
        case DTYPE_Q4_0: {
            size_t n = (size_t)ntile_in * w.nb * 32;
            repack_q4_0<<<grid_for(n), 256, 0, st>>>(s, nrows, w.nb, tile0, ntile_in, w.codes, w.scales, aligned);
            break;
        }
        case DTYPE_TQ2_0: {
            size_t n = (size_t)ntile_in * w.kchunks * 32;
            repack_tq2_0<<<grid_for(n), 256, 0, st>>>(s, nrows, w.nb, w.kchunks, tile0, ntile_in, w.codes,
                                                      w.scales, aligned);
            break;
        }
        case DTYPE_F32:
        case DTYPE_BF16: {
            size_t n = (size_t)ntile_in * w.kchunks * 32;
            int es = w.dtype == DTYPE_F32 ? 4 : 2;
            repack_dense<<<grid_for(n), 256, 0, st>>>(s, nrows, w.cols, es, w.kchunks, tile0, ntile_in, w.codes);
            break;
        }
        default:
            ctx_fail(ctx, "launch_repack", "dtype %s has no device layout", dtype_name(w.dtype));
            return -1;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ctx_fail(ctx, "launch_repack", "launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
