// repack.cu - host block layout -> device layout (see internal.cuh).
//
// Input rows are the reference's packed formats, rows back to back
// (row r starts at r * row_bytes, src/kernels/pool.c:297-301):
//   Q4_0 20-byte and Q8_0 36-byte blocks (include/kernels.h:28-38), TQ2_0 rows
//   (fp32 scale + 8-byte trit blocks), dense F32 / BF16 rows.
// The repack only moves bytes: codes and scales keep their exact bits.
//
// Quantized formats go to the fragment layout: for each 32-row tile and
// 32-column block, the bytes a warp lane (g = lane/4, tig = lane%4) feeds to
// mma.sync m16n8k32 as its A operand are stored contiguously per lane:
//   Q8_0 : per half h (rows 16h+g, 16h+g+8) a uint4 {r0 bytes 4tig..+3,
//          r1 bytes 4tig..+3, r0 bytes 16+4tig..+3, r1 bytes 16+4tig..+3};
//          1024 bytes per (tile, block), half-major then lane.
//   Q4_0 : a uint4 of code word tig (bytes 4tig..4tig+3, i.e. elements
//          8tig..8tig+7) of rows g, g+8, g+16, g+24; 512 bytes per (tile, block).
//   TQ2_0: per pair of blocks (a "unit", 64 columns) a uint4 per lane whose
//          2-bit planes are four A fragments (repack_tq2_0 below); 512 bytes
//          per (tile, unit).
// Scales: per (tile, block) (Q8_0 / Q4_0), 32 floats in the order
// g*4 + i -> row g + 8i; per tile (TQ2_0), 32 floats in row order.  Rows past
// the tensor are zero codes (TQ2_0: code 1, trit 0) with zero scales.
#include "internal.cuh"

namespace {

// Load 4 bytes from a possibly unaligned address.
__device__ __forceinline__ uint32_t ld_u32(const uint8_t *p, bool aligned) {
    if (aligned) return *reinterpret_cast<const uint32_t *>(p);
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Scale slot q (0..31) of a tile holds row (q / 4) + 8 * (q % 4).
__device__ __forceinline__ int scale_row(int q) { return (q >> 2) + 8 * (q & 3); }

// Q8_0: one thread per (tile, block, half, lane).
__global__ void repack_q8_0(const uint8_t *__restrict__ src, int nrows, int nb, int tile0, int ntile_in,
                            uint4 *__restrict__ codes, float *__restrict__ scales, bool aligned) {
    const size_t n = (size_t)ntile_in * nb * 64;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const int h = (int)((i >> 5) & 1);
        const size_t tb = i >> 6;                  // tile_local * nb + b
        const int b = (int)(tb % nb);
        const int tl = (int)(tb / nb);
        const int g = lane >> 2, tig = lane & 3;
        const int r0 = tl * 32 + 16 * h + g, r1 = r0 + 8;
        uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
        if (r0 < nrows) {
            const uint8_t *p = src + ((size_t)r0 * nb + b) * 36 + 4;
            a0 = ld_u32(p + 4 * tig, aligned);
            a2 = ld_u32(p + 16 + 4 * tig, aligned);
        }
        if (r1 < nrows) {
            const uint8_t *p = src + ((size_t)r1 * nb + b) * 36 + 4;
            a1 = ld_u32(p + 4 * tig, aligned);
            a3 = ld_u32(p + 16 + 4 * tig, aligned);
        }
        const size_t tile = (size_t)tile0 + tl;
        codes[((tile * nb + b) * 2 + h) * 32 + lane] = make_uint4(a0, a1, a2, a3);
        if (h == 0) {
            const int r = tl * 32 + scale_row(lane);
            scales[(tile * nb + b) * 32 + lane] =
                r < nrows ? __uint_as_float(ld_u32(src + ((size_t)r * nb + b) * 36, aligned)) : 0.0f;
        }
    }
}

// Q4_0: one thread per (tile, block, lane).
__global__ void repack_q4_0(const uint8_t *__restrict__ src, int nrows, int nb, int tile0, int ntile_in,
                            uint4 *__restrict__ codes, float *__restrict__ scales, bool aligned) {
    const size_t n = (size_t)ntile_in * nb * 32;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const size_t tb = i >> 5;
        const int b = (int)(tb % nb);
        const int tl = (int)(tb / nb);
        const int g = lane >> 2, tig = lane & 3;
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int r = tl * 32 + g + 8 * k;
            w[k] = r < nrows ? ld_u32(src + ((size_t)r * nb + b) * 20 + 4 + 4 * tig, aligned) : 0u;
        }
        const size_t tile = (size_t)tile0 + tl;
        codes[(tile * nb + b) * 32 + lane] = make_uint4(w[0], w[1], w[2], w[3]);
        const int r = tl * 32 + scale_row(lane);
        scales[(tile * nb + b) * 32 + lane] =
            r < nrows ? __uint_as_float(ld_u32(src + ((size_t)r * nb + b) * 20, aligned)) : 0.0f;
    }
}

// TQ2_0 row: 4-byte scale then nb 8-byte blocks.  One thread per (tile,
// unit, lane); unit p holds blocks 2p and 2p+1 as four words per lane whose
// 2-bit planes are four mma A fragments: word i, byte j, bits 2m..2m+1 hold
// the code of row 16*(m&1) + g + 8*(i&1), column
// 32*(2p + (m>>1)) + 16*(i>>1) + 4*tig + j.  Codes of blocks past the row and
// of rows past the tensor are 1 (trit 0).  Scales: 32 floats per tile in row
// order (0 for rows past the tensor).
__global__ void repack_tq2_0(const uint8_t *__restrict__ src, int nrows, int nb, int nunits, int tile0,
                             int ntile_in, uint4 *__restrict__ codes, float *__restrict__ scales, bool aligned) {
    const size_t row_bytes = 4 + (size_t)8 * nb;
    const size_t n = (size_t)ntile_in * nunits * 32;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const size_t tu = i >> 5;
        const int p = (int)(tu % nunits);
        const int tl = (int)(tu / nunits);
        const int g = lane >> 2, tig = lane & 3;
        uint32_t wd[4];
#pragma unroll
        for (int ii = 0; ii < 4; ++ii) {
            uint32_t word = 0;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int r = tl * 32 + 16 * (m & 1) + g + 8 * (ii & 1);
                const int b = 2 * p + (m >> 1);
                // Byte 4*(ii/2) + tig of the block holds columns 16*(ii/2) + 4*tig + j at bits 2j.
                uint32_t byte = 0x55u;
                if (r < nrows && b < nb) byte = src[(size_t)r * row_bytes + 4 + (size_t)8 * b + 4 * (ii >> 1) + tig];
#pragma unroll
                for (int j = 0; j < 4; ++j) word |= ((byte >> (2 * j)) & 3u) << (8 * j + 2 * m);
            }
            wd[ii] = word;
        }
        const size_t tile = (size_t)tile0 + tl;
        codes[(tile * nunits + p) * 32 + lane] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        if (p == 0) {
            const int r = tl * 32 + lane;
            scales[tile * 32 + lane] = r < nrows ? __uint_as_float(ld_u32(src + (size_t)r * row_bytes, aligned)) : 0.0f;
        }
    }
}

// Dense rows (tile layout): W elements of `esize` bytes per 16-byte chunk.
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
            size_t n = (size_t)ntile_in * w.nb * 64;
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
            repack_tq2_0<<<grid_for(n), 256, 0, st>>>(s, nrows, w.nb, w.kchunks, tile0, ntile_in, w.codes, w.scales,
                                                      aligned);
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
