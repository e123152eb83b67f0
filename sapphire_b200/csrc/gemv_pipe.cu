// gemv_pipe.cu - persistent, TMA-pipelined batch-1 GEMV (the decode hot path).
//
// Same products as the reference row kernels (src/kernels/q4_0_avx.c:102-148,
// q8_0_avx.c:16-136, driven per row by src/kernels/pool.c:106-143), plus the
// ternary format and dense F32 / BF16 rows.
//
// Work split.  The weight is cut into items = (32-row tile, K segment).  Items
// are numbered tile-major and every warp of a persistent grid (one CTA per SM)
// takes a contiguous, equal-size range of them, so every SM streams the same
// number of bytes whatever the matrix shape.
//
// Memory pipeline.  Each warp owns a ring of NS shared-memory slots.  Lane 0
// fills a slot with one `cp.async.bulk` of the item's codes and one of its
// scales, completing on the slot's mbarrier (expect_tx).  The warp waits on
// the mbarrier, copies the item into registers, refills the slot with the
// item NS ahead at once, and only then computes - so all NS slots of every
// warp stay in flight while it computes.  (On B200 a read stream needs about
// 150 KB in flight per SM to reach full HBM bandwidth.)
//
// Dot products of the quantized formats run on the integer tensor cores
// (mma.sync m16n8k32, s8 x s8 -> s32): x is split per 32-column block into
// three balanced int8 digits of a 22-bit fixed-point value
//     x_j ~= 2^-e_b * (d0_j + 256 d1_j + 65536 d2_j)
// (error <= 2^-22 of the block's largest |x|), which form the B operand
// (columns 0..2 of an n8 tile).  The codes are the A operand exactly as
// stored (Q8_0), as nibbles with a column-sum correction for the -8 offset
// (Q4_0, u8 x s8), or as 2-bit trits mapped to -1/0/+1 by a byte permute
// (TQ2_0).  Integer products are exact; each block's int32 result is scaled
// by its fp32 scale (and 2^-e_b) in fp32, like the reference's per-block scale.
// Dense F32 / BF16 rows use fp32 FMAs (one lane per row).
//
// Split tiles.  A tile whose segments span several warps is finished by the
// last contributor: each stores its per-row partial (fp32, or the exact int64
// sum for ternary) in the slot of its rank among the tile's contributors,
// fences, and bumps the tile's counter; the one that completes the count sums
// the slots in slot order (deterministic), writes y and resets the counter.
//
// Waits are bounded: a slot that does not fill within kWaitLimit polls sets
// bit 0 of *err; the warp then waits (bounded again) for its copies in flight
// and returns.
#include <cfloat>

#include "internal.cuh"

namespace {

// Warps per CTA (NW) and ring slots per warp (NS) are template parameters;
// the host uses kPipeConfigs[0] (SAPPHIRE_PIPE_CFG selects another one for
// tuning runs).
struct PipeCfg {
    int nw, ns;
};
constexpr PipeCfg kPipeConfigs[] = {{12, 3}, {8, 4}, {16, 2}, {16, 4}, {12, 6}};
constexpr int kMaxPipeWarps = 16;
constexpr unsigned kWaitLimit = 1u << 26;
constexpr int kDigitBytesPerBlock = 96;       // 3 digit rows x 4 lanes x 8 bytes
constexpr int kTq2RegBlocks = 48;             // ternary x blocks per warp held in registers

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// Bulk global -> shared copy (16-byte aligned, multiple of 16 bytes), into this CTA only.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase) {
    for (unsigned i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}

// D += A(16x32, s8 row) * B(32x8, s8 col)
__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A * B + (c0, c1, c0, c1): the start value as the MMA's own C operand
// (no copies into the accumulator registers first).
__device__ __forceinline__ void mma_s8s8_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1, int c0, int c1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}
__device__ __forceinline__ void mma_u8s8_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1, int c0, int c1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

template <typename T>
__device__ __forceinline__ T lds(const uint8_t *p) {
    return *reinterpret_cast<const T *>(p);
}

// ------------------------------------------------------------ formats -----
// Per-format geometry of an item in the device layout (internal.cuh):
// kCodeBpb code bytes per (tile, block), kBpi blocks per item; the dense
// formats use kBpi units of 512 bytes (one 16-byte chunk of 32 rows).
template <tensor_dtype_t DT>
struct Geo;
template <>
struct Geo<DTYPE_Q8_0> {
    static constexpr bool kMma = true;
    static constexpr int kCodeBpb = 1024;
    static constexpr int kBpi = 4;
    static constexpr int kScaleBytes = kBpi * 128;
};
template <>
struct Geo<DTYPE_Q4_0> {
    static constexpr bool kMma = true;
    static constexpr int kCodeBpb = 512;
    static constexpr int kBpi = 4;
    static constexpr int kScaleBytes = kBpi * 128;
};
template <>
struct Geo<DTYPE_TQ2_0> {
    static constexpr bool kMma = true;
    static constexpr int kCodeBpb = 256;
    static constexpr int kBpi = 16;
    static constexpr int kScaleBytes = 0;     // row scale, read at the end of a tile
};
template <>
struct Geo<DTYPE_F32> {
    static constexpr bool kMma = false;
    static constexpr int kCodeBpb = 512;
    static constexpr int kBpi = 8;
    static constexpr int kScaleBytes = 0;
};
template <>
struct Geo<DTYPE_BF16> {
    static constexpr bool kMma = false;
    static constexpr int kCodeBpb = 512;
    static constexpr int kBpi = 8;
    static constexpr int kScaleBytes = 0;
};

template <tensor_dtype_t DT>
__host__ __device__ constexpr int code_bytes() {
    return Geo<DT>::kBpi * Geo<DT>::kCodeBpb;
}
template <tensor_dtype_t DT>
__host__ __device__ constexpr int stage_bytes() {
    return code_bytes<DT>() + Geo<DT>::kScaleBytes;
}

struct PipeParams {
    const uint8_t *codes;
    const float *scales;
    const float *x;
    float *y;
    void *part;                 // [ntiles][kmax][32] partials of split tiles (fp32; int64 for TQ2_0)
    int *cnt;                   // [ntiles] arrival counters, zero between launches
    int *err;                   // error word
    long long total_items;
    int nrows, cols, nb, ntiles, kchunks, nseg, kmax, total_warps;
    // Row-sharded products gathered over peer memory: when ll_n > 0 row r is
    // not stored at y[r] but sent to every rank k as the 8-byte word
    // (ll_epoch << 32 | bits of the value) at ll[k][ll_off + r] (NVLink stores;
    // an aligned 8-byte store arrives whole, so the epoch marks the value
    // valid and no fence is needed).
    int early;                  // weight copies per warp issued before the dependency wait
    int ll_n, ll_off;
    unsigned ll_epoch;
    unsigned long long *ll[kMaxPeers];
};

__device__ __forceinline__ void store_y(const PipeParams &p, size_t r, float v) {
    if (p.ll_n) {
        const unsigned long long word = ((unsigned long long)p.ll_epoch << 32) | __float_as_uint(v);
        for (int k = 0; k < p.ll_n; ++k)
            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p.ll[k] + (size_t)p.ll_off + r), "l"(word) : "memory");
    } else {
        p.y[r] = v;
    }
}

__device__ __forceinline__ long long range_begin(long long w, long long T, long long W) { return (w * T) / W; }
__device__ __forceinline__ int item_owner(long long i, long long T, long long W) {
    long long w = ((i + 1) * W + T - 1) / T - 1;
    return (int)(w < W - 1 ? w : W - 1);
}

// ------------------------------------------------------- x preparation ----
// Shared-memory image of x for the MMA formats:
//   digits[nb][3][4][8]  B fragments (digit rows 0..2, per lane-in-group tig:
//                        word 0 then word 1), a 16-byte zero word after them
//                        for lanes whose B column is 3..7;
//   pexp[0]              2^-e, the one exponent of all of x (room for nb
//                        values is kept);
//   corr[nb][4][2]       Q4_0 only: -8 * (sum of the block's digits of row
//                        2*tig+j), the correction of the unsigned codes.
struct XPrep {
    uint8_t *digits;
    float *pexp;
    int *corr;
    int *nonfinite;
};

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

__host__ __device__ inline size_t xprep_bytes(int nb, bool q4) {
    size_t b = align16((size_t)nb * kDigitBytesPerBlock + 16);
    b += align16((size_t)nb * 4);
    if (q4) b += (size_t)nb * 32;
    return b + 16;
}

// Dense formats stage x as fp32, zero-padded to whole items of 8 chunks so a
// tail item's zero chunks meet zeros.
__host__ __device__ inline int dense_xpad(tensor_dtype_t dt, int kchunks) {
    return ((kchunks + 7) / 8) * 8 * (dt == DTYPE_F32 ? 4 : 8);
}

__host__ __device__ inline size_t ximage_bytes(tensor_dtype_t dt, int nb, int kchunks) {
    size_t b;
    if (dt == DTYPE_Q8_0 || dt == DTYPE_Q4_0 || dt == DTYPE_TQ2_0) b = xprep_bytes(nb, dt == DTYPE_Q4_0);
    else b = (size_t)dense_xpad(dt, kchunks) * 4;
    return (b + 127) & ~(size_t)127;
}

// Balanced base-256 digits of an integer |X| <= 2^22: X = d0 + 256 d1 + 65536 d2.
__device__ __forceinline__ void digits3(int X, int &d0, int &d1, int &d2) {
    d0 = ((X & 0xFF) ^ 0x80) - 0x80;
    const int X1 = (X - d0) >> 8;
    d1 = ((X1 & 0xFF) ^ 0x80) - 0x80;
    d2 = (X1 - d1) >> 8;
}

// Exponent e with max|x| * 2^e < 2^22 (0 for an all-zero block).  For a
// normal m the frexp exponent is the biased exponent field minus 126.
__device__ __forceinline__ int block_exponent(float m) {
    if (!(m > 0.0f)) return 0;
    const int be = (__float_as_int(m) >> 23) & 0xFF;
    int E;
    if (be != 0) {
        E = be - 126;
    } else {
        frexpf(m, &E);
    }
    return 22 - E;
}

// v * 2^e, exact: a multiply by the power of two while 2^e is a normal float.
__device__ __forceinline__ float mul_pow2(float v, int e) {
    return (e >= -126 && e <= 127) ? v * __int_as_float((e + 127) << 23) : ldexpf(v, e);
}

// Byte offset of x position p (0..31) of a block inside its 32-byte digit
// row image [tig][word][byte], for each format's A-fragment k order.
template <tensor_dtype_t DT>
__device__ __forceinline__ int digit_slot(int p) {
    if (DT == DTYPE_Q8_0) {                   // k = p
        const int tig = (p & 15) >> 2, w = p >> 4, j = p & 3;
        return tig * 8 + w * 4 + j;
    } else if (DT == DTYPE_Q4_0) {            // k = tig*4+j <-> p = 8tig+2j (word 0), +1 (word 1)
        const int tig = p >> 3, j = (p & 7) >> 1, w = p & 1;
        return tig * 8 + w * 4 + j;
    } else {                                  // TQ2_0: byte-permute order of the trit decode
        const int hi = p >> 4, q = p & 15, tig = q >> 2, r = q & 3;
        return tig * 8 + (r & 1) * 4 + (r >> 1) + 2 * hi;
    }
}

// `after_loads` runs once this CTA's x loads have been issued (the ternary
// register path) or have returned (the other paths).
template <tensor_dtype_t DT, int NW>
__host__ __device__ constexpr bool tq2_reg_path(int nb) {
    return DT == DTYPE_TQ2_0 && (nb + NW - 1) / NW <= kTq2RegBlocks;
}
struct NoHook {
    __device__ void operator()() const {}
};

// x comes from global memory (p.x), or from an fp32 vector in shared memory
// when xs_smem is given (the fused producers of gemv_direct).
template <tensor_dtype_t DT, int NW, typename Hook = NoHook>
__device__ void prepare_x(const PipeParams &p, XPrep xp, const float *xs_smem = nullptr, Hook after_loads = Hook()) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float s_red[kMaxPipeWarps];
    int gexp = 0;
    if (!xs_smem && tq2_reg_path<DT, NW>(p.nb)) {
        // One exponent for the whole row (the ternary sum runs over all of K
        // in int32).  Warp w converts blocks w + NW*k.  Lane `lane` takes
        // k = 4i + lane/8 and word W = lane%8 of the block's digit rows: the
        // four x positions whose digits share that word (digit_slot), so the
        // rows are written as whole words with the 32 lanes on 32 banks.
        // All values are loaded into registers at once (one L2 round trip),
        // reduced for the exponent and converted from registers.
        constexpr int kIter = kTq2RegBlocks / 4;
        float v[kIter][4];
        const int per = (p.nb + NW - 1) / NW;
        const int W = lane & 7, sub = lane >> 3;
        const int s0 = 4 * (W >> 1) + (W & 1);
        const int src[4] = {s0, s0 + 2, s0 + 16, s0 + 18};
        float m = 0.0f;
        bool bad = false;
#pragma unroll
        for (int i = 0; i < kIter; ++i) {
            const int k = 4 * i + sub, b = warp + NW * k;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c = b * 32 + src[j];
                v[i][j] = (k < per && b < p.nb && c < p.cols) ? __ldg(p.x + c) : 0.0f;
            }
        }
        after_loads();
#pragma unroll
        for (int i = 0; i < kIter; ++i) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                bad |= !isfinite(v[i][j]);
                m = fmaxf(m, fabsf(v[i][j]));
            }
        }
        if (bad) *xp.nonfinite = 1;
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_red[warp] = m;
        __syncthreads();
        m = 0.0f;
        for (int i = 0; i < NW; ++i) m = fmaxf(m, s_red[i]);
        gexp = block_exponent(isfinite(m) ? m : FLT_MAX);
        if (threadIdx.x == 0) xp.pexp[0] = mul_pow2(1.0f, -gexp);
        // x * 2^gexp as two exact multiplies by normal powers of two
        // (gexp <= 170, so the second factor is at most 2^43).
        const int e1 = min(max(gexp, -126), 127);
        const float f1 = __int_as_float((e1 + 127) << 23), f2 = __int_as_float((gexp - e1 + 127) << 23);
#pragma unroll
        for (int i = 0; i < kIter; ++i) {
            const int k = 4 * i + sub, b = warp + NW * k;
            if (k < per && b < p.nb) {
                // Low bytes of the balanced digits (digits3): X, (X + 128) >> 8,
                // and that plus 128, >> 8 again.
                uint32_t b0[4], b1[4], b2[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int X = isfinite(v[i][j]) ? __float2int_rn(v[i][j] * f1 * f2) : 0;
                    const int X1 = (X + 0x80) >> 8;
                    b0[j] = (uint32_t)X;
                    b1[j] = (uint32_t)X1;
                    b2[j] = (uint32_t)((X1 + 0x80) >> 8);
                }
                const uint32_t w0 = __byte_perm(__byte_perm(b0[0], b0[1], 0x40), __byte_perm(b0[2], b0[3], 0x40), 0x5410);
                const uint32_t w1 = __byte_perm(__byte_perm(b1[0], b1[1], 0x40), __byte_perm(b1[2], b1[3], 0x40), 0x5410);
                const uint32_t w2 = __byte_perm(__byte_perm(b2[0], b2[1], 0x40), __byte_perm(b2[2], b2[3], 0x40), 0x5410);
                uint32_t *row = reinterpret_cast<uint32_t *>(xp.digits + (size_t)b * kDigitBytesPerBlock);
                row[0 * 8 + W] = w0;
                row[1 * 8 + W] = w1;
                row[2 * 8 + W] = w2;
            }
        }
        if (threadIdx.x < 4) reinterpret_cast<uint32_t *>(xp.digits + (size_t)p.nb * kDigitBytesPerBlock)[threadIdx.x] = 0;
        return;
    }
    {
        // One exponent for all of x (every format; the ternary rows here are
        // too long for the register path): loads unrolled so each thread has
        // 8 in flight.
        float m = 0.0f;
        bool bad = false;
#pragma unroll 8
        for (int i = threadIdx.x; i < p.cols; i += blockDim.x) {
            const float v = xs_smem ? xs_smem[i] : __ldg(p.x + i);
            bad |= !isfinite(v);
            m = fmaxf(m, fabsf(v));
        }
        after_loads();
        if (bad) *xp.nonfinite = 1;
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_red[warp] = m;
        __syncthreads();
        m = 0.0f;
        for (int i = 0; i < NW; ++i) m = fmaxf(m, s_red[i]);
        gexp = block_exponent(isfinite(m) ? m : FLT_MAX);
        if (threadIdx.x == 0) xp.pexp[0] = mul_pow2(1.0f, -gexp);
    }
    // x * 2^gexp as two exact multiplies by normal powers of two.
    const int e1 = min(max(gexp, -126), 127);
    const float f1 = __int_as_float((e1 + 127) << 23), f2 = __int_as_float((gexp - e1 + 127) << 23);
    // Blocks b = warp + NW*u: the loads of kGroup blocks are issued together,
    // then each block is converted.
    constexpr int kGroup = 8;
    for (int b0 = warp; b0 < p.nb; b0 += NW * kGroup) {
        float vg[kGroup];
#pragma unroll
        for (int u = 0; u < kGroup; ++u) {
            const int c = (b0 + u * NW) * 32 + lane;
            vg[u] = (b0 + u * NW < p.nb && c < p.cols) ? (xs_smem ? xs_smem[c] : __ldg(p.x + c)) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kGroup; ++u) {
            const int b = b0 + u * NW;
            if (b >= p.nb) break;
            const float v = vg[u];
            const int X = isfinite(v) ? __float2int_rn(v * f1 * f2) : 0;
            int d0, d1, d2;
            digits3(X, d0, d1, d2);
            uint8_t *row = xp.digits + (size_t)b * kDigitBytesPerBlock;
            const int off = digit_slot<DT>(lane);
            row[0 * 32 + off] = (uint8_t)(int8_t)d0;
            row[1 * 32 + off] = (uint8_t)(int8_t)d1;
            row[2 * 32 + off] = (uint8_t)(int8_t)d2;
            if (DT == DTYPE_Q4_0) {
                int s0 = d0, s1 = d1, s2 = d2;
                for (int o = 16; o; o >>= 1) {
                    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
                    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
                    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
                }
                // corr[b][tig][j] for digit row lane = 2*tig + j (rows 3..7 are zero)
                if (lane < 8) xp.corr[b * 8 + lane] = lane == 0 ? -8 * s0 : lane == 1 ? -8 * s1 : lane == 2 ? -8 * s2 : 0;
            }
        }
    }
    if (threadIdx.x < 4) reinterpret_cast<uint32_t *>(xp.digits + (size_t)p.nb * kDigitBytesPerBlock)[threadIdx.x] = 0;
}

// ----------------------------------------------------------- item in regs --
// The part of a staged item one lane needs, copied out of shared memory so
// the slot can be refilled before the compute.  Blocks past the end of a row
// are zero codes with zero scales (TQ2_0: code 1, trit 0).
template <tensor_dtype_t DT>
struct ItemRegs;
template <>
struct ItemRegs<DTYPE_Q8_0> {
    uint4 a[4][2];
    float4 s[4];
    __device__ __forceinline__ void load(const uint8_t *st, int nblk, int lane) {
        const int g = lane >> 2;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const bool ok = u < nblk;
            a[u][0] = ok ? lds<uint4>(st + u * 1024 + lane * 16) : make_uint4(0, 0, 0, 0);
            a[u][1] = ok ? lds<uint4>(st + u * 1024 + 512 + lane * 16) : make_uint4(0, 0, 0, 0);
            s[u] = ok ? lds<float4>(st + code_bytes<DTYPE_Q8_0>() + u * 128 + g * 16) : make_float4(0, 0, 0, 0);
        }
    }
};
template <>
struct ItemRegs<DTYPE_Q4_0> {
    uint4 a[4];
    float4 s[4];
    __device__ __forceinline__ void load(const uint8_t *st, int nblk, int lane) {
        const int g = lane >> 2;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const bool ok = u < nblk;
            a[u] = ok ? lds<uint4>(st + u * 512 + lane * 16) : make_uint4(0, 0, 0, 0);
            s[u] = ok ? lds<float4>(st + code_bytes<DTYPE_Q4_0>() + u * 128 + g * 16) : make_float4(0, 0, 0, 0);
        }
    }
};
template <>
struct ItemRegs<DTYPE_TQ2_0> {
    uint2 a[16];
    __device__ __forceinline__ void load(const uint8_t *st, int nblk, int lane) {
#pragma unroll
        for (int u = 0; u < 16; ++u)
            a[u] = u < nblk ? lds<uint2>(st + u * 256 + lane * 8) : make_uint2(0x55555555u, 0x55555555u);
    }
};
struct DenseRegs {
    uint4 c[8];
    __device__ __forceinline__ void load(const uint8_t *st, int nch, int lane) {
#pragma unroll
        for (int u = 0; u < 8; ++u) c[u] = u < nch ? lds<uint4>(st + u * 512 + lane * 16) : make_uint4(0, 0, 0, 0);
    }
};
template <>
struct ItemRegs<DTYPE_F32> : DenseRegs {};
template <>
struct ItemRegs<DTYPE_BF16> : DenseRegs {};

// ------------------------------------------------------------ consumers ---
// Accumulator state of one 32-row tile for a lane (g = lane/4, tig = lane%4).
struct MmaAcc {
    float f[2][4];      // Q8_0 / Q4_0: scaled partial sums per (half, D register)
    int d[2][2][4];     // TQ2_0: exact int32 sums, two independent sets (set, half, reg)
    float dense;        // F32 / BF16: this lane's row
    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                f[h][i] = 0.0f;
                d[0][h][i] = 0;
                d[1][h][i] = 0;
            }
        dense = 0.0f;
    }
};

// B fragment of block b (clamped to the last block; rows past the end of x
// have zero codes, so the clamped digits meet zeros).
__device__ __forceinline__ uint2 load_b(const XPrep &xp, int nb, int b, int lane) {
    const int g = lane >> 2, tig = lane & 3;
    b = b < nb ? b : nb - 1;
    const size_t off = g < 3 ? (size_t)b * kDigitBytesPerBlock + g * 32 + tig * 8 : (size_t)nb * kDigitBytesPerBlock;
    return lds<uint2>(xp.digits + off);
}

// Scaled epilogue of one block's two D tiles (rows g, g+8 | g+16, g+24).
// A lane holds D columns 2tig, 2tig+1 (digits 2tig, 2tig+1; digit 3 is a
// zero column) of rows g, g+8 of each 16-row half.  Digits 0 and 1 are joined
// in integer arithmetic, d0 + 256 d1 (below 2^28: each block sum is below
// 2^22), so a block costs one conversion and one FMA per row and lane; lane
// tig = 1 carries digit 2, weighted by 65536 in tile_rows.  The one exponent
// of x is applied there too.
__device__ __forceinline__ void scale_acc(MmaAcc &acc, const int (&D0)[4], const int (&D1)[4], float4 S) {
    acc.f[0][0] = fmaf(S.x, (float)(D0[0] + 256 * D0[1]), acc.f[0][0]);
    acc.f[0][2] = fmaf(S.y, (float)(D0[2] + 256 * D0[3]), acc.f[0][2]);
    acc.f[1][0] = fmaf(S.z, (float)(D1[0] + 256 * D1[1]), acc.f[1][0]);
    acc.f[1][2] = fmaf(S.w, (float)(D1[2] + 256 * D1[3]), acc.f[1][2]);
}

__device__ __forceinline__ void compute_item(const ItemRegs<DTYPE_Q8_0> &R, int blk0, int nb, int lane,
                                             const XPrep &xp, const float *, MmaAcc &acc) {
#pragma unroll
    for (int u0 = 0; u0 < 4; u0 += 2) {
        uint2 B[2];
        int D[2][2][4];
#pragma unroll
        for (int u = 0; u < 2; ++u) B[u] = load_b(xp, nb, blk0 + u0 + u, lane);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const uint4 a0 = R.a[u0 + u][0], a1 = R.a[u0 + u][1];
            mma_s8s8_c(D[u][0], a0.x, a0.y, a0.z, a0.w, B[u].x, B[u].y, 0, 0);
            mma_s8s8_c(D[u][1], a1.x, a1.y, a1.z, a1.w, B[u].x, B[u].y, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) scale_acc(acc, D[u][0], D[u][1], R.s[u0 + u]);
    }
}

__device__ __forceinline__ void compute_item(const ItemRegs<DTYPE_Q4_0> &R, int blk0, int nb, int lane,
                                             const XPrep &xp, const float *, MmaAcc &acc) {
    const int tig = lane & 3;
    uint2 B[4];
    int2 C[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int b = min(blk0 + u, nb - 1);
        B[u] = load_b(xp, nb, b, lane);
        C[u] = lds<int2>(reinterpret_cast<const uint8_t *>(xp.corr) + (size_t)b * 32 + tig * 8);
    }
    int D[4][2][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const uint4 A = R.a[u];
        const uint32_t lo0 = A.x & 0x0F0F0F0Fu, hi0 = (A.x >> 4) & 0x0F0F0F0Fu;
        const uint32_t lo1 = A.y & 0x0F0F0F0Fu, hi1 = (A.y >> 4) & 0x0F0F0F0Fu;
        const uint32_t lo2 = A.z & 0x0F0F0F0Fu, hi2 = (A.z >> 4) & 0x0F0F0F0Fu;
        const uint32_t lo3 = A.w & 0x0F0F0F0Fu, hi3 = (A.w >> 4) & 0x0F0F0F0Fu;
        // Start from the -8 offset correction of the unsigned codes.
        mma_u8s8_c(D[u][0], lo0, lo1, hi0, hi1, B[u].x, B[u].y, C[u].x, C[u].y);
        mma_u8s8_c(D[u][1], lo2, lo3, hi2, hi3, B[u].x, B[u].y, C[u].x, C[u].y);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) scale_acc(acc, D[u][0], D[u][1], R.s[u]);
}

__device__ __forceinline__ void compute_item(const ItemRegs<DTYPE_TQ2_0> &R, int blk0, int nb, int lane,
                                             const XPrep &xp, const float *, MmaAcc &acc) {
    const uint32_t tbl = 0x020100FFu;   // code c -> c - 1
#pragma unroll
    for (int u0 = 0; u0 < 16; u0 += 4) {
        uint2 B[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) B[u] = load_b(xp, nb, blk0 + u0 + u, lane);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint2 A = R.a[u0 + u];
            const uint32_t m0 = A.x & 0x33333333u, n0 = (A.x >> 2) & 0x33333333u;
            const uint32_t m1 = A.y & 0x33333333u, n1 = (A.y >> 2) & 0x33333333u;
            mma_s8s8(acc.d[u & 1][0], __byte_perm(tbl, 0, m0), __byte_perm(tbl, 0, m0 >> 16), __byte_perm(tbl, 0, n0),
                     __byte_perm(tbl, 0, n0 >> 16), B[u].x, B[u].y);
            mma_s8s8(acc.d[u & 1][1], __byte_perm(tbl, 0, m1), __byte_perm(tbl, 0, m1 >> 16), __byte_perm(tbl, 0, n1),
                     __byte_perm(tbl, 0, n1 >> 16), B[u].x, B[u].y);
        }
    }
}

__device__ __forceinline__ float dense_f32(uint4 c, const float *xs) {
    const float4 v = *reinterpret_cast<const float4 *>(xs);
    float a = __uint_as_float(c.x) * v.x;
    a = fmaf(__uint_as_float(c.y), v.y, a);
    a = fmaf(__uint_as_float(c.z), v.z, a);
    return fmaf(__uint_as_float(c.w), v.w, a);
}
__device__ __forceinline__ float dense_bf16(uint4 c, const float *xs) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xs);
    const float4 v0 = x4[0], v1 = x4[1];
    float a0 = __uint_as_float(c.x << 16) * v0.x, a1 = __uint_as_float(c.x & 0xFFFF0000u) * v0.y;
    a0 = fmaf(__uint_as_float(c.y << 16), v0.z, a0);
    a1 = fmaf(__uint_as_float(c.y & 0xFFFF0000u), v0.w, a1);
    a0 = fmaf(__uint_as_float(c.z << 16), v1.x, a0);
    a1 = fmaf(__uint_as_float(c.z & 0xFFFF0000u), v1.y, a1);
    a0 = fmaf(__uint_as_float(c.w << 16), v1.z, a0);
    a1 = fmaf(__uint_as_float(c.w & 0xFFFF0000u), v1.w, a1);
    return a0 + a1;
}
__device__ __forceinline__ void compute_item(const ItemRegs<DTYPE_F32> &R, int c0, int, int, const XPrep &,
                                             const float *xs, MmaAcc &acc) {
#pragma unroll
    for (int u = 0; u < 8; ++u) acc.dense += dense_f32(R.c[u], xs + (size_t)(c0 + u) * 4);
}
__device__ __forceinline__ void compute_item(const ItemRegs<DTYPE_BF16> &R, int c0, int, int, const XPrep &,
                                             const float *xs, MmaAcc &acc) {
#pragma unroll
    for (int u = 0; u < 8; ++u) acc.dense += dense_bf16(R.c[u], xs + (size_t)(c0 + u) * 8);
}

// Per-row results of a tile.  MMA formats: lanes with tig == 0 hold rows
// g + 8*i (i = 0..3) as 8-byte values (fp32 bits for Q8_0 / Q4_0, the exact
// int64 sum for TQ2_0); all lanes must call (shuffles).  Dense: row = lane.
// Row values of a lane's accumulators: ternary exact int64 sums; Q8_0 / Q4_0
// floats scaled by pe, the x exponent factor 2^-e.
template <tensor_dtype_t DT>
__device__ __forceinline__ void tile_rows(const MmaAcc &acc, unsigned long long (&v)[4], float pe) {
    if constexpr (!Geo<DT>::kMma) {
        v[0] = __float_as_uint(acc.dense);
        return;
    } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (DT == DTYPE_TQ2_0) {
            int d[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) d[i] = acc.d[0][h][i] + acc.d[1][h][i];
            const int up0 = __shfl_down_sync(0xffffffffu, d[0], 1);
            const int up2 = __shfl_down_sync(0xffffffffu, d[2], 1);
            v[2 * h] = (unsigned long long)((long long)d[0] + 256LL * d[1] + 65536LL * up0);
            v[2 * h + 1] = (unsigned long long)((long long)d[2] + 256LL * d[3] + 65536LL * up2);
        } else {
            const float up0 = __shfl_down_sync(0xffffffffu, acc.f[h][0], 1);
            const float up2 = __shfl_down_sync(0xffffffffu, acc.f[h][2], 1);
            v[2 * h] = __float_as_uint((float)(((double)acc.f[h][0] + 65536.0 * up0) * pe));
            v[2 * h + 1] = __float_as_uint((float)(((double)acc.f[h][2] + 65536.0 * up2) * pe));
        }
    }
    }
}

// ---------------------------------------------------------- tile output ---
// Index of row r's scale among a ternary tile's 32 (slot order g*4+i -> row g+8i).
__device__ __forceinline__ int tq2_scale_slot(int r) { return (r & 7) * 4 + (r >> 3); }

// rs: ternary row scale of row r, loaded when the tile started.
template <tensor_dtype_t DT>
__device__ __forceinline__ float finish_row(const XPrep &xp, unsigned long long v, bool nonfinite, float rs) {
    float out;
    if (DT == DTYPE_TQ2_0) {
        out = (float)((double)rs * ((double)(long long)v * (double)xp.pexp[0]));
    } else {
        out = __uint_as_float((uint32_t)v);
    }
    return nonfinite ? __int_as_float(0x7FC00000) : out;
}

// Rows are stored one per lane (row tile*32 + lane); rs is that row's ternary
// scale.
template <tensor_dtype_t DT>
__device__ void flush_tile(const PipeParams &p, const XPrep &xp, int tile, int lane, int my_warp, bool whole,
                           const unsigned long long (&v)[4], bool nonfinite, float rs) {
    constexpr bool kMma = Geo<DT>::kMma;
    const bool owner_lane = kMma ? ((lane & 3) == 0) : true;
    constexpr int kRows = kMma ? 4 : 1;
    auto row_of = [&](int i) { return kMma ? ((lane >> 2) + 8 * i) : lane; };
    if (whole) {
        // One row per lane (a warp's stores are 32 consecutive rows): lane l
        // takes row l = g + 8i from the lane holding it, (l % 8) * 4.
        unsigned long long mine = v[0];
        if constexpr (kMma) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const unsigned long long t = __shfl_sync(0xffffffffu, v[i], (lane & 7) * 4);
                if ((lane >> 3) == i) mine = t;
            }
        }
        if (tile * 32 + lane < p.nrows) store_y(p, (size_t)tile * 32 + lane, finish_row<DT>(xp, mine, nonfinite, rs));
        return;
    }
    // k = contributors of the tile, slot = this warp's rank among them.
    const long long first = (long long)tile * p.nseg;
    int k = 0, slot = -1;
    const int o0 = item_owner(first, p.total_items, p.total_warps);
    if (p.total_items >= p.total_warps) {
        // Every warp owns at least one item, so the tile's owners are the
        // consecutive warps o0..o1 (two 64-bit divisions instead of nseg).
        k = item_owner(first + p.nseg - 1, p.total_items, p.total_warps) - o0 + 1;
        slot = my_warp - o0;
    } else {
        int prev = -1;
        for (int s = 0; s < p.nseg; ++s) {
            const int o = s == 0 ? o0 : item_owner(first + s, p.total_items, p.total_warps);
            if (o != prev) {
                if (o == my_warp) slot = k;
                ++k;
                prev = o;
            }
        }
    }
    long long *base64 = reinterpret_cast<long long *>(p.part) + (size_t)tile * p.kmax * 32;
    float *base32 = reinterpret_cast<float *>(p.part) + (size_t)tile * p.kmax * 32;
    if (owner_lane) {
#pragma unroll
        for (int i = 0; i < kRows; ++i) {
            if (DT == DTYPE_TQ2_0) base64[(size_t)slot * 32 + row_of(i)] = (long long)v[i];
            else base32[(size_t)slot * 32 + row_of(i)] = __uint_as_float((uint32_t)v[i]);
        }
    }
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(p.cnt + tile, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == k - 1) {
        __threadfence();
        // The last contributor sums the slots in slot order, one row per lane.
        const int r = lane;
        unsigned long long sum;
        if (DT == DTYPE_TQ2_0) {
            long long s = 0;
            for (int j = 0; j < k; ++j) s += __ldcg(base64 + (size_t)j * 32 + r);
            sum = (unsigned long long)s;
        } else {
            float s = 0.0f;
            for (int j = 0; j < k; ++j) s += __ldcg(base32 + (size_t)j * 32 + r);
            sum = __float_as_uint(s);
        }
        if (tile * 32 + r < p.nrows) store_y(p, (size_t)tile * 32 + r, finish_row<DT>(xp, sum, nonfinite, rs));
        __syncwarp();
        if (lane == 0) p.cnt[tile] = 0;
    }
}

// --------------------------------------------------------------- kernel ---
template <tensor_dtype_t DT, int NW, int NS>
__global__ void __launch_bounds__(NW * 32, 1) gemv_pipe(const PipeParams p) {
    using G = Geo<DT>;
    constexpr int kStage = stage_bytes<DT>();
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_nonfinite;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Shared memory: [x image][rings][barriers]
    const size_t ximg = ximage_bytes(DT, p.nb, p.kchunks);
    uint8_t *ring = smem + ximg + (size_t)warp * NS * kStage;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + ximg + (size_t)NW * NS * kStage) + warp * NS;
    XPrep xp;
    xp.digits = smem;
    const size_t dig_bytes = align16((size_t)p.nb * kDigitBytesPerBlock + 16);
    xp.pexp = reinterpret_cast<float *>(smem + dig_bytes);
    xp.corr = reinterpret_cast<int *>(smem + dig_bytes + align16((size_t)p.nb * 4));
    xp.nonfinite = &s_nonfinite;
    float *xs = reinterpret_cast<float *>(smem);

    const int gw = blockIdx.x * NW + warp;
    const long long T = p.total_items, W = p.total_warps;
    const long long it0 = range_begin(gw, T, W), it1 = range_begin(gw + 1, T, W);
    const int n_items = (int)(it1 - it0);
    const int units = G::kMma ? p.nb : p.kchunks;   // blocks (quantized) or 512-byte units (dense)

    // (tile, segment) of the next item to copy, advanced without division.
    const int tile0 = (int)(it0 / p.nseg), seg0 = (int)(it0 % p.nseg);
    int q_tile = tile0, q_seg = seg0;
    auto issue = [&](int stage) {
        const int tile = q_tile, seg = q_seg;
        if (++q_seg == p.nseg) {
            q_seg = 0;
            ++q_tile;
        }
        const int u0 = seg * G::kBpi;
        const int nu = min(G::kBpi, units - u0);
        uint8_t *dst = ring + (size_t)stage * kStage;
        const uint8_t *src = p.codes + (size_t)tile * p.kchunks * 512 + (size_t)u0 * G::kCodeBpb;
        const uint32_t bytes = (uint32_t)nu * G::kCodeBpb;
        const uint32_t sbytes = G::kScaleBytes ? (uint32_t)nu * 128 : 0;
        mbar_expect_tx(bars + stage, bytes + sbytes);
        bulk_g2s(dst, src, bytes, bars + stage);
        if (sbytes) bulk_g2s(dst + code_bytes<DT>(), p.scales + ((size_t)tile * p.nb + u0) * 32, sbytes, bars + stage);
    };

    pdl_trigger();
    if (threadIdx.x == 0) s_nonfinite = 0;
    if (lane == 0) {
        for (int s = 0; s < NS; ++s) mbar_init(bars + s, 1);
        fence_mbar_init();
    }
    __syncwarp();
    // The weight copies do not depend on earlier kernels: `early` of them
    // start before the wait for the kernel that produced x, the rest once
    // the x loads are out, which would otherwise queue behind the copies of
    // every SM (none early on the ternary register path, whose x loads are a
    // whole long row per CTA).
    const int early = tq2_reg_path<DT, NW>(p.nb) ? 0 : min(p.early, NS);
    if (lane == 0)
        for (int j = 0; j < early && j < n_items; ++j) issue(j);
    auto issue_rest = [&]() {
        if (lane == 0)
            for (int j = early; j < NS && j < n_items; ++j) issue(j);
    };
    pdl_wait();
    __syncthreads();   // s_nonfinite initialised before x preparation writes it

    // x image, built once per CTA while the first copies are in flight.
    if (G::kMma) {
        prepare_x<DT, NW>(p, xp, nullptr, issue_rest);
    } else {
        issue_rest();
        const int xpad = dense_xpad(DT, p.kchunks);
        for (int i = threadIdx.x; i < xpad; i += blockDim.x) xs[i] = (i < p.cols) ? p.x[i] : 0.0f;
    }
    __syncthreads();
    const bool nonfinite = G::kMma && s_nonfinite != 0;
    const float x_scale = (G::kMma && DT != DTYPE_TQ2_0) ? xp.pexp[0] : 1.0f;

    int cur_tile = -1, c_tile = tile0, c_seg = seg0;
    float row_scale = 0.0f;
    bool cur_whole = false;
    MmaAcc acc;
    acc.reset();
    for (int j = 0; j < n_items; ++j) {
        const int stage = j % NS;
        const uint32_t phase = (uint32_t)(j / NS) & 1u;
        if (!mbar_wait_bounded(bars + stage, phase)) {
            if (lane == 0) atomicOr(p.err, 1);
            for (int q = j; q < n_items && q < j + NS; ++q)
                (void)mbar_wait_bounded(bars + (q % NS), (uint32_t)(q / NS) & 1u);
            return;
        }
        const int tile = c_tile, seg = c_seg;
        if (++c_seg == p.nseg) {
            c_seg = 0;
            ++c_tile;
        }
        // Item into registers, then refill the slot before computing.
        const int u0 = seg * G::kBpi;
        ItemRegs<DT> R;
        R.load(ring + (size_t)stage * kStage, min(G::kBpi, units - u0), lane);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0 && j + NS < n_items) issue(stage);

        if (tile != cur_tile) {
            if (cur_tile >= 0) {
                unsigned long long v[4] = {0, 0, 0, 0};
                tile_rows<DT>(acc, v, x_scale);
                flush_tile<DT>(p, xp, cur_tile, lane, gw, cur_whole, v, nonfinite, row_scale);
            }
            cur_tile = tile;
            acc.reset();
            cur_whole = (seg == 0) && ((long long)tile * p.nseg + p.nseg <= it1);
            // The ternary row scale this lane stores with, loaded now so the
            // flush does not wait for it.
            if (DT == DTYPE_TQ2_0) row_scale = __ldg(p.scales + (size_t)tile * 32 + tq2_scale_slot(lane));
        }
        compute_item(R, u0, p.nb, lane, xp, xs, acc);
    }
    if (cur_tile >= 0) {
        unsigned long long v[4] = {0, 0, 0, 0};
        tile_rows<DT>(acc, v, x_scale);
        flush_tile<DT>(p, xp, cur_tile, lane, gw, cur_whole, v, nonfinite, row_scale);
    }
}

// ----------------------------------------------------------------- host ---
int stage_of(tensor_dtype_t dt) {
    switch (dt) {
        case DTYPE_Q8_0: return stage_bytes<DTYPE_Q8_0>();
        case DTYPE_Q4_0: return stage_bytes<DTYPE_Q4_0>();
        case DTYPE_TQ2_0: return stage_bytes<DTYPE_TQ2_0>();
        case DTYPE_F32: return stage_bytes<DTYPE_F32>();
        case DTYPE_BF16: return stage_bytes<DTYPE_BF16>();
        default: return 0;
    }
}

int bpi_of(tensor_dtype_t dt) {
    switch (dt) {
        case DTYPE_Q8_0: return Geo<DTYPE_Q8_0>::kBpi;
        case DTYPE_Q4_0: return Geo<DTYPE_Q4_0>::kBpi;
        case DTYPE_TQ2_0: return Geo<DTYPE_TQ2_0>::kBpi;
        case DTYPE_F32: return Geo<DTYPE_F32>::kBpi;
        case DTYPE_BF16: return Geo<DTYPE_BF16>::kBpi;
        default: return 1;
    }
}

size_t pipe_smem(tensor_dtype_t dt, int nb, int kchunks, PipeCfg c) {
    const int stage = stage_of(dt);
    if (!stage) return 0;
    return ximage_bytes(dt, nb, kchunks) + (size_t)c.nw * c.ns * stage + (size_t)c.nw * c.ns * 8;
}

// The configuration of a format: 16 warps x 2 slots for TQ2_0 (its 4 KB
// items carry four times the weights of a Q8_0 item, so more warps decoding
// beat deeper rings), 16 x 4 for Q4_0 (2.5 KB items) while its rings and x
// image fit in shared memory, 12 x 3 otherwise.  SAPPHIRE_PIPE_CFG = an index
// into kPipeConfigs selects one for every format (tuning runs).
PipeCfg pipe_cfg(const DevWeight &w) {
    const tensor_dtype_t dt = w.dtype;
    static const int idx = [] {
        const char *v = getenv("SAPPHIRE_PIPE_CFG");
        int i = v ? atoi(v) : -1;
        const int n = (int)(sizeof(kPipeConfigs) / sizeof(kPipeConfigs[0]));
        return (i >= 0 && i < n) ? i : -1;
    }();
    if (idx >= 0) return kPipeConfigs[idx];
    if (dt == DTYPE_TQ2_0) return kPipeConfigs[2];
    if (dt == DTYPE_Q4_0 && pipe_smem(dt, w.nb, w.kchunks, kPipeConfigs[3]) <= 227 * 1024) return kPipeConfigs[3];
    return kPipeConfigs[0];
}

// Weight copies per warp issued before the wait for x's producer: two (C2
// and the Q4_0 LM head measured best with two of 3-4 slots early: the first
// bytes are in flight across the wait, and the x loads queue behind only two
// slots of every warp).  SAPPHIRE_PIPE_EARLY overrides it (tuning runs).
int pipe_early(PipeCfg c) {
    static const int env = [] {
        const char *v = getenv("SAPPHIRE_PIPE_EARLY");
        return v ? atoi(v) : -1;
    }();
    if (env >= 0) return env;
    return std::min(2, c.ns);
}

int item_nseg(const DevWeight &w) {
    const int units = (w.dtype == DTYPE_Q8_0 || w.dtype == DTYPE_Q4_0 || w.dtype == DTYPE_TQ2_0) ? w.nb : w.kchunks;
    const int bpi = bpi_of(w.dtype);
    return (units + bpi - 1) / bpi;
}

// Raises a kernel's dynamic shared-memory opt-in on the context's device only
// when a launch needs more than was set before, so repeated launches (and
// launches recorded into a CUDA graph after a first eager one) make no
// attribute call.
template <typename K>
cudaError_t ensure_smem_optin(K kernel, int device, size_t smem) {
    static std::mutex mu;
    static std::unordered_map<const void *, size_t> set[64];
    if (device < 0 || device >= 64)
        return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    std::lock_guard<std::mutex> lk(mu);
    size_t &cur = set[device][reinterpret_cast<const void *>(kernel)];
    if (smem <= cur) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) cur = smem;
    return e;
}

template <tensor_dtype_t DT>
int launch_cfg(kernel_context_t *ctx, const PipeParams &p, PipeCfg c, int grid, size_t smem, cudaStream_t st) {
    auto run = [&](auto kernel, int threads) -> int {
        cudaError_t e = ensure_smem_optin(kernel, ctx->device, smem);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "launch_gemv_pipe", "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return -1;
        }
        e = launch_pdl(kernel, dim3(grid), dim3(threads), smem, st, p);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) {
            ctx_fail(ctx, "launch_gemv_pipe", "launch failed: %s", cudaGetErrorString(e));
            return -1;
        }
        return 0;
    };
    if (c.nw == 8 && c.ns == 4) return run(gemv_pipe<DT, 8, 4>, 8 * 32);
    if (c.nw == 16 && c.ns == 2) return run(gemv_pipe<DT, 16, 2>, 16 * 32);
    if (c.nw == 16 && c.ns == 4) return run(gemv_pipe<DT, 16, 4>, 16 * 32);
    if (c.nw == 12 && c.ns == 6) return run(gemv_pipe<DT, 12, 6>, 12 * 32);
    return run(gemv_pipe<DT, 12, 3>, 12 * 32);
}

// --------------------------------------------------- latency-bound GEMV --
// Small weights (decode projections, a few hundred KB to a few MB) are bound
// by latency, not bandwidth: gemv_direct gives each 32-row tile one CTA whose
// kDirectWarps warps split the tile's items (at most two per warp), loads
// every item straight into registers before waiting for the kernel that
// produces x (programmatic dependent launch), and reduces the warps' row sums
// in shared memory in warp order - no ring, no split-tile atomics.
constexpr int kDirectWarps = 8;
constexpr int kDirectMaxItems = 2;

template <tensor_dtype_t DT>
__device__ __forceinline__ void load_item_global(ItemRegs<DT> &R, const PipeParams &p, int tile, int u0, int nblk,
                                                 int lane) {
    const int g = lane >> 2;
    const uint8_t *codes = p.codes + (size_t)tile * p.kchunks * 512 + (size_t)u0 * Geo<DT>::kCodeBpb;
    const float *sc = p.scales + ((size_t)tile * p.nb + u0) * 32 + g * 4;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const bool ok = u < nblk;
        if constexpr (DT == DTYPE_Q8_0) {
            R.a[u][0] = ok ? __ldg(reinterpret_cast<const uint4 *>(codes + u * 1024 + lane * 16)) : make_uint4(0, 0, 0, 0);
            R.a[u][1] = ok ? __ldg(reinterpret_cast<const uint4 *>(codes + u * 1024 + 512 + lane * 16))
                           : make_uint4(0, 0, 0, 0);
        } else {
            R.a[u] = ok ? __ldg(reinterpret_cast<const uint4 *>(codes + u * 512 + lane * 16)) : make_uint4(0, 0, 0, 0);
        }
        R.s[u] = ok ? __ldg(reinterpret_cast<const float4 *>(sc + (size_t)u * 32)) : make_float4(0, 0, 0, 0);
    }
}

// Producer of x inside gemv_direct.
enum DirectX : int {
    kXPlain = 0,     // x read from p.x
    kXResNorm = 1,   // h' = h_in + rmsnorm_delta(t, w_post); x = rmsnorm_delta(h', w_next); block 0 stores h'
    kXGeGLU = 2,     // x[i] = gelu(gu[i]) * gu[cols + i]
};
struct DirectFuse {
    const float *t, *w_post, *h_in, *w_next, *gu;
    float *h_out;
    float eps;
};

__device__ __forceinline__ float direct_block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < kDirectWarps ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

// Builds the fp32 x vector of a fused producer in shared memory.  The
// arithmetic is the reference's rmsnorm_delta (src/transformer/normalization.c:
// 103-116) and GeGLU (src/transformer/activations.c:64-82, transformer.c:150-157).
template <int XM>
__device__ void produce_x(const PipeParams &p, const DirectFuse &f, float *xs, float *red) {
    const int n = p.cols;
    if constexpr (XM == kXResNorm) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float v = f.t[i];
            xs[i] = v;
            ss += v * v;
        }
        ss = direct_block_sum(ss, red);
        const float r1 = 1.0f / sqrtf(ss / (float)n + f.eps);
        float hh = 0.0f;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float h = f.h_in[i] + (xs[i] * r1) * (1.0f + (f.w_post ? f.w_post[i] : 0.0f));
            xs[i] = h;
            hh += h * h;
            if (blockIdx.x == 0) f.h_out[i] = h;
        }
        hh = direct_block_sum(hh, red);
        const float r2 = 1.0f / sqrtf(hh / (float)n + f.eps);
        for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = (xs[i] * r2) * (1.0f + (f.w_next ? f.w_next[i] : 0.0f));
    } else if constexpr (XM == kXGeGLU) {
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float x = f.gu[i];
            const float y = 0.7978845608f * (x + 0.044715f * x * x * x);
            xs[i] = (0.5f * x * (1.0f + tanhf(y))) * f.gu[n + i];
        }
    }
    __syncthreads();
}

template <tensor_dtype_t DT, int XM>
__global__ void __launch_bounds__(kDirectWarps * 32) gemv_direct(const PipeParams p, const DirectFuse f) {
    static_assert(DT == DTYPE_Q8_0 || DT == DTYPE_Q4_0, "per-block-scale formats only");
    static_assert(Geo<DT>::kBpi == 4, "items of four blocks");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float part[kDirectWarps][32];
    __shared__ float red[32];
    __shared__ int s_nonfinite;
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    ItemRegs<DT> R[kDirectMaxItems];
#pragma unroll
    for (int k = 0; k < kDirectMaxItems; ++k) {
        const int seg = warp + k * kDirectWarps;
        if (seg < p.nseg) load_item_global<DT>(R[k], p, tile, seg * 4, min(4, p.nb - seg * 4), lane);
    }
    if (threadIdx.x == 0) s_nonfinite = 0;
    pdl_wait();
    __syncthreads();
    unsigned long long v[4];
    if constexpr (DT == DTYPE_Q4_0) {
        // Q4_0: fp32 x in shared memory and FFMA dot products: per block and
        // row sum_j (q_j - 8) x_j, then one multiply by the block scale.  No
        // digit image is built, which is what bounds a GEMV this small.
        float *xs = reinterpret_cast<float *>(smem);
        if constexpr (XM != kXPlain) {
            produce_x<XM>(p, f, xs, red);
        } else {
            // Non-finite x values propagate through the fp32 arithmetic as in
            // the reference's row kernels.
            for (int i = threadIdx.x; i < p.nb * 32; i += blockDim.x) xs[i] = i < p.cols ? __ldg(p.x + i) : 0.0f;
            __syncthreads();
        }
        const int tig = lane & 3;
        float r[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int k = 0; k < kDirectMaxItems; ++k) {
            const int seg = warp + k * kDirectWarps;
            if (seg >= p.nseg) continue;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int b = seg * 4 + u;
                if (b >= p.nb) break;
                const float4 x0 = *reinterpret_cast<const float4 *>(xs + b * 32 + tig * 8);
                const float4 x1 = *reinterpret_cast<const float4 *>(xs + b * 32 + tig * 8 + 4);
                const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const uint32_t w[4] = {R[k].a[u].x, R[k].a[u].y, R[k].a[u].z, R[k].a[u].w};
                const float sc[4] = {R[k].s[u].x, R[k].s[u].y, R[k].s[u].z, R[k].s[u].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
                    float dot = 0.0f;
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        // 0x4B0000nn is the float 2^23 + n; subtracting 2^23 + 8 leaves n - 8 exactly.
                        const float q0 = __int_as_float((int)__byte_perm(lo, 0x4B000000u, 0x7440u | m)) - 8388616.0f;
                        const float q1 = __int_as_float((int)__byte_perm(hi, 0x4B000000u, 0x7440u | m)) - 8388616.0f;
                        dot = fmaf(q0, xv[2 * m], dot);
                        dot = fmaf(q1, xv[2 * m + 1], dot);
                    }
                    r[i] = fmaf(sc[i], dot, r[i]);
                }
            }
        }
        // rows g + 8i: sum the four lanes of the row group
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            r[i] += __shfl_xor_sync(0xffffffffu, r[i], 1);
            r[i] += __shfl_xor_sync(0xffffffffu, r[i], 2);
            v[i] = __float_as_uint(r[i]);
        }
    } else {
        XPrep xp;
        xp.digits = smem;
        const size_t dig_bytes = align16((size_t)p.nb * kDigitBytesPerBlock + 16);
        xp.pexp = reinterpret_cast<float *>(smem + dig_bytes);
        xp.corr = reinterpret_cast<int *>(smem + dig_bytes + align16((size_t)p.nb * 4));
        xp.nonfinite = &s_nonfinite;
        float *xs = nullptr;
        if constexpr (XM != kXPlain) {
            xs = reinterpret_cast<float *>(smem + ((ximage_bytes(DT, p.nb, p.kchunks) + 15) & ~(size_t)15));
            produce_x<XM>(p, f, xs, red);
        }
        prepare_x<DT, kDirectWarps>(p, xp, xs);
        __syncthreads();
        MmaAcc acc;
        acc.reset();
#pragma unroll
        for (int k = 0; k < kDirectMaxItems; ++k) {
            const int seg = warp + k * kDirectWarps;
            if (seg < p.nseg) compute_item(R[k], seg * 4, p.nb, lane, xp, nullptr, acc);
        }
        tile_rows<DT>(acc, v, xp.pexp[0]);
    }
    if ((lane & 3) == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) part[warp][(lane >> 2) + 8 * i] = __uint_as_float((uint32_t)v[i]);
    }
    __syncthreads();
    if (warp == 0) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kDirectWarps; ++w) sum += part[w][lane];
        const int row = tile * 32 + lane;
        if (row < p.nrows) p.y[row] = s_nonfinite ? __int_as_float(0x7FC00000) : sum;
    }
}

}  // namespace

bool direct_supported(const DevWeight &w) {
    if (w.dtype != DTYPE_Q8_0 && w.dtype != DTYPE_Q4_0) return false;
    return w.ntiles > 0 && (w.nb + 3) / 4 <= kDirectWarps * kDirectMaxItems &&
           ximage_bytes(w.dtype, w.nb, w.kchunks) <= 48 * 1024;
}

namespace {
template <int XM>
cudaError_t direct_launch(const DevWeight &w, const PipeParams &p, const DirectFuse &f, size_t smem, cudaStream_t st) {
    if (w.dtype == DTYPE_Q8_0)
        return launch_pdl(gemv_direct<DTYPE_Q8_0, XM>, dim3(w.ntiles), dim3(kDirectWarps * 32), smem, st, p, f);
    return launch_pdl(gemv_direct<DTYPE_Q4_0, XM>, dim3(w.ntiles), dim3(kDirectWarps * 32), smem, st, p, f);
}

int direct_common(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, int mode, const DirectFuse &f,
                  cudaStream_t st) {
    if (w.ntiles == 0) return 0;
    PipeParams p{};
    p.codes = reinterpret_cast<const uint8_t *>(w.codes);
    p.scales = w.scales;
    p.x = x;
    p.y = y;
    p.nrows = w.nrows;
    p.cols = w.cols;
    p.nb = w.nb;
    p.ntiles = w.ntiles;
    p.kchunks = w.kchunks;
    p.nseg = (w.nb + 3) / 4;
    // Q4_0: the fp32 x vector only; Q8_0: the digit image (+ the fp32 vector of a fused producer).
    size_t smem = (size_t)w.nb * 32 * sizeof(float);
    if (w.dtype != DTYPE_Q4_0) {
        smem = ximage_bytes(w.dtype, w.nb, w.kchunks);
        if (mode != kXPlain) smem = ((smem + 15) & ~(size_t)15) + (size_t)w.nb * 32 * sizeof(float);
    }
    cudaError_t e = mode == kXResNorm ? direct_launch<kXResNorm>(w, p, f, smem, st)
                  : mode == kXGeGLU   ? direct_launch<kXGeGLU>(w, p, f, smem, st)
                                      : direct_launch<kXPlain>(w, p, f, smem, st);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        ctx_fail(ctx, "launch_gemv_direct", "launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
}  // namespace

// y = W . x for a small Q8_0 / Q4_0 weight (direct_supported), one CTA per tile.
int launch_gemv_direct(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, cudaStream_t st) {
    return direct_common(ctx, w, x, y, kXPlain, DirectFuse{}, st);
}

int launch_gemv_direct_resnorm(kernel_context_t *ctx, const DevWeight &w, const float *t, const float *w_post,
                               const float *h_in, const float *w_next, float *h_out, float eps, float *y,
                               cudaStream_t st) {
    DirectFuse f{};
    f.t = t;
    f.w_post = w_post;
    f.h_in = h_in;
    f.w_next = w_next;
    f.h_out = h_out;
    f.eps = eps;
    return direct_common(ctx, w, nullptr, y, kXResNorm, f, st);
}

int launch_gemv_direct_geglu(kernel_context_t *ctx, const DevWeight &w, const float *gu, float *y, cudaStream_t st) {
    DirectFuse f{};
    f.gu = gu;
    return direct_common(ctx, w, nullptr, y, kXGeGLU, f, st);
}

// Largest number of warps that can share one tile: ranges hold at least
// floor(T/W) items each, so nseg consecutive items meet at most
// ceil((nseg-1)/L) + 1 of them; with fewer items than warps every range holds
// at most one item.
int pipe_kmax(long long T, long long W, int nseg) {
    if (T <= 0) return 1;
    if (T < W) return nseg;
    const long long L = T / W;
    const long long k = (nseg - 1 + L - 1) / L + 1;
    return (int)(k < nseg ? k : nseg);
}

// Quantized formats run gemv_stream (gemv_stream.cu); dense F32 / BF16 rows
// the pipelined kernel of this file.
bool pipe_supported(kernel_context_t *ctx, const DevWeight &w) {
    if (stream_dtype(w.dtype)) return stream_supported(ctx, w);
    if (w.dtype != DTYPE_F32 && w.dtype != DTYPE_BF16) return false;
    return pipe_smem(w.dtype, w.nb, w.kchunks, pipe_cfg(w)) <= 227 * 1024;
}

// Scratch in float units: partials [ntiles][kmax][32] (two floats per entry
// for the int64 ternary sums), counters [ntiles].
void pipe_scratch_size(kernel_context_t *ctx, const DevWeight &w, size_t *part_floats, size_t *cnt_ints) {
    if (stream_dtype(w.dtype)) {
        stream_scratch_size(ctx, w, part_floats, cnt_ints);
        return;
    }
    const int nseg = item_nseg(w);
    const long long T = (long long)w.ntiles * nseg;
    const long long W = (long long)sm_count(ctx->device) * pipe_cfg(w).nw;
    *part_floats = (size_t)w.ntiles * pipe_kmax(T, W, nseg) * 32 * (w.dtype == DTYPE_TQ2_0 ? 2 : 1);
    *cnt_ints = (size_t)w.ntiles;
}

// Batch-1 product y[r] = W[r,:] . x with the pipelined kernel.  part / cnt /
// err: scratch sized by pipe_scratch_size (counters zero), error word.
int launch_gemv_pipe(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, float *part, int *cnt,
                     int *err, cudaStream_t st) {
    return launch_gemv_pipe_ll(ctx, w, x, y, part, cnt, err, nullptr, nullptr, st);
}

int launch_gemv_pipe_ll(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, float *part, int *cnt,
                        int *err, const GatherArgs *g, bool *gathered, cudaStream_t st) {
    if (gathered) *gathered = false;
    if (stream_dtype(w.dtype)) {
        if (gathered && g) *gathered = w.ntiles > 0;
        return launch_gemv_stream(ctx, w, x, y, part, cnt, err, g, st);
    }
    if (w.ntiles == 0) return 0;
    const int ll_n = g ? g->n : 0;
    if (ll_n < 0 || ll_n > kMaxPeers) {
        ctx_fail(ctx, "launch_gemv_pipe", "%d gather targets (at most %d)", ll_n, kMaxPeers);
        return -1;
    }
    const PipeCfg c = pipe_cfg(w);
    PipeParams p;
    p.early = pipe_early(c);
    p.ll_n = ll_n;
    p.ll_off = g ? g->row_off : 0;
    p.ll_epoch = g ? g->epoch : 0u;
    for (int k = 0; k < kMaxPeers; ++k) p.ll[k] = k < ll_n ? g->targets[k] : nullptr;
    p.codes = reinterpret_cast<const uint8_t *>(w.codes);
    p.scales = w.scales;
    p.x = x;
    p.y = y;
    p.part = part;
    p.cnt = cnt;
    p.err = err;
    p.nrows = w.nrows;
    p.cols = w.cols;
    p.nb = w.nb;
    p.ntiles = w.ntiles;
    p.kchunks = w.kchunks;
    p.nseg = item_nseg(w);
    p.total_items = (long long)w.ntiles * p.nseg;
    // One CTA per SM, or fewer when the weight has fewer items than a full
    // grid has warps (small decode projections): every warp gets work.
    const long long want = (p.total_items + c.nw - 1) / c.nw;
    const int grid = (int)std::min<long long>(sm_count(ctx->device), std::max<long long>(1, want));
    p.total_warps = grid * c.nw;
    p.kmax = pipe_kmax(p.total_items, p.total_warps, p.nseg);
    const size_t smem = pipe_smem(w.dtype, w.nb, w.kchunks, c);
    switch (w.dtype) {
        case DTYPE_F32: return launch_cfg<DTYPE_F32>(ctx, p, c, grid, smem, st);
        case DTYPE_BF16: return launch_cfg<DTYPE_BF16>(ctx, p, c, grid, smem, st);
        default:
            ctx_fail(ctx, "launch_gemv_pipe", "unsupported dtype");
            return -1;
    }
}
