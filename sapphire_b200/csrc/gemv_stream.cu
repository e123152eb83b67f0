// gemv_stream.cu - batch-1 GEMV of the quantized formats (Q8_0, Q4_0, TQ2_0):
// the decode hot path behind kernel_gemv.
//
// Same products as the reference row kernels (src/kernels/q4_0_avx.c:102-148,
// q8_0_avx.c:16-136, driven per row by src/kernels/pool.c:106-143), plus the
// ternary format.
//
// Work split.  A "unit" is 32 rows x 64 columns (two 32-column blocks) of a
// 32-row tile.  Units are numbered tile-major and every consumer warp of the
// persistent grid (one CTA per SM) takes a contiguous range of them whose
// length differs from the others' by at most one unit, so every SM streams
// the same number of bytes whatever the shape.  A warp walks its range in
// items of up to UPI units, cut at tile boundaries and at the range's end.
//
// Memory pipeline.  Warp NC of each CTA is the producer: its lane c streams
// consumer c's items into that consumer's ring of NS shared-memory slots with
// cp.async.bulk, completing on the slot's "full" mbarrier (expect_tx).  A
// consumer waits on "full", copies the item into registers, arrives on the
// slot's "empty" mbarrier (release; the producer's acquire-wait on it orders
// the refill after the reads, so no proxy fence is needed) and only then
// computes.  Consumers issue no copies.
//
// Dot products run on the integer tensor cores (mma.sync m16n8k32).  x is
// converted once per CTA to a 22-bit fixed-point image X_j = round(x_j 2^e)
// (one exponent e for all of x) split into three balanced int8 digits
// X = d0 + 256 d1 + 65536 d2, stored per 32-column block as the B fragments
// of digit columns 0..2 plus a zero column.
//   Q8_0 / Q4_0: a unit's two blocks share one C tile - block 2p in digit
//     columns 0..2, block 2p+1 in columns 4..6 - so one epilogue (digit join,
//     conversion, per-block scale FMA, like the reference's per-block
//     (q - 8) * scale) serves two blocks.  Q4_0 nibbles are fed as unsigned
//     codes with -8 * (digit sum) as the MMA's start value.
//   TQ2_0: the codes c = t + 1 of four 16-row x 32-column fragments are
//     interleaved as the four 2-bit planes of the same bytes, so each MMA
//     register is one AND with a plane mask (plane m carries 4^m c); the four
//     planes accumulate exactly in int32 across all of K, are joined by exact
//     shifts at the end of a tile, and sum_j X_j is subtracted once per row.
//
// Split tiles.  A tile whose items span several warps is finished by the
// warp that owns its first segment - for that warp it is the last tile of its
// range, while the other owners meet it first, so their parts are long done
// when it gets there.  The others store their per-row partials (fp32, or the
// exact int64 sum for ternary) as 8-byte words tagged with the launch's epoch
// in the slot of their rank among the tile's owners; the finisher waits
// (bounded) for each word to carry the epoch and sums in slot order
// (deterministic).  An aligned 8-byte store arrives whole, so the tag marks
// the value valid: no fence, atomic or counter is needed.
//
// Waits are bounded.  A consumer whose slot does not fill sets bit 0 of *err
// and its abort flag, and leaves the loop; the producer lane serving it stops
// waiting for it; before the CTA exits every producer lane waits (bounded) for
// the copies it issued that may still be in flight.
#include <cfloat>

#include "internal.cuh"

namespace {

constexpr unsigned kWaitLimit = 1u << 26;     // polls of a bounded wait
constexpr int kImgBlock = 128;                // digit rows d0, d1, d2 and a zero row, 32 bytes each
constexpr int kMaxConsumers = 16;

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ uint32_t saddr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// Bulk global -> shared copy (16-byte aligned, multiple of 16 bytes), into this CTA only.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(saddr(dst)),
        "l"(src), "r"(bytes), "r"(saddr(bar))
        : "memory");
}

// D = A(16x32) * B(32x8) + C, 8-bit operands, int32 accumulate.
__device__ __forceinline__ void mma_s8(int (&d)[4], uint4 a, uint2 b, const int (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}
__device__ __forceinline__ void mma_u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b,
                                       const int (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}

template <typename T>
__device__ __forceinline__ T lds(const uint8_t *p) {
    return *reinterpret_cast<const T *>(p);
}

// ------------------------------------------------------------ formats -----
// Bytes of one unit in the device layout (internal.cuh / repack.cu): codes
// and (per-block formats) scales; per-block formats store a unit as two
// consecutive blocks, so the last unit of an odd-block row is one block.
template <tensor_dtype_t DT>
struct Fmt;
template <>
struct Fmt<DTYPE_Q8_0> {
    static constexpr int kBlockCode = 1024;
    static constexpr bool kBlockScales = true;
};
template <>
struct Fmt<DTYPE_Q4_0> {
    static constexpr int kBlockCode = 512;
    static constexpr bool kBlockScales = true;
};
template <>
struct Fmt<DTYPE_TQ2_0> {
    static constexpr int kBlockCode = 256;
    static constexpr bool kBlockScales = false;    // one fp32 scale per row, read when a tile starts
};
template <tensor_dtype_t DT>
__host__ __device__ constexpr int unit_code() { return 2 * Fmt<DT>::kBlockCode; }
template <tensor_dtype_t DT>
__host__ __device__ constexpr int unit_scale() { return Fmt<DT>::kBlockScales ? 256 : 0; }
template <tensor_dtype_t DT, int UPI>
__host__ __device__ constexpr int slot_bytes() { return UPI * (unit_code<DT>() + unit_scale<DT>()); }

struct StreamParams {
    const uint8_t *codes;
    const float *scales;
    const float *x;
    float *y;
    unsigned long long *part;   // [ntiles][kmax][32][words] epoch-tagged partials of split tiles
                                // (one word of fp32 bits; two of int64 halves for TQ2_0)
    int *err;                   // error word (bit 0: a bounded wait expired)
    unsigned epoch;             // tag of this launch's partial words (never 0)
    long long total_units;      // ntiles * nunits
    int nrows, cols, nb, nunits, ntiles, kmax, total_warps;
    int early;                  // items per consumer the producer issues before the x loads are out
    unsigned wait_limit;        // test hook: polls before the unarmed consumer's first wait gives up
    int test_unarmed;           // test hook: consumer 0 of CTA 0 gets no copy for its first item
    // Row-sharded products gathered over peer memory: when ll_n > 0 row r is
    // not stored at y[r] but sent to every rank k as the 8-byte word
    // (ll_epoch << 32 | bits of the value) at ll[k][ll_off + r] (NVLink stores;
    // an aligned 8-byte store arrives whole, so the epoch marks the value
    // valid and no fence is needed).
    int ll_n, ll_off;
    unsigned ll_epoch;
    unsigned long long *ll[kMaxPeers];
    // The gather itself: once a consumer warp has finished its items it
    // waits for rows [gw*R/W, (gw+1)*R/W) of its own buffer `ll_self` to
    // carry the epoch (bounded by ll_wait_ns) and writes them to y_full.
    const unsigned long long *ll_self;
    float *y_full;
    long long rows_full;
    unsigned long long ll_wait_ns;
};

__device__ __forceinline__ void store_y(const StreamParams &p, size_t r, float v) {
    if (p.ll_n) {
        const unsigned long long word = ((unsigned long long)p.ll_epoch << 32) | __float_as_uint(v);
        for (int k = 0; k < p.ll_n; ++k)
            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p.ll[k] + (size_t)p.ll_off + r), "l"(word) : "memory");
    } else {
        p.y[r] = v;
    }
}

// Warp w of W owns units [w*U/W, (w+1)*U/W); unit_owner(i) is the warp whose
// range holds unit i.
__device__ __forceinline__ long long range_begin(long long w, long long U, long long W) { return (w * U) / W; }
__device__ __forceinline__ int unit_owner(long long i, long long U, long long W) {
    long long w = ((i + 1) * W + U - 1) / U - 1;
    return (int)(w < W - 1 ? w : W - 1);
}

// Walks a warp's unit range item by item (producer lanes and consumers walk
// the same sequence).
struct Cursor {
    long long u, ub;      // next unit, end of the range
    int tile, pu;         // tile of unit u and its position in the tile
    __device__ __forceinline__ void start(long long ua, long long ub_, int nunits) {
        u = ua;
        ub = ub_;
        tile = (int)(ua / nunits);
        pu = (int)(ua - (long long)tile * nunits);
    }
    __device__ __forceinline__ bool more() const { return u < ub; }
    // Units in the next item (at most upi, not past the tile or the range).
    __device__ __forceinline__ int count(int upi, int nunits) const {
        return (int)min((long long)min(upi, nunits - pu), ub - u);
    }
    __device__ __forceinline__ void advance(int nu, int nunits) {
        u += nu;
        pu += nu;
        if (pu == nunits) {
            pu = 0;
            ++tile;
        }
    }
};

// Named barrier over the NC consumer warps (the producer warp never joins).
__device__ __forceinline__ void consumers_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// ------------------------------------------------------- x preparation ----
// Shared-memory image of x, built by the consumer warps:
//   img[nbp][4][4][8]  per block: digit rows d0, d1, d2 (B fragments: per
//                      lane-in-group tig, K slots 4tig..4tig+3 then
//                      16+4tig..16+4tig+3) and a zero row; nbp = nb rounded
//                      up to even, the extra block all zero;
//   corr[nbp][4]       Q4_0: -8 * (sum of the block's digits d0, d1, d2), 0;
//   sx                 TQ2_0: sum over all columns of X_j (int64);
//   pexp               2^-e.
struct XImage {
    uint8_t *img;
    int *corr;
    long long *sx;
    float *pexp;
    int *nonfinite;
};

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }
__host__ __device__ inline int nb_even(int nb) { return (nb + 1) & ~1; }
__host__ __device__ inline size_t ximg_bytes(int nb, bool q4) {
    size_t b = (size_t)nb_even(nb) * kImgBlock;
    if (q4) b += (size_t)nb_even(nb) * 16;
    return align16(b) + 16 + 16;          // + sx (8) + pexp (4), padded
}

// Exponent e with max|x| * 2^e < 2^22 (0 for all-zero x).
__device__ __forceinline__ int x_exponent(float m) {
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

// Byte offset, inside a 32-byte digit row, of the K slot that carries
// element p (0..31) of a block.  Q8_0 / TQ2_0: slot = p.  Q4_0: the low nibble
// of code byte 4t+j (element 8t+2j) is slot 4t+j, the high nibble (element
// 8t+2j+1) slot 16+4t+j.
template <tensor_dtype_t DT>
__device__ __forceinline__ int digit_byte(int p) {
    if (DT == DTYPE_Q4_0) return (p >> 3) * 8 + (p & 1) * 4 + ((p & 7) >> 1);
    return ((p & 15) >> 2) * 8 + (p >> 4) * 4 + (p & 3);
}

// Loads of x in flight per consumer thread in the staging pass.
constexpr int kXLoads = 16;

// Builds the x image.  Pass 1 stages x as fp32 in the image region itself
// (block b's 128 bytes hold x[32b .. 32b+32) as floats; columns past `cols`
// are zero) with every load of a thread issued at once, and reduces max|x|.
// Pass 2 converts block b in place: the warp that owns it reads the block's
// 32 floats, then overwrites the same 128 bytes with the digit rows.
template <tensor_dtype_t DT, int NC>
__device__ void prepare_x(const StreamParams &p, const XImage &xi) {
    constexpr int kThreads = NC * 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    __shared__ unsigned s_max[kMaxConsumers];
    __shared__ long long s_sx[kMaxConsumers];
    const int nbp = nb_even(p.nb);
    float *stage = reinterpret_cast<float *>(xi.img);
    // Pass 1.  The bits of a non-negative float order like the float, so an
    // unsigned maximum gives max|x| (NaN bits sort above every finite value).
    unsigned m = 0;
    bool bad = false;
    auto take = [&](float t) {
        bad |= !isfinite(t);
        m = max(m, __float_as_uint(fabsf(t)));
    };
    // Every thread issues a first batch of loads, then all consumer threads
    // arrive on barrier 2 together (the x loads are out: the producer may
    // issue the rest of the rings); later batches, for long rows, follow.
    if (((uintptr_t)p.x & 15) == 0 && (p.cols & 3) == 0) {
        const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
        const int n4 = p.cols >> 2;
        for (int i0 = tid, first = 1; first || i0 < n4; i0 += kXLoads * kThreads, first = 0) {
            float4 t[kXLoads];
#pragma unroll
            for (int q = 0; q < kXLoads; ++q) {
                const int i = i0 + q * kThreads;
                t[q] = i < n4 ? __ldg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (first) asm volatile("bar.arrive 2, %0;" ::"r"(kThreads + 32) : "memory");
#pragma unroll
            for (int q = 0; q < kXLoads; ++q) {
                const int i = i0 + q * kThreads;
                if (i < n4) {
                    reinterpret_cast<float4 *>(stage)[i] = t[q];
                    take(t[q].x);
                    take(t[q].y);
                    take(t[q].z);
                    take(t[q].w);
                }
            }
        }
    } else {
        for (int i0 = tid, first = 1; first || i0 < p.cols; i0 += kXLoads * kThreads, first = 0) {
            float t[kXLoads];
#pragma unroll
            for (int q = 0; q < kXLoads; ++q) {
                const int i = i0 + q * kThreads;
                t[q] = i < p.cols ? __ldg(p.x + i) : 0.0f;
            }
            if (first) asm volatile("bar.arrive 2, %0;" ::"r"(kThreads + 32) : "memory");
#pragma unroll
            for (int q = 0; q < kXLoads; ++q) {
                const int i = i0 + q * kThreads;
                if (i < p.cols) {
                    stage[i] = t[q];
                    take(t[q]);
                }
            }
        }
    }
    for (int i = p.cols + tid; i < nbp * 32; i += kThreads) stage[i] = 0.0f;
    if (bad) *xi.nonfinite = 1;
    m = __reduce_max_sync(0xffffffffu, m);
    if (lane == 0) s_max[warp] = m;
    consumers_sync(kThreads);
    m = 0;
    for (int i = 0; i < NC; ++i) m = max(m, s_max[i]);
    const float mf = __uint_as_float(m);
    const int e = x_exponent(isfinite(mf) ? mf : FLT_MAX);
    if (threadIdx.x == 0) *xi.pexp = (e >= -126 && e <= 127) ? __int_as_float((127 - e) << 23) : ldexpf(1.0f, -e);
    // x * 2^e as two exact multiplies by normal powers of two (e <= 170).
    const int e1 = min(max(e, -126), 127);
    const float f1 = __int_as_float((e1 + 127) << 23), f2 = __int_as_float((e - e1 + 127) << 23);
    // Pass 2: digits of blocks b = warp + NC*k (the padding block of an
    // odd-block row is staged as zeros, so its digits and correction are 0),
    // the Q4_0 corrections and the ternary x sum.
    long long sx = 0;
    if (DT != DTYPE_Q4_0) {
        // Q8_0 / TQ2_0: elements 4k .. 4k+3 of a block land in four
        // consecutive bytes, (k & 3) * 8 + (k >> 2) * 4, of each digit row
        // (digit_byte), so lane 8q + k converts them from one 16-byte load
        // and stores one word per row: a warp converts blocks 4w + 4NC i + q.
        const int q = lane >> 3, k = lane & 7;
        const int wb = (k & 3) * 8 + (k >> 2) * 4;
        long long sxl = 0;
        for (int b0 = 4 * warp; b0 < nbp; b0 += 4 * NC) {
            const int b = b0 + q;
            const float4 t = b < nbp ? *reinterpret_cast<const float4 *>(stage + (size_t)b * 32 + 4 * k)
                                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            __syncwarp();
            if (b < nbp) {
                const float tv[4] = {t.x, t.y, t.z, t.w};
                uint32_t w0 = 0, w1 = 0, w2 = 0;
                int sb = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int X = isfinite(tv[e]) ? __float2int_rn(tv[e] * f1 * f2) : 0;
                    const int d0 = ((X & 0xFF) ^ 0x80) - 0x80;
                    const int X1 = (X - d0) >> 8;
                    const int d1 = ((X1 & 0xFF) ^ 0x80) - 0x80;
                    const int d2 = (X1 - d1) >> 8;
                    w0 |= (uint32_t)(d0 & 0xFF) << (8 * e);
                    w1 |= (uint32_t)(d1 & 0xFF) << (8 * e);
                    w2 |= (uint32_t)(d2 & 0xFF) << (8 * e);
                    sb += X;       // |X| < 2^22: four fit int32
                }
                uint8_t *blk = xi.img + (size_t)b * kImgBlock;
                *reinterpret_cast<uint32_t *>(blk + wb) = w0;
                *reinterpret_cast<uint32_t *>(blk + 32 + wb) = w1;
                *reinterpret_cast<uint32_t *>(blk + 64 + wb) = w2;
                *reinterpret_cast<uint32_t *>(blk + 96 + wb) = 0u;
                sxl += sb;
            }
        }
        if (DT == DTYPE_TQ2_0) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sxl += __shfl_xor_sync(0xffffffffu, sxl, o);
            sx = sxl;
        }
    }
    const int off = digit_byte<DT>(lane);
#pragma unroll 2
    for (int b = warp; DT == DTYPE_Q4_0 && b < nbp; b += NC) {
        uint8_t *blk = xi.img + (size_t)b * kImgBlock;
        const float t = stage[b * 32 + lane];
        __syncwarp();
        const int X = isfinite(t) ? __float2int_rn(t * f1 * f2) : 0;
        const int d0 = ((X & 0xFF) ^ 0x80) - 0x80;
        const int X1 = (X - d0) >> 8;
        const int d1 = ((X1 & 0xFF) ^ 0x80) - 0x80;
        const int d2 = (X1 - d1) >> 8;
        blk[off] = (uint8_t)d0;
        blk[32 + off] = (uint8_t)d1;
        blk[64 + off] = (uint8_t)d2;
        blk[96 + lane] = 0;
        if (DT == DTYPE_Q4_0) {
            const int s0 = __reduce_add_sync(0xffffffffu, d0);
            const int s1 = __reduce_add_sync(0xffffffffu, d1);
            const int s2 = __reduce_add_sync(0xffffffffu, d2);
            if (lane < 4) xi.corr[b * 4 + lane] = lane == 0 ? -8 * s0 : lane == 1 ? -8 * s1 : lane == 2 ? -8 * s2 : 0;
        }
        if (DT == DTYPE_TQ2_0) sx += __reduce_add_sync(0xffffffffu, X);   // |X| < 2^22: a block sum fits int32
    }
    if (DT == DTYPE_TQ2_0) {
        if (lane == 0) s_sx[warp] = sx;
        consumers_sync(kThreads);
        if (threadIdx.x == 0) {
            long long t = 0;
            for (int i = 0; i < NC; ++i) t += s_sx[i];
            *xi.sx = t;
        }
    }
}

// ----------------------------------------------------------- item in regs --
// The part of a staged item one lane needs (unit u of UPI; units past the
// item's count are not loaded).
template <tensor_dtype_t DT, int UPI>
struct Item;
template <int UPI>
struct Item<DTYPE_Q8_0, UPI> {
    uint4 a[UPI][2][2];   // [unit][block of the unit][16-row half]: the A fragment
    float4 s[UPI];        // scales of rows g, g+8, g+16, g+24 of block 2p + tig/2
    template <bool FULL>
    __device__ __forceinline__ void load(const uint8_t *st, int nu, int lane, bool last_half) {
        const int g = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int u = 0; u < UPI; ++u) {
            if (FULL || u < nu) {
#pragma unroll
                for (int k = 0; k < 2; ++k)
#pragma unroll
                    for (int h = 0; h < 2; ++h) a[u][k][h] = lds<uint4>(st + (2 * u + k) * 1024 + h * 512 + lane * 16);
                // Block 2p+1 of an odd-block row's last unit is not copied:
                // its lanes (tig >= 2) use zero scales, not the slot's stale bytes.
                const float4 t = lds<float4>(st + UPI * 2048 + u * 256 + (tig >> 1) * 128 + g * 16);
                const bool z = last_half && u == nu - 1 && tig >= 2;
                s[u] = make_float4(z ? 0.f : t.x, z ? 0.f : t.y, z ? 0.f : t.z, z ? 0.f : t.w);
            }
        }
    }
};
template <int UPI>
struct Item<DTYPE_Q4_0, UPI> {
    uint4 a[UPI][2];      // [unit][block]: code word tig of rows g, g+8, g+16, g+24
    float4 s[UPI];
    template <bool FULL>
    __device__ __forceinline__ void load(const uint8_t *st, int nu, int lane, bool last_half) {
        const int g = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int u = 0; u < UPI; ++u) {
            if (FULL || u < nu) {
#pragma unroll
                for (int k = 0; k < 2; ++k) a[u][k] = lds<uint4>(st + (2 * u + k) * 512 + lane * 16);
                const float4 t = lds<float4>(st + UPI * 1024 + u * 256 + (tig >> 1) * 128 + g * 16);
                const bool z = last_half && u == nu - 1 && tig >= 2;
                s[u] = make_float4(z ? 0.f : t.x, z ? 0.f : t.y, z ? 0.f : t.z, z ? 0.f : t.w);
            }
        }
    }
};
template <int UPI>
struct Item<DTYPE_TQ2_0, UPI> {
    uint4 a[UPI];         // four words: 2-bit planes of four A fragments
    template <bool FULL>
    __device__ __forceinline__ void load(const uint8_t *st, int nu, int lane, bool) {
#pragma unroll
        for (int u = 0; u < UPI; ++u)
            if (FULL || u < nu) a[u] = lds<uint4>(st + u * 512 + lane * 16);
    }
};

// Accumulators of one 32-row tile for a lane (g = lane/4, tig = lane%4).
struct Acc {
    float f[2][2];        // Q8_0 / Q4_0: [half][row g / g+8] scaled sums (digit columns of this lane)
    int d[2][4][4];       // TQ2_0: [set: unit parity][plane][C register] exact sums (two independent
                          // MMA chains)
    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int h = 0; h < 2; ++h) f[h][0] = f[h][1] = 0.0f;
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int m = 0; m < 4; ++m)
#pragma unroll
                for (int i = 0; i < 4; ++i) d[q][m][i] = 0;
    }
};

// Lane constants for the B loads: offsets inside a unit's 256-byte image
// (blocks 2p, 2p+1).  Q8_0 / Q4_0: block 2p feeds digit columns 0..2 (lanes
// g < 3, g == 3 reads the zero row), block 2p+1 columns 4..6 (lanes g = 4..6;
// all other lanes read a zero row).  TQ2_0: both blocks feed columns 0..2.
struct LaneOff {
    int b0, b1;
};
template <tensor_dtype_t DT>
__device__ __forceinline__ LaneOff lane_offsets(int lane) {
    const int g = lane >> 2, tig = lane & 3;
    LaneOff o;
    if (DT == DTYPE_TQ2_0) {
        o.b0 = min(g, 3) * 32 + tig * 8;
        o.b1 = kImgBlock + o.b0;
    } else {
        o.b0 = (g < 4 ? g : 3) * 32 + tig * 8;
        o.b1 = kImgBlock + (g >= 4 ? min(g - 4, 3) : 3) * 32 + tig * 8;
    }
    return o;
}

// Joins digits 0 and 1 of a C register pair (below 2^28: a block's digit
// products are below 2^22) and adds scale * value.
__device__ __forceinline__ void scale2(float (&acc)[2], const int (&D)[4], float s0, float s1) {
    acc[0] = fmaf(s0, (float)(D[0] + 256 * D[1]), acc[0]);
    acc[1] = fmaf(s1, (float)(D[2] + 256 * D[3]), acc[1]);
}

template <bool FULL, int UPI>
__device__ __forceinline__ void compute(const Item<DTYPE_Q8_0, UPI> &R, int nu, int p0, const XImage &xi,
                                        LaneOff lo, int, Acc &acc) {
    const int zero[4] = {0, 0, 0, 0};
#pragma unroll
    for (int u = 0; u < UPI; ++u) {
        if (FULL || u < nu) {
            const uint8_t *bi = xi.img + (size_t)(p0 + u) * (2 * kImgBlock);
            const uint2 B0 = lds<uint2>(bi + lo.b0), B1 = lds<uint2>(bi + lo.b1);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                int D[4];
                mma_s8(D, R.a[u][0][h], B0, zero);
                mma_s8(D, R.a[u][1][h], B1, D);
                scale2(acc.f[h], D, h ? R.s[u].z : R.s[u].x, h ? R.s[u].w : R.s[u].y);
            }
        }
    }
}

template <bool FULL, int UPI>
__device__ __forceinline__ void compute(const Item<DTYPE_Q4_0, UPI> &R, int nu, int p0, const XImage &xi,
                                        LaneOff lo, int tig, Acc &acc) {
#pragma unroll
    for (int u = 0; u < UPI; ++u) {
        if (FULL || u < nu) {
            const uint8_t *bi = xi.img + (size_t)(p0 + u) * (2 * kImgBlock);
            const uint2 B0 = lds<uint2>(bi + lo.b0), B1 = lds<uint2>(bi + lo.b1);
            const int2 C = *reinterpret_cast<const int2 *>(xi.corr + (size_t)(p0 + u) * 8 + tig * 2);
            const int c0[4] = {C.x, C.y, C.x, C.y};
            const uint4 A0 = R.a[u][0], A1 = R.a[u][1];
            // Half 0 (rows g, g+8): words x, y; half 1 (rows g+16, g+24): z, w.
            // Low nibbles are K slots 0..15, high nibbles 16..31.
            {
                int D[4];
                mma_u8(D, A0.x & 0x0F0F0F0Fu, A0.y & 0x0F0F0F0Fu, (A0.x >> 4) & 0x0F0F0F0Fu, (A0.y >> 4) & 0x0F0F0F0Fu,
                       B0, c0);
                mma_u8(D, A1.x & 0x0F0F0F0Fu, A1.y & 0x0F0F0F0Fu, (A1.x >> 4) & 0x0F0F0F0Fu, (A1.y >> 4) & 0x0F0F0F0Fu,
                       B1, D);
                scale2(acc.f[0], D, R.s[u].x, R.s[u].y);
            }
            {
                int D[4];
                mma_u8(D, A0.z & 0x0F0F0F0Fu, A0.w & 0x0F0F0F0Fu, (A0.z >> 4) & 0x0F0F0F0Fu, (A0.w >> 4) & 0x0F0F0F0Fu,
                       B0, c0);
                mma_u8(D, A1.z & 0x0F0F0F0Fu, A1.w & 0x0F0F0F0Fu, (A1.z >> 4) & 0x0F0F0F0Fu, (A1.w >> 4) & 0x0F0F0F0Fu,
                       B1, D);
                scale2(acc.f[1], D, R.s[u].z, R.s[u].w);
            }
        }
    }
}

template <bool FULL, int UPI>
__device__ __forceinline__ void compute(const Item<DTYPE_TQ2_0, UPI> &R, int nu, int p0, const XImage &xi,
                                        LaneOff lo, int, Acc &acc) {
#pragma unroll
    for (int u = 0; u < UPI; ++u) {
        if (FULL || u < nu) {
            const uint8_t *bi = xi.img + (size_t)(p0 + u) * (2 * kImgBlock);
            const uint2 B0 = lds<uint2>(bi + lo.b0), B1 = lds<uint2>(bi + lo.b1);
            const uint4 W = R.a[u];
            // Plane m (bits 2m, 2m+1 of every byte) is the fragment of half
            // m & 1 and block 2p + (m >> 1), scaled by 4^m.  Even and odd
            // units accumulate into separate sets (independent MMA chains).
            int(&a)[4][4] = acc.d[u & 1];
            mma_u8(a[0], W.x & 0x03030303u, W.y & 0x03030303u, W.z & 0x03030303u, W.w & 0x03030303u, B0, a[0]);
            mma_u8(a[1], W.x & 0x0C0C0C0Cu, W.y & 0x0C0C0C0Cu, W.z & 0x0C0C0C0Cu, W.w & 0x0C0C0C0Cu, B0, a[1]);
            mma_u8(a[2], W.x & 0x30303030u, W.y & 0x30303030u, W.z & 0x30303030u, W.w & 0x30303030u, B1, a[2]);
            mma_u8(a[3], W.x & 0xC0C0C0C0u, W.y & 0xC0C0C0C0u, W.z & 0xC0C0C0C0u, W.w & 0xC0C0C0C0u, B1, a[3]);
        }
    }
}

// Per-row results of a tile: lanes with tig == 0 hold rows g + 8i (i = 0..3)
// as 8-byte values (fp32 bits for Q8_0 / Q4_0, already scaled by 2^-e; the
// exact int64 sum of c * X for TQ2_0).  All lanes must call (shuffles).
template <tensor_dtype_t DT>
__device__ __forceinline__ void tile_rows(const Acc &acc, unsigned long long (&v)[4], float pe) {
    if (DT == DTYPE_TQ2_0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int D[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int p0 = acc.d[0][h][i] + acc.d[1][h][i], p2 = acc.d[0][h + 2][i] + acc.d[1][h + 2][i];
                D[i] = h == 0 ? p0 + (p2 >> 4) : (p0 >> 2) + (p2 >> 6);
            }
            const int up0 = __shfl_down_sync(0xffffffffu, D[0], 1);
            const int up2 = __shfl_down_sync(0xffffffffu, D[2], 1);
            v[2 * h] = (unsigned long long)((long long)D[0] + 256LL * D[1] + 65536LL * up0);
            v[2 * h + 1] = (unsigned long long)((long long)D[2] + 256LL * D[3] + 65536LL * up2);
        }
    } else {
        // Lanes tig 0 / 2: digits 0-1 of blocks 2p / 2p+1; tig 1 / 3: digit 2.
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                float t = fmaf(65536.0f, __shfl_down_sync(0xffffffffu, acc.f[h][i], 1), acc.f[h][i]);
                t += __shfl_down_sync(0xffffffffu, t, 2);
                v[2 * h + i] = __float_as_uint(t * pe);
            }
    }
}

// rs: ternary row scale of row tile*32 + lane, loaded when the tile started.
template <tensor_dtype_t DT>
__device__ __forceinline__ float finish_row(const XImage &xi, unsigned long long v, bool nonfinite, float rs) {
    float out;
    if (DT == DTYPE_TQ2_0) {
        out = (float)((double)rs * ((double)((long long)v - *xi.sx) * (double)*xi.pexp));
    } else {
        out = __uint_as_float((uint32_t)v);
    }
    return nonfinite ? __int_as_float(0x7FC00000) : out;
}

// Epoch-tagged 8-byte words of the split-tile partials: (epoch << 32) | bits.
__device__ __forceinline__ void put_word(unsigned long long *p, unsigned epoch, uint32_t bits) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((unsigned long long)epoch << 32) | bits)
                 : "memory");
}
__device__ __forceinline__ unsigned long long ld_part(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Polls a word until it carries `epoch` (bounded); false if the wait ran out.
__device__ __forceinline__ bool get_word(const unsigned long long *p, unsigned epoch, uint32_t &bits) {
    for (unsigned i = 0; i < kWaitLimit; ++i) {
        unsigned long long w;
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
        if ((unsigned)(w >> 32) == epoch) {
            bits = (uint32_t)w;
            return true;
        }
        __nanosleep(64);
    }
    return false;
}

// Stores a finished tile (one row per lane), or its part of a tile shared
// with other warps (see "Split tiles" above).
template <tensor_dtype_t DT>
__device__ void flush_tile(const StreamParams &p, const XImage &xi, int tile, int lane, int my_warp, bool whole,
                           const unsigned long long (&v)[4], bool nonfinite, float rs) {
    // Lane l takes row l = g + 8i from the lane holding it, (l % 8) * 4.
    unsigned long long mine = v[0];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const unsigned long long t = __shfl_sync(0xffffffffu, v[i], (lane & 7) * 4);
        if ((lane >> 3) == i) mine = t;
    }
    const bool row_ok = tile * 32 + lane < p.nrows;
    if (whole) {
        if (row_ok) store_y(p, (size_t)tile * 32 + lane, finish_row<DT>(xi, mine, nonfinite, rs));
        return;
    }
    // k = owners of the tile's units, slot = this warp's rank among them.
    const long long first = (long long)tile * p.nunits;
    int k = 0, slot = -1;
    const int o0 = unit_owner(first, p.total_units, p.total_warps);
    if (p.total_units >= p.total_warps) {
        // Every warp owns at least one unit, so the tile's owners are the
        // consecutive warps o0..o1.
        k = unit_owner(first + p.nunits - 1, p.total_units, p.total_warps) - o0 + 1;
        slot = my_warp - o0;
    } else {
        int prev = -1;
        for (int s = 0; s < p.nunits; ++s) {
            const int o = s == 0 ? o0 : unit_owner(first + s, p.total_units, p.total_warps);
            if (o != prev) {
                if (o == my_warp) slot = k;
                ++k;
                prev = o;
            }
        }
    }
    constexpr int kWords = DT == DTYPE_TQ2_0 ? 2 : 1;
    unsigned long long *base = p.part + (size_t)tile * p.kmax * 32 * kWords;
    if (slot > 0) {
        unsigned long long *w = base + ((size_t)slot * 32 + lane) * kWords;
        put_word(w, p.epoch, (uint32_t)mine);
        if (kWords == 2) put_word(w + 1, p.epoch, (uint32_t)(mine >> 32));
        return;
    }
    // The finisher: sum the parts in slot order.  The words of kSlots slots
    // are loaded at once (one round trip per batch rather than one per word,
    // which matters when a short shard spreads a tile over dozens of warps);
    // only a word that does not carry the epoch yet is polled again.
    constexpr int kSlots = 8 / kWords;
    bool ok = true;
    long long ti = (long long)mine;
    float tf = __uint_as_float((uint32_t)mine);
    for (int j0 = 1; j0 < k; j0 += kSlots) {
        unsigned long long w[kSlots][kWords];
#pragma unroll
        for (int q = 0; q < kSlots; ++q)
#pragma unroll
            for (int h = 0; h < kWords; ++h)
                w[q][h] = j0 + q < k ? ld_part(base + ((size_t)(j0 + q) * 32 + lane) * kWords + h) : 0ull;
#pragma unroll
        for (int q = 0; q < kSlots; ++q) {
            if (j0 + q >= k) break;
            uint32_t bits[kWords];
#pragma unroll
            for (int h = 0; h < kWords; ++h) {
                bits[h] = (uint32_t)w[q][h];
                if ((unsigned)(w[q][h] >> 32) != p.epoch)
                    ok = ok && get_word(base + ((size_t)(j0 + q) * 32 + lane) * kWords + h, p.epoch, bits[h]);
            }
            if (DT == DTYPE_TQ2_0)
                ti += (long long)(((unsigned long long)bits[kWords - 1] << 32) | bits[0]);
            else
                tf += __uint_as_float(bits[0]);
        }
    }
    const unsigned long long sum = DT == DTYPE_TQ2_0 ? (unsigned long long)ti : __float_as_uint(tf);
    if (!ok) atomicOr(p.err, 1);
    if (row_ok) store_y(p, (size_t)tile * 32 + lane, ok ? finish_row<DT>(xi, sum, nonfinite, rs) : __int_as_float(0x7FC00000));
}

// The gather step of a row-sharded product: rows [r0, r1) of this rank's
// buffer.  Each lane loads up to kGatherBatch words at once (one round trip
// for the whole slice), then waits only for words that do not carry the
// epoch yet.  A word that does not arrive within wait_ns sets bit 3 of *err
// and the CTA-wide flag `expired`, after which the CTA's warps stop waiting
// and store NaN for stale words.
constexpr int kGatherBatch = 8;

__device__ __forceinline__ unsigned long long ld_sys(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__device__ void gather_rows(const StreamParams &p, long long r0, long long r1, int lane, int *expired) {
    for (long long rb = r0 + lane; rb < r1; rb += 32 * kGatherBatch) {
        unsigned long long w[kGatherBatch];
#pragma unroll
        for (int q = 0; q < kGatherBatch; ++q) {
            const long long r = rb + 32 * q;
            w[q] = r < r1 ? ld_sys(p.ll_self + r) : 0ull;
        }
#pragma unroll
        for (int q = 0; q < kGatherBatch; ++q) {
            const long long r = rb + 32 * q;
            if (r >= r1) break;
            if ((unsigned)(w[q] >> 32) != p.ll_epoch) {
                uint64_t t0;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
                for (;;) {
                    if (*reinterpret_cast<volatile int *>(expired)) {
                        w[q] = 0x7FC00000ull;
                        break;
                    }
                    __nanosleep(64);
                    w[q] = ld_sys(p.ll_self + r);
                    if ((unsigned)(w[q] >> 32) == p.ll_epoch) break;
                    uint64_t t;
                    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                    if (t - t0 > p.ll_wait_ns) {
                        atomicOr(p.err, 8);
                        *reinterpret_cast<volatile int *>(expired) = 1;
                        w[q] = 0x7FC00000ull;
                        break;
                    }
                }
            }
            p.y_full[r] = __uint_as_float((unsigned)(w[q] & 0xFFFFFFFFull));
        }
    }
}

// --------------------------------------------------------------- kernel ---
template <tensor_dtype_t DT, int NC, int NS, int UPI>
__global__ void __launch_bounds__((NC + 1) * 32, 1) gemv_stream(const StreamParams p) {
    constexpr int kSlot = slot_bytes<DT, UPI>();
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_nonfinite;
    __shared__ int s_abort[kMaxConsumers];
    __shared__ int s_expired;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Shared memory: [rings][x image], barriers in static shared memory.
    __shared__ __align__(8) uint64_t full[kMaxConsumers][NS];
    __shared__ __align__(8) uint64_t empty[kMaxConsumers][NS];
    uint8_t *rings = smem;
    uint8_t *ximg = smem + (size_t)NC * NS * kSlot;
    XImage xi;
    xi.img = ximg;
    const size_t img_b = (size_t)nb_even(p.nb) * kImgBlock;
    xi.corr = reinterpret_cast<int *>(ximg + img_b);
    const size_t tail = align16(img_b + (DT == DTYPE_Q4_0 ? (size_t)nb_even(p.nb) * 16 : 0));
    xi.sx = reinterpret_cast<long long *>(ximg + tail);
    xi.pexp = reinterpret_cast<float *>(ximg + tail + 16);
    xi.nonfinite = &s_nonfinite;

    const long long U = p.total_units, W = p.total_warps;
    pdl_trigger();
    if (threadIdx.x < NC * NS) {
        mbar_init(&full[0][0] + threadIdx.x, 1);
        mbar_init(&empty[0][0] + threadIdx.x, 32);
    }
    if (threadIdx.x < kMaxConsumers) s_abort[threadIdx.x] = 0;
    if (threadIdx.x == 0) {
        s_nonfinite = 0;
        s_expired = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NC) {
        // ------------------------------------------------------ producer --
        // Lane c streams consumer c's items.  The lanes poll their consumers'
        // "empty" barriers with the non-blocking test_wait in lockstep, so a
        // lane whose consumer is still computing never holds up the others
        // (a blocking wait would suspend the whole warp).  The weight does
        // not depend on earlier kernels, so `early` items per consumer go
        // out before the programmatic-launch wait; the rest wait until the
        // consumers have issued their x loads (named barrier 2), which would
        // otherwise queue behind every ring's copies.
        const int c = lane;
        Cursor cur;
        cur.start(0, 0, p.nunits);
        if (c < NC) {
            const int gw = blockIdx.x * NC + c;
            cur.start(range_begin(gw, U, W), range_begin(gw + 1, U, W), p.nunits);
        }
        uint8_t *ring = rings + (size_t)min(c, NC - 1) * NS * kSlot;
        int j = 0, issued = 0;
        unsigned idle = 0;
        bool live = c < NC && cur.more();
        bool gate = true;                  // the x-load barrier is still ahead
        const int early = min(p.early, NS);
        for (;;) {
            if (gate && !__any_sync(0xffffffffu, live && j < early)) {
                asm volatile("bar.sync 2, %0;" ::"r"((NC + 1) * 32) : "memory");
                gate = false;
            }
            if (!__any_sync(0xffffffffu, live)) break;
            bool ready = false;
            if (live && !(gate && j >= early)) {
                ready = j < NS || mbar_test_wait(&empty[c][j % NS], (uint32_t)((j / NS) - 1) & 1u);
                // A consumer that gave up reports the error; stop serving it.
                if (!ready && (*reinterpret_cast<volatile int *>(&s_abort[c]) || ++idle > kWaitLimit)) live = false;
            }
            if (ready) {
                idle = 0;
                const int s = j % NS;
                const int nu = cur.count(UPI, p.nunits);
                const int u0 = cur.pu;
                uint8_t *dst = ring + (size_t)s * kSlot;
                if (!(p.test_unarmed && blockIdx.x == 0 && c == 0 && j == 0)) {
                    if (Fmt<DT>::kBlockScales) {
                        const int b0 = 2 * u0, nblk = min(2 * nu, p.nb - b0);
                        const uint32_t cb = (uint32_t)nblk * Fmt<DT>::kBlockCode, sb = (uint32_t)nblk * 128u;
                        mbar_expect_tx(&full[c][s], cb + sb);
                        bulk_g2s(dst, p.codes + ((size_t)cur.tile * p.nb + b0) * Fmt<DT>::kBlockCode, cb,
                                 &full[c][s]);
                        bulk_g2s(dst + UPI * unit_code<DT>(), p.scales + ((size_t)cur.tile * p.nb + b0) * 32, sb,
                                 &full[c][s]);
                    } else {
                        const uint32_t cb = (uint32_t)nu * unit_code<DT>();
                        mbar_expect_tx(&full[c][s], cb);
                        bulk_g2s(dst, p.codes + ((size_t)cur.tile * p.nunits + u0) * unit_code<DT>(), cb,
                                 &full[c][s]);
                    }
                    issued = j + 1;
                }
                cur.advance(nu, p.nunits);
                ++j;
                if (!cur.more()) live = false;
            }
            if (!__any_sync(0xffffffffu, ready)) __nanosleep(32);
        }
        if (gate) asm volatile("bar.sync 2, %0;" ::"r"((NC + 1) * 32) : "memory");
        // Copies still in flight land before the CTA exits: wait for the
        // last NS issued items' slots (their consumer may have left).
        if (c < NC) {
            for (int q = max(0, issued - NS); q < issued; ++q) {
                if (p.test_unarmed && blockIdx.x == 0 && c == 0 && q == 0) continue;
                for (unsigned i = 0; i < kWaitLimit; ++i)
                    if (mbar_try_wait(&full[c][q % NS], (uint32_t)(q / NS) & 1u)) break;
            }
        }
    } else {
        // ------------------------------------------------------ consumers --
        const int gw = blockIdx.x * NC + warp;
        const long long ua = range_begin(gw, U, W), ub = range_begin(gw + 1, U, W);
        const int tig = lane & 3;
        pdl_wait();
        prepare_x<DT, NC>(p, xi);
        consumers_sync(NC * 32);
        const bool nonfinite = s_nonfinite != 0;
        const float pe = *xi.pexp;
        const LaneOff lo = lane_offsets<DT>(lane);
        const bool odd_nb = (p.nb & 1) != 0;

        Cursor cur;
        cur.start(ua, ub, p.nunits);
        int cur_tile = -1;
        float row_scale = 0.0f;
        bool cur_whole = false;
        Acc acc;
        acc.reset();
        for (int j = 0; cur.more(); ++j) {
            const int s = j % NS;
            const uint32_t ph = (uint32_t)(j / NS) & 1u;
            const unsigned limit = (j == 0 && p.test_unarmed && blockIdx.x == 0 && warp == 0) ? p.wait_limit
                                                                                              : kWaitLimit;
            bool ok = false;
            for (unsigned i = 0; i < limit; ++i)
                if (mbar_try_wait(&full[warp][s], ph)) {
                    ok = true;
                    break;
                }
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) {
                    atomicOr(p.err, 1);
                    s_abort[warp] = 1;
                }
                __syncwarp();
                cur_tile = -1;     // nothing is stored for an unfinished tile
                break;
            }
            const int u0 = cur.pu;
            const int nu = cur.count(UPI, p.nunits);
            const int tile = cur.tile;
            const bool full_item = nu == UPI;
            Item<DT, UPI> R;
            const uint8_t *slot = rings + ((size_t)warp * NS + s) * kSlot;
            const bool last_half = odd_nb && u0 + nu == p.nunits;
            if (full_item) R.template load<true>(slot, nu, lane, last_half);
            else R.template load<false>(slot, nu, lane, last_half);
            mbar_arrive(&empty[warp][s]);

            if (tile != cur_tile) {
                if (cur_tile >= 0) {
                    unsigned long long v[4] = {0, 0, 0, 0};
                    tile_rows<DT>(acc, v, pe);
                    flush_tile<DT>(p, xi, cur_tile, lane, gw, cur_whole, v, nonfinite, row_scale);
                }
                cur_tile = tile;
                acc.reset();
                cur_whole = u0 == 0 && (long long)tile * p.nunits + p.nunits <= ub;
                if (DT == DTYPE_TQ2_0) row_scale = __ldg(p.scales + (size_t)tile * 32 + lane);
            }
            if (full_item) compute<true, UPI>(R, nu, u0, xi, lo, tig, acc);
            else compute<false, UPI>(R, nu, u0, xi, lo, tig, acc);
            cur.advance(nu, p.nunits);
        }
        if (cur_tile >= 0) {
            unsigned long long v[4] = {0, 0, 0, 0};
            tile_rows<DT>(acc, v, pe);
            flush_tile<DT>(p, xi, cur_tile, lane, gw, cur_whole, v, nonfinite, row_scale);
        }
        if (p.ll_n && p.ll_self)
            gather_rows(p, range_begin(gw, p.rows_full, W), range_begin(gw + 1, p.rows_full, W), lane, &s_expired);
    }
    __syncthreads();
}

// ----------------------------------------------------------------- host ---
struct StreamCfg {
    int nc, ns, upi;
};

size_t stream_smem(tensor_dtype_t dt, int nb, StreamCfg c) {
    int slot = 0;
    switch (dt) {
        case DTYPE_Q8_0: slot = c.upi * (unit_code<DTYPE_Q8_0>() + unit_scale<DTYPE_Q8_0>()); break;
        case DTYPE_Q4_0: slot = c.upi * (unit_code<DTYPE_Q4_0>() + unit_scale<DTYPE_Q4_0>()); break;
        case DTYPE_TQ2_0: slot = c.upi * unit_code<DTYPE_TQ2_0>(); break;
        default: return 0;
    }
    return (size_t)c.nc * c.ns * slot + ximg_bytes(nb, dt == DTYPE_Q4_0);
}
// Configurations instantiated per format: (consumer warps, slots, units per
// item).  SAPPHIRE_STREAM_CFG = an index selects one (tuning runs);
// otherwise the first whose rings and x image fit shared memory.  Work is
// balanced to a unit whatever the item size, so the order is by measured
// speed.  Consumer counts of 7, 11 and 15 make 8, 12 and 16 warps with the
// producer: a whole number of warps per SM sub-partition, so no
// sub-partition's register file caps the others' registers per thread.
constexpr StreamCfg kQ8Cfgs[] = {{11, 3, 2}, {15, 2, 2}, {11, 2, 3}, {7, 4, 2}, {11, 2, 4}};
constexpr StreamCfg kQ4Cfgs[] = {{11, 2, 5}, {15, 2, 5}, {11, 3, 4}, {15, 2, 4}, {11, 2, 8}};
constexpr StreamCfg kTq2Cfgs[] = {{15, 2, 10}, {11, 3, 10}, {15, 3, 6}, {15, 4, 5}, {15, 2, 8}};

// Dynamic shared memory a configuration may use (the static barriers and
// reduction arrays take the rest of the 227 KB per block).
constexpr size_t kStreamSmemMax = 225 * 1024;

// {0, 0, 0} when no configuration fits (rows too long for the x image).
template <size_t N>
StreamCfg pick(const StreamCfg (&cfgs)[N], const DevWeight &w, int env) {
    if (env >= 0 && env < (int)N && stream_smem(w.dtype, w.nb, cfgs[env]) <= kStreamSmemMax) return cfgs[env];
    for (size_t i = 0; i < N; ++i)
        if (stream_smem(w.dtype, w.nb, cfgs[i]) <= kStreamSmemMax) return cfgs[i];
    return StreamCfg{0, 0, 0};
}

StreamCfg stream_cfg(const DevWeight &w) {
    static const int env = [] {
        const char *v = getenv("SAPPHIRE_STREAM_CFG");
        return v ? atoi(v) : -1;
    }();
    switch (w.dtype) {
        case DTYPE_Q8_0: return pick(kQ8Cfgs, w, env);
        case DTYPE_Q4_0: return pick(kQ4Cfgs, w, env);
        default: return pick(kTq2Cfgs, w, env);
    }
}

template <typename K>
cudaError_t smem_optin(K kernel, int device, size_t smem) {
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

template <tensor_dtype_t DT, int NC, int NS, int UPI>
int run_cfg(kernel_context_t *ctx, const StreamParams &p, int grid, size_t smem, cudaStream_t st) {
    auto kernel = gemv_stream<DT, NC, NS, UPI>;
    cudaError_t e = smem_optin(kernel, ctx->device, smem);
    if (e != cudaSuccess) {
        ctx_fail(ctx, "launch_gemv_stream", "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        return -1;
    }
    e = launch_pdl(kernel, dim3(grid), dim3((NC + 1) * 32), smem, st, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        ctx_fail(ctx, "launch_gemv_stream", "launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

#define SAPPHIRE_STREAM_TRY(DT, NC, NS, UPI) \
    if (c.nc == NC && c.ns == NS && c.upi == UPI) return run_cfg<DT, NC, NS, UPI>(ctx, p, grid, smem, st);

int dispatch(kernel_context_t *ctx, tensor_dtype_t dt, StreamCfg c, const StreamParams &p, int grid, size_t smem,
             cudaStream_t st) {
    if (dt == DTYPE_Q8_0) {
        SAPPHIRE_STREAM_TRY(DTYPE_Q8_0, 11, 3, 2)
        SAPPHIRE_STREAM_TRY(DTYPE_Q8_0, 15, 2, 2)
        SAPPHIRE_STREAM_TRY(DTYPE_Q8_0, 11, 2, 3)
        SAPPHIRE_STREAM_TRY(DTYPE_Q8_0, 7, 4, 2)
        SAPPHIRE_STREAM_TRY(DTYPE_Q8_0, 11, 2, 4)
    } else if (dt == DTYPE_Q4_0) {
        SAPPHIRE_STREAM_TRY(DTYPE_Q4_0, 11, 2, 5)
        SAPPHIRE_STREAM_TRY(DTYPE_Q4_0, 15, 2, 5)
        SAPPHIRE_STREAM_TRY(DTYPE_Q4_0, 11, 3, 4)
        SAPPHIRE_STREAM_TRY(DTYPE_Q4_0, 15, 2, 4)
        SAPPHIRE_STREAM_TRY(DTYPE_Q4_0, 11, 2, 8)
    } else if (dt == DTYPE_TQ2_0) {
        SAPPHIRE_STREAM_TRY(DTYPE_TQ2_0, 15, 2, 10)
        SAPPHIRE_STREAM_TRY(DTYPE_TQ2_0, 11, 3, 10)
        SAPPHIRE_STREAM_TRY(DTYPE_TQ2_0, 15, 3, 6)
        SAPPHIRE_STREAM_TRY(DTYPE_TQ2_0, 15, 4, 5)
        SAPPHIRE_STREAM_TRY(DTYPE_TQ2_0, 15, 2, 8)
    }
    ctx_fail(ctx, "launch_gemv_stream", "no kernel instantiated for this configuration");
    return -1;
}
#undef SAPPHIRE_STREAM_TRY

// Largest number of warps that can share one tile: ranges hold at least
// floor(U/W) units each, so a tile's n consecutive units meet at most
// ceil((n-1)/L) + 1 of them; with fewer units than warps every range holds
// at most one unit.
int stream_kmax(long long U, long long W, int n) {
    if (U <= 0) return 1;
    if (U < W) return n;
    const long long L = U / W;
    const long long k = (n - 1 + L - 1) / L + 1;
    return (int)(k < n ? k : n);
}

// Items per consumer issued before the consumers' x loads (SAPPHIRE_STREAM_EARLY
// overrides the default of 1 for tuning runs).
int stream_early() {
    static const int v = [] {
        const char *e = getenv("SAPPHIRE_STREAM_EARLY");
        return e ? atoi(e) : 1;
    }();
    return v;
}

struct Geometry {
    StreamCfg c;
    int nunits, grid;
    long long units;
};

Geometry geometry(kernel_context_t *ctx, const DevWeight &w) {
    Geometry g;
    const int sms = sm_count(ctx->device);
    g.c = stream_cfg(w);
    g.nunits = (w.nb + 1) / 2;
    g.units = (long long)w.ntiles * g.nunits;
    if (g.c.nc == 0) {
        g.grid = 0;
        return g;
    }
    // One CTA per SM, or fewer when the weight has fewer items of UPI units
    // than a full grid has consumer warps: every warp gets work.
    const long long items = (long long)w.ntiles * ((g.nunits + g.c.upi - 1) / g.c.upi);
    const long long want = (items + g.c.nc - 1) / g.c.nc;
    g.grid = (int)std::min<long long>(sms, std::max<long long>(1, want));
    return g;
}

// Tags of the split-tile partial words: one per launch, process-wide (a
// partial buffer may be shared by contexts), never 0 so zeroed memory never
// reads as valid.
std::atomic<unsigned> g_epoch{0};
unsigned next_epoch() {
    unsigned e;
    do {
        e = g_epoch.fetch_add(1) + 1;
    } while (e == 0);
    return e;
}

// Test hook (sapphire_test_stream_unarmed): 1 = the next launches leave consumer
// 0 of CTA 0 without its first copy, with a short wait limit.
std::atomic<int> g_test_unarmed{0};

}  // namespace

bool stream_dtype(tensor_dtype_t dt) { return dt == DTYPE_Q8_0 || dt == DTYPE_Q4_0 || dt == DTYPE_TQ2_0; }

bool stream_supported(kernel_context_t *ctx, const DevWeight &w) {
    if (!stream_dtype(w.dtype) || w.nb <= 0) return false;
    // TQ2_0 plane sums: 64 * 2 * 128 per element over half the blocks of a
    // row stay below 2^31 for up to 8192 blocks.
    if (w.dtype == DTYPE_TQ2_0 && w.nb > 8192) return false;
    return geometry(ctx, w).c.nc > 0;
}

// Scratch in float units: epoch-tagged partial words [ntiles][kmax][32] (two
// floats per word; two words per row for TQ2_0).  No counters.
void stream_scratch_size(kernel_context_t *ctx, const DevWeight &w, size_t *part_floats, size_t *cnt_ints) {
    const Geometry g = geometry(ctx, w);
    const long long W = (long long)g.grid * g.c.nc;
    *part_floats = (size_t)w.ntiles * stream_kmax(g.units, W, g.nunits) * 32 * (w.dtype == DTYPE_TQ2_0 ? 4 : 2);
    *cnt_ints = 0;
}

int launch_gemv_stream(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, float *part, int *,
                       int *err, const GatherArgs *ga, cudaStream_t st) {
    if (w.ntiles == 0) return 0;
    const int ll_n = ga ? ga->n : 0;
    if (ll_n < 0 || ll_n > kMaxPeers) {
        ctx_fail(ctx, "launch_gemv_stream", "%d gather targets (at most %d)", ll_n, kMaxPeers);
        return -1;
    }
    const Geometry g = geometry(ctx, w);
    if (g.c.nc == 0) {
        ctx_fail(ctx, "launch_gemv_stream", "%s weight with %d columns exceeds the kernel's shared-memory budget",
                 dtype_name(w.dtype), w.cols);
        return -1;
    }
    StreamParams p{};
    p.codes = reinterpret_cast<const uint8_t *>(w.codes);
    p.scales = w.scales;
    p.x = x;
    p.y = y;
    p.part = reinterpret_cast<unsigned long long *>(part);
    p.err = err;
    p.epoch = next_epoch();
    p.nrows = w.nrows;
    p.cols = w.cols;
    p.nb = w.nb;
    p.nunits = g.nunits;
    p.ntiles = w.ntiles;
    p.total_units = g.units;
    p.total_warps = g.grid * g.c.nc;
    p.kmax = stream_kmax(g.units, p.total_warps, g.nunits);
    p.early = stream_early();
    p.test_unarmed = g_test_unarmed.load() ? 1 : 0;
    p.wait_limit = p.test_unarmed ? (1u << 12) : kWaitLimit;
    p.ll_n = ll_n;
    p.ll_off = ga ? ga->row_off : 0;
    p.ll_epoch = ga ? ga->epoch : 0u;
    for (int k = 0; k < kMaxPeers; ++k) p.ll[k] = k < ll_n ? ga->targets[k] : nullptr;
    p.ll_self = ga ? ga->self : nullptr;
    p.y_full = ga ? ga->y_full : nullptr;
    p.rows_full = ga ? ga->rows_full : 0;
    p.ll_wait_ns = ga ? ga->wait_ns : 0;
    const size_t smem = stream_smem(w.dtype, w.nb, g.c);
    return dispatch(ctx, w.dtype, g.c, p, g.grid, smem, st);
}

// Test-only: makes the following quantized batch-1 GEMV launches leave one
// consumer warp without its first copy (an mbarrier nothing arms) and give it
// a short wait limit, so the bounded wait runs out and the error path runs.
// No GPU fault is involved.  on = 0 restores normal launches.
extern "C" SAPPHIRE_API int sapphire_test_stream_unarmed(int on) {
    g_test_unarmed.store(on ? 1 : 0);
    return 0;
}
