// gemm_tc.cu - batched prefill product on the 5th-generation tensor cores
// (tcgen05, sm_100a):  Y[t * ldy + r] = sum_k W[r, k] * X[t * ldx + k]  for a
// Q4_0 weight W and many activation rows (tokens) X.
//
// The reference has no working quantized batched product: kernel_gemm with a
// Q4_0 weight returns -1 (src/kernels/pool.c:318-321), so its prefill runs
// the row kernel once per token.  This kernel computes the same products in
// one pass: each weight is dequantised exactly as the row kernel does it,
// (q - 8) * scale in fp32 (src/kernels/q4_0_avx.c:40-41), and the activations
// are rounded to bf16, the activation type of the tensor-core prefill path.
//
// Numerics.  The tensor cores multiply bf16 x bf16 exactly and accumulate in
// fp32.  A dequantised weight w (fp32) is split into w_hi = bf16(w) and
// w_lo = bf16(w - w_hi), |w - w_hi - w_lo| <= 2^-17 |w|, and every K step
// issues two MMAs (A = w_hi, A = w_lo) against the same activation tile.  The
// result therefore matches the fp32 row kernel run on the bf16-rounded
// activations to fp32 accumulation error, instead of the 2^-9 relative error
// of a single bf16 copy of the weights.
//
// Kernel: persistent, one CTA per SM, 320 threads.
//   tile       128 weight rows (M) x 256 tokens (N); K in stages of 64
//   warps 0-3  epilogue: TMEM -> registers -> Y (fp32); warp q reads TMEM
//              lanes 32q..32q+31, i.e. weight rows 32q + lane of the tile
//   warp 4     copy producer: activation tile [256 tokens][64 k] bf16 with
//              the 128-byte swizzle (tensor TMA), plus the stage's raw Q4_0
//              codes and scales (bulk copies), into this CTA's shared memory
//   warp 5     allocates TMEM (2 x 256 fp32 columns) and issues tcgen05.mma
//   warps 6-9  dequantise the raw weight bytes (device layout, repack.cu:
//              lane (g, tig) holds elements 8tig..8tig+7 of rows g + 8i) into
//              shared memory, K-major with the 128-byte swizzle, hi and lo
// Shared memory: 3 stages x (32 KB activations + 2 x 16 KB weights + 5 KB
// raw Q4_0).  Two TMEM accumulators let the epilogue of one tile overlap the
// next tile's MMAs.
//
// Synchronisation (mbarriers): xfull[s] (TMA bytes), afull[s] (4 dequant
// warps), empty[s] (tcgen05.commit after the stage's MMAs), tfull[b] (commit
// after a tile's last MMA), tempty[b] (4 epilogue warps).  Every wait is
// bounded by time; one that expires sets bit 1 of *err and an abort flag that
// ends the other roles' loops, each role then waits (bounded again) for its
// own asynchronous work in flight, and the CTA frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <mutex>

#include "internal.cuh"

namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 3;
constexpr int kThreads = 320;
constexpr int kWarpTma = 4, kWarpMma = 5, kWarpDeq0 = 6, kDeqWarps = 4, kEpiWarps = 4;
constexpr uint32_t kXBytes = kBN * kBK * 2;             // 32 KB
constexpr uint32_t kABytes = kBM * kBK * 2;             // 16 KB per half
constexpr uint32_t kStageBytes = kXBytes + 2 * kABytes; // 64 KB
// Raw Q4_0 bytes of one stage, copied by the TMA warp: for each of the four
// 32-row groups, two blocks of codes (2 x 512 B) and of scales (2 x 128 B).
constexpr uint32_t kRawCodeBytes = 4 * 1024, kRawScaleBytes = 4 * 256;
constexpr uint32_t kRawBytes = kRawCodeBytes + kRawScaleBytes;
constexpr uint32_t kTmemCols = 2 * kBN;
constexpr int kBarriers = 3 * kStages + 2 + 2 + 1;
constexpr size_t kSmemBytes = (size_t)kStages * (kStageBytes + kRawBytes) + 256 + 1024;  // + barriers + slack
constexpr unsigned long long kWaitNs = 2000000000ull;   // 2 s per wait

// Instruction descriptor: bf16 x bf16 -> fp32, A and B K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4)            // D format f32
                          | (1u << 7)            // A format bf16
                          | (1u << 10)           // B format bf16
                          | ((uint32_t)(kBN >> 3) << 17)
                          | ((uint32_t)(kBM >> 4) << 24);
// The same with N = 128, for the half-width tiles of the last wave.
constexpr uint32_t kIdescHalf = (kIdesc & ~(0x3Fu << 17)) | ((uint32_t)((kBN / 2) >> 3) << 17);

struct GemmParams {
    const uint4 *codes;   // device layout of the Q4_0 weight
    const float *scales;
    float *y;
    int *err;
    int nrows, nb, ntiles32, batch, ldy, mtiles, total_tiles, kstages;
    // Tiles [0, full_tiles) are 128 x 256; the rest are the 128 x 128 halves
    // of full tiles full_tiles, full_tiles + 1, ... (the last wave, split so
    // that twice as many SMs share it).
    int full_tiles;
};

struct TileGeom {
    int m, n0, width;   // 128-row group, first token, tokens
};
__device__ __forceinline__ TileGeom tile_geom(const GemmParams &p, int tile) {
    if (tile < p.full_tiles) return {tile % p.mtiles, (tile / p.mtiles) * kBN, kBN};
    const int h = tile - p.full_tiles, f = p.full_tiles + (h >> 1);
    return {f % p.mtiles, (f / p.mtiles) * kBN + (h & 1) * (kBN / 2), kBN / 2};
}

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ uint32_t saddr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase of `bar` with the given parity; false after kWaitNs or,
// when abort_flag is given, once another role has set it.
__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    for (int i = 0; i < 64; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort_flag && *abort_flag) return false;
        if (globaltimer() - t0 > kWaitNs) return false;
    }
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            saddr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(saddr(bar))
        : "memory");
}
// Bulk global -> shared copy into this CTA (16-byte aligned, multiple of 16 bytes).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     saddr(dst)),
                 "l"(src), "r"(bytes), "r"(saddr(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand with the 128-byte
// swizzle: rows of 64 bf16 (128 B), 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;                 // leading byte offset (unused when swizzled)
    d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;                 // descriptor version of sm_100
    d |= (uint64_t)2 << 61;                 // 128-byte swizzle
    return d;
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------ dequantise --
// Eight weights (one code word: bytes -> elements 2m (low nibble), 2m+1 (high
// nibble)) times the row's block scale, split into bf16 hi / lo and stored as
// one 16-byte chunk of each half.
__device__ __forceinline__ void dequant8(uint32_t word, float s, uint8_t *hi_dst, uint8_t *lo_dst) {
    const uint32_t lo_n = word & 0x0F0F0F0Fu, hi_n = (word >> 4) & 0x0F0F0F0Fu;
    uint32_t h[4], l[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        // 0x4B0000nn is the float 2^23 + n; subtracting 2^23 + 8 leaves n - 8 exactly.
        const float f0 = __int_as_float((int)__byte_perm(lo_n, 0x4B000000u, 0x7440u | m));
        const float f1 = __int_as_float((int)__byte_perm(hi_n, 0x4B000000u, 0x7440u | m));
        const float w0 = __fmul_rn(__fsub_rn(f0, 8388616.0f), s);
        const float w1 = __fmul_rn(__fsub_rn(f1, 8388616.0f), s);
        const __nv_bfloat162 hp = __floats2bfloat162_rn(w0, w1);
        const uint32_t hb = *reinterpret_cast<const uint32_t *>(&hp);
        const float r0 = __fsub_rn(w0, __uint_as_float(hb << 16));
        const float r1 = __fsub_rn(w1, __uint_as_float(hb & 0xFFFF0000u));
        const __nv_bfloat162 lp = __floats2bfloat162_rn(r0, r1);
        h[m] = hb;
        l[m] = *reinterpret_cast<const uint32_t *>(&lp);
    }
    *reinterpret_cast<uint4 *>(hi_dst) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4 *>(lo_dst) = make_uint4(l[0], l[1], l[2], l[3]);
}

// ---------------------------------------------------------------- kernel --
__global__ void __launch_bounds__(kThreads, 1)
    gemm_q4_0_tc(const __grid_constant__ CUtensorMap xmap, const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)kStages * (kStageBytes + kRawBytes));
    uint64_t *xfull = bars, *afull = bars + kStages, *empty = bars + 2 * kStages;
    uint64_t *tfull = bars + 3 * kStages, *tempty = tfull + 2, *mdone = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + kBarriers);
    __shared__ int s_abort;
    volatile int *abort_flag = &s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto stage_x = [&](int s) { return smem + (size_t)s * kStageBytes; };
    auto stage_hi = [&](int s) { return smem + (size_t)s * kStageBytes + kXBytes; };
    auto stage_lo = [&](int s) { return smem + (size_t)s * kStageBytes + kXBytes + kABytes; };
    auto stage_raw = [&](int s) { return smem + (size_t)kStages * kStageBytes + (size_t)s * kRawBytes; };
    auto fail = [&]() {
        *abort_flag = 1;
        atomicOr(p.err, 2);
    };

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(xfull + s, 1);
            mbar_init(afull + s, kDeqWarps);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull + b, 1);
            mbar_init(tempty + b, kEpiWarps);
        }
        mbar_init(mdone, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kWarpTma) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            long long kc = 0;
            for (int tile = blockIdx.x; tile < p.total_tiles && !*abort_flag; tile += gridDim.x) {
                // A half-width tile still loads the full 256-token box (its
                // MMAs read the first 128 rows).
                const TileGeom tg = tile_geom(p, tile);
                const int n0 = tg.n0;
                const int t32_0 = tg.m * 4;
                const int ngroups = min(4, p.ntiles32 - t32_0);
                for (int ks = 0; ks < p.kstages; ++ks, ++kc) {
                    const int s = (int)(kc % kStages);
                    const uint32_t ph = (uint32_t)(kc / kStages) & 1u;
                    if (!wait_bounded(empty + s, ph ^ 1u, abort_flag)) {
                        fail();
                        break;
                    }
                    // Blocks 2ks, 2ks+1 of each 32-row group: codes and scales
                    // of consecutive blocks are contiguous in the device layout.
                    const int nblk = min(2, p.nb - 2 * ks);
                    mbar_expect_tx(xfull + s, kXBytes + (uint32_t)(ngroups * nblk * (512 + 128)));
                    tma_load_2d(stage_x(s), &xmap, ks * kBK, n0, xfull + s);
                    uint8_t *raw = stage_raw(s);
                    for (int d = 0; d < ngroups; ++d) {
                        const size_t u = (size_t)(t32_0 + d) * p.nb + 2 * ks;
                        bulk_g2s(raw + d * 1024, p.codes + u * 32, (uint32_t)nblk * 512u, xfull + s);
                        bulk_g2s(raw + kRawCodeBytes + d * 256, p.scales + u * 32, (uint32_t)nblk * 128u, xfull + s);
                    }
                }
            }
            // Drain: the last copy issued into each stage has landed.
            for (long long q = kc - 1; q >= 0 && q >= kc - kStages; --q)
                (void)wait_bounded(xfull + (int)(q % kStages), (uint32_t)(q / kStages) & 1u, nullptr);
        }
        __syncwarp();
    } else if (warp == kWarpMma) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            long long kc = 0;
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x, ++it) {
                const int b = it & 1;
                if (!wait_bounded(tempty + b, ((uint32_t)(it >> 1) & 1u) ^ 1u, abort_flag)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(b * kBN);
                const uint32_t idesc = tile_geom(p, tile).width == kBN ? kIdesc : kIdescHalf;
                for (int ks = 0; ks < p.kstages; ++ks, ++kc) {
                    const int s = (int)(kc % kStages);
                    const uint32_t ph = (uint32_t)(kc / kStages) & 1u;
                    if (!wait_bounded(xfull + s, ph, abort_flag) || !wait_bounded(afull + s, ph, abort_flag)) {
                        fail();
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xa = saddr(stage_x(s)), ha = saddr(stage_hi(s)), la = saddr(stage_lo(s));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint64_t bdesc = sw128_desc(xa + kk * 32);
                        umma_bf16(d_tmem, sw128_desc(ha + kk * 32), bdesc, idesc, (ks | kk) != 0);
                        umma_bf16(d_tmem, sw128_desc(la + kk * 32), bdesc, idesc, 1u);
                    }
                    umma_commit(empty + s);   // frees the stage once these MMAs have read it
                }
                if (ok) umma_commit(tfull + b);
            }
            // All MMAs issued by this thread have completed before TMEM is freed.
            umma_commit(mdone);
            (void)wait_bounded(mdone, 0u, nullptr);
        }
        __syncwarp();
    } else if (warp >= kWarpDeq0) {
        // ------------------------------------------------- dequant producers
        const int d = warp - kWarpDeq0;           // 32-row group of the 128-row tile
        const int g = lane >> 2, tig = lane & 3;
        long long kc = 0;
        for (int tile = blockIdx.x; tile < p.total_tiles && !*abort_flag; tile += gridDim.x) {
            const int t32 = tile_geom(p, tile).m * 4 + d;
            const bool tile_ok = t32 < p.ntiles32;
            bool ok = true;
            for (int ks = 0; ks < p.kstages; ++ks, ++kc) {
                const int s = (int)(kc % kStages);
                const uint32_t ph = (uint32_t)(kc / kStages) & 1u;
                // The stage's raw bytes have landed; its previous MMAs are done
                // (the TMA warp waited for that before copying).
                if (!wait_bounded(xfull + s, ph, abort_flag)) {
                    if (lane == 0) fail();
                    ok = false;
                    break;
                }
                const uint8_t *raw = stage_raw(s);
                uint8_t *hi = stage_hi(s), *lo = stage_lo(s);
#pragma unroll
                for (int jo = 0; jo < 2; ++jo) {
                    // Odd g stores its blocks in the other order, so each group
                    // of 8 lanes covers the eight 16-byte bank slots once.
                    const int j = jo ^ (g & 1);
                    uint4 c = make_uint4(0, 0, 0, 0);
                    float4 sc = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (tile_ok && 2 * ks + j < p.nb) {
                        c = *reinterpret_cast<const uint4 *>(raw + d * 1024 + j * 512 + lane * 16);
                        sc = *reinterpret_cast<const float4 *>(raw + kRawCodeBytes + d * 256 + j * 128 + g * 16);
                    }
                    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
                    const float sv[4] = {sc.x, sc.y, sc.z, sc.w};
                    const int chunk = 4 * j + tig;            // 16-byte chunk of the 128-byte row
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        // row 32d + g + 8i: 8-row group 4d + i, row g inside it
                        const uint32_t off = (uint32_t)(4 * d + i) * 1024u + (uint32_t)g * 128u +
                                             (uint32_t)((chunk ^ g) << 4);
                        dequant8(w[i], sv[i], hi + off, lo + off);
                    }
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(afull + s);
            }
            if (!ok) break;
        }
    } else {
        // -------------------------------------------------------- epilogue
        const int q = warp;                        // TMEM lanes 32q..32q+31
        int it = 0;
        for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++it) {
            const int b = it & 1;
            if (!wait_bounded(tfull + b, (uint32_t)(it >> 1) & 1u, abort_flag)) {
                if (lane == 0) fail();
                break;
            }
            tc_fence_after();
            const TileGeom tg = tile_geom(p, tile);
            const int row = tg.m * kBM + 32 * q + lane;
            const int t0 = tg.n0;
            const bool row_ok = row < p.nrows;
#pragma unroll 1
            for (int c0 = 0; c0 < tg.width; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kBN + c0), v);
                const int tmax = min(32, p.batch - (t0 + c0));
                if (row_ok) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < tmax) p.y[(size_t)(t0 + c0 + j) * p.ldy + row] = __uint_as_float(v[j]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty + b);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

// Activations fp32 [batch][ldx] -> bf16 [batch][kp] (round to nearest even),
// zero past `cols`.  One thread per 8 outputs.
__global__ void x_to_bf16(const float *__restrict__ x, int ldx, int cols, int batch, int kp,
                          uint4 *__restrict__ xb) {
    const int per_row = kp / 8;
    const size_t n = (size_t)batch * per_row;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_row);
        const int k0 = (int)(i % per_row) * 8;
        const float *row = x + (size_t)t * ldx;
        uint32_t w[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int k = k0 + 2 * m;
            const float a = k < cols ? row[k] : 0.0f;
            const float b = k + 1 < cols ? row[k + 1] : 0.0f;
            const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
            w[m] = *reinterpret_cast<const uint32_t *>(&h);
        }
        xb[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

int sm_count_of(int dev) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 148;
    }
    return n;
}

}  // namespace

bool gemm_tc_supported(const DevWeight &w, int batch) {
    return w.dtype == DTYPE_Q4_0 && batch >= kGemmTcMinBatch && w.ntiles > 0;
}

int launch_gemm_tc(kernel_context_t *ctx, const DevWeight &w, const float *x, int ldx, float *y, int ldy, int batch,
                   int *err, cudaStream_t st) {
    if (batch <= 0 || w.ntiles == 0) return 0;
    const int kp = ((w.nb * 32 + kBK - 1) / kBK) * kBK;
    const size_t xb_bytes = (size_t)batch * kp * 2;
    if (ensure_scratch(ctx, &ctx->d_xb, &ctx->d_xb_cap, xb_bytes)) return -1;
    const size_t nvec = (size_t)batch * (kp / 8);
    const int cgrid = (int)std::min<size_t>((nvec + 255) / 256, (size_t)sm_count_of(ctx->device) * 8);
    x_to_bf16<<<cgrid, 256, 0, st>>>(x, ldx, w.cols, batch, kp, reinterpret_cast<uint4 *>(ctx->d_xb));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ctx_fail(ctx, "launch_gemm_tc", "activation conversion launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return launch_gemm_tc_bf16(ctx, w, ctx->d_xb, kp, y, ldy, batch, err, st);
}

int launch_gemm_tc_bf16(kernel_context_t *ctx, const DevWeight &w, const void *xb, int ldxb, float *y, int ldy,
                        int batch, int *err, cudaStream_t st) {
    if (w.dtype != DTYPE_Q4_0) {
        ctx_fail(ctx, "launch_gemm_tc", "only Q4_0 weights have a tensor-core batched path");
        return -1;
    }
    if (batch <= 0 || w.ntiles == 0) return 0;
    if (ldxb < w.nb * 32 || ldxb % 8 != 0 || (reinterpret_cast<uintptr_t>(xb) & 15) != 0) {
        ctx_fail(ctx, "launch_gemm_tc", "bf16 activations need 16-byte aligned rows of at least %d values "
                 "(row stride %d)", w.nb * 32, ldxb);
        return -1;
    }
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) {
        ctx_fail(ctx, "launch_gemm_tc", "cuTensorMapEncodeTiled is not available from the driver");
        return -1;
    }
    const int kp = ((w.nb * 32 + kBK - 1) / kBK) * kBK;
    cudaError_t e;
    CUtensorMap xmap;
    // Columns past the row (k >= ldxb, up to the last 64-wide stage) read as
    // zero; they meet zero weights.
    const cuuint64_t dims[2] = {(cuuint64_t)std::min(kp, ldxb), (cuuint64_t)batch};
    const cuuint64_t strides[1] = {(cuuint64_t)ldxb * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBN};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(xb), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        ctx_fail(ctx, "launch_gemm_tc", "cuTensorMapEncodeTiled failed (%d)", (int)r);
        return -1;
    }

    GemmParams p;
    p.codes = w.codes;
    p.scales = w.scales;
    p.y = y;
    p.err = err;
    p.nrows = w.nrows;
    p.nb = w.nb;
    p.ntiles32 = w.ntiles;
    p.batch = batch;
    p.ldy = ldy;
    p.mtiles = (w.ntiles + 3) / 4;
    const int full = p.mtiles * ((batch + kBN - 1) / kBN);
    // Several waves whose last is partial: its r tiles run as 2r half-width
    // tiles when those still fit one wave (C5: 640 tiles on 148 SMs, the last
    // 48 become 96 halves).
    const int sms_all = sm_count_of(ctx->device);
    const int rest = full > sms_all ? full % sms_all : 0;
    const bool split = rest > 0 && 2 * rest <= sms_all;
    p.full_tiles = split ? full - rest : full;
    p.total_tiles = split ? full + rest : full;
    p.kstages = kp / kBK;
    const int grid = std::min(p.total_tiles, sm_count_of(ctx->device));

    // The shared-memory opt-in is a per-device function attribute.
    static std::mutex attr_mu;
    static bool attr_set[64] = {false};
    {
        std::lock_guard<std::mutex> lk(attr_mu);
        const int dev = ctx->device;
        if (dev < 0 || dev >= 64 || !attr_set[dev]) {
            e = cudaFuncSetAttribute(gemm_q4_0_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
            if (e != cudaSuccess) {
                ctx_fail(ctx, "launch_gemm_tc", "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
                return -1;
            }
            if (dev >= 0 && dev < 64) attr_set[dev] = true;
        }
    }
    gemm_q4_0_tc<<<grid, kThreads, kSmemBytes, st>>>(xmap, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        ctx_fail(ctx, "launch_gemm_tc", "launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
