// gemv_pipe.cu - persistent, TMA-pipelined batch-1 GEMV (the decode hot path).
//
// Same products as gemv.cu (reference row kernels src/kernels/q4_0_avx.c,
// q8_0_avx.c, applied to every row by src/kernels/pool.c:106-143, plus the
// ternary and dense formats), over the same tile layout (internal.cuh).
//
// Work split.  The weight is cut into items = (32-row tile, K segment of SEG
// 16-byte chunks).  Items are numbered tile-major and every warp of a
// persistent grid (one CTA per SM) takes a contiguous, equal-size range of
// them, so all SMs stream the same number of bytes whatever the matrix shape.
//
// Memory pipeline.  Each warp owns a ring of STAGES shared-memory slots.  Lane
// 0 fills a slot with one `cp.async.bulk` of the item's codes (SEG x 512
// contiguous bytes) and one of its scales, completing on the slot's mbarrier
// (expect_tx); the warp waits on the mbarrier, decodes and accumulates from
// shared memory, and refills the slot with the item STAGES ahead.  That keeps
// STAGES items of every warp in flight while it computes.
//
// Split tiles.  A tile whose segments span several warps is finished by the
// last contributor to arrive: each contributor stores its per-row partial in
// the scratch slot of its rank among the tile's contributors, fences, and bumps
// the tile's counter; the one that sees the count complete sums the slots in
// slot order (deterministic), writes y and resets the counter to 0.
//
// Waits are bounded: a slot that does not fill within kWaitLimit polls sets
// bit 0 of *err, the warp waits (bounded again) for its copies in flight and
// returns.
#include "internal.cuh"

namespace {

constexpr int kPipeWarps = 8;
constexpr int kPipeThreads = kPipeWarps * 32;
constexpr int kStages = 4;
constexpr int kSeg = 8;                       // 16-byte chunks per item (4 KB of codes)
constexpr float kTwo23 = 8388608.0f;
constexpr unsigned kWaitLimit = 1u << 26;

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
// Bulk global -> shared copy of `bytes` (16-byte aligned, multiple of 16),
// completing on `bar`.  No multicast.
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
// Poll until the phase completes; false after kWaitLimit polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase) {
    for (unsigned i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}

__device__ __forceinline__ float byte_plus_2p23(uint32_t w, const int k) {
    return __int_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (unsigned)k));
}
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }

// --------------------------------------------------------- format traits --
// Per-format constants and the consumer step of one 16-byte chunk (the lane's
// row) against the shared-memory copy of x.
template <tensor_dtype_t DT>
struct Fmt;

template <>
struct Fmt<DTYPE_Q8_0> {
    static constexpr int kCPB = 2;            // chunks per 32-weight block
    static constexpr int kW = 16;             // weights per chunk
    static constexpr bool kBlockScale = true;
    static __device__ __forceinline__ float chunk(uint4 c, const float *xs) {
        const uint32_t w[4] = {c.x ^ 0x80808080u, c.y ^ 0x80808080u, c.z ^ 0x80808080u, c.w ^ 0x80808080u};
        const float4 *x4 = reinterpret_cast<const float4 *>(xs);
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 v = x4[i];
            a0 = fmaf(byte_plus_2p23(w[i], 0) - (kTwo23 + 128.0f), v.x, a0);
            a1 = fmaf(byte_plus_2p23(w[i], 1) - (kTwo23 + 128.0f), v.y, a1);
            a0 = fmaf(byte_plus_2p23(w[i], 2) - (kTwo23 + 128.0f), v.z, a0);
            a1 = fmaf(byte_plus_2p23(w[i], 3) - (kTwo23 + 128.0f), v.w, a1);
        }
        return a0 + a1;
    }
};

template <>
struct Fmt<DTYPE_Q4_0> {
    static constexpr int kCPB = 1;
    static constexpr int kW = 32;
    static constexpr bool kBlockScale = true;
    static __device__ __forceinline__ float chunk(uint4 c, const float *xs) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        const float4 *x4 = reinterpret_cast<const float4 *>(xs);
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = w[i] & 0x0F0F0F0Fu;
            const uint32_t hi = (w[i] >> 4) & 0x0F0F0F0Fu;
            const float4 v0 = x4[2 * i], v1 = x4[2 * i + 1];
            a0 = fmaf(byte_plus_2p23(lo, 0) - (kTwo23 + 8.0f), v0.x, a0);
            a1 = fmaf(byte_plus_2p23(hi, 0) - (kTwo23 + 8.0f), v0.y, a1);
            a0 = fmaf(byte_plus_2p23(lo, 1) - (kTwo23 + 8.0f), v0.z, a0);
            a1 = fmaf(byte_plus_2p23(hi, 1) - (kTwo23 + 8.0f), v0.w, a1);
            a0 = fmaf(byte_plus_2p23(lo, 2) - (kTwo23 + 8.0f), v1.x, a0);
            a1 = fmaf(byte_plus_2p23(hi, 2) - (kTwo23 + 8.0f), v1.y, a1);
            a0 = fmaf(byte_plus_2p23(lo, 3) - (kTwo23 + 8.0f), v1.z, a0);
            a1 = fmaf(byte_plus_2p23(hi, 3) - (kTwo23 + 8.0f), v1.w, a1);
        }
        return a0 + a1;
    }
};

template <>
struct Fmt<DTYPE_TQ2_0> {
    static constexpr int kCPB = 1;            // unused: row scale, not block scale
    static constexpr int kW = 64;
    static constexpr bool kBlockScale = false;
    // (c - 1) * 4^p decoded in place, position-wise accumulators rescaled here.
    static __device__ __forceinline__ float chunk(uint4 c, const float *xs) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        const float4 *x4 = reinterpret_cast<const float4 *>(xs);
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t bb = __byte_perm(w[i], 0x4B000000u, 0x7440u | (unsigned)k);
                const float4 v = x4[4 * i + k];
                a0 = fmaf(__int_as_float(bb & 0x4B000003u) - (kTwo23 + 1.0f), v.x, a0);
                a1 = fmaf(__int_as_float(bb & 0x4B00000Cu) - (kTwo23 + 4.0f), v.y, a1);
                a2 = fmaf(__int_as_float(bb & 0x4B000030u) - (kTwo23 + 16.0f), v.z, a2);
                a3 = fmaf(__int_as_float(bb & 0x4B0000C0u) - (kTwo23 + 64.0f), v.w, a3);
            }
        }
        return a0 + 0.25f * a1 + 0.0625f * a2 + 0.015625f * a3;
    }
};

template <>
struct Fmt<DTYPE_F32> {
    static constexpr int kCPB = 1;
    static constexpr int kW = 4;
    static constexpr bool kBlockScale = false;
    static __device__ __forceinline__ float chunk(uint4 c, const float *xs) {
        const float4 v = *reinterpret_cast<const float4 *>(xs);
        float a = __uint_as_float(c.x) * v.x;
        a = fmaf(__uint_as_float(c.y), v.y, a);
        a = fmaf(__uint_as_float(c.z), v.z, a);
        return fmaf(__uint_as_float(c.w), v.w, a);
    }
};

template <>
struct Fmt<DTYPE_BF16> {
    static constexpr int kCPB = 1;
    static constexpr int kW = 8;
    static constexpr bool kBlockScale = false;
    static __device__ __forceinline__ float chunk(uint4 c, const float *xs) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        const float4 *x4 = reinterpret_cast<const float4 *>(xs);
        const float4 v0 = x4[0], v1 = x4[1];
        float a0 = __uint_as_float(w[0] << 16) * v0.x, a1 = __uint_as_float(w[0] & 0xFFFF0000u) * v0.y;
        a0 = fmaf(__uint_as_float(w[1] << 16), v0.z, a0);
        a1 = fmaf(__uint_as_float(w[1] & 0xFFFF0000u), v0.w, a1);
        a0 = fmaf(__uint_as_float(w[2] << 16), v1.x, a0);
        a1 = fmaf(__uint_as_float(w[2] & 0xFFFF0000u), v1.y, a1);
        a0 = fmaf(__uint_as_float(w[3] << 16), v1.z, a0);
        a1 = fmaf(__uint_as_float(w[3] & 0xFFFF0000u), v1.w, a1);
        return a0 + a1;
    }
};

template <tensor_dtype_t DT>
struct Layout {
    static constexpr int kCodeBytes = kSeg * 512;
    static constexpr int kScaleBytes = Fmt<DT>::kBlockScale ? (kSeg / Fmt<DT>::kCPB) * 128 : 0;
    static constexpr int kStageBytes = kCodeBytes + kScaleBytes;   // multiple of 128
};

struct PipeParams {
    const uint4 *codes;
    const float *scales;
    const float *x;
    float *y;
    float *part;              // [ntiles][kmax][32] partial sums of split tiles
    int *cnt;                 // [ntiles] arrival counters, zero between calls
    int *err;                 // error word (host-mapped)
    long long total_items;
    int nrows, cols, nb, ntiles, kchunks, nseg, kmax, total_warps;
};

__device__ __forceinline__ long long range_begin(long long w, long long T, long long W) { return (w * T) / W; }
// Warp whose range holds item i (ranges are [begin(w), begin(w+1))).
__device__ __forceinline__ int item_owner(long long i, long long T, long long W) {
    long long w = ((i + 1) * W + T - 1) / T - 1;
    return (int)(w < W - 1 ? w : W - 1);
}

template <tensor_dtype_t DT>
__device__ __forceinline__ float finalize(const PipeParams &p, int tile, int lane, float v) {
    if (DT == DTYPE_TQ2_0) return __ldg(p.scales + (size_t)tile * 32 + lane) * v;
    return v;
}

// Write a tile's result, or hand a partial to the split-tile combine.
template <tensor_dtype_t DT>
__device__ void flush_tile(const PipeParams &p, int tile, int lane, int my_warp, bool whole, float acc) {
    const int row = tile * 32 + lane;
    if (whole) {
        if (row < p.nrows) p.y[row] = finalize<DT>(p, tile, lane, acc);
        return;
    }
    // Contributors are the distinct owners of the tile's items, in item order.
    const long long first = (long long)tile * p.nseg;
    int k = 0, slot = -1, prev = -1;
    for (int s = 0; s < p.nseg; ++s) {
        const int o = item_owner(first + s, p.total_items, p.total_warps);
        if (o != prev) {
            if (o == my_warp) slot = k;
            ++k;
            prev = o;
        }
    }
    float *base = p.part + (size_t)tile * p.kmax * 32;
    base[(size_t)slot * 32 + lane] = acc;
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(p.cnt + tile, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == k - 1) {
        __threadfence();
        float sum = 0.0f;
        for (int j = 0; j < k; ++j) sum += __ldcg(base + (size_t)j * 32 + lane);
        if (row < p.nrows) p.y[row] = finalize<DT>(p, tile, lane, sum);
        __syncwarp();
        if (lane == 0) p.cnt[tile] = 0;
    }
}

template <tensor_dtype_t DT>
__global__ void __launch_bounds__(kPipeThreads, 1) gemv_pipe(const PipeParams p) {
    using F = Fmt<DT>;
    using L = Layout<DT>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int xpad = p.kchunks * F::kW;
    float *xs = reinterpret_cast<float *>(smem);
    uint8_t *ring_all = smem + (((size_t)xpad * 4 + 127) & ~(size_t)127);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *ring = ring_all + (size_t)warp * kStages * L::kStageBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring_all + (size_t)kPipeWarps * kStages * L::kStageBytes) +
                     warp * kStages;

    const int gw = blockIdx.x * kPipeWarps + warp;
    const long long T = p.total_items, W = p.total_warps;
    const long long it0 = range_begin(gw, T, W), it1 = range_begin(gw + 1, T, W);
    const int n_items = (int)(it1 - it0);

    auto issue = [&](long long item, int stage) {
        const int tile = (int)(item / p.nseg), seg = (int)(item % p.nseg);
        const int c0 = seg * kSeg;
        const int nch = min(kSeg, p.kchunks - c0);
        uint8_t *dst = ring + (size_t)stage * L::kStageBytes;
        const uint8_t *src = reinterpret_cast<const uint8_t *>(p.codes) + ((size_t)tile * p.kchunks + c0) * 512;
        uint32_t bytes = (uint32_t)nch * 512;
        uint32_t sbytes = 0;
        const float *ssrc = nullptr;
        if (F::kBlockScale) {
            const int b0 = c0 / F::kCPB, nblk = nch / F::kCPB;
            ssrc = p.scales + ((size_t)tile * p.nb + b0) * 32;
            sbytes = (uint32_t)nblk * 128;
        }
        mbar_expect_tx(bars + stage, bytes + sbytes);
        bulk_g2s(dst, src, bytes, bars + stage);
        if (sbytes) bulk_g2s(dst + L::kCodeBytes, ssrc, sbytes, bars + stage);
    };

    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(bars + s, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (lane == 0)
        for (int j = 0; j < kStages && j < n_items; ++j) issue(it0 + j, j);

    // x (zero-padded to whole chunks) staged once per CTA, overlapping the
    // first copies.
    for (int i = threadIdx.x; i < xpad; i += blockDim.x) xs[i] = (i < p.cols) ? p.x[i] : 0.0f;
    __syncthreads();

    int cur_tile = -1;
    bool cur_whole = false;
    float acc = 0.0f;
    for (int j = 0; j < n_items; ++j) {
        const long long item = it0 + j;
        const int stage = j % kStages;
        const uint32_t phase = (uint32_t)(j / kStages) & 1u;
        if (!mbar_wait_bounded(bars + stage, phase)) {
            if (lane == 0) atomicOr(p.err, 1);
            // Drain this warp's copies still in flight (bounded), then leave.
            for (int q = j; q < n_items && q < j + kStages; ++q)
                (void)mbar_wait_bounded(bars + (q % kStages), (uint32_t)(q / kStages) & 1u);
            return;
        }
        const int tile = (int)(item / p.nseg), seg = (int)(item % p.nseg);
        if (tile != cur_tile) {
            if (cur_tile >= 0) flush_tile<DT>(p, cur_tile, lane, gw, cur_whole, acc);
            cur_tile = tile;
            acc = 0.0f;
            // whole = this warp holds every segment of the tile
            cur_whole = (seg == 0) && ((long long)tile * p.nseg + p.nseg <= it1);
        }
        const int c0 = seg * kSeg;
        const int nch = min(kSeg, p.kchunks - c0);
        const uint8_t *st = ring + (size_t)stage * L::kStageBytes;
        if (F::kBlockScale) {
            constexpr int kBlk = kSeg / F::kCPB;
            const int nblk = nch / F::kCPB;
            const float *sc = reinterpret_cast<const float *>(st + L::kCodeBytes);
#pragma unroll
            for (int b = 0; b < kBlk; ++b) {
                if (b < nblk) {
                    float part = 0.0f;
#pragma unroll
                    for (int h = 0; h < F::kCPB; ++h) {
                        const int ch = b * F::kCPB + h;
                        part += F::chunk(lds128(st + (size_t)ch * 512 + lane * 16), xs + (size_t)(c0 + ch) * F::kW);
                    }
                    acc = fmaf(sc[b * 32 + lane], part, acc);
                }
            }
        } else {
#pragma unroll
            for (int ch = 0; ch < kSeg; ++ch)
                if (ch < nch) acc += F::chunk(lds128(st + (size_t)ch * 512 + lane * 16), xs + (size_t)(c0 + ch) * F::kW);
        }
        // Refill this slot with the item kStages ahead: order this warp's
        // reads of the slot before the asynchronous write into it.
        fence_proxy_async();
        __syncwarp();
        if (lane == 0 && j + kStages < n_items) issue(item + kStages, stage);
    }
    if (cur_tile >= 0) flush_tile<DT>(p, cur_tile, lane, gw, cur_whole, acc);
}

size_t pipe_smem(tensor_dtype_t dt, int kchunks, int chunk_w) {
    size_t stage = 0;
    switch (dt) {
        case DTYPE_Q8_0: stage = Layout<DTYPE_Q8_0>::kStageBytes; break;
        case DTYPE_Q4_0: stage = Layout<DTYPE_Q4_0>::kStageBytes; break;
        case DTYPE_TQ2_0: stage = Layout<DTYPE_TQ2_0>::kStageBytes; break;
        case DTYPE_F32: stage = Layout<DTYPE_F32>::kStageBytes; break;
        case DTYPE_BF16: stage = Layout<DTYPE_BF16>::kStageBytes; break;
        default: return 0;
    }
    const size_t xbytes = ((size_t)kchunks * chunk_w * 4 + 127) & ~(size_t)127;
    return xbytes + (size_t)kPipeWarps * kStages * stage + (size_t)kPipeWarps * kStages * 8;
}

int sm_count(int dev) {
    static int cached[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace

// Largest number of warps that can share one tile: ranges have at least
// floor(T/W) items each, so n = nseg consecutive items meet at most
// ceil((n-1)/L) + 1 of them; with fewer items than warps every range holds at
// most one item.
int pipe_kmax(long long T, long long W, int nseg) {
    if (T <= 0) return 1;
    if (T < W) return nseg;
    const long long L = T / W;
    const long long k = (nseg - 1 + L - 1) / L + 1;
    return (int)(k < nseg ? k : nseg);
}

bool pipe_supported(const DevWeight &w) {
    if (w.dtype != DTYPE_Q8_0 && w.dtype != DTYPE_Q4_0 && w.dtype != DTYPE_TQ2_0 && w.dtype != DTYPE_F32 &&
        w.dtype != DTYPE_BF16)
        return false;
    return pipe_smem(w.dtype, w.kchunks, chunk_weights(w.dtype)) <= 227 * 1024;
}

// Batch-1 product y[r] = W[r,:] . x with the pipelined kernel.  part / cnt:
// scratch of at least ntiles*kmax*32 floats and ntiles zeroed ints (see
// pipe_scratch_floats); err: device-visible error word.
int launch_gemv_pipe(kernel_context_t *ctx, const DevWeight &w, const float *x, float *y, float *part, int *cnt,
                     int *err, cudaStream_t st) {
    if (w.ntiles == 0) return 0;
    PipeParams p;
    p.codes = w.codes;
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
    p.nseg = (w.kchunks + kSeg - 1) / kSeg;
    p.total_items = (long long)w.ntiles * p.nseg;
    const int grid = sm_count(ctx->device);
    p.total_warps = grid * kPipeWarps;
    p.kmax = pipe_kmax(p.total_items, p.total_warps, p.nseg);
    const size_t smem = pipe_smem(w.dtype, w.kchunks, chunk_weights(w.dtype));
    auto launch = [&](auto kernel) -> int {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "launch_gemv_pipe", "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return -1;
        }
        kernel<<<grid, kPipeThreads, smem, st>>>(p);
        e = cudaGetLastError();
        if (e != cudaSuccess) {
            ctx_fail(ctx, "launch_gemv_pipe", "launch failed: %s", cudaGetErrorString(e));
            return -1;
        }
        return 0;
    };
    switch (w.dtype) {
        case DTYPE_Q8_0: return launch(gemv_pipe<DTYPE_Q8_0>);
        case DTYPE_Q4_0: return launch(gemv_pipe<DTYPE_Q4_0>);
        case DTYPE_TQ2_0: return launch(gemv_pipe<DTYPE_TQ2_0>);
        case DTYPE_F32: return launch(gemv_pipe<DTYPE_F32>);
        case DTYPE_BF16: return launch(gemv_pipe<DTYPE_BF16>);
        default:
            ctx_fail(ctx, "launch_gemv_pipe", "unsupported dtype");
            return -1;
    }
}

// Scratch the pipelined kernel needs for a weight on this device.
void pipe_scratch_size(kernel_context_t *ctx, const DevWeight &w, size_t *part_floats, size_t *cnt_ints) {
    const int nseg = (w.kchunks + kSeg - 1) / kSeg;
    const long long T = (long long)w.ntiles * nseg;
    const long long W = (long long)sm_count(ctx->device) * kPipeWarps;
    *part_floats = (size_t)w.ntiles * pipe_kmax(T, W, nseg) * 32;
    *cnt_ints = (size_t)w.ntiles;
}
