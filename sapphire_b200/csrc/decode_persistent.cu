// decode_persistent.cu - one Gemma-3 decode step as ONE persistent kernel.
//
// The step of decode.cu (the reference's inference_forward,
// src/inference/inference.c:616-651, with the layer stages of
// src/transformer/attention.c:311-375 and transformer.c:96-283) is a chain of
// small dependent products: per layer 0.2 - 1.6 MB of Q4_0 weights, each
// needing the whole output of the stage before.  Run as one kernel per stage
// it is bound by launch and drain latency (5 - 12 us per kernel for 1 - 3 us
// of memory traffic).  Here one CTA per SM runs the whole token, and a stage
// waits for exactly the data it reads: every stage output is written as
// epoch-tagged 8-byte words, and a consumer polls the words it needs until
// they carry the stage's epoch (no grid barrier, no separate flag):
//
//   per layer l:
//     QKV   every CTA: h += rmsnorm_delta(down_out, ffn_post[l-1]) (l > 0),
//           x = rmsnorm_delta(h, attn[l]); its rows of [Wq; Wk; Wv] . x
//     ATT   CTA c < nsplit: q / k rmsnorm_delta + RoPE of the token, keys
//           [k0, k0 + chunk) of the layer's window: scores, softmax partial
//           (max m, sum l, sum p v) per query head -> part[c] (m and l as
//           tagged words stored with release after the sums); the CTA whose
//           range holds pos writes the token's K / V rows
//     O     every CTA: attn = combine of the nsplit partials, its rows of Wo . attn
//     GU    every CTA: h += rmsnorm_delta(o_out, attn_post[l]),
//           x = rmsnorm_delta(h, ffn[l]); its (gate, up) row pairs . x, and
//           gelu_tanh(gate) * up of each pair
//     DOWN  every CTA: its rows of Wdown . (the GU stage's outputs)
//   then CTA 0: h += rmsnorm_delta(down_out, ffn_post[L-1]) and either the
//   final norm (the LM head's input) or the prompt-state advance.
//
// Buffers need no double buffering: every CTA has rows in every product, so
// before any CTA can write a stage's buffer again (one layer later) it must
// have consumed outputs that every CTA produced after its last read of that
// buffer.
//
// Every CTA keeps its own copy of the residual stream h in shared memory and
// updates it with the same arithmetic in the same order, so the copies stay
// identical and h never crosses CTAs.  A CTA's rows of each product are a
// contiguous range of the row layout (PersistParams::wrows), fetched into
// shared memory with one cp.async.bulk per stage a whole layer ahead (right
// after the same stage of the layer before used the buffer); the keys of a
// CTA's attention split and the norm weights are fetched the same way one
// layer ahead.  So a stage reads only its small input vector from L2.
//
// Arithmetic is fp32 and per element the same as decode.cu's kernels (and the
// reference): Q4_0 dot products as sum_b scale_b * sum_j (q_j - 8) x_j, one
// lane per 8 weights of a block, then a warp tree; sums run in a different
// order than the reference's, so results agree to rounding.
//
// Waits are bounded: a word that does not arrive within wait_ns sets
// kErrStepWait in the error word and a device abort flag, after which no
// CTA waits again (the step's results are then garbage, and the host reports
// the error); an mbarrier wait that expires sets bit 0.  All CTAs must be
// resident at once: the kernel is launched cooperatively (one CTA per SM).
#include <cmath>
#include <cstdlib>

#include "internal.cuh"
#include "decode_common.cuh"

namespace {

constexpr int kPWarps = kPersistThreads / 32;
constexpr int kDefaultChunk = 16;

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ uint32_t saddr(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(saddr(dst)),
        "l"(src), "r"(bytes), "r"(saddr(bar))
        : "memory");
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
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Every thread waits for phase `parity` of an mbarrier (bounded).
__device__ __forceinline__ void mbar_wait(uint64_t *bar, uint32_t parity, const PersistParams &p) {
    if (mbar_try_wait(bar, parity)) return;
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (gtimer() - t0 > p.wait_ns) {
            atomicOr(p.err, 1);
            return;
        }
    }
}

// ------------------------------------------------------ tagged words ----
// A stage's outputs are 8-byte words (epoch << 32 | fp32 bits): an aligned
// 8-byte store is seen whole, so a word that carries the stage's epoch holds
// its value and needs no separate flag or barrier.  Every launch has its own
// range of epochs (ctl[1], the launches so far, never repeats within 2^32
// stages), and every word a consumer waits for is rewritten in every launch.
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_word_acquire(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_word(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_word_release(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long tagged(unsigned epoch, float v) {
    return ((unsigned long long)epoch << 32) | __float_as_uint(v);
}

// Gives up the launch's waits after an expiry: sets kErrStepWait, the
// device abort flag and the CTA's own flag.
__device__ __noinline__ void give_up(const PersistParams &p, int *s_abort) {
    atomicOr(p.err, kErrStepWait);
    atomicExch(p.ctl, 1u);
    *reinterpret_cast<volatile int *>(s_abort) = 1;
}

// True while the wait begun at t0 may go on (bounded by wait_ns; false once
// this CTA or any other has given up).  The clock and the device abort flag
// are read every 16th poll only, so a poll costs one round trip.
__device__ __forceinline__ bool keep_waiting(const PersistParams &p, int *s_abort, uint64_t t0, unsigned &it) {
    if (*reinterpret_cast<volatile int *>(s_abort)) return false;
    if ((++it & 15u) == 0 && (gtimer() - t0 > p.wait_ns || *reinterpret_cast<volatile unsigned *>(p.ctl) != 0)) {
        give_up(p, s_abort);
        return false;
    }
    return true;
}

// dst[i] = value of src[i] for i < n once every word carries `epoch`.  A
// thread issues the loads of all its words (up to kFetch at a time) before
// checking any, and re-loads all of its words still pending together, so a
// wait costs one L2 round trip per poll, not one per word.  Ends with
// __syncthreads.
constexpr int kFetch = 8;
__device__ void fetch_vec(const unsigned long long *src, int n, unsigned epoch, float *dst, const PersistParams &p,
                          int *s_abort) {
    for (int base = 0; base < n; base += kFetch * kPersistThreads) {
        unsigned long long v[kFetch];
        unsigned pending = 0;
#pragma unroll
        for (int k = 0; k < kFetch; ++k) {
            const int i = base + k * kPersistThreads + threadIdx.x;
            v[k] = i < n ? ld_word(src + i) : ((unsigned long long)epoch << 32);
        }
#pragma unroll
        for (int k = 0; k < kFetch; ++k)
            if ((unsigned)(v[k] >> 32) != epoch) pending |= 1u << k;
        if (pending) {
            const uint64_t t0 = gtimer();
            unsigned it = 0;
            while (pending && keep_waiting(p, s_abort, t0, it)) {
#pragma unroll
                for (int k = 0; k < kFetch; ++k)
                    if (pending & (1u << k)) v[k] = ld_word(src + base + k * kPersistThreads + threadIdx.x);
#pragma unroll
                for (int k = 0; k < kFetch; ++k)
                    if ((unsigned)(v[k] >> 32) == epoch) pending &= ~(1u << k);
            }
        }
#pragma unroll
        for (int k = 0; k < kFetch; ++k) {
            const int i = base + k * kPersistThreads + threadIdx.x;
            if (i < n) dst[i] = __uint_as_float((unsigned)v[k]);
        }
    }
    __syncthreads();
}

// Rows [r0, r1) of stage s that CTA c computes (balanced split of the rows).
// Stage GU holds gate row i and up row i as rows 2i and 2i + 1, split by
// pairs, so a block holds both rows of each of its pairs.  (32-bit
// arithmetic: persist_plan admits rows * grid < 2^32.)
__device__ __forceinline__ void stage_rows(const PersistParams &p, int s, int &r0, int &r1) {
    const unsigned G = gridDim.x, c = blockIdx.x;
    if (s == kStGu) {
        const unsigned P = (unsigned)p.stage_rows[s] / 2;
        r0 = (int)(2 * (c * P / G));
        r1 = (int)(2 * ((c + 1) * P / G));
    } else {
        const unsigned R = (unsigned)p.stage_rows[s];
        r0 = (int)(c * R / G);
        r1 = (int)((c + 1) * R / G);
    }
}

// Attention work of CTA c at layer l: query head h = c / splits and keys
// [k0, k0 + n) of split b = c % splits (n = 0: none); the window of the
// layer (all positions for a global layer, the last `window` otherwise) is
// cut into nsplit splits of `chunk` keys.
struct Split {
    int h, b, k0, n, chunk, nsplit;
};
__device__ __forceinline__ Split split_of(const PersistParams &p, int l, int pos, int c) {
    Split sp;
    const int seq = pos + 1;
    const bool global = (p.global_mask >> l) & 1ull;
    const int start = (!global && seq > p.window) ? seq - p.window : 0;
    const int len = seq - start;
    sp.chunk = max(p.chunk, (len + p.splits - 1) / p.splits);
    sp.nsplit = (len + sp.chunk - 1) / sp.chunk;
    sp.h = c / p.splits;
    sp.b = c % p.splits;
    sp.k0 = start + sp.b * sp.chunk;
    sp.n = (sp.h < p.heads && sp.b < sp.nsplit) ? min(sp.chunk, seq - sp.k0) : 0;
    return sp;
}

// Thread 0: fetch this CTA's rows of stage s of layer l into its buffer.
__device__ void issue_stage(const PersistParams &p, int l, int s, uint8_t *smem, uint64_t *bar) {
    int r0, r1;
    stage_rows(p, s, r0, r1);
    const uint32_t bytes = (uint32_t)(r1 - r0) * (uint32_t)p.stage_stride[s];
    if (bytes == 0) {
        mbar_arrive(bar);
        return;
    }
    mbar_arrive_tx(bar, bytes);
    const uint8_t *src = p.wrows + (size_t)l * p.layer_bytes + p.stage_off[s] + (size_t)r0 * p.stage_stride[s];
    bulk_g2s(smem + p.off_w[s], src, bytes, bar);
}

// Thread 0: fetch the K and V rows of this CTA's split of layer l (of its
// head's KV head).  The row of pos itself is stale (this step writes it) and
// is replaced after the wait.
__device__ void issue_kv(const PersistParams &p, int l, int pos, uint8_t *smem, uint64_t *bar) {
    const Split sp = split_of(p, l, pos, blockIdx.x);
    if (sp.n <= 0) {
        mbar_arrive(bar);
        return;
    }
    const int kh = sp.h / (p.heads / p.kv_heads);
    const uint32_t bytes = (uint32_t)sp.n * (uint32_t)p.hd * 4u;
    mbar_arrive_tx(bar, 2u * bytes);
    const size_t off = (((size_t)l * p.kv_heads + kh) * p.context + sp.k0) * p.hd;
    bulk_g2s(smem + p.off_k, p.kcache + off, bytes, bar);
    bulk_g2s(smem + p.off_v, p.vcache + off, bytes, bar);
}

// Thread 0: fetch layer l's norm weights into buffer l & 1 (and, with `rope`,
// the RoPE rows of pos for both tables, which stay for the whole step).
__device__ void issue_norms(const PersistParams &p, int l, int pos, bool rope, uint8_t *smem, uint64_t *bar) {
    const uint32_t nbytes = (uint32_t)p.norm_stride * 4u, rbytes = (uint32_t)p.hd * 4u;
    mbar_arrive_tx(bar, nbytes + (rope ? 4u * rbytes : 0u));
    bulk_g2s(smem + p.off_nrm[l & 1], p.norms + (size_t)l * p.norm_stride, nbytes, bar);
    if (rope) {
        const size_t r = (size_t)pos * p.hd;
        bulk_g2s(smem + p.off_rope, p.rope_cos_g + r, rbytes, bar);
        bulk_g2s(smem + p.off_rope + rbytes, p.rope_sin_g + r, rbytes, bar);
        bulk_g2s(smem + p.off_rope + 2 * rbytes, p.rope_cos_l + r, rbytes, bar);
        bulk_g2s(smem + p.off_rope + 3 * rbytes, p.rope_sin_l + r, rbytes, bar);
    }
}

// hidden += rmsnorm_delta(t, w) for t the tagged output of the stage before,
// given as `nparts` partial vectors added in order (fetched through vin into
// xs).  Same per-element arithmetic as residual_norm_kernel.
__device__ void residual_add(float *hidden, const unsigned long long *t, int nparts, unsigned epoch, const float *w,
                             int n, float *xs, float *vin, float *red, const PersistParams &p, int *s_abort) {
    if (nparts == 1) {
        fetch_vec(t, n, epoch, xs, p, s_abort);
    } else {
        fetch_vec(t, nparts * n, epoch, vin, p, s_abort);
        for (int i = threadIdx.x; i < n; i += kPersistThreads) {
            float v = vin[i];
            for (int k = 1; k < nparts; ++k) v += vin[(size_t)k * n + i];
            xs[i] = v;
        }
    }
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += kPersistThreads) ss += xs[i] * xs[i];
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss / (float)n + p.eps);
    for (int i = threadIdx.x; i < n; i += kPersistThreads) hidden[i] = hidden[i] + (xs[i] * r) * (1.0f + w[i]);
}

// out = rmsnorm_delta(hidden, w), zero-padded to `padded` values.
__device__ void norm_to(const float *hidden, const float *w, int n, int padded, float eps, float *out, float *red) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += kPersistThreads) ss += hidden[i] * hidden[i];
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = threadIdx.x; i < padded; i += kPersistThreads) out[i] = i < n ? (hidden[i] * r) * (1.0f + w[i]) : 0.0f;
}

// Partial dot product of one 4-byte Q4_0 code word (8 weights) with its x values.
__device__ __forceinline__ float q4_word_dot(uint32_t code, float4 x0, float4 x1) {
    const uint32_t lo = code & 0x0F0F0F0Fu, hi = (code >> 4) & 0x0F0F0F0Fu;
    // 0x4B0000nn is the float 2^23 + n; subtracting 2^23 + 8 leaves n - 8 exactly.
#define Q4F(word, m) (__int_as_float((int)__byte_perm((word), 0x4B000000u, 0x7440u | (m))) - 8388616.0f)
    float dot = 0.0f;
    dot = fmaf(Q4F(lo, 0), x0.x, dot);
    dot = fmaf(Q4F(hi, 0), x0.y, dot);
    dot = fmaf(Q4F(lo, 1), x0.z, dot);
    dot = fmaf(Q4F(hi, 1), x0.w, dot);
    dot = fmaf(Q4F(lo, 2), x1.x, dot);
    dot = fmaf(Q4F(hi, 2), x1.y, dot);
    dot = fmaf(Q4F(lo, 3), x1.z, dot);
    dot = fmaf(Q4F(hi, 3), x1.w, dot);
#undef Q4F
    return dot;
}

// y[r] = W[r] . xs (as tagged words of `epoch`, in `replicas` copies) for
// this CTA's rows of stage s (weights in shared memory), one warp per row, two rows at a time; lane k
// of a row takes 4-byte code word k (8 weights of block k / 4) and its x
// values xs[8k .. 8k + 8).
//
// Stage GU (pairs): a warp takes rows 2j and 2j + 1 (gate and up of output j)
// and writes one word, gelu_tanh(gate) * up, to y[j] (the DOWN stage's input).
__device__ void gemv_stage(const PersistParams &p, int s, const uint8_t *w, const float *xs, unsigned long long *y,
                           unsigned epoch, int replicas, int seg = 0, int seg0 = 0) {
    int r0, r1;
    stage_rows(p, s, r0, r1);
    const int nb = p.stage_nb[s], stride = p.stage_stride[s], nwords = nb * 4, nr = r1 - r0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool pairs = s == kStGu;
    const int ny = pairs ? p.stage_rows[s] / 2 : p.stage_rows[s];   // outputs per copy
    for (int i = warp; pairs ? 2 * i < nr : i < nr; i += pairs ? kPWarps : 2 * kPWarps) {
        const int r = pairs ? 2 * i : i;
        const int r2 = pairs ? r + 1 : r + kPWarps;
        const bool two = r2 < nr;
        const uint8_t *row = w + (size_t)r * stride, *row2 = w + (size_t)(two ? r2 : r) * stride;
        const float *sc = reinterpret_cast<const float *>(row + (size_t)nb * 16);
        const float *sc2 = reinterpret_cast<const float *>(row2 + (size_t)nb * 16);
        // With seg > 0, row r' of the stage reads x segment r' / seg - seg0
        // (nb * 32 values each); otherwise every row reads xs.
        const float *x1p = seg ? xs + (size_t)((r0 + r) / seg - seg0) * nb * 32 : xs;
        const float *x2p = seg ? xs + (size_t)((r0 + (two ? r2 : r)) / seg - seg0) * nb * 32 : xs;
        float acc = 0.0f, acc2 = 0.0f;
        for (int k = lane; k < nwords; k += 32) {
            const uint32_t c1 = *reinterpret_cast<const uint32_t *>(row + 4 * k);
            const uint32_t c2 = *reinterpret_cast<const uint32_t *>(row2 + 4 * k);
            const float4 a0 = *reinterpret_cast<const float4 *>(x1p + 8 * k);
            const float4 a1 = *reinterpret_cast<const float4 *>(x1p + 8 * k + 4);
            // Rows of one x (every stage but the head-split O) share the loads.
            const float4 b0 = seg ? *reinterpret_cast<const float4 *>(x2p + 8 * k) : a0;
            const float4 b1 = seg ? *reinterpret_cast<const float4 *>(x2p + 8 * k + 4) : a1;
            acc = fmaf(sc[k >> 2], q4_word_dot(c1, a0, a1), acc);
            acc2 = fmaf(sc2[k >> 2], q4_word_dot(c2, b0, b1), acc2);
        }
        acc = warp_sum(acc);
        acc2 = warp_sum(acc2);
        // Every lane holds the sums (xor reduction): lane k writes copy k.
        if (pairs) {
            // GeGLU of the reference (src/transformer/activations.c:64-82).
            const float g = geglu_tanh(acc, acc2);
            if (lane < replicas) st_word(y + (size_t)lane * ny + (r0 + r) / 2, tagged(epoch, g));
        } else if (lane < replicas) {
            unsigned long long *yk = y + (size_t)lane * ny;
            st_word(yk + r0 + r, tagged(epoch, acc));
            if (two) st_word(yk + r0 + r2, tagged(epoch, acc2));
        }
    }
}

// rmsnorm_delta of one head (hd values at x in shared memory) then the
// half-split rotation (rope_apply_fast, src/transformer/rope.c:65-80), by one
// warp; lane owns the pairs (i, i + hd/2) for i = lane + 32 j.  The same
// arithmetic as warp_norm_rope.
__device__ void norm_rope_smem(const float *x, const float *w, float eps, const float *cs, const float *sn, int hd,
                               float *dst) {
    const int lane = threadIdx.x & 31, half = hd >> 1;
    float a[kMaxHeadDim / 64], b[kMaxHeadDim / 64];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxHeadDim / 64; ++j) {
        const int i = lane + 32 * j;
        a[j] = i < half ? x[i] : 0.0f;
        b[j] = i < half ? x[i + half] : 0.0f;
        ss += a[j] * a[j] + b[j] * b[j];
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)hd + eps);
#pragma unroll
    for (int j = 0; j < kMaxHeadDim / 64; ++j) {
        const int i = lane + 32 * j;
        if (i < half) {
            const float y0 = (a[j] * r) * (1.0f + w[i]);
            const float y1 = (b[j] * r) * (1.0f + w[i + half]);
            const float c = cs[i], sv = sn[i];
            dst[i] = y0 * c - y1 * sv;
            dst[i + half] = y1 * c + y0 * sv;
        }
    }
}

// Attention of the current token for query head h over the keys of split b
// at layer l (see the file comment); the partial result goes to
// p.part[b * heads + h]: [m, l, -, -, acc...], the m / l words last.
// nrm: the layer's norm weights in shared memory; the RoPE rows of pos are in
// shared memory too.
__device__ void attention_stage(const PersistParams &p, int l, int pos, uint8_t *smem, uint64_t *kv_bar,
                                const float *nrm, unsigned e_qkv, unsigned epoch, int *s_abort) {
    __shared__ float s_ml[2];
    const Split sp = split_of(p, l, pos, blockIdx.x);
    mbar_wait(kv_bar, (uint32_t)(l & 1), p);
    if (sp.n <= 0) return;
    const int heads = p.heads, kvh = p.kv_heads, hd = p.hd, group = heads / kvh, n = sp.n, h = sp.h;
    const int kh = h / group;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *vin = reinterpret_cast<float *>(smem + p.off_vin);
    fetch_vec(p.qkv, (heads + 2 * kvh) * hd, e_qkv, vin, p, s_abort);
    const bool global = (p.global_mask >> l) & 1ull;
    const float *rope = reinterpret_cast<const float *>(smem + p.off_rope) + (global ? 0 : 2 * hd);
    const float *wq = nrm + 4 * p.hidden, *wk = wq + hd;
    float *qs = reinterpret_cast<float *>(smem + p.off_q);
    float *kcur = reinterpret_cast<float *>(smem + p.off_kcur);
    float *vcur = reinterpret_cast<float *>(smem + p.off_vcur);
    float *K = reinterpret_cast<float *>(smem + p.off_k);
    float *V = reinterpret_cast<float *>(smem + p.off_v);
    float *sc = reinterpret_cast<float *>(smem + p.off_sc);
    float *accs = reinterpret_cast<float *>(smem + p.off_acc);

    // The token's q of head h and k of its KV head (rmsnorm_delta with
    // q_norm / k_norm, then RoPE at pos), and v.
    if (warp == 0) norm_rope_smem(vin + (size_t)h * hd, wq, p.eps, rope, rope + hd, hd, qs);
    if (warp == 1) norm_rope_smem(vin + (size_t)(heads + kh) * hd, wk, p.eps, rope, rope + hd, hd, kcur);
    for (int i = threadIdx.x; i < hd; i += kPersistThreads) vcur[i] = vin[(size_t)(heads + kvh + kh) * hd + i];
    __syncthreads();
    if (pos >= sp.k0 && pos < sp.k0 + n) {
        // This split holds the token: its K / V rows replace the stale rows
        // fetched with the split; the group's first head stores them for
        // later steps.
        const int t = pos - sp.k0;
        const bool store = h % group == 0;
        const size_t g = (((size_t)l * kvh + kh) * p.context + pos) * hd;
        for (int d = threadIdx.x; d < hd; d += kPersistThreads) {
            K[(size_t)t * hd + d] = kcur[d];
            V[(size_t)t * hd + d] = vcur[d];
            if (store) {
                p.kcache[g + d] = kcur[d];
                p.vcache[g + d] = vcur[d];
            }
        }
        // The next layer's keys are fetched into these buffers by the async
        // proxy: order these generic writes before that.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
    }
    constexpr int NJ = kMaxHeadDim / 32;
    const int nj = hd / 32;
    // Scores: one warp per key, q in registers (lane holds d = lane + 32 j).
    {
        float q[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) q[j] = j < nj ? qs[lane + 32 * j] : 0.0f;
        for (int t = warp; t < n; t += kPWarps) {
            float a = 0.0f;
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                if (j < nj) a = fmaf(q[j], K[(size_t)t * hd + lane + 32 * j], a);
            a = warp_sum(a);
            if (lane == 0) sc[t] = a * p.att_scale;
        }
    }
    __syncthreads();
    // Softmax partial: m = max score, p = exp(s - m), l = sum p.
    if (warp == 0) {
        float m = -INFINITY;
        for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[t]);
        m = warp_max(m);
        float s = 0.0f;
        for (int t = lane; t < n; t += 32) {
            const float e = expf(sc[t] - m);
            sc[t] = e;
            s += e;
        }
        s = warp_sum(s);
        if (lane == 0) {
            s_ml[0] = m;
            s_ml[1] = s;
        }
    }
    __syncthreads();
    // acc = sum_t p_t v_t: thread (part q, dimension d) sums the keys
    // t = q, q + parts, ...; then the parts are added in order.
    const int parts = kPersistThreads / hd;
    {
        const int d = threadIdx.x % hd, q = threadIdx.x / hd;
        float a = 0.0f;
        for (int t = q; t < n; t += parts) a = fmaf(sc[t], V[(size_t)t * hd + d], a);
        accs[(size_t)q * hd + d] = a;
    }
    __syncthreads();
    float *row = p.part + ((size_t)sp.b * heads + h) * (hd + 4);
    for (int d = threadIdx.x; d < hd; d += kPersistThreads) {
        float a = accs[d];
        for (int q = 1; q < parts; ++q) a += accs[(size_t)q * hd + d];
        row[4 + d] = a;
    }
    __syncthreads();
    // The m and l words last, with release: a consumer that sees both tagged
    // with this epoch also sees the acc values.
    if (threadIdx.x == 0) {
        unsigned long long *hw = reinterpret_cast<unsigned long long *>(row);
        st_word_release(hw, tagged(epoch, s_ml[0]));
        st_word_release(hw + 1, tagged(epoch, s_ml[1]));
    }
}

// attn_h = sum_b w_b acc_b with w_b = exp(m_b - M) / sum_b' exp(m_b' - M) l_b'
// (M = max_b m_b) over the splits of layer l, for the heads h0 .. h0 + nh - 1
// that this CTA's rows of the head-split O product use, into xs ([nh][hd]).
// First one warp per head waits for the (m, l) words of every split (acquire:
// the acc values behind them are then visible) and forms the weights; then
// thread (part q, quad j) sums splits b = q, q + P, ... of outputs
// 4j .. 4j + 3 with all loads of a batch in flight; the parts are added in
// order.  Returns h0.
__device__ int combine_stage(const PersistParams &p, int l, int pos, float *xs, float *scratch, float *wts,
                             unsigned epoch, int *s_abort) {
    int r0, r1;
    stage_rows(p, kStO, r0, r1);
    const int H = p.hidden, hd = p.hd, heads = p.heads, S = p.splits;
    const int h0 = r0 / H, nh = (r1 - 1) / H - h0 + 1;
    const int nsplit = split_of(p, l, pos, 0).nsplit;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t hstride = (size_t)hd + 4;
    for (int w = warp; w < nh; w += kPWarps) {
        const int h = h0 + w;
        float *wm = wts + (size_t)w * 2 * S, *wl = wm + S;
        float mx = -INFINITY;
        for (int b = lane; b < nsplit; b += 32) {
            const unsigned long long *hw =
                reinterpret_cast<const unsigned long long *>(p.part + ((size_t)b * heads + h) * hstride);
            unsigned long long m = ld_word_acquire(hw), lv = ld_word_acquire(hw + 1);
            if ((unsigned)(m >> 32) != epoch || (unsigned)(lv >> 32) != epoch) {
                const uint64_t t0 = gtimer();
                unsigned it = 0;
                while (((unsigned)(m >> 32) != epoch || (unsigned)(lv >> 32) != epoch) &&
                       keep_waiting(p, s_abort, t0, it)) {
                    m = ld_word_acquire(hw);
                    lv = ld_word_acquire(hw + 1);
                }
            }
            wm[b] = __uint_as_float((unsigned)m);
            wl[b] = __uint_as_float((unsigned)lv);
            mx = fmaxf(mx, wm[b]);
        }
        const float M = warp_max(mx);
        float L = 0.0f;
        for (int b = lane; b < nsplit; b += 32) {
            const float e = expf(wm[b] - M);
            wm[b] = e;
            L += e * wl[b];
        }
        const float inv = 1.0f / warp_sum(L);
        for (int b = lane; b < nsplit; b += 32) wm[b] *= inv;
    }
    __syncthreads();
    const int quads = nh * hd / 4;
    const int P = max(1, kPersistThreads / quads);
    constexpr int kBatch = 8;
    for (int i = threadIdx.x; i < P * quads; i += kPersistThreads) {
        const int q = i / quads, j = i % quads;
        const int w = (4 * j) / hd, d = (4 * j) % hd;
        const float *base = p.part + (size_t)(h0 + w) * hstride + 4 + d;
        const float *wm = wts + (size_t)w * 2 * S;
        float4 O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int b0 = q; b0 < nsplit; b0 += P * kBatch) {
            float4 a[kBatch];
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const int b = b0 + P * k;
                a[k] = b < nsplit ? __ldcg(reinterpret_cast<const float4 *>(base + (size_t)b * heads * hstride))
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const int b = b0 + P * k;
                const float wb = b < nsplit ? wm[b] : 0.0f;
                O.x = fmaf(wb, a[k].x, O.x);
                O.y = fmaf(wb, a[k].y, O.y);
                O.z = fmaf(wb, a[k].z, O.z);
                O.w = fmaf(wb, a[k].w, O.w);
            }
        }
        reinterpret_cast<float4 *>(scratch)[i] = O;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < quads; j += kPersistThreads) {
        float4 o = reinterpret_cast<const float4 *>(scratch)[j];
        for (int q = 1; q < P; ++q) {
            const float4 a = reinterpret_cast<const float4 *>(scratch)[(size_t)q * quads + j];
            o = make_float4(o.x + a.x, o.y + a.y, o.z + a.z, o.w + a.w);
        }
        reinterpret_cast<float4 *>(xs)[j] = o;
    }
    __syncthreads();
    return h0;
}

__global__ void __launch_bounds__(kPersistThreads, 1) decode_persistent_kernel(const __grid_constant__ PersistParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    // mbarriers: one per weight stage, the keys, the two norm buffers.
    constexpr int kBarKv = kNumStages, kBarNorm = kNumStages + 1, kNumBars = kNumStages + 3;
    __shared__ __align__(8) uint64_t mbar[kNumBars];
    __shared__ float red[32];
    __shared__ int s_abort;
    float *hidden = reinterpret_cast<float *>(smem + p.off_hidden);
    float *xs = reinterpret_cast<float *>(smem + p.off_x);
    float *scratch = reinterpret_cast<float *>(smem + p.off_acc);
    float *vin = reinterpret_cast<float *>(smem + p.off_vin);
    const int H = p.hidden;
    // This CTA's copies of the vectors every CTA reads.
    const int rep = blockIdx.x % kPersistReplicas;
    const unsigned long long *o_rep = p.o_out + (size_t)rep * p.stage_rows[kStO],
                             *down_rep = p.down_out + (size_t)rep * H,
                             *gu_rep = p.gu + (size_t)rep * p.ffn;
    // The state and the launch count are read once, at the start: CTA 0
    // changes them only after it has consumed the last stage, which every
    // CTA contributed to.
    const int pos = *reinterpret_cast<volatile const int *>(&p.st->pos);
    int tok = *reinterpret_cast<volatile const int *>(&p.st->cur_token);
    const unsigned launch = *reinterpret_cast<volatile const unsigned *>(p.ctl + 1);
    // Epochs of this launch: 5 per layer (qkv, partials, o, gu, down).
    const unsigned e0 = launch * (5u * (unsigned)p.layers + 1u);

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int i = 0; i < kNumBars; ++i) mbar_init(&mbar[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        issue_norms(p, 0, pos, true, smem, &mbar[kBarNorm]);
        if (p.layers > 1) issue_norms(p, 1, pos, false, smem, &mbar[kBarNorm + 1]);
        for (int s = 0; s < kNumStages; ++s) issue_stage(p, 0, s, smem, &mbar[s]);
        issue_kv(p, 0, pos, smem, &mbar[kBarKv]);
    }
    // h = embedding row * sqrt(hidden) (transformer.c:367-380).
    if (tok < 0 || tok >= p.vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, kErrToken);
        tok = 0;
    }
    const uint16_t *erow = p.embed + (size_t)tok * H;
    for (int i = threadIdx.x; i < H; i += kPersistThreads)
        hidden[i] = __uint_as_float((uint32_t)__ldg(erow + i) << 16) * p.emb_scale;

    for (int l = 0; l < p.layers; ++l) {
        const uint32_t par = (uint32_t)(l & 1);
        const bool more = l + 1 < p.layers;
        const unsigned e_qkv = e0 + 5u * l + 1u, e_part = e_qkv + 1u, e_o = e_qkv + 2u, e_gu = e_qkv + 3u,
                       e_down = e_qkv + 4u;
        // Norm weights of this layer (buffer l & 1, phase l / 2 of its barrier).
        mbar_wait(&mbar[kBarNorm + (l & 1)], (uint32_t)((l >> 1) & 1), p);
        const float *nrm = reinterpret_cast<const float *>(smem + p.off_nrm[l & 1]);
        const float *prev = reinterpret_cast<const float *>(smem + p.off_nrm[(l + 1) & 1]);
        __syncthreads();
        // QKV
        if (l > 0) residual_add(hidden, down_rep, 1, e_qkv - 1u, prev + 3 * H, H, xs, vin, red, p, &s_abort);
        norm_to(hidden, nrm, H, p.stage_nb[kStQkv] * 32, p.eps, xs, red);
        mbar_wait(&mbar[kStQkv], par, p);
        __syncthreads();
        if (!(p.test_stall && l == 0 && blockIdx.x == gridDim.x - 1))
            gemv_stage(p, kStQkv, smem + p.off_w[kStQkv], xs, p.qkv, e_qkv, 1);
        __syncthreads();
        if (threadIdx.x == 0) {
            if (more) issue_stage(p, l + 1, kStQkv, smem, &mbar[kStQkv]);
            // The previous layer's norms are no longer read: fetch layer l + 1's.
            if (l >= 1 && more) issue_norms(p, l + 1, pos, false, smem, &mbar[kBarNorm + ((l + 1) & 1)]);
        }
        // ATT
        attention_stage(p, l, pos, smem, &mbar[kBarKv], nrm, e_qkv, e_part, &s_abort);
        __syncthreads();
        if (threadIdx.x == 0 && more) issue_kv(p, l + 1, pos, smem, &mbar[kBarKv]);
        // O
        const int h0 = combine_stage(p, l, pos, xs, scratch, vin, e_part, &s_abort);
        mbar_wait(&mbar[kStO], par, p);
        gemv_stage(p, kStO, smem + p.off_w[kStO], xs, p.o_out, e_o, kPersistReplicas, H, h0);
        __syncthreads();
        if (threadIdx.x == 0 && more) issue_stage(p, l + 1, kStO, smem, &mbar[kStO]);
        // GU
        residual_add(hidden, o_rep, p.heads, e_o, nrm + H, H, xs, vin, red, p, &s_abort);
        norm_to(hidden, nrm + 2 * H, H, p.stage_nb[kStGu] * 32, p.eps, xs, red);
        mbar_wait(&mbar[kStGu], par, p);
        __syncthreads();
        gemv_stage(p, kStGu, smem + p.off_w[kStGu], xs, p.gu, e_gu, kPersistReplicas);
        __syncthreads();
        if (threadIdx.x == 0 && more) issue_stage(p, l + 1, kStGu, smem, &mbar[kStGu]);
        // DOWN: x = gelu_tanh(gate) * up, formed by the GU stage's blocks.
        {
            const int F = p.ffn, width = p.stage_nb[kStDown] * 32;
            for (int i = F + threadIdx.x; i < width; i += kPersistThreads) xs[i] = 0.0f;
            fetch_vec(gu_rep, F, e_gu, xs, p, &s_abort);
        }
        mbar_wait(&mbar[kStDown], par, p);
        __syncthreads();
        gemv_stage(p, kStDown, smem + p.off_w[kStDown], xs, p.down_out, e_down, kPersistReplicas);
        __syncthreads();
        if (threadIdx.x == 0 && more) issue_stage(p, l + 1, kStDown, smem, &mbar[kStDown]);
    }

    if (blockIdx.x == 0) {
        const float *last = reinterpret_cast<const float *>(smem + p.off_nrm[(p.layers - 1) & 1]);
        // h + rmsnorm_delta(down_out, ffn_post) of the last layer; waiting for
        // it also means every CTA has passed its last read of this launch.
        residual_add(hidden, down_rep, 1, e0 + 5u * p.layers, last + 3 * H, H, xs, vin, red, p, &s_abort);
        if (p.generate) {
            // logits input: rmsnorm_delta(h, final) (transformer.c:393-408)
            float ss = 0.0f;
            for (int i = threadIdx.x; i < H; i += kPersistThreads) ss += hidden[i] * hidden[i];
            ss = block_sum(ss, red);
            const float r = 1.0f / sqrtf(ss / (float)H + p.eps);
            for (int i = threadIdx.x; i < H; i += kPersistThreads)
                p.norm_out[i] = (hidden[i] * r) * (1.0f + __ldg(p.w_final + i));
        }
        if (threadIdx.x == 0) {
            if (!p.generate) {
                // Prompt phase: the next prompt token becomes the input at the next position.
                const int i = p.st->prompt_index + 1;
                p.st->prompt_index = i;
                p.st->pos = pos + 1;
                if (i < p.st->n_prompt) p.st->cur_token = p.prompt[i];
            }
            p.ctl[1] = launch + 1u;
        }
    }
}

size_t align128(size_t v) { return (v + 127) & ~(size_t)127; }

// Dynamic shared-memory layout for grid G and at least `chunk` keys per
// split: fills p's offsets and attention geometry and returns the total bytes.
size_t smem_layout(PersistParams &p, int G, int chunk) {
    p.splits = G / p.heads;
    p.chunk = chunk;
    // Every window up to the context fits `splits` splits of chunk_max keys.
    p.chunk_max = std::max(chunk, (p.context + p.splits - 1) / p.splits);
    size_t off = 0;
    for (int st = 0; st < kNumStages; ++st) {
        p.off_w[st] = (unsigned)off;
        const size_t rows_max = st == kStGu ? 2 * (((size_t)p.stage_rows[st] / 2 + G - 1) / G)
                                            : ((size_t)p.stage_rows[st] + G - 1) / G;
        off = align128(off + rows_max * p.stage_stride[st]);
    }
    const size_t kv_bytes = (size_t)p.chunk_max * p.hd * 4;
    p.off_k = (unsigned)off;
    off = align128(off + kv_bytes);
    p.off_v = (unsigned)off;
    off = align128(off + kv_bytes);
    p.off_hidden = (unsigned)off;
    off = align128(off + (size_t)p.hidden * 4);
    size_t xw = std::max((size_t)p.heads * p.hd, (size_t)p.hidden);
    for (int st = 0; st < kNumStages; ++st) xw = std::max(xw, (size_t)p.stage_nb[st] * 32);
    p.off_x = (unsigned)off;
    off = align128(off + xw * 4);
    p.off_q = (unsigned)off;
    off = align128(off + (size_t)p.hd * 4);
    p.off_kcur = (unsigned)off;
    off = align128(off + (size_t)p.hd * 4);
    p.off_vcur = (unsigned)off;
    off = align128(off + (size_t)p.hd * 4);
    p.off_sc = (unsigned)off;
    off = align128(off + (size_t)p.chunk_max * 4);
    for (int b = 0; b < 2; ++b) {
        p.off_nrm[b] = (unsigned)off;
        off = align128(off + (size_t)p.norm_stride * 4);
    }
    p.off_rope = (unsigned)off;
    off = align128(off + (size_t)4 * p.hd * 4);
    // Scratch of the weighted key sums (parts x hd) and of the split combine
    // (at most max(threads, heads * hd / 4) float4).
    p.off_acc = (unsigned)off;
    off = align128(off + std::max((size_t)4 * kPersistThreads, (size_t)p.heads * p.hd) * 4);
    // Staged input vectors (qkv, gate / up, the heads' O rows) and the
    // combine's (m, l) pairs.
    size_t vin = std::max((size_t)(p.heads + 2 * p.kv_heads) * p.hd, (size_t)2 * p.ffn);
    vin = std::max(vin, std::max((size_t)p.heads * p.hidden, (size_t)2 * G));
    p.off_vin = (unsigned)off;
    off = align128(off + vin * 4);
    return off;
}

}  // namespace

PersistPlan persist_plan(int device, const PersistParams &s, const char **why) {
    PersistPlan plan;
    *why = nullptr;
    const int G = sm_count(device);
    if (G <= 0) {
        *why = "no SM count";
        return plan;
    }
    // One attention block serves one query head, so any grouping of query
    // heads over KV heads works.
    if (s.hd % 64 || s.hd > kMaxHeadDim || s.kv_heads <= 0 || s.heads % s.kv_heads) {
        *why = "head shape";
        return plan;
    }
    if (s.hidden % 4 || s.ffn % 4 || s.norm_stride != 4 * s.hidden + 2 * s.hd || kPersistThreads % s.hd) {
        *why = "hidden / ffn / head_dim alignment";
        return plan;
    }
    if (s.layers > 64 || G < s.heads) {
        *why = "more than 64 layers or fewer SMs than heads";
        return plan;
    }
    // Every CTA must have rows in every product (the buffers' reuse relies on
    // it; stage GU counts pairs).
    for (int st = 0; st < kNumStages; ++st)
        if (s.stage_stride[st] % 16 || s.stage_rows[st] < (st == kStGu ? 2 * G : G) || (unsigned long long)s.stage_rows[st] * G >= (1ull << 32)) {
            *why = "row layout";
            return plan;
        }
    int chunk = kDefaultChunk;
    if (const char *e = getenv("SAPPHIRE_DECODE_CHUNK")) {
        const int v = atoi(e);
        if (v >= 1 && v <= 256) chunk = v;
    }
    PersistParams lay = s;
    const size_t bytes = smem_layout(lay, G, chunk);
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    const size_t static_bytes = 1024;   // mbarriers, reduction scratch, flags
    if (bytes + static_bytes > (size_t)optin) {
        *why = "shared memory";
        return plan;
    }
    if (cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
        cudaSuccess) {
        cudaGetLastError();
        *why = "shared-memory attribute";
        return plan;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persistent_kernel, kPersistThreads, bytes) !=
            cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        *why = "occupancy";
        return plan;
    }
    plan.ok = true;
    plan.grid = G;
    plan.chunk = chunk;
    plan.smem = bytes;
    // One partial row per (split, head): splits * heads <= G rows.
    plan.part_floats = (size_t)G * (s.hd + 4);
    return plan;
}

void persist_layout(const PersistPlan &plan, PersistParams &p) { smem_layout(p, plan.grid, plan.chunk); }

cudaError_t launch_persist(const PersistPlan &plan, const PersistParams &p, bool cooperative, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(kPersistThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cooperative ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, decode_persistent_kernel, p);
}
