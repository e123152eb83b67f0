// decode.cu - device-resident Gemma-3 decoder (include/sapphire_decode.h).
//
// One token's step mirrors the reference's inference_forward
// (src/inference/inference.c:616-651) and its layer stages
// (src/transformer/attention.c:311-375, src/transformer/transformer.c:96-283):
//
//   hidden = bf16 embedding row * sqrt(hidden)              (transformer.c:367-380)
//   per layer:
//     norm   = rmsnorm_delta(hidden, attn)                   (attention.c:321-325)
//     qkv    = [Wq; Wk; Wv] . norm        one Q4_0 GEMV over the concatenated rows
//     q, k   = rmsnorm_delta per head (q_norm / k_norm), RoPE at pos (half split)
//     K, V cache[pos] = k, v                                 (attention.c:292-309)
//     attn   = softmax(q . K / sqrt(query_pre_attn_scalar)) . V over the layer's
//              window (all positions for global layers)      (attention.c:93-163)
//     hidden += rmsnorm_delta(Wo . attn, attn_post)          (attention.c:348-366)
//     norm   = rmsnorm_delta(hidden, ffn)                    (transformer.c:119-121)
//     gu     = [Wgate; Wup] . norm        one Q4_0 GEMV
//     hidden += rmsnorm_delta(Wdown . (gelu(gate) * up), ffn_post)
//   logits = Wlm . rmsnorm_delta(hidden, final)              (transformer.c:393-408)
//   token  = greedy argmax, lowest index on ties             (src/utils/utils.c:145-156)
//
// All arithmetic is fp32 like the reference; sums run in a different order, so
// the results agree to rounding, not bit for bit.  The RoPE tables are
// computed on the host with the reference's formula and libm calls
// (src/transformer/rope.c:19-37), so they are the same numbers.
//
// Kernels of one token (5 per layer): the QKV GEMV (whose x stage also applies
// the previous layer's FFN residual and this layer's pre-attention norm), the
// attention (with QK-norm, RoPE and the KV-cache write), the O GEMV, the
// gate/up GEMV (attention residual + pre-FFN norm in its x stage) and the down
// GEMV (GeGLU in its x stage); then, for a generated token, the final norm,
// the LM-head GEMV and the argmax.  Every kernel is launched with programmatic
// dependent launch, so each GEMV streams its weights while the previous kernel
// runs.  The current token, position and output index live in device memory,
// and a step is captured once into a CUDA graph per step kind (prompt step,
// generated step); a generation is a sequence of graph launches with no host
// round trip.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "internal.cuh"
#include "decode_common.cuh"
#include "../../include/sapphire_decode.h"
#include "../../include/sapphire_safetensors.h"

namespace {

constexpr int kNormThreads = 256;
constexpr int kAttnSplit = 32;        // CTAs per layer's attention
static_assert(kAttnSplit == 32, "the combine maps one split to one warp lane");
constexpr int kAttnThreads = 256;
constexpr int kArgmaxBlocks = 148;
constexpr int kArgmaxThreads = 512;

// Sharded LM head: every rank's mapped exchange buffer, [2 parities][kMaxPeers
// ranks][4 words] of (epoch << 32 | 32 bits).
struct PeerSlots {
    unsigned long long *p[kMaxPeers];
};
constexpr int kExchWords = 4;
constexpr unsigned long long kExchWaitNs = 2000000000ull;

// out[i] = (in[i] * rms_inv) * (1 + w[i]),  rms_inv = 1 / sqrt(mean(in^2) + eps)
// (rmsnorm_delta, src/transformer/normalization.c:103-116).  One block; in and
// out may alias.
__device__ void rms_delta_block(const float *in, const float *w, float *out, int n, float eps, float *red) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += in[i] * in[i];
    ss = block_sum(ss, red);
    const float rms_inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float scale = 1.0f + (w ? w[i] : 0.0f);
        out[i] = (in[i] * rms_inv) * scale;
    }
}

// --------------------------------------------------------------- kernels --
// hidden = embed[token] * sqrt(hidden); norm = rmsnorm_delta(hidden, w).
__global__ void embed_norm_kernel(const DecState *st, const uint16_t *__restrict__ embed, int vocab, int dim,
                                  float scale, const float *w, float eps, float *hidden, float *norm, int *err) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    int tok = st->cur_token;
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, kErrToken);
        tok = 0;
    }
    const uint16_t *row = embed + (size_t)tok * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) hidden[i] = __uint_as_float((uint32_t)row[i] << 16) * scale;
    __syncthreads();
    rms_delta_block(hidden, w, norm, dim, eps, red);
}

// hidden += rmsnorm_delta(t, w_post); norm = rmsnorm_delta(hidden, w_next).
__global__ void residual_norm_kernel(const float *t, const float *w_post, float *hidden, const float *w_next,
                                     float *norm, int dim, float eps) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += t[i] * t[i];
    ss = block_sum(ss, red);
    const float rms_inv = 1.0f / sqrtf(ss / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        const float n = (t[i] * rms_inv) * (1.0f + (w_post ? w_post[i] : 0.0f));
        hidden[i] = hidden[i] + n;
    }
    __syncthreads();
    rms_delta_block(hidden, w_next, norm, dim, eps, red);
}

// Attention of the current token over positions [start, pos] of one layer.
// Grid: kAttnSplit blocks, each a contiguous key range for every KV head.  A
// block stages its keys kSub at a time (K and V rows into shared memory, all
// loads in flight together), scores them for the KV head's query group and
// keeps a running max m, sum l and unnormalised output acc = sum exp(s - m) v
// per query head; the last block to finish combines the splits in block order
// (deterministic) and resets the arrival counter.
//
// The block also finishes the projections of the current token first (what
// the reference does in attention_apply_rope_cache, attention.c:292-309):
// rmsnorm_delta per head with q_norm / k_norm, RoPE at pos (rope_apply_fast,
// src/transformer/rope.c:65-80), and block 0 writes the new K and V rows;
// the block whose range holds pos reads them from shared memory.
constexpr int kSub = 16;

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    const DecState *st, const float *qkv, float *kcache, float *vcache, float *out, float *part, int *counter,
    int heads, int kv_heads, int hd, int context, int window, int is_global, float scale, const float *q_norm,
    const float *k_norm, float eps, const float *rope_cos, const float *rope_sin) {
    pdl_trigger();
    pdl_wait();
    __shared__ __align__(16) float qs[kMaxGroup * kMaxHeadDim];
    __shared__ __align__(16) float ks[kSub * kMaxHeadDim];
    __shared__ __align__(16) float vs[kSub * kMaxHeadDim];
    __shared__ __align__(16) float kpos[kMaxHeadDim], vpos[kMaxHeadDim];
    __shared__ float sc[kMaxGroup * kSub];
    __shared__ float mh[kMaxGroup], lh[kMaxGroup], ch[kMaxGroup];
    __shared__ float wsplit[kMaxHeads * kAttnSplit];
    __shared__ int last;
    const int pos = st->pos;
    const int seq = pos + 1;
    const int start = (!is_global && seq > window) ? seq - window : 0;
    const int len = seq - start;
    // Keys per block: a multiple of kSub, so short sequences use few blocks
    // (one block, and no combine, up to kSub keys).
    const int chunk = max(kSub, ((len + kAttnSplit - 1) / kAttnSplit + kSub - 1) / kSub * kSub);
    const int nsplit = (len + chunk - 1) / chunk;
    const int k0 = start + blockIdx.x * chunk;
    const int k1 = min(seq, k0 + chunk);
    const int n = max(0, k1 - k0);
    const int group = heads / kv_heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const size_t part_stride = (size_t)hd + 2;
    const int d = threadIdx.x;                  // output dimension of this thread (hd <= blockDim)

    const float *cs = rope_cos + (size_t)pos * hd, *sn = rope_sin + (size_t)pos * hd;
    for (int kh = 0; kh < kv_heads; ++kh) {
        float *kb = kcache + (size_t)kh * context * hd;
        float *vb = vcache + (size_t)kh * context * hd;
        // Normed, rotated q of the group, k and v of the current token.
        for (int h = warp; h < group + 2; h += nwarps) {
            if (h < group) {
                warp_norm_rope(qkv + (size_t)(kh * group + h) * hd, q_norm, eps, cs, sn, hd, qs + h * hd);
            } else if (h == group) {
                warp_norm_rope(qkv + (size_t)(heads + kh) * hd, k_norm, eps, cs, sn, hd, kpos);
            } else {
                const float *v = qkv + (size_t)(heads + kv_heads + kh) * hd;
                for (int i = lane; i < hd; i += 32) vpos[i] = v[i];
            }
        }
        if (threadIdx.x < group) {
            mh[threadIdx.x] = -INFINITY;
            lh[threadIdx.x] = 0.0f;
        }
        float acc[kMaxGroup];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.0f;
        __syncthreads();
        if (blockIdx.x == 0) {
            for (int i = threadIdx.x; i < hd; i += blockDim.x) {
                kb[(size_t)pos * hd + i] = kpos[i];
                vb[(size_t)pos * hd + i] = vpos[i];
            }
        }
        for (int t0 = 0; t0 < n; t0 += kSub) {
            const int ns = min(kSub, n - t0);
            // Stage ns rows of K and V (all loads issued before any use).
            const float4 *k4 = reinterpret_cast<const float4 *>(kb + (size_t)(k0 + t0) * hd);
            const float4 *v4 = reinterpret_cast<const float4 *>(vb + (size_t)(k0 + t0) * hd);
            const int nv = ns * hd / 4;
            const int row4 = hd / 4;
            for (int i = threadIdx.x; i < nv; i += blockDim.x) {
                float4 a, b;
                if (k0 + t0 + i / row4 == pos) {          // written by this kernel: take it from shared memory
                    a = reinterpret_cast<const float4 *>(kpos)[i % row4];
                    b = reinterpret_cast<const float4 *>(vpos)[i % row4];
                } else {
                    a = __ldcg(k4 + i);
                    b = __ldcg(v4 + i);
                }
                reinterpret_cast<float4 *>(ks)[i] = a;
                reinterpret_cast<float4 *>(vs)[i] = b;
            }
            __syncthreads();
            // scores of the staged keys (one warp per key)
            for (int t = warp; t < ns; t += nwarps) {
                float a[kMaxGroup];
#pragma unroll
                for (int h = 0; h < kMaxGroup; ++h) a[h] = 0.0f;
                for (int dd = lane; dd < hd; dd += 32) {
                    const float kv = ks[t * hd + dd];
#pragma unroll
                    for (int h = 0; h < kMaxGroup; ++h)
                        if (h < group) a[h] += qs[h * hd + dd] * kv;
                }
#pragma unroll
                for (int h = 0; h < kMaxGroup; ++h) {
                    if (h < group) {
                        const float v = warp_sum(a[h]);
                        if (lane == 0) sc[h * kSub + t] = v * scale;
                    }
                }
            }
            __syncthreads();
            // running max / sum per head (one warp per head, lane = key)
            for (int h = warp; h < group; h += nwarps) {
                const float sv = lane < ns ? sc[h * kSub + lane] : -INFINITY;
                const float m_old = mh[h];
                const float m_new = fmaxf(m_old, warp_max(sv));
                const float p = lane < ns ? expf(sv - m_new) : 0.0f;
                const float psum = warp_sum(p);
                const float c = expf(m_old - m_new);     // 0 while m_old is -inf
                if (lane < ns) sc[h * kSub + lane] = p;
                if (lane == 0) {
                    ch[h] = c;
                    mh[h] = m_new;
                    lh[h] = lh[h] * c + psum;
                }
            }
            __syncthreads();
            if (d < hd) {
#pragma unroll
                for (int h = 0; h < kMaxGroup; ++h) {
                    if (h < group) {
                        float a = acc[h] * ch[h];
                        for (int t = 0; t < ns; ++t) a += sc[h * kSub + t] * vs[t * hd + d];
                        acc[h] = a;
                    }
                }
            }
            __syncthreads();
        }
        if (d < hd) {
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h) {
                if (h < group) {
                    float *pp = part + ((size_t)(blockIdx.x * kv_heads + kh) * group + h) * part_stride;
                    pp[2 + d] = acc[h];
                }
            }
        }
        if (threadIdx.x < group) {
            float *pp = part + ((size_t)(blockIdx.x * kv_heads + kh) * group + threadIdx.x) * part_stride;
            pp[0] = mh[threadIdx.x];
            pp[1] = lh[threadIdx.x];
        }
        __syncthreads();
    }

    if (nsplit == 1) {
        // A single block holds every key: normalise and store directly.
        if (blockIdx.x == 0) {
            for (int j = threadIdx.x; j < heads * hd; j += blockDim.x) {
                const int h = j / hd, kh = h / group, hh = h % group;
                const float *pp = part + ((size_t)kh * group + hh) * part_stride;
                out[j] = __ldcg(pp + 2 + j % hd) / __ldcg(pp + 1);
            }
        }
        return;
    }
    if ((int)blockIdx.x >= nsplit) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = (atomicAdd(counter, 1) == nsplit - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    // Combine: weight of split b for head h is exp(m_b - M) / sum_b' l_b' exp(m_b' - M)
    // (one warp per head, lane = split), then out = sum_b weight_b acc_b.
    for (int h = warp; h < heads; h += nwarps) {
        const int kh = h / group, hh = h % group;
        float m = -INFINITY, l = 0.0f;
        if (lane < nsplit) {
            const float *pp = part + ((size_t)(lane * kv_heads + kh) * group + hh) * part_stride;
            m = __ldcg(pp);
            l = __ldcg(pp + 1);
        }
        const float M = warp_max(m);
        const float e = (m == -INFINITY) ? 0.0f : expf(m - M);
        const float L = warp_sum(l * e);
        wsplit[h * kAttnSplit + lane] = e / L;
    }
    __syncthreads();
    // Each thread sums its outputs over the splits; the loads of kOut outputs
    // of one split are independent, so several splits' loads are in flight.
    constexpr int kOut = 4;
    for (int j0 = threadIdx.x; j0 < heads * hd; j0 += blockDim.x * kOut) {
        float O[kOut];
        int base[kOut], wrow[kOut];
#pragma unroll
        for (int k = 0; k < kOut; ++k) {
            const int j = j0 + k * blockDim.x;
            const int h = j / hd, kh = h / group, hh = h % group;
            O[k] = 0.0f;
            base[k] = j < heads * hd ? (int)(((size_t)kh * group + hh) * part_stride + 2 + j % hd) : -1;
            wrow[k] = h * kAttnSplit;
        }
#pragma unroll 4
        for (int b = 0; b < nsplit; ++b) {
            const size_t boff = (size_t)b * kv_heads * group * part_stride;
#pragma unroll
            for (int k = 0; k < kOut; ++k)
                if (base[k] >= 0) O[k] += __ldcg(part + boff + base[k]) * wsplit[wrow[k] + b];
        }
#pragma unroll
        for (int k = 0; k < kOut; ++k)
            if (base[k] >= 0) out[j0 + k * blockDim.x] = O[k];
    }
    if (threadIdx.x == 0) *counter = 0;
}

// Top-1 (value, lowest index on ties) and top-2 value.
struct Top2 {
    float v1;
    int i1;
    float v2;
};
__device__ __forceinline__ void top2_push(Top2 &a, float v, int i) {
    if (v > a.v1 || (v == a.v1 && i < a.i1)) {
        a.v2 = fmaxf(a.v2, a.v1);
        a.v1 = v;
        a.i1 = i;
    } else if (v > a.v2) {
        a.v2 = v;
    }
}
__device__ __forceinline__ Top2 top2_merge(const Top2 &a, const Top2 &b) {
    const bool b_first = b.v1 > a.v1 || (b.v1 == a.v1 && b.i1 < a.i1);
    Top2 r;
    if (b_first) {
        r.v1 = b.v1;
        r.i1 = b.i1;
        r.v2 = fmaxf(b.v2, a.v1);
    } else {
        r.v1 = a.v1;
        r.i1 = a.i1;
        r.v2 = fmaxf(a.v2, b.v1);
    }
    return r;
}
__device__ Top2 block_top2(Top2 t, Top2 *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Top2 u;
        u.v1 = __shfl_xor_sync(0xffffffffu, t.v1, o);
        u.i1 = __shfl_xor_sync(0xffffffffu, t.i1, o);
        u.v2 = __shfl_xor_sync(0xffffffffu, t.v2, o);
        t = top2_merge(t, u);
    }
    __syncthreads();
    if (lane == 0) sh[warp] = t;
    __syncthreads();
    Top2 r = sh[0];
    for (int w = 1; w < nw; ++w) r = top2_merge(r, sh[w]);
    return r;
}

// Greedy token of the logits; the last block writes it as the next input,
// records it (and the top-1 minus top-2 margin) and advances the position.
__global__ void argmax_advance_kernel(const float *logits, int n, Top2 *part, int *counter, DecState *st,
                                      int *out_tokens, float *out_margins) {
    pdl_trigger();
    pdl_wait();
    __shared__ Top2 sh[32];
    __shared__ int last;
    Top2 t{-INFINITY, 0x7fffffff, -INFINITY};
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) top2_push(t, logits[i], i);
    t = block_top2(t, sh);
    if (threadIdx.x == 0) {
        part[blockIdx.x] = t;
        __threadfence();
        last = (atomicAdd(counter, 1) == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    Top2 r{-INFINITY, 0x7fffffff, -INFINITY};
    for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
        Top2 u;
        u.v1 = __ldcg(&part[b].v1);
        u.i1 = __ldcg(&part[b].i1);
        u.v2 = __ldcg(&part[b].v2);
        r = top2_merge(r, u);
    }
    r = block_top2(r, sh);
    if (threadIdx.x == 0) {
        const int tok = (r.i1 >= 0 && r.i1 < n) ? r.i1 : 0;
        const int g = st->gen_index;
        out_tokens[g] = tok;
        out_margins[g] = r.v1 - r.v2;
        st->gen_index = g + 1;
        st->cur_token = tok;
        st->pos = st->pos + 1;
        *counter = 0;
    }
}

// Greedy token of a row-sharded LM head: every rank reduces its slice of the
// logits (rows row0 .. row0 + n) to (top-1 value, its global index, top-2
// value) like argmax_advance_kernel; the last block sends the three values to
// every rank as epoch-tagged 8-byte words (an aligned 8-byte store arrives
// whole), waits (bounded) for every rank's words of this epoch, and merges
// them in rank order with the same rule, lowest index on ties - so every rank
// picks the same token as the unsharded argmax (src/utils/utils.c:145-156)
// having exchanged 8 * 3 bytes per rank instead of the logits.  Buffers
// alternate by epoch parity: a rank writes parity p again two steps later,
// after its own wait of the step between, which needed every rank's words of
// that step, written after that rank's kernel of this step had completed.
__global__ void argmax_sharded_kernel(const float *logits, int n, int row0, Top2 *part, int *counter, DecState *st,
                                      int *out_tokens, float *out_margins, PeerSlots peers, int world, int rank,
                                      const unsigned long long *mine, int *err) {
    pdl_trigger();
    pdl_wait();
    __shared__ Top2 sh[32];
    __shared__ int last;
    __shared__ Top2 ranks[kMaxPeers];
    Top2 t{-INFINITY, 0x7fffffff, -INFINITY};
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        top2_push(t, logits[i], row0 + i);
    t = block_top2(t, sh);
    if (threadIdx.x == 0) {
        part[blockIdx.x] = t;
        __threadfence();
        last = (atomicAdd(counter, 1) == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    Top2 r{-INFINITY, 0x7fffffff, -INFINITY};
    for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
        Top2 u;
        u.v1 = __ldcg(&part[b].v1);
        u.i1 = __ldcg(&part[b].i1);
        u.v2 = __ldcg(&part[b].v2);
        r = top2_merge(r, u);
    }
    r = block_top2(r, sh);
    const unsigned epoch = st->epoch + 1;
    const int parity = (int)(epoch & 1u);
    const unsigned long long tag = (unsigned long long)epoch << 32;
    if (threadIdx.x < world) {
        unsigned long long *dst = peers.p[threadIdx.x] + ((size_t)parity * kMaxPeers + rank) * kExchWords;
        const unsigned long long w0 = tag | __float_as_uint(r.v1), w1 = tag | (unsigned)r.i1,
                                 w2 = tag | __float_as_uint(r.v2);
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(w0) : "memory");
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + 1), "l"(w1) : "memory");
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + 2), "l"(w2) : "memory");
    }
    if (threadIdx.x < world) {
        const unsigned long long *src = mine + ((size_t)parity * kMaxPeers + threadIdx.x) * kExchWords;
        unsigned long long w[3];
        bool ok = true;
        uint64_t t0;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        for (int k = 0; k < 3 && ok; ++k) {
            for (;;) {
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[k]) : "l"(src + k) : "memory");
                if ((unsigned)(w[k] >> 32) == epoch) break;
                uint64_t now;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
                if (now - t0 > kExchWaitNs) {
                    ok = false;
                    break;
                }
                __nanosleep(32);
            }
        }
        Top2 u{-INFINITY, 0x7fffffff, -INFINITY};
        if (ok) {
            u.v1 = __uint_as_float((unsigned)w[0]);
            u.i1 = (int)(unsigned)w[1];
            u.v2 = __uint_as_float((unsigned)w[2]);
        } else {
            atomicOr(err, 8);
        }
        ranks[threadIdx.x] = u;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        Top2 g = ranks[0];
        for (int k = 1; k < world; ++k) g = top2_merge(g, ranks[k]);
        const int tok = (g.i1 >= 0 && g.i1 < 0x7fffffff) ? g.i1 : 0;
        const int gi = st->gen_index;
        out_tokens[gi] = tok;
        out_margins[gi] = g.v1 - g.v2;
        st->gen_index = gi + 1;
        st->cur_token = tok;
        st->pos = st->pos + 1;
        st->epoch = epoch;
        *counter = 0;
    }
}

// Prompt phase: the next prompt token becomes the input at the next position.
__global__ void prompt_advance_kernel(DecState *st, const int *prompt) {
    pdl_trigger();
    pdl_wait();
    const int i = st->prompt_index + 1;
    st->prompt_index = i;
    st->pos = st->pos + 1;
    if (i < st->n_prompt) st->cur_token = prompt[i];
}

}  // namespace

// ------------------------------------------------------------- the engine --
struct sapphire_decoder {
    kernel_context_t *ctx = nullptr;
    sapphire_gemma3_config_t cfg{};
    int q_dim = 0, kv_dim = 0;

    // Host copies backing the uploaded weights (tensor views over them).
    std::vector<std::vector<uint8_t>> host;
    std::vector<tensor_t *> tensors;
    struct Layer {
        tensor_t *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
        float *w_attn = nullptr, *w_attn_post = nullptr, *w_ffn = nullptr, *w_ffn_post = nullptr;
        float *w_q = nullptr, *w_k = nullptr;
        bool global = false;
    };
    std::vector<Layer> layers;
    tensor_t *lm_head = nullptr;
    float *w_final = nullptr;

    // Device buffers.
    uint16_t *embed = nullptr;
    float *rope_cos_g = nullptr, *rope_sin_g = nullptr, *rope_cos_l = nullptr, *rope_sin_l = nullptr;
    float *kcache = nullptr, *vcache = nullptr;
    float *hidden = nullptr, *hidden2 = nullptr, *norm = nullptr, *qkv = nullptr, *attn = nullptr, *tmp = nullptr,
          *gu = nullptr, *logits = nullptr, *attn_part = nullptr;
    void *top2_part = nullptr;
    int *counters = nullptr;        // [0] attention, [1] argmax
    DecState *state = nullptr;
    int *prompt = nullptr, *out_tokens = nullptr;
    float *out_margins = nullptr;
    std::vector<void *> allocations;

    // Sharded LM head (context with world > 1): exchange buffers and the
    // number of generated steps so far (the next step's epoch - 1).
    bool sharded = false;
    void *exch_local = nullptr;
    void *exch_peers[kMaxPeers] = {};
    unsigned epochs = 0;
    float *logits_all = nullptr;    // [world * ceil(vocab / world)] gathered logits (last_logits)

    // Persistent step (decode_persistent.cu): used when the model fits its
    // plan, unless SAPPHIRE_DECODE_PERSISTENT=0.  Projections live in its
    // row layout only; the LM head stays a context weight.
    bool persist = false;
    bool coop = true;               // launched cooperatively (false: capture refused it)
    PersistPlan plan;
    PersistParams pp{};
    uint8_t *wrows = nullptr;
    unsigned *ctl = nullptr;        // [0] abort flag, [1] launches so far

    cudaGraphExec_t g_prompt = nullptr, g_gen = nullptr;
    int launches_prompt = 0, launches_gen = 0;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    float last_prompt_ms = 0, last_gen_ms = 0;
};

namespace {

// Test hook (sapphire_test_decode_stall): decoders created while it is set
// run a persistent step in which one block withholds its output.
std::atomic<int> g_test_decode_stall{0};

int dev_alloc(sapphire_decoder_t *d, void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        ctx_fail(d->ctx, "sapphire_decoder_create", "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
        return -1;
    }
    d->allocations.push_back(*p);
    return 0;
}

int upload_floats(sapphire_decoder_t *d, float **dst, const float *src, size_t n) {
    if (dev_alloc(d, (void **)dst, n * sizeof(float))) return -1;
    cudaError_t e = src ? cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice)
                        : cudaMemset(*dst, 0, n * sizeof(float));
    if (e != cudaSuccess) {
        ctx_fail(d->ctx, "sapphire_decoder_create", "norm weight upload failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// A Q4_0 tensor over the concatenation of `parts` (rows back to back),
// uploaded to the context.
// Every rank of a sharded context holds the whole weight unless `whole` is
// false (the LM head, whose rows are sharded).
tensor_t *concat_q4(sapphire_decoder_t *d, const std::vector<std::pair<const void *, int>> &parts, int cols,
                    bool whole = true) {
    const size_t rb = sapphire_row_bytes_internal(DTYPE_Q4_0, cols);
    int rows = 0;
    for (auto &p : parts) rows += p.second;
    d->host.emplace_back((size_t)rows * rb);
    std::vector<uint8_t> &buf = d->host.back();
    size_t off = 0;
    for (auto &p : parts) {
        if (!p.first) {
            ctx_fail(d->ctx, "sapphire_decoder_create", "a projection pointer is NULL");
            return nullptr;
        }
        memcpy(buf.data() + off, p.first, (size_t)p.second * rb);
        off += (size_t)p.second * rb;
    }
    int shape[2] = {rows, cols};
    tensor_t *t = tensor_create_view(DTYPE_Q4_0, 2, shape, buf.data());
    if (!t) {
        ctx_fail(d->ctx, "sapphire_decoder_create", "tensor_create_view failed");
        return nullptr;
    }
    d->tensors.push_back(t);
    if (!ctx_weight(d->ctx, t, whole)) return nullptr;
    return t;
}

const DevWeight *weight_of(sapphire_decoder_t *d, tensor_t *t) { return ctx_weight(d->ctx, t, t != d->lm_head); }

// The reference's table (rope_precompute_freqs, src/transformer/rope.c:19-37):
// half-split storage, cos / sin of pos * base^(-2m/d) in float.
void rope_table(std::vector<float> &c, std::vector<float> &s, int hd, int context, float base) {
    const int half = hd / 2;
    c.assign((size_t)context * hd, 0.0f);
    s.assign((size_t)context * hd, 0.0f);
    for (int pos = 0; pos < context; ++pos) {
        for (int m = 0; m < half; ++m) {
            const float freq = 1.0f / powf(base, 2.0f * (float)m / (float)hd);
            const float angle = (float)pos * freq;
            const float cv = cosf(angle), sv = sinf(angle);
            c[(size_t)pos * hd + m] = cv;
            c[(size_t)pos * hd + m + half] = cv;
            s[(size_t)pos * hd + m] = sv;
            s[(size_t)pos * hd + m + half] = sv;
        }
    }
}

int check_launch(sapphire_decoder_t *d, const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ctx_fail(d->ctx, "sapphire_decoder", "%s launch failed: %s", what, cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// Enqueue one step: embedding, the layers and either the prompt advance or
// the LM head + greedy argmax.  Returns the number of kernels, -1 on error.
// The LM head and the greedy argmax of a generated step (the argmax advances
// the state).  Returns the number of kernels, -1 on error.
int enqueue_head(sapphire_decoder_t *d, cudaStream_t st) {
    kernel_context_t *ctx = d->ctx;
    const DevWeight *head = weight_of(d, d->lm_head);
    if (!head) return -1;
    if (launch_gemv_best(ctx, *head, d->norm, d->logits, st)) return -1;
    if (d->sharded) {
        PeerSlots peers{};
        for (int k = 0; k < ctx->world; ++k) peers.p[k] = static_cast<unsigned long long *>(d->exch_peers[k]);
        launch_pdl(argmax_sharded_kernel, dim3(kArgmaxBlocks), dim3(kArgmaxThreads), 0, st, (const float *)d->logits,
                   head->nrows, head->row0, reinterpret_cast<Top2 *>(d->top2_part), d->counters + 1, d->state,
                   d->out_tokens, d->out_margins, peers, ctx->world, ctx->rank, (const unsigned long long *)d->exch_local,
                   ctx->d_err);
    } else {
        launch_pdl(argmax_advance_kernel, dim3(kArgmaxBlocks), dim3(kArgmaxThreads), 0, st, (const float *)d->logits,
                   d->cfg.vocab, reinterpret_cast<Top2 *>(d->top2_part), d->counters + 1, d->state, d->out_tokens,
                   d->out_margins);
    }
    if (check_launch(d, "argmax")) return -1;
    return 2;
}

int enqueue_step(sapphire_decoder_t *d, bool generate, cudaStream_t st) {
    const sapphire_gemma3_config_t &c = d->cfg;
    kernel_context_t *ctx = d->ctx;
    int launches = 0;
    if (d->persist) {
        // One persistent kernel for the layers (and the prompt advance or the
        // final norm), then the LM head and the argmax.
        d->pp.generate = generate ? 1 : 0;
        cudaError_t e = launch_persist(d->plan, d->pp, d->coop, st);
        if (e != cudaSuccess) {
            cudaGetLastError();
            ctx_fail(ctx, "sapphire_decoder", "persistent step launch failed: %s", cudaGetErrorString(e));
            return -1;
        }
        if (!generate) return 1;
        const int h = enqueue_head(d, st);
        return h < 0 ? -1 : 1 + h;
    }
    const float eps = c.rms_eps;
    const float emb_scale = sqrtf((float)c.hidden);
    const float att_scale = 1.0f / sqrtf(c.query_pre_attn_scalar > 0.0f ? c.query_pre_attn_scalar : (float)c.head_dim);

    launch_pdl(embed_norm_kernel, dim3(1), dim3(kNormThreads), 0, st, (const DecState *)d->state,
               (const uint16_t *)d->embed, c.vocab, c.hidden, emb_scale, (const float *)d->layers[0].w_attn, eps,
               d->hidden, d->norm, ctx->d_err);
    if (check_launch(d, "embedding")) return -1;
    ++launches;
    // The residual stream alternates between two buffers: a fused GEMV reads
    // one and its first block writes the updated stream to the other.
    float *cur = d->hidden, *other = d->hidden2;
    for (int l = 0; l < c.layers; ++l) {
        sapphire_decoder::Layer &L = d->layers[l];
        const DevWeight *qkv = weight_of(d, L.qkv), *o = weight_of(d, L.o), *gu = weight_of(d, L.gu),
                        *down = weight_of(d, L.down);
        if (!qkv || !o || !gu || !down) return -1;
        // qkv = W_qkv . rmsnorm_delta(h, attn); for l > 0, h = h + rmsnorm_delta(down_out, ffn_post) first.
        if (l == 0) {
            if (launch_gemv_direct(ctx, *qkv, d->norm, d->qkv, st)) return -1;
        } else {
            if (launch_gemv_direct_resnorm(ctx, *qkv, d->tmp, d->layers[l - 1].w_ffn_post, cur, L.w_attn, other,
                                           eps, d->qkv, st))
                return -1;
            std::swap(cur, other);
        }
        float *kc = d->kcache + (size_t)l * c.kv_heads * c.context * c.head_dim;
        float *vc = d->vcache + (size_t)l * c.kv_heads * c.context * c.head_dim;
        launch_pdl(attention_kernel, dim3(kAttnSplit), dim3(kAttnThreads), 0, st, (const DecState *)d->state,
                   (const float *)d->qkv, kc, vc, d->attn, d->attn_part, d->counters, c.heads, c.kv_heads,
                   c.head_dim, c.context, c.sliding_window > 0 ? c.sliding_window : 1024, L.global ? 1 : 0,
                   att_scale, (const float *)L.w_q, (const float *)L.w_k, eps,
                   (const float *)(L.global ? d->rope_cos_g : d->rope_cos_l),
                   (const float *)(L.global ? d->rope_sin_g : d->rope_sin_l));
        if (check_launch(d, "attention")) return -1;
        if (launch_gemv_direct(ctx, *o, d->attn, d->tmp, st)) return -1;
        // gu = W_gu . rmsnorm_delta(h + rmsnorm_delta(o_out, attn_post), ffn)
        if (launch_gemv_direct_resnorm(ctx, *gu, d->tmp, L.w_attn_post, cur, L.w_ffn, other, eps, d->gu, st))
            return -1;
        std::swap(cur, other);
        // down_out = W_down . (gelu(gate) * up)
        if (launch_gemv_direct_geglu(ctx, *down, d->gu, d->tmp, st)) return -1;
        launches += 5;
    }
    if (generate) {
        // h = h + rmsnorm_delta(down_out, ffn_post); logits = W_lm . rmsnorm_delta(h, final)
        launch_pdl(residual_norm_kernel, dim3(1), dim3(kNormThreads), 0, st, (const float *)d->tmp,
                   (const float *)d->layers[c.layers - 1].w_ffn_post, cur, (const float *)d->w_final, d->norm,
                   c.hidden, eps);
        if (check_launch(d, "final norm")) return -1;
        const int h = enqueue_head(d, st);
        if (h < 0) return -1;
        launches += 1 + h;
    } else {
        launch_pdl(prompt_advance_kernel, dim3(1), dim3(1), 0, st, d->state, (const int *)d->prompt);
        if (check_launch(d, "prompt advance")) return -1;
        launches += 1;
    }
    return launches;
}

int capture(sapphire_decoder_t *d, bool generate, cudaGraphExec_t *exec, int *launches) {
    cudaStream_t st = d->ctx->stream;
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) {
        ctx_fail(d->ctx, "sapphire_decoder_create", "stream capture failed to start: %s", cudaGetErrorString(e));
        return -1;
    }
    const int n = enqueue_step(d, generate, st);
    e = cudaStreamEndCapture(st, &g);
    if (n < 0 || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        if (n >= 0) ctx_fail(d->ctx, "sapphire_decoder_create", "stream capture failed: %s", cudaGetErrorString(e));
        return -1;
    }
    e = cudaGraphInstantiate(exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        ctx_fail(d->ctx, "sapphire_decoder_create", "graph instantiation failed: %s", cudaGetErrorString(e));
        return -1;
    }
    *launches = n;
    return 0;
}

int set_state(sapphire_decoder_t *d, int first_token, int n_prompt, cudaStream_t st) {
    DecState s{0, first_token, 0, n_prompt, 0, d->epochs};
    CUDA_TRY(d->ctx, cudaMemcpyAsync(d->state, &s, sizeof s, cudaMemcpyHostToDevice, st));
    return 0;
}

}  // namespace

extern "C" SAPPHIRE_API void sapphire_decoder_destroy(sapphire_decoder_t *d) {
    if (!d) return;
    {
        std::lock_guard<std::recursive_mutex> lk(d->ctx->exec_mutex);
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(d->ctx->device);
        cudaStreamSynchronize(d->ctx->stream);
        if (d->g_prompt) cudaGraphExecDestroy(d->g_prompt);
        if (d->g_gen) cudaGraphExecDestroy(d->g_gen);
        for (cudaEvent_t e : d->ev)
            if (e) cudaEventDestroy(e);
        for (void *p : d->allocations) cudaFree(p);
        if (d->exch_local) shard_unmap_buffers(d->ctx, d->exch_local, d->exch_peers);
        if (prev >= 0) cudaSetDevice(prev);
    }
    for (tensor_t *t : d->tensors) tensor_release(t);   // drops the device copies
    delete d;
}

extern "C" SAPPHIRE_API sapphire_decoder_t *sapphire_decoder_create(kernel_context_t *ctx,
                                                                    const sapphire_gemma3_config_t *cfg,
                                                                    const sapphire_gemma3_weights_t *w) {
    if (!ctx || !cfg || !w || !w->embed_bf16 || !w->lm_head || !w->proj) {
        LOG_ERROR("sapphire_decoder_create: NULL argument");
        return nullptr;
    }
    const sapphire_gemma3_config_t &c = *cfg;
    if (c.layers <= 0 || c.hidden <= 0 || c.ffn <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads ||
        c.heads / c.kv_heads > kMaxGroup || c.heads > kMaxHeads || c.head_dim <= 0 || c.head_dim > kMaxHeadDim || c.head_dim % 64 ||
        c.vocab <= 0 || c.context <= 0 || c.context > kMaxContext || c.rms_eps < 0.0f) {
        ctx_fail(ctx, "sapphire_decoder_create",
                 "unsupported shape (heads %% kv_heads == 0, group <= %d, head_dim a multiple of 64 up to %d, "
                 "context <= %d)", kMaxGroup, kMaxHeadDim, kMaxContext);
        return nullptr;
    }
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (!ctx->initialized || ctx->world > kMaxPeers) {
        ctx_fail(ctx, "sapphire_decoder_create", "needs an initialized context of at most %d ranks", kMaxPeers);
        return nullptr;
    }
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    sapphire_decoder_t *d = new sapphire_decoder();
    d->ctx = ctx;
    d->cfg = c;
    d->sharded = ctx->world > 1;
    d->q_dim = c.heads * c.head_dim;
    d->kv_dim = c.kv_heads * c.head_dim;
    bool ok = false;
    do {
        d->layers.resize(c.layers);
        // The persistent step when the model fits it.
        PersistParams &pp = d->pp;
        pp.layers = c.layers;
        pp.hidden = c.hidden;
        pp.ffn = c.ffn;
        pp.heads = c.heads;
        pp.kv_heads = c.kv_heads;
        pp.hd = c.head_dim;
        pp.context = c.context;
        pp.vocab = c.vocab;
        pp.window = c.sliding_window > 0 ? c.sliding_window : 1024;
        pp.norm_stride = 4 * c.hidden + 2 * c.head_dim;
        // Stage O is split by head: its row h * hidden + r is row r of Wo
        // over head h's head_dim columns.
        const int stage_shape[kNumStages][2] = {{d->q_dim + 2 * d->kv_dim, c.hidden},
                                                 {c.heads * c.hidden, c.head_dim},
                                                 {2 * c.ffn, c.hidden},
                                                 {c.hidden, c.ffn}};
        pp.global_mask = 0;
        for (int l = 0; l < c.layers && l < 64; ++l)
            if (c.global_mask ? ((c.global_mask >> l) & 1ULL) != 0 : ((l + 1) % 6 == 0)) pp.global_mask |= 1ULL << l;
        unsigned long long lb = 0;
        for (int s = 0; s < kNumStages; ++s) {
            pp.stage_rows[s] = stage_shape[s][0];
            pp.stage_nb[s] = (stage_shape[s][1] + 31) / 32;
            pp.stage_stride[s] = (pp.stage_nb[s] * 20 + 15) / 16 * 16;
            pp.stage_off[s] = lb;
            lb += (unsigned long long)pp.stage_rows[s] * pp.stage_stride[s];
        }
        pp.layer_bytes = lb;
        {
            const char *why = nullptr;
            const char *env = getenv("SAPPHIRE_DECODE_PERSISTENT");
            d->plan = persist_plan(ctx->device, pp, &why);
            d->persist = d->plan.ok && !(env && strcmp(env, "0") == 0);
            if (!d->plan.ok) LOG_INFO("decoder: one kernel per stage (persistent step does not fit: %s)", why);
        }
        bool null_proj = false;
        for (int k = 0; k < 7 * c.layers; ++k) null_proj = null_proj || !w->proj[k];
        if (null_proj) {
            ctx_fail(ctx, "sapphire_decoder_create", "a projection pointer is NULL");
            break;
        }
        if (d->persist) {
            // Projections in the persistent step's row layout: per row the nb
            // blocks' 16 code bytes, then their nb fp32 scales.
            std::vector<uint8_t> rows((size_t)lb * c.layers, 0);
            for (int l = 0; l < c.layers; ++l) {
                const void *const *p = w->proj + 7 * l;
                // Blocks [b0, b0 + nb) of a packed Q4_0 row into one row of the layout.
                auto put_row = [](uint8_t *dst, const uint8_t *src, int nb, int b0) {
                    for (int b = 0; b < nb; ++b) {
                        memcpy(dst + 16 * b, src + 20 * (b0 + b) + 4, 16);
                        memcpy(dst + 16 * nb + 4 * b, src + 20 * (b0 + b), 4);
                    }
                };
                // (source, rows, source columns) of each stage; stage O by head.
                const struct {
                    const void *src;
                    int rows, cols;
                } parts[kNumStages][3] = {{{p[0], d->q_dim, c.hidden}, {p[1], d->kv_dim, c.hidden}, {p[2], d->kv_dim, c.hidden}},
                                          {{p[3], c.hidden, d->q_dim}, {nullptr, 0, 0}, {nullptr, 0, 0}},
                                          {{p[4], c.ffn, c.hidden}, {p[5], c.ffn, c.hidden}, {nullptr, 0, 0}},
                                          {{p[6], c.hidden, c.ffn}, {nullptr, 0, 0}, {nullptr, 0, 0}}};
                for (int s = 0; s < kNumStages; ++s) {
                    const int nb = pp.stage_nb[s], stride = pp.stage_stride[s];
                    uint8_t *dst = rows.data() + (size_t)l * lb + pp.stage_off[s];
                    if (s == kStGu) {
                        // Gate row i and up row i as rows 2i and 2i + 1.
                        const size_t src_rb = sapphire_row_bytes_internal(DTYPE_Q4_0, c.hidden);
                        const uint8_t *gate = static_cast<const uint8_t *>(p[4]), *up = static_cast<const uint8_t *>(p[5]);
                        for (int i = 0; i < c.ffn; ++i, dst += 2 * stride) {
                            put_row(dst, gate + (size_t)i * src_rb, nb, 0);
                            put_row(dst + stride, up + (size_t)i * src_rb, nb, 0);
                        }
                        continue;
                    }
                    const int pieces = s == kStO ? c.heads : 1;
                    for (int h = 0; h < pieces; ++h)
                        for (const auto &part : parts[s]) {
                            if (!part.src) continue;
                            const size_t src_rb = sapphire_row_bytes_internal(DTYPE_Q4_0, part.cols);
                            const uint8_t *src = static_cast<const uint8_t *>(part.src);
                            for (int r = 0; r < part.rows; ++r, dst += stride, src += src_rb) put_row(dst, src, nb, h * nb);
                        }
                }
            }
            if (dev_alloc(d, (void **)&d->wrows, rows.size()) ||
                cudaMemcpy(d->wrows, rows.data(), rows.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
                ctx_fail(ctx, "sapphire_decoder_create", "projection upload failed");
                break;
            }
        }
        for (int l = 0; l < c.layers; ++l) {
            const void *const *p = w->proj + 7 * l;
            sapphire_decoder::Layer &L = d->layers[l];
            L.global = c.global_mask ? ((c.global_mask >> l) & 1ULL) != 0 : ((l + 1) % 6 == 0);
            if (!d->persist) {
                if (!(L.qkv = concat_q4(d, {{p[0], d->q_dim}, {p[1], d->kv_dim}, {p[2], d->kv_dim}}, c.hidden))) break;
                if (!(L.o = concat_q4(d, {{p[3], c.hidden}}, d->q_dim))) break;
                if (!(L.gu = concat_q4(d, {{p[4], c.ffn}, {p[5], c.ffn}}, c.hidden))) break;
                if (!(L.down = concat_q4(d, {{p[6], c.hidden}}, c.ffn))) break;
            }
            const float *const *nw = w->norms ? w->norms + 6 * l : nullptr;
            if (upload_floats(d, &L.w_attn, nw ? nw[0] : nullptr, c.hidden) ||
                upload_floats(d, &L.w_attn_post, nw ? nw[1] : nullptr, c.hidden) ||
                upload_floats(d, &L.w_ffn, nw ? nw[2] : nullptr, c.hidden) ||
                upload_floats(d, &L.w_ffn_post, nw ? nw[3] : nullptr, c.hidden) ||
                upload_floats(d, &L.w_q, nw ? nw[4] : nullptr, c.head_dim) ||
                upload_floats(d, &L.w_k, nw ? nw[5] : nullptr, c.head_dim))
                break;
            if (l + 1 == c.layers) ok = true;
        }
        if (!ok) break;
        ok = false;
        bool direct = true;
        for (auto &L : d->layers)
            for (tensor_t *t : {L.qkv, L.o, L.gu, L.down}) {
                if (d->persist) break;
                const DevWeight *dw = weight_of(d, t);
                direct = direct && dw && dw->ntiles <= kDirectMaxTiles && direct_supported(*dw);
            }
        if (!direct) {
            ctx_fail(ctx, "sapphire_decoder_create",
                     "projection shapes outside the fused decode GEMV (at most %d rows and 2048 columns)",
                     kDirectMaxTiles * 32);
            break;
        }
        if (!(d->lm_head = concat_q4(d, {{w->lm_head, c.vocab}}, c.hidden, !d->sharded))) break;
        if (d->sharded) {
            // Collective: every rank creates its decoder at the same point.
            if (shard_map_buffers(ctx, (size_t)2 * kMaxPeers * kExchWords * sizeof(unsigned long long),
                                  &d->exch_local, d->exch_peers))
                break;
            const size_t per = ((size_t)c.vocab + ctx->world - 1) / ctx->world;
            if (dev_alloc(d, (void **)&d->logits_all, per * (ctx->world + 1) * sizeof(float))) break;
        }
        if (upload_floats(d, &d->w_final, w->final_norm, c.hidden)) break;
        const size_t emb = (size_t)c.vocab * c.hidden;
        if (dev_alloc(d, (void **)&d->embed, emb * 2)) break;
        if (cudaMemcpy(d->embed, w->embed_bf16, emb * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
            ctx_fail(ctx, "sapphire_decoder_create", "embedding upload failed");
            break;
        }
        std::vector<float> cs, sn;
        const size_t rope_n = (size_t)c.context * c.head_dim;
        rope_table(cs, sn, c.head_dim, c.context, c.rope_theta);
        if (upload_floats(d, &d->rope_cos_g, cs.data(), rope_n) || upload_floats(d, &d->rope_sin_g, sn.data(), rope_n))
            break;
        rope_table(cs, sn, c.head_dim, c.context, c.rope_local_theta);
        if (upload_floats(d, &d->rope_cos_l, cs.data(), rope_n) || upload_floats(d, &d->rope_sin_l, sn.data(), rope_n))
            break;
        const size_t kv = (size_t)c.layers * c.kv_heads * c.context * c.head_dim;
        if (upload_floats(d, &d->kcache, nullptr, kv) || upload_floats(d, &d->vcache, nullptr, kv)) break;
        if (dev_alloc(d, (void **)&d->hidden, c.hidden * 4) || dev_alloc(d, (void **)&d->hidden2, c.hidden * 4) ||
            dev_alloc(d, (void **)&d->norm, c.hidden * 4) ||
            dev_alloc(d, (void **)&d->qkv, (size_t)(d->q_dim + 2 * d->kv_dim) * 4) ||
            dev_alloc(d, (void **)&d->attn, (size_t)d->q_dim * 4) ||
            dev_alloc(d, (void **)&d->tmp, (size_t)c.hidden * 4) ||
            dev_alloc(d, (void **)&d->gu, (size_t)2 * c.ffn * 4) ||
            dev_alloc(d, (void **)&d->logits, (size_t)c.vocab * 4) ||
            dev_alloc(d, (void **)&d->attn_part, (size_t)kAttnSplit * c.heads * (c.head_dim + 2) * 4) ||
            dev_alloc(d, &d->top2_part, (size_t)kArgmaxBlocks * sizeof(Top2)) ||
            dev_alloc(d, (void **)&d->state, sizeof(DecState)) ||
            dev_alloc(d, (void **)&d->prompt, (size_t)c.context * 4) ||
            dev_alloc(d, (void **)&d->out_tokens, (size_t)c.context * 4) ||
            dev_alloc(d, (void **)&d->out_margins, (size_t)c.context * 4))
            break;
        if (dev_alloc(d, (void **)&d->counters, 16) || cudaMemset(d->counters, 0, 16) != cudaSuccess) break;
        if (d->persist) {
            // Norm weights of every layer back to back (attn, attn_post, ffn,
            // ffn_post, q, k), copied from their uploaded vectors.
            float *d_norms = nullptr;
            if (dev_alloc(d, (void **)&d_norms, (size_t)c.layers * pp.norm_stride * 4)) break;
            bool copied = true;
            for (int l = 0; l < c.layers && copied; ++l) {
                const sapphire_decoder::Layer &L = d->layers[l];
                float *dst = d_norms + (size_t)l * pp.norm_stride;
                const std::pair<const float *, int> parts[6] = {{L.w_attn, c.hidden},   {L.w_attn_post, c.hidden},
                                                                {L.w_ffn, c.hidden},    {L.w_ffn_post, c.hidden},
                                                                {L.w_q, c.head_dim},    {L.w_k, c.head_dim}};
                for (const auto &pr : parts) {
                    copied = copied && cudaMemcpy(dst, pr.first, (size_t)pr.second * 4, cudaMemcpyDeviceToDevice) ==
                                           cudaSuccess;
                    dst += pr.second;
                }
            }
            if (!copied ||
                dev_alloc(d, (void **)&pp.qkv, (size_t)(d->q_dim + 2 * d->kv_dim) * 8) ||
                dev_alloc(d, (void **)&pp.o_out, (size_t)c.heads * c.hidden * 8 * kPersistReplicas) ||
                dev_alloc(d, (void **)&pp.gu, (size_t)c.ffn * 8 * kPersistReplicas) ||
                dev_alloc(d, (void **)&pp.down_out, (size_t)c.hidden * 8 * kPersistReplicas) ||
                dev_alloc(d, (void **)&pp.part, d->plan.part_floats * 4) ||
                dev_alloc(d, (void **)&d->ctl, 4 * sizeof(unsigned)))
                break;
            // Tagged words start with epoch 0, which no launch uses.
            if (cudaMemset(pp.qkv, 0, (size_t)(d->q_dim + 2 * d->kv_dim) * 8) != cudaSuccess ||
                cudaMemset(pp.o_out, 0, (size_t)c.heads * c.hidden * 8 * kPersistReplicas) != cudaSuccess ||
                cudaMemset(pp.gu, 0, (size_t)c.ffn * 8 * kPersistReplicas) != cudaSuccess ||
                cudaMemset(pp.down_out, 0, (size_t)c.hidden * 8 * kPersistReplicas) != cudaSuccess ||
                cudaMemset(pp.part, 0, d->plan.part_floats * 4) != cudaSuccess ||
                cudaMemset(d->ctl, 0, 4 * sizeof(unsigned)) != cudaSuccess) {
                ctx_fail(ctx, "sapphire_decoder_create", "persistent step buffers could not be cleared");
                break;
            }
            pp.st = d->state;
            pp.prompt = d->prompt;
            pp.eps = c.rms_eps;
            pp.emb_scale = sqrtf((float)c.hidden);
            pp.att_scale = 1.0f / sqrtf(c.query_pre_attn_scalar > 0.0f ? c.query_pre_attn_scalar : (float)c.head_dim);
            pp.embed = d->embed;
            pp.wrows = d->wrows;
            pp.norms = d_norms;
            pp.w_final = d->w_final;
            pp.rope_cos_g = d->rope_cos_g;
            pp.rope_sin_g = d->rope_sin_g;
            pp.rope_cos_l = d->rope_cos_l;
            pp.rope_sin_l = d->rope_sin_l;
            pp.kcache = d->kcache;
            pp.vcache = d->vcache;
            pp.norm_out = d->norm;
            pp.ctl = d->ctl;
            pp.err = ctx->d_err;
            pp.test_stall = g_test_decode_stall.load();
            pp.wait_ns = pp.test_stall ? 1000000ull : 2000000000ull;
            persist_layout(d->plan, pp);
        }
        // Scratch of the GEMVs sized for the largest weight, before capture.
        size_t pf = 0, ci = 0;
        std::vector<tensor_t *> all = {d->lm_head};
        if (!d->persist)
            for (auto &L : d->layers) all.insert(all.end(), {L.qkv, L.o, L.gu, L.down});
        for (tensor_t *t : all) {
            const DevWeight *dw = weight_of(d, t);
            if (!dw) break;
            size_t a = 0, b = 0;
            pipe_scratch_size(ctx, *dw, &a, &b);
            pf = std::max(pf, a);
            ci = std::max(ci, b);
        }
        if (ensure_pipe_scratch(ctx, pf, ci)) break;
        // One eager pass of each step kind (also checks every launch), then capture.
        cudaStream_t st = ctx->stream;
        if (set_state(d, 0, 1, st) || enqueue_step(d, false, st) < 0 || enqueue_step(d, true, st) < 0) break;
        d->epochs += 1;
        const cudaError_t se = cudaStreamSynchronize(st);
        if (se != cudaSuccess) {
            ctx_fail(ctx, "sapphire_decoder_create", "warm-up step failed: %s", cudaGetErrorString(se));
            break;
        }
        // A kernel error of the warm-up (its message names the cause).
        if (check_kernel_error(ctx, "sapphire_decoder_create warm-up step")) break;
        if (capture(d, false, &d->g_prompt, &d->launches_prompt) ||
            capture(d, true, &d->g_gen, &d->launches_gen)) {
            if (!d->persist || !d->coop) break;
            // Capture refused the cooperative launch: capture a plain one (its
            // CTAs are resident together all the same - one per SM, with
            // nothing else running during the step - and its waits are bounded).
            cudaGetLastError();
            if (d->g_prompt) cudaGraphExecDestroy(d->g_prompt);
            d->g_prompt = nullptr;
            d->coop = false;
            LOG_WARN("decoder: persistent step captured without the cooperative attribute");
            if (capture(d, false, &d->g_prompt, &d->launches_prompt) ||
                capture(d, true, &d->g_gen, &d->launches_gen))
                break;
        }
        bool evs = true;
        for (cudaEvent_t &e : d->ev) evs = evs && cudaEventCreate(&e) == cudaSuccess;
        if (!evs) break;
        ok = true;
    } while (false);
    if (prev >= 0) cudaSetDevice(prev);
    if (!ok) {
        cudaGetLastError();
        sapphire_decoder_destroy(d);
        return nullptr;
    }
    return d;
}

extern "C" SAPPHIRE_API int sapphire_decoder_generate(sapphire_decoder_t *d, const int *prompt, int n_prompt,
                                                      int n_gen, int *out_ids, float *out_margins) {
    if (!d || !prompt || n_prompt < 1 || n_gen < 0 || (n_gen && !out_ids)) {
        LOG_ERROR("sapphire_decoder_generate: bad arguments");
        return -1;
    }
    kernel_context_t *ctx = d->ctx;
    std::lock_guard<std::recursive_mutex> lk(ctx->exec_mutex);
    if (n_prompt + n_gen > d->cfg.context) {
        ctx_fail(ctx, "sapphire_decoder_generate", "prompt %d + generated %d exceed the context %d", n_prompt, n_gen,
                 d->cfg.context);
        return -1;
    }
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= d->cfg.vocab) {
            ctx_fail(ctx, "sapphire_decoder_generate", "prompt token %d out of range", prompt[i]);
            return -1;
        }
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    cudaStream_t st = ctx->stream;
    int rc = -1;
    do {
        if (cudaMemcpyAsync(d->prompt, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) break;
        if (set_state(d, prompt[0], n_prompt, st)) break;
        // Clear the persistent step's abort flag (a step that gave up waiting
        // leaves it set); the launch count stays.
        if (d->persist && cudaMemsetAsync(d->ctl, 0, sizeof(unsigned), st) != cudaSuccess) break;
        if (cudaEventRecord(d->ev[0], st) != cudaSuccess) break;
        bool ok = true;
        for (int i = 0; ok && i + 1 < n_prompt; ++i) ok = cudaGraphLaunch(d->g_prompt, st) == cudaSuccess;
        ok = ok && cudaEventRecord(d->ev[1], st) == cudaSuccess;
        for (int i = 0; ok && i < n_gen; ++i) ok = cudaGraphLaunch(d->g_gen, st) == cudaSuccess;
        ok = ok && cudaEventRecord(d->ev[2], st) == cudaSuccess;
        if (!ok) {
            ctx_fail(ctx, "sapphire_decoder_generate", "graph launch failed: %s", cudaGetErrorString(cudaGetLastError()));
            break;
        }
        if (n_gen) {
            if (cudaMemcpyAsync(out_ids, d->out_tokens, (size_t)n_gen * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
                break;
            if (out_margins &&
                cudaMemcpyAsync(out_margins, d->out_margins, (size_t)n_gen * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
                break;
        }
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) {
            ctx_fail(ctx, "sapphire_decoder_generate", "GPU execution failed: %s", cudaGetErrorString(e));
            break;
        }
        d->epochs += (unsigned)n_gen;
        if (check_kernel_error(ctx, "sapphire_decoder_generate")) break;
        cudaEventElapsedTime(&d->last_prompt_ms, d->ev[0], d->ev[1]);
        cudaEventElapsedTime(&d->last_gen_ms, d->ev[1], d->ev[2]);
        rc = 0;
    } while (false);
    if (rc) cudaGetLastError();
    if (prev >= 0) cudaSetDevice(prev);
    return rc;
}

extern "C" SAPPHIRE_API int sapphire_decoder_last_logits(sapphire_decoder_t *d, float *out) {
    if (!d || !out) return -1;
    std::lock_guard<std::recursive_mutex> lk(d->ctx->exec_mutex);
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d->ctx->device);
    const float *src = d->logits;
    cudaError_t e = cudaSuccess;
    if (d->sharded) {
        // Collective: the slices of every rank, all-gathered (NCCL).
        kernel_context_t *ctx = d->ctx;
        const size_t per = ((size_t)d->cfg.vocab + ctx->world - 1) / ctx->world;
        const DevWeight *head = weight_of(d, d->lm_head);
        float *send = d->logits_all + per * ctx->world;
        e = cudaMemsetAsync(send, 0, per * sizeof(float), ctx->stream);
        if (e == cudaSuccess && head && head->nrows > 0)
            e = cudaMemcpyAsync(send, d->logits, (size_t)head->nrows * sizeof(float), cudaMemcpyDeviceToDevice,
                                ctx->stream);
        if (e == cudaSuccess && shard_allgather(ctx, send, d->logits_all, per, ctx->stream)) e = cudaErrorUnknown;
        src = d->logits_all;
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, src, (size_t)d->cfg.vocab * 4, cudaMemcpyDefault, d->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->ctx->stream);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) {
        ctx_fail(d->ctx, "sapphire_decoder_last_logits", "copy failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" SAPPHIRE_API int sapphire_decoder_last_times(sapphire_decoder_t *d, float *prompt_ms, float *generate_ms) {
    if (!d) return -1;
    if (prompt_ms) *prompt_ms = d->last_prompt_ms;
    if (generate_ms) *generate_ms = d->last_gen_ms;
    return 0;
}

extern "C" SAPPHIRE_API int sapphire_test_decode_stall(int on) { return g_test_decode_stall.exchange(on ? 1 : 0); }

extern "C" SAPPHIRE_API int sapphire_decoder_launches_per_token(sapphire_decoder_t *d) {
    return d ? d->launches_gen : -1;
}

extern "C" SAPPHIRE_API int sapphire_decoder_launches_per_prompt_token(sapphire_decoder_t *d) {
    return d ? d->launches_prompt : -1;
}

// ------------------------------------------------- model from a file ------
// Names as the reference's tensor map (src/loader/gemma3_map.c).
namespace {
const void *st_data(sapphire_safetensors_t *st, const std::string &name, tensor_dtype_t dt, int rows, int cols,
                    kernel_context_t *ctx) {
    tensor_t *t = sapphire_safetensors_tensor(st, name.c_str());
    if (!t) {
        ctx_fail(ctx, "sapphire_decoder_create_from_safetensors", "tensor '%s' missing", name.c_str());
        return nullptr;
    }
    const int *sh = tensor_shape(t);
    if (tensor_dtype(t) != dt || tensor_ndim(t) != 2 || sh[0] != rows || sh[1] != cols) {
        ctx_fail(ctx, "sapphire_decoder_create_from_safetensors", "tensor '%s' is not %s [%d, %d]", name.c_str(),
                 dtype_name(dt), rows, cols);
        return nullptr;
    }
    return tensor_data(t);
}

// A norm vector as fp32 in `out` (zeros when absent); false on a bad tensor.
bool st_norm(sapphire_safetensors_t *st, const std::string &name, int n, std::vector<float> &out,
             kernel_context_t *ctx) {
    out.assign((size_t)n, 0.0f);
    tensor_t *t = sapphire_safetensors_tensor(st, name.c_str());
    if (!t) return true;
    if (tensor_ndim(t) != 1 || tensor_shape(t)[0] != n ||
        (tensor_dtype(t) != DTYPE_F32 && tensor_dtype(t) != DTYPE_BF16)) {
        ctx_fail(ctx, "sapphire_decoder_create_from_safetensors", "norm '%s' is not F32 or BF16 [%d]", name.c_str(),
                 n);
        return false;
    }
    if (tensor_dtype(t) == DTYPE_F32) {
        memcpy(out.data(), tensor_data(t), (size_t)n * sizeof(float));
    } else {
        const uint16_t *b = static_cast<const uint16_t *>(tensor_data(t));
        for (int i = 0; i < n; ++i) {
            const uint32_t bits = (uint32_t)b[i] << 16;
            memcpy(&out[i], &bits, sizeof bits);
        }
    }
    return true;
}
}  // namespace

extern "C" SAPPHIRE_API sapphire_decoder_t *sapphire_decoder_create_from_safetensors(
    kernel_context_t *ctx, const sapphire_gemma3_config_t *cfg, sapphire_safetensors_t *st) {
    if (!ctx || !cfg || !st) {
        LOG_ERROR("NULL argument");
        return nullptr;
    }
    const sapphire_gemma3_config_t &c = *cfg;
    if (c.layers <= 0 || c.hidden <= 0 || c.ffn <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.head_dim <= 0 ||
        c.vocab <= 0) {
        ctx_fail(ctx, "sapphire_decoder_create_from_safetensors", "invalid model shape");
        return nullptr;
    }
    const int qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim;
    std::vector<const void *> proj((size_t)7 * c.layers);
    std::vector<std::vector<float>> norm_store((size_t)6 * c.layers + 1);
    std::vector<const float *> norms((size_t)6 * c.layers);
    for (int l = 0; l < c.layers; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        const struct {
            const char *name;
            int rows, cols;
        } pr[7] = {{"self_attn.q_proj.weight", qd, c.hidden},   {"self_attn.k_proj.weight", kvd, c.hidden},
                   {"self_attn.v_proj.weight", kvd, c.hidden},  {"self_attn.o_proj.weight", c.hidden, qd},
                   {"mlp.gate_proj.weight", c.ffn, c.hidden},   {"mlp.up_proj.weight", c.ffn, c.hidden},
                   {"mlp.down_proj.weight", c.hidden, c.ffn}};
        for (int k = 0; k < 7; ++k)
            if (!(proj[(size_t)7 * l + k] = st_data(st, p + pr[k].name, DTYPE_Q4_0, pr[k].rows, pr[k].cols, ctx)))
                return nullptr;
        const struct {
            const char *name;
            int n;
        } nr[6] = {{"input_layernorm.weight", c.hidden},           {"post_attention_layernorm.weight", c.hidden},
                   {"pre_feedforward_layernorm.weight", c.hidden}, {"post_feedforward_layernorm.weight", c.hidden},
                   {"self_attn.q_norm.weight", c.head_dim},        {"self_attn.k_norm.weight", c.head_dim}};
        for (int k = 0; k < 6; ++k) {
            std::vector<float> &v = norm_store[(size_t)6 * l + k];
            if (!st_norm(st, p + nr[k].name, nr[k].n, v, ctx)) return nullptr;
            norms[(size_t)6 * l + k] = v.data();
        }
    }
    std::vector<float> &final_norm = norm_store.back();
    if (!st_norm(st, "model.norm.weight", c.hidden, final_norm, ctx)) return nullptr;
    const void *embed = st_data(st, "model.embed_tokens.weight", DTYPE_BF16, c.vocab, c.hidden, ctx);
    const void *head = embed ? st_data(st, "lm_head.weight", DTYPE_Q4_0, c.vocab, c.hidden, ctx) : nullptr;
    if (!embed || !head) return nullptr;
    sapphire_gemma3_weights_t w{};
    w.embed_bf16 = static_cast<const uint16_t *>(embed);
    w.lm_head = head;
    w.final_norm = final_norm.data();
    w.proj = proj.data();
    w.norms = norms.data();
    return sapphire_decoder_create(ctx, cfg, &w);
}
