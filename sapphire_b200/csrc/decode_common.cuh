// decode_common.cuh - pieces shared by the two decode step implementations
// (decode.cu: one kernel per stage; decode_persistent.cu: one persistent
// kernel per token).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

constexpr int kMaxGroup = 8;          // query heads per KV head
constexpr int kMaxHeads = 32;
constexpr int kMaxHeadDim = 256;
constexpr int kMaxContext = 4096;

// Device-side step state.
struct DecState {
    int pos;            // position of the token being processed
    int cur_token;      // token being processed
    int prompt_index;   // index of cur_token in the prompt during the prompt phase
    int n_prompt;
    int gen_index;      // next output slot
    unsigned epoch;     // sharded LM head: generated steps so far (tag of the exchange words)
};

// Error bits of the context's error word set by the decode kernels.
constexpr int kErrToken = 4;          // a token id outside the vocabulary
constexpr int kErrStepWait = 16;     // a persistent step gave up waiting for another CTA's output

#ifdef __CUDACC__
static __device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
static __device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Sum over the block (blockDim.x a multiple of 32, at most 1024); every thread
// receives the result.  `red` holds 32 floats.
static __device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.0f;
    return warp_sum(t);
}

// rmsnorm_delta of one head (hd values at x, written by an earlier kernel or
// an earlier stage of this one, hence L2 loads) then the half-split rotation
// (rope_apply_fast, src/transformer/rope.c:65-80), by one warp; lane owns the
// pairs (i, i + hd/2) for i = lane + 32 j.
static __device__ __forceinline__ void warp_norm_rope(const float *x, const float *w, float eps, const float *cs,
                                                      const float *sn, int hd, float *dst) {
    const int lane = threadIdx.x & 31, half = hd >> 1;
    float a[kMaxHeadDim / 64], b[kMaxHeadDim / 64];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxHeadDim / 64; ++j) {
        const int i = lane + 32 * j;
        a[j] = i < half ? __ldcg(x + i) : 0.0f;
        b[j] = i < half ? __ldcg(x + i + half) : 0.0f;
        ss += a[j] * a[j] + b[j] * b[j];
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)hd + eps);
#pragma unroll
    for (int j = 0; j < kMaxHeadDim / 64; ++j) {
        const int i = lane + 32 * j;
        if (i < half) {
            const float y0 = (a[j] * r) * (1.0f + (w ? w[i] : 0.0f));
            const float y1 = (b[j] * r) * (1.0f + (w ? w[i + half] : 0.0f));
            const float c = cs[i], sv = sn[i];
            dst[i] = y0 * c - y1 * sv;
            dst[i + half] = y1 * c + y0 * sv;
        }
    }
}

// GeGLU of the reference (src/transformer/activations.c:64-82): tanh form of gelu(x), times u.
static __device__ __forceinline__ float geglu_tanh(float x, float u) {
    const float y = 0.7978845608f * (x + 0.044715f * x * x * x);
    return (0.5f * x * (1.0f + tanhf(y))) * u;
}
#endif

// ------------------------------------------------ persistent decode step --
// Stages of a layer in the persistent kernel's weight layout.
enum PersistStage : int { kStQkv = 0, kStO = 1, kStGu = 2, kStDown = 3, kNumStages = 4 };

// Everything one launch of the persistent step reads (decode_persistent.cu).
struct PersistParams {
    DecState *st;
    const int *prompt;
    int generate;                 // 1: leave the final norm in norm_out; 0: advance the prompt state
    int layers, hidden, ffn, heads, kv_heads, hd, context, window, vocab;
    float eps, emb_scale, att_scale;
    const uint16_t *embed;        // bf16 [vocab][hidden]
    // Projections in the row layout: row r of a stage is row_stride bytes,
    // nb 16-byte code groups (the Q4_0 blocks' code bytes in order) then nb
    // fp32 scales; stage s of layer l starts at wrows + l * layer_bytes + stage_off[s].
    const uint8_t *wrows;
    unsigned long long layer_bytes;
    unsigned long long stage_off[kNumStages];
    int stage_rows[kNumStages], stage_nb[kNumStages], stage_stride[kNumStages];
    // Norm weights, per layer norm_stride floats: attn, attn_post, ffn,
    // ffn_post (hidden each), q, k (hd each).
    const float *norms;
    int norm_stride;
    const float *w_final;
    unsigned long long global_mask;   // bit l: layer l attends globally (layers <= 64)
    const float *rope_cos_g, *rope_sin_g, *rope_cos_l, *rope_sin_l;
    float *kcache, *vcache;       // [layers][kv_heads][context][hd]
    // Stage outputs as epoch-tagged words (epoch << 32 | fp32 bits): a
    // consumer polls the words it needs until they carry the stage's epoch.
    // o_out, gu and down_out, which every CTA reads, are written in
    // kPersistReplicas copies ([replica][row]); CTA c polls copy c % kPersistReplicas.
    unsigned long long *qkv, *o_out, *gu, *down_out;
    // gu holds gelu_tanh(gate) * up (ffn words per copy): the GU stage's rows
    // are gate / up pairs (row 2i = gate row i, 2i + 1 = up row i).
    // Attention partials per split and head, part[(b * heads + h)]: [m word,
    // l word, acc (hd floats)] (the m / l words are tagged and stored with
    // release after acc).  The O product is split by head: stage O's row
    // h * hidden + r is row r of Wo restricted to head h's columns, and the
    // residual adds the heads' partial rows in head order.
    float *part;
    float *norm_out;              // the LM head's input (plain floats)
    // Attention: CTA c works for query head c / splits on split c % splits;
    // a window of len keys is cut into splits of max(chunk, ceil(len / splits))
    // keys (at most chunk_max, what the key buffers hold).
    int chunk, chunk_max, splits;
    unsigned *ctl;                // [0] abort flag, [1] launches so far (never cleared: the epoch base)
    int *err;
    unsigned long long wait_ns;   // bound of every wait
    int test_stall;               // test hook: the last CTA withholds its layer-0 qkv rows
    // Dynamic shared-memory offsets (bytes).
    unsigned off_w[kNumStages], off_k, off_v, off_hidden, off_x, off_q, off_kcur, off_vcur, off_sc;
    unsigned off_nrm[2], off_rope, off_acc, off_vin;
};

// Host side (decode_persistent.cu).
constexpr int kPersistThreads = 512;
constexpr int kPersistReplicas = 8;
struct PersistPlan {
    bool ok = false;
    int grid = 0, chunk = 0;
    size_t smem = 0;
    size_t part_floats = 0;
};
// Shared-memory plan of the persistent step for a model; ok = false (with the
// reason in *why) when the model does not fit it.
PersistPlan persist_plan(int device, const PersistParams &shape, const char **why);
// Fills p's shared-memory offsets from the plan.
void persist_layout(const PersistPlan &plan, PersistParams &p);
cudaError_t launch_persist(const PersistPlan &plan, const PersistParams &p, bool cooperative, cudaStream_t st);
