/*
 * decode_ref.c - test-side harness that runs the reference's own Gemma-3
 * decode (its inference session, transformer layers, attention, KV cache and
 * Q4_0 kernel_gemv, compiled unmodified into oracle/_ref/libsapphire_ref.so)
 * on a random-init model held in memory.  It is the oracle of the decode
 * workload: tests compare the GPU decoder's greedy token ids with its output,
 * and bench.py times it as the CPU baseline.  Never linked by the product.
 *
 * What it drives (reference files):
 *   - inference_session_create (src/inference/inference.c:499-584) with a
 *     model_spec_t whose llm_model / variant_config are filled here;
 *   - inference_forward (inference.c:612-651), one token at a time for the
 *     prompt, following the position convention of perform_inference
 *     (inference.c:238-255): positions 0..n-2 prefill, then the last prompt
 *     token at position n-1 starts generation;
 *   - the LM head as in lm_head (src/transformer/transformer.c:393-408):
 *     rmsnorm_delta with the final norm weights, then kernel_gemv, but with a
 *     separate Q4_0 head, because the reference's embedding lookup reads the
 *     embedding table as BF16 (transformer.c:367-380) and its tied head would
 *     be a BF16 GEMV;
 *   - sample_greedy (src/utils/utils.c:145-156).
 * Norm weights are zero (Gemma's (1 + w) RMSNorm: scale 1), q_norm / k_norm
 * have head_dim entries (broadcast over heads, attention.c:228-269), and
 * layer_types_mask = 0 selects the 5:1 local/global pattern
 * (src/transformer/layer_config_loader.c:6-16).
 */
#define _POSIX_C_SOURCE 200809L
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "gemma3_270m_config.h"
#include "inference.h"
#include "kernels.h"
#include "llm_model.h"
#include "model_spec.h"
#include "tensor.h"
#include "utils.h"

#define EXPORT __attribute__((visibility("default")))

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

static tensor_t *view2(tensor_dtype_t dt, int rows, int cols, const void *data) {
    int shape[2] = {rows, cols};
    return tensor_create_view(dt, 2, shape, (void *)data);
}

static tensor_t *view1(int n, const float *data) {
    int shape[1] = {n};
    return tensor_create_view(DTYPE_F32, 1, shape, (void *)data);
}

/*
 * weights: n_layers * 7 pointers to packed Q4_0 rows, per layer in the order
 * q [heads*head_dim, hidden], k, v [kv_heads*head_dim, hidden],
 * o [hidden, heads*head_dim], gate, up [ffn, hidden], down [hidden, ffn].
 * Outputs: out_tokens / out_margin (top-1 minus top-2 logit) per generated
 * token, out_logits0 (vocab floats, may be NULL) of the first generated step,
 * and the wall time of the prompt and generation phases.
 * Returns 0, or -1 on a setup failure.
 */
EXPORT int decode_ref_run(const int *prompt, int n_prompt, int n_gen, const uint16_t *embed_bf16,
                          const void *const *weights, const void *lm_head_q4, int n_layers, int hidden, int ffn,
                          int heads, int kv_heads, int head_dim, int vocab, int context, int sliding_window,
                          int *out_tokens, float *out_margin, float *out_logits0, double *out_prefill_s,
                          double *out_decode_s) {
    if (!prompt || n_prompt < 1 || n_gen < 0 || !embed_bf16 || !weights || !lm_head_q4 ||
        n_layers <= 0 || n_layers > SAPPHIRE_MAX_LAYERS || n_prompt + n_gen > context)
        return -1;
    int rc = -1;
    gemma3_270m_config_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.attn_logit_softcapping = NAN;
    cfg.final_logit_softcapping = NAN;
    cfg.rope_scaling = NAN;
    cfg.head_dim = head_dim;
    cfg.hidden_size = hidden;
    cfg.intermediate_size = ffn;
    cfg.layer_types_mask = 0;
    cfg.layer_types_count = n_layers;
    cfg.max_position_embeddings = context;
    cfg.num_attention_heads = heads;
    cfg.num_hidden_layers = n_layers;
    cfg.num_key_value_heads = kv_heads;
    cfg.query_pre_attn_scalar = (float)head_dim;
    cfg.rms_norm_eps = 1e-6f;
    cfg.rope_local_base_freq = 10000.0f;
    cfg.rope_theta = 1000000.0f;
    cfg.sliding_window = sliding_window;
    cfg.vocab_size = vocab;
    cfg.sliding_window_pattern = 6;

    const int q_dim = heads * head_dim, kv_dim = kv_heads * head_dim;
    float *zeros = calloc((size_t)(hidden > q_dim ? hidden : q_dim) + 64, sizeof(float));
    float *hidden_norm = aligned_alloc(32, ((size_t)hidden + 64) * sizeof(float));
    float *logits = malloc((size_t)vocab * sizeof(float));
    model_layer_weights_t *layers = calloc((size_t)n_layers, sizeof *layers);
    llm_model_t model;
    memset(&model, 0, sizeof model);
    model_spec_t spec;
    memset(&spec, 0, sizeof spec);
    inference_session_t *s = NULL;
    tensor_t *lm_head = NULL, *final_norm = NULL;
    if (!zeros || !hidden_norm || !logits || !layers) goto out;

    model.embedding_weight = view2(DTYPE_BF16, vocab, hidden, embed_bf16);
    final_norm = view1(hidden, zeros);
    model.norm_final_weight = final_norm;
    lm_head = view2(DTYPE_Q4_0, vocab, hidden, lm_head_q4);
    model.lm_head_weight = lm_head;
    model.layers = layers;
    for (int l = 0; l < n_layers; ++l) {
        const void *const *w = weights + 7 * l;
        model_layer_weights_t *L = &layers[l];
        L->norm_attn_weight = view1(hidden, zeros);
        L->norm_attn_post_weight = view1(hidden, zeros);
        L->norm_ffn_weight = view1(hidden, zeros);
        L->norm_ffn_post_weight = view1(hidden, zeros);
        L->q_norm_weight = view1(head_dim, zeros);
        L->k_norm_weight = view1(head_dim, zeros);
        L->q_proj_weight = view2(DTYPE_Q4_0, q_dim, hidden, w[0]);
        L->k_proj_weight = view2(DTYPE_Q4_0, kv_dim, hidden, w[1]);
        L->v_proj_weight = view2(DTYPE_Q4_0, kv_dim, hidden, w[2]);
        L->out_proj_weight = view2(DTYPE_Q4_0, hidden, q_dim, w[3]);
        L->gate_proj_weight = view2(DTYPE_Q4_0, ffn, hidden, w[4]);
        L->up_proj_weight = view2(DTYPE_Q4_0, ffn, hidden, w[5]);
        L->down_proj_weight = view2(DTYPE_Q4_0, hidden, ffn, w[6]);
    }
    spec.model_id = "gemma3-270m-random-init";
    spec.llm_model = &model;
    spec.variant_config = &cfg;

    s = inference_session_create(&spec, context);
    if (!s) goto out;

    double t0 = now_s();
    for (int p = 0; p + 1 < n_prompt; ++p) inference_forward(s, prompt[p], p, NULL);
    double t1 = now_s();
    int last = prompt[n_prompt - 1];
    for (int g = 0; g < n_gen; ++g) {
        const int pos = n_prompt - 1 + g;
        inference_forward(s, last, pos, NULL);
        rmsnorm_delta(hidden_norm, s->scratch_buffer, zeros, 1e-6f, hidden);
        if (kernel_gemv(s->gemv_ctx, logits, lm_head, hidden_norm) != 0) goto out;
        const int tok = sample_greedy(logits, vocab);
        float second = -FLT_MAX;
        for (int i = 0; i < vocab; ++i)
            if (i != tok && logits[i] > second) second = logits[i];
        out_tokens[g] = tok;
        if (out_margin) out_margin[g] = logits[tok] - second;
        if (g == 0 && out_logits0) memcpy(out_logits0, logits, (size_t)vocab * sizeof(float));
        last = tok;
    }
    double t2 = now_s();
    if (out_prefill_s) *out_prefill_s = t1 - t0;
    if (out_decode_s) *out_decode_s = t2 - t1;
    rc = 0;
out:
    if (s) destroy_inference_session(s);
    if (layers) {
        for (int l = 0; l < n_layers; ++l) {
            tensor_t **fields[] = {&layers[l].norm_attn_weight, &layers[l].norm_attn_post_weight,
                                   &layers[l].norm_ffn_weight, &layers[l].norm_ffn_post_weight,
                                   &layers[l].q_norm_weight, &layers[l].k_norm_weight, &layers[l].q_proj_weight,
                                   &layers[l].k_proj_weight, &layers[l].v_proj_weight, &layers[l].out_proj_weight,
                                   &layers[l].gate_proj_weight, &layers[l].up_proj_weight,
                                   &layers[l].down_proj_weight};
            for (size_t f = 0; f < sizeof fields / sizeof fields[0]; ++f)
                if (*fields[f]) tensor_release(*fields[f]);
        }
        free(layers);
    }
    if (model.embedding_weight) tensor_release(model.embedding_weight);
    if (final_norm) tensor_release(final_norm);
    if (lm_head) tensor_release(lm_head);
    free(zeros);
    free(hidden_norm);
    free(logits);
    return rc;
}
