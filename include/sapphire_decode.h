/*
 * sapphire_decode.h - device-resident Gemma-3 decoder built on the GEMV path.
 *
 * No single reference function has this signature: it replaces the decode
 * loop the reference runs on the host - inference_session_create
 * (src/inference/inference.c:499-584), one inference_forward per token
 * (inference.c:612-651, src/transformer/transformer.c:318-345,
 * src/transformer/attention.c:311-375), the LM head (transformer.c:393-408)
 * and sample_greedy (src/utils/utils.c:145-156) - with the same arithmetic,
 * kept on one GPU: every projection is a Q4_0 GEMV of the library, the norms,
 * QK-norm, RoPE, attention over the KV cache, GeGLU and the greedy argmax are
 * kernels, and one token's whole step is a CUDA graph, so a token costs no
 * host round trip.
 *
 * When the model fits it (any Gemma-3 shape whose products have at least one
 * row per SM and whose per-SM slices fit shared memory), all layers of a
 * token run as ONE persistent kernel, one block per SM, whose stages wait for
 * each other's outputs through epoch-tagged words in global memory; a
 * generated token adds the LM-head GEMV and the argmax (3 kernels).
 * Otherwise - or with the environment variable SAPPHIRE_DECODE_PERSISTENT=0
 * at creation - each stage is its own kernel (5 per layer).  Both give the
 * reference's greedy ids.
 */
#ifndef SAPPHIRE_DECODE_H
#define SAPPHIRE_DECODE_H

#include <stdint.h>

#include "kernels.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct sapphire_decoder sapphire_decoder_t;

/* Model shape (the fields of gemma3_270m_config_t the decode uses). */
typedef struct {
    int layers, hidden, ffn, heads, kv_heads, head_dim, vocab;
    int context;          /* KV-cache length (max positions) */
    int sliding_window;   /* local layers attend to the last `sliding_window` positions */
    float rope_theta;     /* global layers */
    float rope_local_theta;
    float query_pre_attn_scalar;   /* scores scaled by 1/sqrt(this) */
    float rms_eps;
    /* Layer l uses global attention iff bit l of global_mask is set; with a
     * zero mask, iff (l + 1) % 6 == 0 (the reference's 5:1 default). */
    unsigned long long global_mask;
} sapphire_gemma3_config_t;

/* Host weights; they are copied to the GPU by sapphire_decoder_create. */
typedef struct {
    const uint16_t *embed_bf16;   /* [vocab][hidden] bf16 bit patterns, scaled by sqrt(hidden) on lookup */
    const void *lm_head;          /* Q4_0 rows [vocab][hidden] */
    const float *final_norm;      /* [hidden], NULL = zeros ((1 + w) RMSNorm) */
    /* [layers * 7] Q4_0 rows: q [heads*head_dim][hidden], k, v [kv_heads*head_dim][hidden],
     * o [hidden][heads*head_dim], gate, up [ffn][hidden], down [hidden][ffn]. */
    const void *const *proj;
    /* [layers * 6] or NULL: attn, attn_post, ffn, ffn_post [hidden], q_norm, k_norm [head_dim];
     * a NULL entry means zeros. */
    const float *const *norms;
} sapphire_gemma3_weights_t;

/** Upload a model and allocate the KV cache on the context's GPU.  NULL on error
 *  (message in kernel_ctx_last_error).  On a sharded context
 *  (kernel_ctx_init_sharded) every rank holds the whole model except the LM
 *  head, whose rows are sharded: each rank computes its slice of the logits
 *  and the ranks agree on the greedy token by exchanging 8-byte (value,
 *  index) words over peer memory instead of gathering the logits.  Then
 *  create, generate and last_logits are collective: every rank calls them in
 *  the same order with the same arguments. */
SAPPHIRE_API sapphire_decoder_t *sapphire_decoder_create(kernel_context_t *ctx, const sapphire_gemma3_config_t *cfg,
                                                         const sapphire_gemma3_weights_t *w);
/** Greedy generation as the reference's perform_inference orders it
 *  (inference.c:238-325): prompt[0..n_prompt-2] fill the KV cache at
 *  positions 0..n_prompt-2, then prompt[n_prompt-1] at position n_prompt-1
 *  starts n_gen greedy steps.  out_ids receives the generated ids; out_margins
 *  (may be NULL) the top-1 minus top-2 logit of each step.  The cache is reset
 *  first.  n_prompt + n_gen must not exceed the context.  0 / -1. */
SAPPHIRE_API int sapphire_decoder_generate(sapphire_decoder_t *d, const int *prompt, int n_prompt, int n_gen,
                                           int *out_ids, float *out_margins);
/** Logits of the last generated step ([vocab] floats, host or device pointer);
 *  on a sharded decoder the ranks' slices are all-gathered (NCCL) first. */
SAPPHIRE_API int sapphire_decoder_last_logits(sapphire_decoder_t *d, float *out);
/** Device time in milliseconds of the prompt and generation phases of the last
 *  sapphire_decoder_generate (CUDA events on the context stream). */
SAPPHIRE_API int sapphire_decoder_last_times(sapphire_decoder_t *d, float *prompt_ms, float *generate_ms);
/** Kernel launches of one generated token (graph nodes). */
SAPPHIRE_API int sapphire_decoder_launches_per_token(sapphire_decoder_t *d);
/** Kernels a prompt token's step launches (no LM head, no argmax). */
SAPPHIRE_API int sapphire_decoder_launches_per_prompt_token(sapphire_decoder_t *d);
SAPPHIRE_API void sapphire_decoder_destroy(sapphire_decoder_t *d);

/** Test hook (no reference counterpart): on != 0 makes decoders created
 *  afterwards run a persistent step in which one block withholds its layer-0
 *  q / k / v rows and every wait is limited to 1 ms, so the step's bounded
 *  waits run out without any GPU fault; creation then fails with the expiry
 *  in kernel_ctx_last_error and the context stays usable.  Returns the
 *  previous setting.  Process-wide. */
SAPPHIRE_API int sapphire_test_decode_stall(int on);

#ifdef __cplusplus
}
#endif

#endif /* SAPPHIRE_DECODE_H */
