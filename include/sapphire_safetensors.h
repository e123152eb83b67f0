/*
 * sapphire_safetensors.h - safetensors files holding quantized weights.
 *
 * Extends the reference's reader (src/io/safetensors_reader.c:401-449, which
 * accepts F32 / BF16 / F16 only) so Q4_0 / Q8_0 / TQ2_0 weights can be loaded
 * from a file and uploaded at model load.  The container is unchanged: an
 * 8-byte little-endian header length, a JSON header mapping every tensor name
 * to {"dtype", "shape", "data_offsets": [begin, end]} (offsets relative to the
 * data section that follows the header), then the data.  Added dtypes:
 *
 *   "Q4_0", "Q8_0"  rows of the reference's ggml_block_q4_0 / ggml_block_q8_0
 *                   (include/kernels.h), back to back;
 *   "TQ2_0"         rows of this library's ternary format (sapphire_cuda.h);
 *
 * "shape" is the logical [rows, cols] and the payload must hold exactly
 * rows * sapphire_row_bytes(dtype, cols) bytes.  "__metadata__" is ignored.
 * The file is memory-mapped; tensors are zero-copy tensor_t views owned by
 * the handle (do not release them; they live until sapphire_safetensors_close).
 */
#ifndef SAPPHIRE_SAFETENSORS_H
#define SAPPHIRE_SAFETENSORS_H

#include "kernels.h"
#include "tensor.h"
#include "sapphire_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

#define SAPPHIRE_ST_MAX_DIMS 8

typedef struct sapphire_safetensors sapphire_safetensors_t;

/** Map a file and parse its header; NULL (with a logged reason) on a missing
 *  file, a malformed header, an unknown dtype or a payload whose size does
 *  not match its dtype and shape. */
SAPPHIRE_API sapphire_safetensors_t *sapphire_safetensors_open(const char *path);
/** Tensors in the file (-1 for NULL). */
SAPPHIRE_API int sapphire_safetensors_count(const sapphire_safetensors_t *st);
/** Name of tensor `index` in header order, NULL when out of range. */
SAPPHIRE_API const char *sapphire_safetensors_name(const sapphire_safetensors_t *st, int index);
/** View of a tensor's bytes in the mapping (owned by st), NULL if absent. */
SAPPHIRE_API tensor_t *sapphire_safetensors_tensor(sapphire_safetensors_t *st, const char *name);
SAPPHIRE_API void sapphire_safetensors_close(sapphire_safetensors_t *st);

/** A Gemma-3 decoder from a quantized file, with the reference's tensor names
 *  (src/loader/gemma3_map.c): model.embed_tokens.weight (BF16 [vocab, hidden]),
 *  model.layers.L.self_attn.{q,k,v,o}_proj.weight and
 *  model.layers.L.mlp.{gate,up,down}_proj.weight (Q4_0), lm_head.weight (Q4_0
 *  [vocab, hidden]; the reference ties it to the embedding, which it reads as
 *  BF16 - here it must be a Q4_0 tensor), and the norms
 *  model.layers.L.{input_layernorm, post_attention_layernorm,
 *  pre_feedforward_layernorm, post_feedforward_layernorm}.weight,
 *  model.layers.L.self_attn.{q,k}_norm.weight, model.norm.weight (F32 or BF16;
 *  absent means zeros).  Shapes are checked against cfg.  Everything is copied
 *  to the context's GPU; the file may be closed afterwards.  NULL on error. */
SAPPHIRE_API sapphire_decoder_t *sapphire_decoder_create_from_safetensors(kernel_context_t *ctx,
                                                                          const sapphire_gemma3_config_t *cfg,
                                                                          sapphire_safetensors_t *st);

#ifdef __cplusplus
}
#endif

#endif /* SAPPHIRE_SAFETENSORS_H */
