/*
 * sapphire_cuda.h - entry points of libsapphire_cuda.so that the reference
 * API does not have.  None of them replaces a reference function; each one
 * extends the reference boundary (include/kernels.h) in the direction the
 * reference's own design notes point to: device-resident weights uploaded at
 * model load, an asynchronous device-pointer path, row sharding over several
 * GPUs, quantisers, and the ternary format.
 *
 * All pointers are plain C pointers.  Where a pointer may be either host or
 * device memory the function says so; the library tells them apart with
 * cudaPointerGetAttributes.  Streams are passed as void* (a cudaStream_t).
 * Return convention: 0 on success, -1 on error (details via LOG_ERROR and
 * kernel_ctx_last_error), as in the reference's kernel_gemv.
 */
#ifndef SAPPHIRE_CUDA_H
#define SAPPHIRE_CUDA_H

#include <stddef.h>
#include <stdint.h>
#include "kernels.h"
#include "tensor.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------- *
 * Ternary format (DTYPE_TQ2_0).  No reference counterpart: the reference has
 * no ternary code.  A packed row is
 *     float scale;  sapphire_block_tq2_0 blocks[ceil(cols/32)];
 * (4 + 8*ceil(cols/32) bytes, rows stored back to back).  Trit j of a block is
 * the 2-bit code c = t + 1 (t in {-1, 0, +1}, c in {0, 1, 2}) at bits
 * 2*(j%4) .. 2*(j%4)+1 of byte j/4.  Weight = t * scale, decoded as c - 1.
 * ------------------------------------------------------------------------- */
typedef struct {
    uint8_t q_data[8];
} sapphire_block_tq2_0;

/** One ternary row dot product (row = fp32 scale + block_count blocks); host
 *  pointers, computed on the GPU like the other row-kernel entry points.
 *  block_size must be 32 (0.0f otherwise). */
SAPPHIRE_API float quantized_gemv_tq2_0(const void *W_row, const float *x, int block_count, int block_size);

/** Bytes of one packed host row of `cols` columns: Q4_0 20*nb, Q8_0 36*nb,
 *  TQ2_0 4+8*nb (nb = ceil(cols/32)), F32 4*cols, BF16/F16 2*cols. */
SAPPHIRE_API size_t sapphire_row_bytes(tensor_dtype_t dtype, int cols);

/* ------------------------------------------------------------------------- *
 * Device residency.  Extends the reference's weight handling (weights are
 * host views, src/tensor/tensor.c:133-152, read by every kernel_gemv call):
 * here a weight is copied to the context's GPU once, re-laid out for
 * coalesced streaming, and reused until evicted, destroyed or released.
 * A weight whose host bytes change after upload must be evicted by the caller.
 * ------------------------------------------------------------------------- */

/** Upload (and re-lay out) A now instead of at its first GEMV.  Idempotent. */
SAPPHIRE_API int kernel_tensor_upload(kernel_context_t *ctx, const tensor_t *A);
/** Drop the device copy of A, if any. */
SAPPHIRE_API int kernel_tensor_evict(kernel_context_t *ctx, const tensor_t *A);
/** Bytes of device memory held by resident weights of this context. */
SAPPHIRE_API size_t kernel_ctx_resident_bytes(kernel_context_t *ctx);

/* ------------------------------------------------------------------------- *
 * Asynchronous device path.  y / x / Y / X are device pointers on the
 * context's GPU; work is enqueued on the context stream and the call returns
 * without waiting.  Ordering is the stream's: a later call on the same
 * context, or kernel_ctx_synchronize, sees the result.
 * ------------------------------------------------------------------------- */
SAPPHIRE_API int kernel_gemv_device(kernel_context_t *ctx, float *y, const tensor_t *A, const float *x);
/** Y[b*rows + r] = A[r,:] . X[b*cols ..] for b < batch_size (device pointers).
 *  A Q4_0 weight with batch_size >= 16 (here and in kernel_gemm) runs the
 *  tensor-core prefill product: activations rounded to bf16 (nearest even),
 *  weights dequantised exactly, fp32 accumulation - unless the context keeps
 *  fp32 products (kernel_ctx_set_fp32_products). */
SAPPHIRE_API int kernel_gemm_device(kernel_context_t *ctx, float *Y, const tensor_t *A, const float *X, int batch_size);
/** Tensor-core prefill product from bf16 activations already on the device
 *  (no counterpart in the reference, whose Q4_0 kernel_gemm returns -1):
 *  Y[b*rows + r] = A[r,:] . Xb[b*x_stride ..] for b < batch_size.  A: Q4_0.
 *  Xb: bf16 values, 16-byte aligned, x_stride a multiple of 8 and at least
 *  32 * ceil(cols / 32), zero from column `cols` to the end of the last
 *  block.  Unsharded contexts only.  Asynchronous like kernel_gemm_device. */
SAPPHIRE_API int kernel_gemm_device_bf16(kernel_context_t *ctx, float *Y, const tensor_t *A, const void *Xb,
                                         int batch_size, int x_stride);
/** Batch-1 y = A @ x like kernel_gemv_device, for callers that must not
 *  allocate device memory when they multiply (a serving loop with a fixed
 *  memory budget or pool, or a path where an allocation's implicit device
 *  synchronisation would stall other work).  No counterpart in the reference.
 *  Calls no cudaMalloc / cudaFree: A must already be resident
 *  (kernel_tensor_upload, which allocates, at model load); y and x are device
 *  pointers on the context's GPU; the work is enqueued on the context stream.
 *  Scratch is a fixed 4 MiB device array inside the library, held by every
 *  GPU that loads it until exit.  The scratch grows with the row count (about
 *  260 bytes per 32 rows for Q8_0 / Q4_0 and twice that for TQ2_0 at 640
 *  columns: the 262144-row Q8_0 LM head needs 2.1 MB); a weight that needs
 *  more than 4 MiB is rejected with -1 and an error message.  The first call
 *  on a device looks up the array's device address, so make that call before
 *  any stream capture.  All calls share the array and it keeps the last
 *  call's contents (each call clears what must start at zero): calls that
 *  overlap on the GPU, from any context or stream, race.  A kernel error (an
 *  expired bounded wait) is recorded in the context's error word and returned
 *  as -1 by the next kernel_ctx_synchronize.  Not for sharded contexts. */
SAPPHIRE_API int kernel_gemv_device_noalloc(kernel_context_t *ctx, float *y, const tensor_t *A, const float *x);
/** Waits for the context stream; -1 if it failed or if a kernel enqueued by
 *  an asynchronous call since the last check reported an expired bounded
 *  wait (details via kernel_ctx_last_error). */
SAPPHIRE_API int kernel_ctx_synchronize(kernel_context_t *ctx);
/** The context's cudaStream_t (as void*). */
SAPPHIRE_API void* kernel_ctx_get_stream(kernel_context_t *ctx);
/** Use an external stream (void* cudaStream_t, NULL = legacy default stream). */
SAPPHIRE_API int kernel_ctx_set_stream(kernel_context_t *ctx, void *stream);
/** CUDA ordinal the context is bound to, -1 for NULL. */
SAPPHIRE_API int kernel_ctx_get_device(kernel_context_t *ctx);
/** Choose the GPU of a context before kernel_ctx_init (default: the calling
 *  thread's current device at kernel_ctx_create).  -1 after init or when the
 *  device does not exist. */
SAPPHIRE_API int kernel_ctx_set_device(kernel_context_t *ctx, int device);
/** on != 0: batched Q4_0 products of this context (kernel_gemm,
 *  kernel_gemm_device) keep fp32 activations - one fp32 row product per
 *  activation row, the reference's arithmetic - instead of the bf16
 *  tensor-core product from batch 16 on.  Off by default.  No reference
 *  counterpart (the reference's Q4_0 kernel_gemm returns -1).  0, or -1 for
 *  a NULL context. */
SAPPHIRE_API int kernel_ctx_set_fp32_products(kernel_context_t *ctx, int on);
/** Message of the last error recorded on the context ("" if none). */
SAPPHIRE_API const char* kernel_ctx_last_error(kernel_context_t *ctx);

/** Pinned host memory (cudaHostAlloc) for activation buffers, so host-pointer
 *  GEMV calls copy without a driver staging pass. */
SAPPHIRE_API void* kernel_host_alloc(size_t bytes);
SAPPHIRE_API void kernel_host_free(void *p);

/* ------------------------------------------------------------------------- *
 * Quantisers and unpackers (run on the context's GPU).  src / dst may be host
 * or device pointers.  No reference counterpart: the reference ships no
 * quantiser (its tensor_get_f32 dequant is a stub, src/tensor/tensor.c:238-244).
 *  Q4_0 block:  m = element of largest |x| (first one on ties), d = m / -8,
 *               id = d ? 1/d : 0, q = min(15, trunc(x*id + 8.5)) (NaN -> 0).
 *  Q8_0 block:  a = max |x|, d = a / 127, id = d ? 1/d : 0,
 *               q = clamp(round_half_away(x*id), -127, 127) (NaN -> 0).
 *  Columns past `cols` in the last block quantise as zeros.
 * ------------------------------------------------------------------------- */
SAPPHIRE_API int kernel_quantize_q4_0(kernel_context_t *ctx, void *dst, const float *src, int rows, int cols);
SAPPHIRE_API int kernel_quantize_q8_0(kernel_context_t *ctx, void *dst, const float *src, int rows, int cols);
/** Pack trits (int8 in {-1,0,1}, row-major [rows, cols]) and per-row scales
 *  into TQ2_0 rows.  Values outside {-1,0,1} are an error. */
SAPPHIRE_API int kernel_pack_tq2_0(kernel_context_t *ctx, void *dst, const int8_t *trits, const float *row_scales, int rows, int cols);
/** Unpack a quantized or dense 2-D tensor to fp32 [rows, cols] (dst host or device). */
SAPPHIRE_API int kernel_dequantize(kernel_context_t *ctx, float *dst, const tensor_t *A);

/* ------------------------------------------------------------------------- *
 * Row sharding over several GPUs (one process per GPU).  No reference
 * counterpart: the reference is single-process CPU code.
 * Rank r of W owns rows [r*ceil(R/W), min(R, (r+1)*ceil(R/W))); kernel_gemv on
 * a sharded context computes its slice and all-gathers the full y with NCCL.
 * ------------------------------------------------------------------------- */
#define SAPPHIRE_UNIQUE_ID_BYTES 128
/** Fill id_out (SAPPHIRE_UNIQUE_ID_BYTES bytes) with a new NCCL unique id;
 *  rank 0 calls it and the caller broadcasts the bytes to every rank. */
SAPPHIRE_API int kernel_shard_unique_id(void *id_out);
/** Join the sharded group (after kernel_ctx_init).  world_size 1 is a no-op. */
SAPPHIRE_API int kernel_ctx_init_sharded(kernel_context_t *ctx, int rank, int world_size, const void *unique_id);
/** This context's rank and world size (0 / 1 when not sharded). */
SAPPHIRE_API int kernel_ctx_shard_info(kernel_context_t *ctx, int *rank, int *world_size);
/** Rows [*row0, *row0 + *nrows) of a `rows`-row weight owned by `rank` of
 *  `world_size` (the rule above; *nrows may be 0 for trailing ranks).
 *  Pure arithmetic, no GPU.  0 on success, -1 on bad arguments. */
SAPPHIRE_API int sapphire_shard_rows(int rows, int rank, int world_size, int *row0, int *nrows);

/* ------------------------------------------------------------------------- *
 * Test hooks for the bounded-wait error paths.  No reference counterpart
 * (the reference has no device waits).  They make a wait run out without any
 * GPU fault - a barrier or a flag that nothing sets - so tests can check that
 * the error is reported and the context stays usable.
 * ------------------------------------------------------------------------- */
/** on != 0: the following quantized batch-1 GEMV launches (kernel_gemv,
 *  kernel_gemv_device, kernel_gemv_device_noalloc) give one consumer warp a
 *  shared-memory slot that no copy fills and a short wait limit; the call (or
 *  the next kernel_ctx_synchronize) returns -1.  on = 0 restores normal
 *  launches.  Process-wide. */
SAPPHIRE_API int sapphire_test_stream_unarmed(int on);
/** Runs the peer-gather pull of a sharded product over a local buffer of
 *  `rows` words that nothing writes, with a wait limit of wait_ns
 *  nanoseconds: y (device, `rows` floats) receives NaN and the call returns -1
 *  with the expiry recorded in kernel_ctx_last_error. */
SAPPHIRE_API int sapphire_test_pull_expiry(kernel_context_t *ctx, float *y, long long rows,
                                           unsigned long long wait_ns);

#ifdef __cplusplus
}
#endif

#endif /* SAPPHIRE_CUDA_H */
