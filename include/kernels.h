/*
 * kernels.h - GEMV entry points of the B200 library (libsapphire_cuda.so).
 *
 * Drop-in for the reference header include/kernels.h.  Every declaration
 * marked SAPPHIRE_API keeps the reference's name, signature and return
 * convention, and is exported by libsapphire_cuda.so.  The GEMV work behind
 * kernel_gemv / kernel_gemm / kernel_gemv_* runs on the GPU (sm_100a kernels);
 * there is no CPU fallback on that path.
 *
 * The activation / normalisation / vector helpers at the end are declared for
 * source compatibility only: in the reference they live in the host
 * application's own objects (src/transformer/activations.c, normalization.c,
 * src/utils/utils.c) and this library does not define them.
 *
 * Additive entry points (device residency, sharding, quantisers, ternary) are
 * in sapphire_cuda.h.
 */
#ifndef KERNELS_H
#define KERNELS_H

#include <stdint.h>
#include <stddef.h>
#include "tensor.h"

#ifndef SAPPHIRE_API
#define SAPPHIRE_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------- *
 * Packed block formats (byte-compatible with reference include/kernels.h:28-38)
 * ------------------------------------------------------------------------- */

/** Q4_0 block: weight j of the block is (q_j - 8) * scale, q_j in [0, 15].
 *  Byte i of q_data holds q_{2i} in bits 0-3 and q_{2i+1} in bits 4-7
 *  (interleaved order, reference src/kernels/q4_0_avx.c:61-65).  20 bytes. */
typedef struct {
    float scale;
    uint8_t q_data[16];
} ggml_block_q4_0;

/** Q8_0 block: weight j is (int8_t)q_data[j] * scale.  36 bytes. */
typedef struct {
    float scale;
    uint8_t q_data[32];
} ggml_block_q8_0;

/* ------------------------------------------------------------------------- *
 * Context (reference include/kernels.h:45-72, src/kernels/pool.c:157-268)
 * ------------------------------------------------------------------------- */

/** Opaque execution context.  Here it owns one GPU (the device current at
 *  creation), a CUDA stream, the device copies of uploaded weights, scratch
 *  and a small host worker pool for kernel_parallel_for. */
typedef struct sapphire_context kernel_context_t;

/** Create a context bound to the current CUDA device.  num_threads sizes the
 *  host pool used by kernel_parallel_for (<= 0: all online CPUs); chunk_size
 *  <= 0 means 16.  No GPU work happens until kernel_ctx_init.  NULL on error. */
SAPPHIRE_API kernel_context_t* kernel_ctx_create(int num_threads, int chunk_size);

/** Create the stream, device scratch and host workers.  Idempotent.
 *  0 on success, -1 on failure (logged). */
SAPPHIRE_API int kernel_ctx_init(kernel_context_t *ctx);

/** Release device copies, stream, scratch and workers.  NULL-safe. */
SAPPHIRE_API void kernel_ctx_destroy(kernel_context_t *ctx);

/* ------------------------------------------------------------------------- *
 * Row-kernel ABI (reference include/kernels.h:78-130)
 * ------------------------------------------------------------------------- */

typedef float (*kernel_fn_t)(const void* w_row, const float* x, int blocks, int block_size);
typedef float (*gemv_kernel_t)(const void* w_row, const float* x, int blocks, int block_size);

typedef struct {
    const void* w_row;
    const float* X;
    float* Y;
    int batch_size;
    int d_model;
    int out_stride;
    int blocks;
    int block_size;
} gemm_args_t;

typedef void (*gemm_kernel_t)(const gemm_args_t* args);

/** Host callback run by kernel_parallel_for. */
typedef void (*parallel_for_fn_t)(void* arg, int idx);

/** Run fn(arg, i) for i in [0, n) on the context's host workers and wait.
 *  This is a host facility (the reference uses it for per-token attention);
 *  it launches no GPU work.  0 on success, -1 on bad arguments. */
SAPPHIRE_API int kernel_parallel_for(kernel_context_t *ctx, parallel_for_fn_t fn, void* arg, int n);

/* One-row dot products.  W_row and x are host pointers; the row is computed
 * on the GPU of a process-wide default context: every call copies the row
 * and x to the device, launches one kernel and synchronises with the GPU
 * before it returns (tens of microseconds per call, against well under a
 * microsecond for the reference's AVX2 row on the host).  They are correct
 * but slow: they exist for ABI compatibility with callers of the reference
 * row kernels (its tests and benches); whole products belong in kernel_gemv.
 * block_size must be 32 for the quantized forms (the reference returns 0.0f
 * otherwise, and so do these). */
SAPPHIRE_API float quantized_gemv_q4_0_aligned(const void *W_row, const float *x, int block_count, int block_size);
SAPPHIRE_API float quantized_gemv_q4_0_unaligned(const void *W_row, const float *x, int block_count, int block_size);
SAPPHIRE_API float quantized_gemv_q8_0_aligned(const void *W_row, const float *x, int block_count, int block_size);
SAPPHIRE_API float quantized_gemv_q8_0_unaligned(const void *W_row, const float *x, int block_count, int block_size);
SAPPHIRE_API float quantized_gemv_bf16_avx2(const void *W_row, const float *x, int block_count, int block_size);
SAPPHIRE_API float quantized_gemv_bf16_scalar(const void *W_row, const float *x, int block_count, int block_size);
SAPPHIRE_API float quantized_gemv_f32_avx2(const void *W_row, const float *x, int block_count, int block_size);
SAPPHIRE_API float quantized_gemv_f32_scalar(const void *W_row, const float *x, int block_count, int block_size);

/* Batched one-row kernels: Y[i*out_stride] = dot(w_row, X[i*d_model .. +d_model)). */
SAPPHIRE_API void kernel_gemm_f32_avx2(const gemm_args_t* args);
SAPPHIRE_API void kernel_gemm_bf16_avx2(const gemm_args_t* args);

/* ------------------------------------------------------------------------- *
 * Tensor GEMV (reference include/kernels.h:136-166, src/kernels/dispatch.c)
 * ------------------------------------------------------------------------- */

/** y[rows] = A[rows, cols] @ x[cols].  A: F32, BF16, Q4_0, Q8_0 or TQ2_0.
 *  Quantized A needs a context (NULL gives -1, as in the reference); F32/BF16
 *  with a NULL context run on a process-wide default context.  x and y may be
 *  host or device pointers; the call is synchronous (y is valid on return).
 *  A page-locked host y (cudaHostAlloc / kernel_host_alloc / registered) is
 *  written by the kernel through its device mapping while the product runs;
 *  other host y receive a copy after it.
 *  The first call with a given weight tensor uploads it (see
 *  kernel_tensor_upload in sapphire_cuda.h).  0 on success, -1 on error. */
SAPPHIRE_API int kernel_gemv(kernel_context_t *ctx, float *y, const tensor_t *A, const float *x);

/** Batched product.  With out_stride != 0: Y[b*rows + r] = A[r,:] . X[b*cols ..],
 *  b < batch_size (the reference passes out_stride as its "is GEMM" flag and
 *  always uses a row stride of `rows`, src/kernels/dispatch.c:98, pool.c:133).
 *  With out_stride == 0 only X[0..cols) is used, like kernel_gemv.
 *  Q4_0 / Q8_0 / TQ2_0 are supported here (the reference returns -1 for them).
 *  A Q4_0 product of 16 or more rows runs on the tensor cores with bf16
 *  activations unless kernel_ctx_set_fp32_products (sapphire_cuda.h) keeps
 *  fp32 (one row product per activation row). */
SAPPHIRE_API int kernel_gemm(kernel_context_t *ctx, float *Y, const tensor_t *A, const float *X, int batch_size, int out_stride);

/** y = A @ x for 1-D F32 tensors x, y (shape-checked). */
SAPPHIRE_API int kernel_gemv_tensor(kernel_context_t *ctx, const tensor_t *y, const tensor_t *A, const tensor_t *x);

/** y += alpha * (A @ x).  The temporary lives in context scratch (no malloc per call). */
SAPPHIRE_API int kernel_gemv_add(kernel_context_t *ctx, float *y, const tensor_t *A, const float *x, float alpha);

/** Y[k*rows ..] = A @ X[k*cols ..] for k < batch_size. */
SAPPHIRE_API int kernel_gemv_batch(kernel_context_t *ctx, float *Y, const tensor_t *A, const float *X, int batch_size);

/** Host float padding the caller should apply to activation buffers: 8 for the
 *  float and quantized dtypes (unchanged from the reference), 1 otherwise. */
SAPPHIRE_API int kernel_get_simd_lane_count(tensor_dtype_t dtype);

/* ------------------------------------------------------------------------- *
 * Host-side helpers of the reference header.  NOT defined by this library:
 * the host application links them from its own transformer/utils objects.
 * ------------------------------------------------------------------------- */
float silu(float x);
void silu_inplace(float *x, int n);
float relu(float x);
void relu_inplace(float *x, int n);
float gelu(float x);
void gelu_inplace(float *x, int n);
float geglu(float x, float y);
int sapphire_geglu(float *output, const float *input, size_t size);
int rmsnorm(float *out, const float *in, const float *weight, float epsilon, int dim);
int rmsnorm_delta(float *out, const float *in, const float *weight, float epsilon, int dim);
int rmsnorm_batch(float *out, const float *in, const float *weight, float epsilon, int batch_size, int dim);
void softmax(float *scores, int n);
void vec_softcap(float *x, int n, float cap);
void vec_add(float *dst, const float *src, int n);
void vec_scale(float *x, float s, int n);
void vec_copy(float *dst, const float *src, int n);
float vec_dot(const float *a, const float *b, int n);
void bf16_to_f32_vec(float *dst, const uint16_t *src, int n);
const float* get_norm_weights(const tensor_t *weight, float *scratch, int n);

/* ------------------------------------------------------------------------- *
 * Legacy names (reference include/kernels.h:228-238)
 * ------------------------------------------------------------------------- */
#define sapphire_context_create kernel_ctx_create
#define sapphire_context_destroy kernel_ctx_destroy
#define tensor_gemv_ctx_create kernel_ctx_create
#define tensor_gemv_ctx_destroy kernel_ctx_destroy
#define tensor_gemv_with_ctx kernel_gemv
#define tensor_gemm_with_ctx kernel_gemm
#define tensor_gemv_tensor_with_ctx kernel_gemv_tensor
#define tensor_gemv_add_with_ctx kernel_gemv_add
#define tensor_gemv_batch_with_ctx kernel_gemv_batch
#define tensor_gemv_simd_lane_count_for_dtype kernel_get_simd_lane_count
#define sapphire_batched_gemv kernel_gemv

#ifdef __cplusplus
}
#endif

#endif /* KERNELS_H */
