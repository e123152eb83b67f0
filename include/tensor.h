/*
 * tensor.h - tensor handle of the B200 GEMV library.
 *
 * Drop-in for the reference header include/tensor.h: every function below has
 * the same name, signature and return convention as the reference
 * (include/tensor.h:60-208, implemented in src/tensor/tensor.c:81-390), so the
 * Gemma-3 host code compiles against this header unchanged.
 *
 * Differences that a caller can observe:
 *  - DTYPE_TQ2_0 is APPENDED to tensor_dtype_t (value 5).  It is the ternary
 *    format this library defines (the reference has none): each row is an fp32
 *    scale followed by ceil(cols/32) 8-byte blocks of 2-bit trit codes.
 *  - tensor_nbytes() keeps the reference's element-count arithmetic for Q4_0
 *    and Q8_0 (numel/2 and numel bytes, pinned by the reference's
 *    src/test/test_tensor.c:97,104).  Those numbers do NOT describe the packed
 *    block storage; the GEMV path computes the real byte size from the shape
 *    (rows * ceil(cols/32) * {20, 36} bytes; TQ2_0: rows * (4 + 8*ceil(cols/32))).
 */
#ifndef TENSOR_H
#define TENSOR_H

#include <stddef.h>
#include <stdint.h>

#ifndef SAPPHIRE_API
#define SAPPHIRE_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/** Element formats.  Values 0..4 match the reference enum (include/tensor.h:17-23). */
typedef enum {
    DTYPE_F32,     /* 4-byte IEEE float                                          */
    DTYPE_BF16,    /* 2-byte bfloat16                                            */
    DTYPE_F16,     /* 2-byte IEEE half (storage only; no GEMV kernel)            */
    DTYPE_Q4_0,    /* 32-weight blocks: fp32 scale + 16 bytes of 4-bit codes     */
    DTYPE_Q8_0,    /* 32-weight blocks: fp32 scale + 32 int8 codes               */
    DTYPE_TQ2_0,   /* ternary rows: fp32 row scale + 8-byte blocks of 2-bit trits */
} tensor_dtype_t;

/** Storage order (reference include/tensor.h:31-34). Only row-major is produced. */
typedef enum {
    LAYOUT_ROW_MAJOR,
    LAYOUT_COLUMN_MAJOR,
} memory_layout_t;

/** Opaque tensor handle; fields are private to tensor.c. */
typedef struct tensor_t tensor_t;

/** Allocate a zero-filled tensor of ndim (1..8) dimensions; refcount starts at 1. NULL on error. */
SAPPHIRE_API tensor_t* tensor_create(int ndim, const int *shape, tensor_dtype_t dtype);

/** New F32 tensor holding the transpose of a 2-D F32 tensor. 0 on success, -1 otherwise. */
SAPPHIRE_API int tensor_transpose(const tensor_t *src, tensor_t **dst);

/** Deep copy (new allocation, same shape/dtype/layout/bytes). NULL on error. */
SAPPHIRE_API tensor_t* tensor_clone(const tensor_t *src);

/** Product of the shape; 0 for NULL. */
SAPPHIRE_API size_t tensor_numel(const tensor_t *t);

/** Bytes per element used for tensor_nbytes: F32 4, BF16/F16 2, Q4_0/Q8_0/TQ2_0 1. */
SAPPHIRE_API size_t dtype_element_size(tensor_dtype_t dtype);

/** Printable name of a dtype ("F32", "Q4_0", ... or "UNKNOWN"). */
SAPPHIRE_API const char* dtype_name(tensor_dtype_t dtype);

/** Element read by linear index.  F32 only; quantized dtypes log a warning and give 0. */
SAPPHIRE_API float tensor_get_f32(const tensor_t *t, size_t idx);

/** Element write by linear index (F32 only).  0 on success, -1 otherwise. */
SAPPHIRE_API int tensor_set_f32(tensor_t *t, size_t idx, float val);

/** Reference counting.  tensor_release frees owned data when the count reaches 0. */
SAPPHIRE_API void tensor_ref_inc(tensor_t *t);
SAPPHIRE_API void tensor_release(tensor_t *t);

/** Log one line of metadata (shape, dtype, layout, bytes, refcount). */
SAPPHIRE_API void tensor_print_info(const tensor_t *t);

/** Accessors (NULL-safe: 0 / NULL / DTYPE_F32 for a NULL tensor). */
SAPPHIRE_API int tensor_ndim(const tensor_t *t);
SAPPHIRE_API const int* tensor_shape(const tensor_t *t);
SAPPHIRE_API const void* tensor_data(const tensor_t *t);
SAPPHIRE_API float* tensor_data_f32(const tensor_t *t);
SAPPHIRE_API void* tensor_data_mutable(const tensor_t *t);
SAPPHIRE_API tensor_dtype_t tensor_dtype(const tensor_t *t);
SAPPHIRE_API size_t tensor_nbytes(const tensor_t *t);
SAPPHIRE_API int tensor_ref_count(const tensor_t *t);

/** Non-owning view over caller memory (e.g. an mmap'd checkpoint).  The data
 *  pointer may be host memory or device memory of the context's GPU. */
SAPPHIRE_API tensor_t* tensor_create_view(tensor_dtype_t dtype, int ndim, const int *shape, void *data);

#ifdef __cplusplus
}
#endif

#endif /* TENSOR_H */
