// tensor.c - tensor_t handle (include/tensor.h).
//
// Behaviour follows the reference src/tensor/tensor.c: the same byte counts
// (Q4_0 = ceil(numel/2), Q8_0 = numel, views use numel*element_size,
// :108-112 and :149), the same NULL conventions of the accessors (:348-390),
// and reference counting that frees only owned data (:283-293).
// Additions: each handle carries a process-unique id so the GPU side can key
// device copies of weights, and tensor_release tells the GPU side to drop
// them before the handle goes away.
#define _POSIX_C_SOURCE 200809L
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "common.h"

struct tensor_t {
    void *data;
    int ndim;
    int shape[8];
    tensor_dtype_t dtype;
    memory_layout_t layout;
    size_t nbytes;
    int ref_count;
    int is_external;
    uint64_t uid;
};

static atomic_uint_fast64_t g_next_uid = 1;

static uint64_t next_uid(void) { return (uint64_t)atomic_fetch_add(&g_next_uid, 1); }

size_t dtype_element_size(tensor_dtype_t dtype) {
    switch (dtype) {
        case DTYPE_F32:   return 4;
        case DTYPE_BF16:  return 2;
        case DTYPE_F16:   return 2;
        case DTYPE_Q4_0:  return 1;
        case DTYPE_Q8_0:  return 1;
        case DTYPE_TQ2_0: return 1;
        default:          return 0;
    }
}

const char* dtype_name(tensor_dtype_t dtype) {
    switch (dtype) {
        case DTYPE_F32:   return "F32";
        case DTYPE_BF16:  return "BF16";
        case DTYPE_F16:   return "F16";
        case DTYPE_Q4_0:  return "Q4_0";
        case DTYPE_Q8_0:  return "Q8_0";
        case DTYPE_TQ2_0: return "TQ2_0";
        default:          return "UNKNOWN";
    }
}

static size_t numel_of(int ndim, const int *shape) {
    size_t n = 1;
    for (int i = 0; i < ndim; ++i) n *= (size_t)shape[i];
    return n;
}

tensor_t* tensor_create(int ndim, const int *shape, tensor_dtype_t dtype) {
    if (ndim < 1 || ndim > 8 || !shape) {
        LOG_ERROR("ndim %d out of range or shape missing", ndim);
        return NULL;
    }
    tensor_t *t = (tensor_t *)calloc(1, sizeof *t);
    if (!t) {
        LOG_ERROR("out of memory for the handle");
        return NULL;
    }
    t->ndim = ndim;
    t->dtype = dtype;
    t->layout = LAYOUT_ROW_MAJOR;
    memcpy(t->shape, shape, (size_t)ndim * sizeof(int));
    size_t numel = numel_of(ndim, shape);
    t->nbytes = (dtype == DTYPE_Q4_0) ? (numel + 1) / 2 : numel * dtype_element_size(dtype);
    t->data = calloc(t->nbytes ? t->nbytes : 1, 1);
    if (!t->data) {
        LOG_ERROR("out of memory for %zu bytes", t->nbytes);
        free(t);
        return NULL;
    }
    t->ref_count = 1;
    t->is_external = 0;
    t->uid = next_uid();
    return t;
}

tensor_t* tensor_create_view(tensor_dtype_t dtype, int ndim, const int *shape, void *data) {
    if (ndim < 1 || ndim > 8 || !shape) {
        LOG_ERROR("ndim %d out of range or shape missing", ndim);
        return NULL;
    }
    tensor_t *t = (tensor_t *)calloc(1, sizeof *t);
    if (!t) return NULL;
    t->data = data;
    t->ndim = ndim;
    t->dtype = dtype;
    t->layout = LAYOUT_ROW_MAJOR;
    memcpy(t->shape, shape, (size_t)ndim * sizeof(int));
    t->nbytes = numel_of(ndim, shape) * dtype_element_size(dtype);
    t->ref_count = 1;
    t->is_external = 1;
    t->uid = next_uid();
    return t;
}

tensor_t* tensor_clone(const tensor_t *src) {
    if (!src) return NULL;
    tensor_t *c = tensor_create(src->ndim, src->shape, src->dtype);
    if (!c) return NULL;
    c->layout = src->layout;
    if (src->data && src->nbytes) memcpy(c->data, src->data, src->nbytes);
    return c;
}

int tensor_transpose(const tensor_t *src, tensor_t **dst) {
    if (!src || !dst || src->ndim != 2 || src->dtype != DTYPE_F32) return -1;
    int m = src->shape[0], n = src->shape[1];
    int dims[2] = {n, m};
    tensor_t *t = tensor_create(2, dims, DTYPE_F32);
    if (!t) return -1;
    const float *s = (const float *)src->data;
    float *d = (float *)t->data;
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) d[(size_t)j * m + i] = s[(size_t)i * n + j];
    *dst = t;
    return 0;
}

size_t tensor_numel(const tensor_t *t) { return t ? numel_of(t->ndim, t->shape) : 0; }

float tensor_get_f32(const tensor_t *t, size_t idx) {
    if (!t || idx >= tensor_numel(t)) {
        LOG_ERROR("index %zu out of range", idx);
        return 0.0f;
    }
    if (t->dtype == DTYPE_F32) return ((const float *)t->data)[idx];
    // The reference returns 0 for quantized element reads
    // (src/tensor/tensor.c:238-244); use kernel_dequantize for real values.
    LOG_WARN("tensor_get_f32 on %s returns 0; use kernel_dequantize", dtype_name(t->dtype));
    return 0.0f;
}

int tensor_set_f32(tensor_t *t, size_t idx, float val) {
    if (!t || idx >= tensor_numel(t)) {
        LOG_ERROR("index %zu out of range", idx);
        return -1;
    }
    if (t->dtype != DTYPE_F32) {
        LOG_ERROR("the tensor is not F32");
        return -1;
    }
    ((float *)t->data)[idx] = val;
    return 0;
}

void tensor_ref_inc(tensor_t *t) {
    if (t) t->ref_count++;
}

void tensor_release(tensor_t *t) {
    if (!t) return;
    if (--t->ref_count > 0) return;
    sapphire_on_tensor_release(t->uid);
    if (t->data && !t->is_external) free(t->data);
    free(t);
}

void tensor_print_info(const tensor_t *t) {
    if (!t) {
        LOG_INFO("(null tensor)");
        return;
    }
    char shape[8 * 12 + 3];
    int pos = snprintf(shape, sizeof shape, "[");
    for (int i = 0; i < t->ndim && pos < (int)sizeof shape; ++i)
        pos += snprintf(shape + pos, sizeof shape - (size_t)pos, i ? ",%d" : "%d", t->shape[i]);
    if (pos < (int)sizeof shape) snprintf(shape + pos, sizeof shape - (size_t)pos, "]");
    LOG_INFO("shape %s, %s, %s layout, %zu bytes, %d references", shape,
             dtype_name(t->dtype), t->layout == LAYOUT_ROW_MAJOR ? "row-major" : "col-major",
             t->nbytes, t->ref_count);
}

int tensor_ndim(const tensor_t *t) { return t ? t->ndim : 0; }
const int* tensor_shape(const tensor_t *t) { return t ? t->shape : NULL; }
const void* tensor_data(const tensor_t *t) { return t ? t->data : NULL; }

float* tensor_data_f32(const tensor_t *t) {
    if (!t) return NULL;
    if (t->dtype != DTYPE_F32) {
        LOG_WARN("dtype %d is not F32", (int)t->dtype);
        return NULL;
    }
    return (float *)t->data;
}

void* tensor_data_mutable(const tensor_t *t) { return t ? t->data : NULL; }
tensor_dtype_t tensor_dtype(const tensor_t *t) { return t ? t->dtype : DTYPE_F32; }
size_t tensor_nbytes(const tensor_t *t) { return t ? t->nbytes : 0; }
int tensor_ref_count(const tensor_t *t) { return t ? t->ref_count : 0; }

uint64_t sapphire_tensor_uid(const tensor_t *t) { return t ? t->uid : 0; }
