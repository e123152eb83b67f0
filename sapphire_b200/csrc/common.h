// common.h - internal declarations shared by the libsapphire_cuda.so sources.
//
// Not installed; callers use include/kernels.h, include/tensor.h and
// include/sapphire_cuda.h.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/kernels.h"
#include "../../include/tensor.h"
#include "../../include/sapphire_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

// ---------------------------------------------------------------- logging --
// Levels and the SAPPHIRE_LOG_LEVEL variable follow the reference logger
// (src/log.c:46-66): debug < info < warn < error < none.
enum { SAPPHIRE_LOG_DEBUG = 10, SAPPHIRE_LOG_INFO = 20, SAPPHIRE_LOG_WARN = 30,
       SAPPHIRE_LOG_ERROR = 40, SAPPHIRE_LOG_NONE = 100 };
void sapphire_log(int level, const char *file, int line, const char *func, const char *fmt, ...)
    __attribute__((format(printf, 5, 6)));
#define LOG_DEBUG(...) sapphire_log(SAPPHIRE_LOG_DEBUG, __FILE__, __LINE__, __func__, __VA_ARGS__)
#define LOG_INFO(...)  sapphire_log(SAPPHIRE_LOG_INFO,  __FILE__, __LINE__, __func__, __VA_ARGS__)
#define LOG_WARN(...)  sapphire_log(SAPPHIRE_LOG_WARN,  __FILE__, __LINE__, __func__, __VA_ARGS__)
#define LOG_ERROR(...) sapphire_log(SAPPHIRE_LOG_ERROR, __FILE__, __LINE__, __func__, __VA_ARGS__)

// ------------------------------------------------------- tensor internals --
// Process-unique id of a tensor handle (never reused), used to key device copies.
uint64_t sapphire_tensor_uid(const tensor_t *t);
// Called by tensor_release() before a handle is freed: drops device copies.
void sapphire_on_tensor_release(uint64_t uid);

// ------------------------------------------------------------ formats -----
// Bytes of one packed host row (the reference's block layout), 0 for dtypes
// without a GEMV path.
size_t sapphire_row_bytes_internal(tensor_dtype_t dtype, int cols);

#ifdef __cplusplus
}
#endif
