/*
 * sapphire_oracle.c - CPU restatement of the reference's quantized GEMV
 * arithmetic.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and
 * the CPU-baseline leg of bench.py call it as the checker; the product library
 * (libsapphire_cuda.so) never links, loads or calls it.
 *
 * Parity pin: tests/test_oracle_pins.py checks every function here against the
 * reference's own kernels compiled from its sources (oracle/_ref, built by
 * oracle/Makefile) and against the golden fixtures in tests/golden/ that were
 * generated from those kernels.  The quantisers and the ternary format have
 * no reference implementation (the reference has no quantiser and no ternary
 * code); they are pinned only to the formulas stated below ("parity unpinned"
 * for those two items).
 *
 * Build: oracle/Makefile, with -ffp-contract=off so no FMA contraction changes
 * a rounding.
 */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define OR_API __attribute__((visibility("default")))

enum { OR_F32 = 0, OR_BF16 = 1, OR_F16 = 2, OR_Q4_0 = 3, OR_Q8_0 = 4, OR_TQ2_0 = 5 };

static float ld_f32(const uint8_t *p) {
    float f;
    memcpy(&f, p, 4);
    return f;
}

OR_API size_t oracle_row_bytes(int dtype, int cols) {
    size_t nb = ((size_t)cols + 31) / 32;
    switch (dtype) {
        case OR_Q4_0: return nb * 20;             /* include/kernels.h:28-32 */
        case OR_Q8_0: return nb * 36;             /* include/kernels.h:34-38 */
        case OR_TQ2_0: return 4 + nb * 8;         /* this library's ternary row */
        case OR_F32: return (size_t)cols * 4;
        case OR_BF16: return (size_t)cols * 2;
        default: return 0;
    }
}

/* ------------------------------------------------------------ codes ------ */
/* Q4_0 code j of a block: byte j/2, low nibble for even j, high for odd j
 * (src/kernels/q4_0_avx.c:61-65, src/test/bench/bench_q4.c:26-32). */
static int q4_code(const uint8_t *blk, int j) {
    uint8_t v = blk[4 + j / 2];
    return (j & 1) ? (v >> 4) : (v & 0x0F);
}
/* Q8_0 code j: signed byte (src/kernels/q8_0_avx.c:45-48). */
static int q8_code(const uint8_t *blk, int j) { return (int8_t)blk[4 + j]; }
/* TQ2_0 trit j of an 8-byte block: (bits 2*(j%4) of byte j/4) - 1. */
static int tq2_trit(const uint8_t *blk8, int j) { return ((blk8[j / 4] >> (2 * (j % 4))) & 3) - 1; }

/* ------------------------------------------------------- row products ---- */
/* Q4_0 row, fp32, in the scalar reference's order: sum += scale*(q-8)*x per
 * element (src/test/bench/bench_q4.c:18-36). */
OR_API float oracle_row_q4_0(const void *row, const float *x, int nb) {
    const uint8_t *p = (const uint8_t *)row;
    float sum = 0.0f;
    for (int b = 0; b < nb; ++b) {
        const uint8_t *blk = p + (size_t)b * 20;
        float scale = ld_f32(blk);
        for (int j = 0; j < 32; ++j) sum += scale * (float)(q4_code(blk, j) - 8) * x[b * 32 + j];
    }
    return sum;
}

/* Q8_0 row, fp32: w = q*scale, then sum += w*x (src/kernels/q8_0_avx.c:40-64). */
OR_API float oracle_row_q8_0(const void *row, const float *x, int nb) {
    const uint8_t *p = (const uint8_t *)row;
    float sum = 0.0f;
    for (int b = 0; b < nb; ++b) {
        const uint8_t *blk = p + (size_t)b * 36;
        float scale = ld_f32(blk);
        for (int j = 0; j < 32; ++j) sum += ((float)q8_code(blk, j) * scale) * x[b * 32 + j];
    }
    return sum;
}

/* TQ2_0 row, fp32: scale * sum (t*x). */
OR_API float oracle_row_tq2_0(const void *row, const float *x, int nb) {
    const uint8_t *p = (const uint8_t *)row;
    float scale = ld_f32(p);
    float sum = 0.0f;
    for (int b = 0; b < nb; ++b)
        for (int j = 0; j < 32; ++j) sum += (float)tq2_trit(p + 4 + (size_t)b * 8, j) * x[b * 32 + j];
    return scale * sum;
}

/* Exact-as-possible row product in double (order-independent ground truth). */
static double row_f64(int dtype, const uint8_t *p, const float *x, int cols) {
    int nb = (cols + 31) / 32;
    double sum = 0.0;
    if (dtype == OR_Q4_0 || dtype == OR_Q8_0) {
        size_t bsz = dtype == OR_Q4_0 ? 20 : 36;
        for (int b = 0; b < nb; ++b) {
            const uint8_t *blk = p + (size_t)b * bsz;
            double scale = ld_f32(blk), part = 0.0;
            for (int j = 0; j < 32 && b * 32 + j < cols; ++j) {
                int q = dtype == OR_Q4_0 ? q4_code(blk, j) - 8 : q8_code(blk, j);
                part += (double)q * (double)x[b * 32 + j];
            }
            sum += scale * part;
        }
    } else if (dtype == OR_TQ2_0) {
        double scale = ld_f32(p);
        for (int c = 0; c < cols; ++c) sum += (double)tq2_trit(p + 4 + (size_t)(c / 32) * 8, c % 32) * x[c];
        sum *= scale;
    } else if (dtype == OR_F32) {
        for (int c = 0; c < cols; ++c) sum += (double)ld_f32(p + (size_t)c * 4) * x[c];
    } else if (dtype == OR_BF16) {
        for (int c = 0; c < cols; ++c) {
            uint32_t u = ((uint32_t)p[2 * c] | ((uint32_t)p[2 * c + 1] << 8)) << 16;
            float w;
            memcpy(&w, &u, 4);
            sum += (double)w * x[c];
        }
    }
    return sum;
}

/* ------------------------------------------------------------- GEMV ------ */
typedef struct {
    int dtype, rows, cols, batch, r0, r1;
    const uint8_t *W;
    const float *X;
    void *Y;
    int f64;
} gemv_job_t;

static void *gemv_worker(void *arg) {
    gemv_job_t *j = (gemv_job_t *)arg;
    size_t rb = oracle_row_bytes(j->dtype, j->cols);
    for (int b = 0; b < j->batch; ++b) {
        const float *x = j->X + (size_t)b * j->cols;
        for (int r = j->r0; r < j->r1; ++r) {
            const uint8_t *row = j->W + (size_t)r * rb;
            if (j->f64) {
                ((double *)j->Y)[(size_t)b * j->rows + r] = row_f64(j->dtype, row, x, j->cols);
            } else {
                float v = 0.0f;
                int nb = (j->cols + 31) / 32;
                if (j->dtype == OR_Q4_0) v = oracle_row_q4_0(row, x, nb);
                else if (j->dtype == OR_Q8_0) v = oracle_row_q8_0(row, x, nb);
                else if (j->dtype == OR_TQ2_0) v = oracle_row_tq2_0(row, x, nb);
                else v = (float)row_f64(j->dtype, row, x, j->cols);
                ((float *)j->Y)[(size_t)b * j->rows + r] = v;
            }
        }
    }
    return NULL;
}

/* Y[b*rows + r] = W[r,:] . X[b*cols ..] for all rows.  Quantized rows read
 * x[0 .. nb*32): callers pad x with zeros past `cols` (the reference's
 * sessions pad activations the same way, src/inference/inference.c:377-431).
 * f64 != 0 writes doubles (ground truth), else floats in the reference's
 * scalar order.  nthreads <= 0: one thread per online CPU. */
static int run_gemv(int dtype, const void *W, int rows, int cols, const float *X, int batch, void *Y, int f64,
                    int nthreads) {
    if (!W || !X || !Y || rows <= 0 || cols <= 0 || batch <= 0) return -1;
    if (nthreads <= 0) {
        long n = sysconf(_SC_NPROCESSORS_ONLN);
        nthreads = n > 0 ? (int)n : 1;
    }
    if (nthreads > rows) nthreads = rows;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    gemv_job_t jobs[256];
    int per = (rows + nthreads - 1) / nthreads;
    int joined[256];
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = (gemv_job_t){dtype, rows, cols, batch, t * per, (t + 1) * per > rows ? rows : (t + 1) * per,
                               (const uint8_t *)W, X, Y, f64};
        joined[t] = 0;
        if (jobs[t].r0 >= jobs[t].r1) continue;
        if (pthread_create(&th[t], NULL, gemv_worker, &jobs[t]) != 0) gemv_worker(&jobs[t]);
        else joined[t] = 1;
    }
    for (int t = 0; t < nthreads; ++t)
        if (joined[t]) pthread_join(th[t], NULL);
    return 0;
}

OR_API int oracle_gemv(int dtype, const void *W, int rows, int cols, const float *X, int batch, float *Y,
                       int nthreads) {
    return run_gemv(dtype, W, rows, cols, X, batch, Y, 0, nthreads);
}

OR_API int oracle_gemv_f64(int dtype, const void *W, int rows, int cols, const float *X, int batch, double *Y,
                           int nthreads) {
    return run_gemv(dtype, W, rows, cols, X, batch, Y, 1, nthreads);
}

/* ------------------------------------------------------------ quantisers - */
/* Q4_0 block quantiser (the formula BASELINE.json names; the reference has
 * none): m = element of largest |x| (first on ties), d = m/-8,
 * id = d ? 1/d : 0, q = min(15, trunc(x*id + 8.5)) with NaN -> 0, packed in
 * the reference's interleaved nibble order. */
static void quant_q4_block(const float *v, uint8_t *out) {
    float amax = 0.0f, m = 0.0f;
    for (int j = 0; j < 32; ++j) {
        float a = fabsf(v[j]);
        if (a > amax) {
            amax = a;
            m = v[j];
        }
    }
    float d = m / -8.0f;
    float id = (d != 0.0f) ? 1.0f / d : 0.0f;
    memcpy(out, &d, 4);
    int q[32];
    for (int j = 0; j < 32; ++j) {
        float prod = v[j] * id;
        float t = prod + 8.5f;
        q[j] = (t >= 15.0f) ? 15 : (t >= 1.0f ? (int)t : 0);
    }
    for (int i = 0; i < 16; ++i) out[4 + i] = (uint8_t)(q[2 * i] | (q[2 * i + 1] << 4));
}

/* Q8_0: a = max|x|, d = a/127, id = d ? 1/d : 0, q = clamp(roundf(x*id)). */
static void quant_q8_block(const float *v, uint8_t *out) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    float d = amax / 127.0f;
    float id = (d != 0.0f) ? 1.0f / d : 0.0f;
    memcpy(out, &d, 4);
    for (int j = 0; j < 32; ++j) {
        float prod = v[j] * id;
        float t = roundf(prod);
        int q = (t != t) ? 0 : (t > 127.0f ? 127 : (t < -127.0f ? -127 : (int)t));
        out[4 + j] = (uint8_t)(int8_t)q;
    }
}

OR_API int oracle_quantize(int dtype, const float *src, int rows, int cols, void *dst) {
    if (!src || !dst || rows <= 0 || cols <= 0 || (dtype != OR_Q4_0 && dtype != OR_Q8_0)) return -1;
    int nb = (cols + 31) / 32;
    size_t bsz = dtype == OR_Q4_0 ? 20 : 36;
    uint8_t *o = (uint8_t *)dst;
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) {
            float v[32];
            for (int j = 0; j < 32; ++j) {
                int c = b * 32 + j;
                v[j] = c < cols ? src[(size_t)r * cols + c] : 0.0f;
            }
            uint8_t *blk = o + ((size_t)r * nb + b) * bsz;
            if (dtype == OR_Q4_0) quant_q4_block(v, blk);
            else quant_q8_block(v, blk);
        }
    return 0;
}

/* Ternary rows: fp32 scale, then per 32 columns 8 bytes of codes c = t + 1. */
OR_API int oracle_pack_tq2_0(const int8_t *trits, const float *scales, int rows, int cols, void *dst) {
    if (!trits || !scales || !dst || rows <= 0 || cols <= 0) return -1;
    int nb = (cols + 31) / 32;
    size_t rb = 4 + (size_t)8 * nb;
    uint8_t *o = (uint8_t *)dst;
    for (int r = 0; r < rows; ++r) {
        uint8_t *row = o + (size_t)r * rb;
        memcpy(row, &scales[r], 4);
        for (int b = 0; b < nb; ++b)
            for (int byte = 0; byte < 8; ++byte) {
                unsigned v = 0;
                for (int p = 0; p < 4; ++p) {
                    int c = b * 32 + byte * 4 + p;
                    int t = c < cols ? trits[(size_t)r * cols + c] : 0;
                    if (t < -1 || t > 1) return -1;
                    v |= (unsigned)(t + 1) << (2 * p);
                }
                row[4 + (size_t)b * 8 + byte] = (uint8_t)v;
            }
    }
    return 0;
}

/* Unpack to fp32 [rows, cols]: Q4_0 (q-8)*scale, Q8_0 q*scale, TQ2_0 t*scale. */
OR_API int oracle_dequantize(int dtype, const void *src, int rows, int cols, float *dst) {
    if (!src || !dst || rows <= 0 || cols <= 0) return -1;
    size_t rb = oracle_row_bytes(dtype, cols);
    if (!rb) return -1;
    const uint8_t *p = (const uint8_t *)src;
    for (int r = 0; r < rows; ++r) {
        const uint8_t *row = p + (size_t)r * rb;
        for (int c = 0; c < cols; ++c) {
            int b = c / 32, j = c % 32;
            float v;
            if (dtype == OR_Q4_0) v = (float)(q4_code(row + (size_t)b * 20, j) - 8) * ld_f32(row + (size_t)b * 20);
            else if (dtype == OR_Q8_0) v = (float)q8_code(row + (size_t)b * 36, j) * ld_f32(row + (size_t)b * 36);
            else if (dtype == OR_TQ2_0) v = (float)tq2_trit(row + 4 + (size_t)b * 8, j) * ld_f32(row);
            else if (dtype == OR_F32) v = ld_f32(row + (size_t)c * 4);
            else {
                uint32_t u = ((uint32_t)row[2 * c] | ((uint32_t)row[2 * c + 1] << 8)) << 16;
                memcpy(&v, &u, 4);
            }
            dst[(size_t)r * cols + c] = v;
        }
    }
    return 0;
}
