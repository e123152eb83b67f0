/*
 * fuzz_safetensors.c - mutation fuzzer of the safetensors reader
 * (sapphire_b200/csrc/safetensors.c), built from source with AddressSanitizer
 * and UndefinedBehaviorSanitizer by tests/test_safetensors.py.
 *
 * A file is untrusted input.  Every iteration mutates a valid file that holds
 * one tensor of each dtype the reader accepts, writes it to a temporary path,
 * opens it, takes a view of every tensor it lists and touches the first and
 * last payload byte of each, then closes it.  Half of the iterations change
 * only digits (the JSON stays well formed, so shapes and data_offsets reach
 * the size checks); the others flip bits, overwrite bytes with JSON
 * punctuation, insert, delete, truncate or rewrite the header length.  The
 * sanitizers turn any out-of-bounds access, use after free, leak or overflow
 * into a non-zero exit.
 *
 *   fuzz_safetensors <iterations> <seed> <scratch path>
 *
 * Linked with the reader's own sources (safetensors.c, tensor.c, log.c) and
 * the two library hooks those call, defined below.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "sapphire_safetensors.h"
#include "tensor.h"

/* Library hooks the reader's sources call (normally in context.cu). */
void sapphire_on_tensor_release(uint64_t uid) { (void)uid; }
size_t sapphire_row_bytes(tensor_dtype_t dt, int cols) {
    const size_t blocks = ((size_t)cols + 31) / 32;
    switch (dt) {
        case DTYPE_Q4_0: return blocks * 20;
        case DTYPE_Q8_0: return blocks * 36;
        case DTYPE_TQ2_0: return 4 + blocks * 8;
        default: return 0;
    }
}

static uint64_t state;
static uint64_t next(void) {
    state ^= state << 13;
    state ^= state >> 7;
    state ^= state << 17;
    return state;
}

/* A valid file: an 8-byte little-endian header length, the JSON header, then
 * 172 payload bytes (F32 2x3, BF16 4, Q4_0 2x64, Q8_0 1x32, TQ2_0 2x40). */
static size_t valid_file(uint8_t *buf) {
    static const char header[] =
        "{\"__metadata__\":{\"format\":\"pt\",\"note\":[1,{\"k\":\"\\u0041\\n\"}]},"
        "\"a\":{\"dtype\":\"F32\",\"shape\":[2,3],\"data_offsets\":[0,24]},"
        "\"b\":{\"dtype\":\"BF16\",\"shape\":[4],\"data_offsets\":[24,32]},"
        "\"q4\":{\"dtype\":\"Q4_0\",\"shape\":[2,64],\"data_offsets\":[32,112]},"
        "\"q8\":{\"dtype\":\"Q8_0\",\"shape\":[1,32],\"data_offsets\":[112,148]},"
        "\"t\":{\"dtype\":\"TQ2_0\",\"shape\":[2,40],\"data_offsets\":[148,172]}}";
    const size_t h = sizeof header - 1;
    for (int i = 0; i < 8; ++i) buf[i] = (uint8_t)((uint64_t)h >> (8 * i));
    memcpy(buf + 8, header, h);
    for (size_t i = 0; i < 172; ++i) buf[8 + h + i] = (uint8_t)next();
    return 8 + h + 172;
}

static size_t payload_bytes(const tensor_t *t) {
    const tensor_dtype_t dt = tensor_dtype(t);
    const int *shape = tensor_shape(t);
    if (dt == DTYPE_Q4_0 || dt == DTYPE_Q8_0 || dt == DTYPE_TQ2_0)
        return (size_t)shape[0] * sapphire_row_bytes(dt, shape[1]);
    return tensor_nbytes(t);
}

int main(int argc, char **argv) {
    if (argc != 4) {
        fprintf(stderr, "usage: %s <iterations> <seed> <scratch path>\n", argv[0]);
        return 2;
    }
    const long iterations = atol(argv[1]);
    state = 0x9E3779B97F4A7C15ull * (uint64_t)(atoll(argv[2]) + 1);
    const char *path = argv[3];
    static uint8_t base[1024], buf[2048];
    const size_t n0 = valid_file(base);
    static const char punct[] = "{}[]\",:\\0123456789-eE. u";
    long opened = 0, views = 0;
    for (long it = 0; it < iterations; ++it) {
        size_t n = n0;
        memcpy(buf, base, n);
        const int mutations = 1 + (int)(next() % 3);
        const int digits_only = (int)(next() & 1);
        for (int m = 0; m < mutations; ++m) {
            const size_t pos = (size_t)(next() % n);
            if (digits_only) {
                /* The next digit at or after pos becomes another digit. */
                for (size_t i = pos; i < n; ++i)
                    if (i >= 8 && buf[i] >= '0' && buf[i] <= '9') {
                        buf[i] = (uint8_t)('0' + next() % 10);
                        break;
                    }
                continue;
            }
            switch (next() % 6) {
                case 0: buf[pos] ^= (uint8_t)(1u << (next() % 8)); break;
                case 1: buf[pos] = (uint8_t)punct[next() % (sizeof punct - 1)]; break;
                case 2: n = pos > 0 ? pos : 1; break;
                case 3:
                    if (n + 1 < sizeof buf) {
                        memmove(buf + pos + 1, buf + pos, n - pos);
                        buf[pos] = (uint8_t)punct[next() % (sizeof punct - 1)];
                        ++n;
                    }
                    break;
                case 4:
                    if (n > 1) {
                        memmove(buf + pos, buf + pos + 1, n - pos - 1);
                        --n;
                    }
                    break;
                default: buf[next() % 8] = (uint8_t)next(); break;
            }
        }
        FILE *f = fopen(path, "wb");
        if (!f || fwrite(buf, 1, n, f) != n) {
            fprintf(stderr, "cannot write %s\n", path);
            return 2;
        }
        fclose(f);
        sapphire_safetensors_t *st = sapphire_safetensors_open(path);
        if (!st) continue;
        ++opened;
        const int count = sapphire_safetensors_count(st);
        for (int i = 0; i < count; ++i) {
            tensor_t *t = sapphire_safetensors_tensor(st, sapphire_safetensors_name(st, i));
            if (!t) continue;
            ++views;
            const uint8_t *d = (const uint8_t *)tensor_data(t);
            const size_t bytes = payload_bytes(t);
            volatile uint8_t sink = 0;
            if (d && bytes) sink = (uint8_t)(d[0] ^ d[bytes - 1]);
            (void)sink;
        }
        sapphire_safetensors_close(st);
    }
    printf("iterations %ld opened %ld views %ld\n", iterations, opened, views);
    return 0;
}
