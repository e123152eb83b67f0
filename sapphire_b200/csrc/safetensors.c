// safetensors.c - safetensors files with quantized tensors, mapped without a
// copy (include/sapphire_safetensors.h).
//
// The reference reads F32 / BF16 / F16 tensors only
// (src/io/safetensors_reader.c:40-60, 401-449: any other dtype is an error),
// so quantized weights cannot come from a file.  This reader accepts the same
// container - an 8-byte little-endian header length, a JSON header mapping
// each name to {"dtype", "shape", "data_offsets": [begin, end]} relative to
// the data section, then the data - and adds the dtypes "Q4_0", "Q8_0" and
// "TQ2_0": the payload is the packed rows of include/kernels.h /
// include/sapphire_cuda.h, back to back, and "shape" is the logical
// [rows, cols] (the payload holds rows * row_bytes(cols) bytes).  Tensors are
// tensor_t views into the mapped file, owned by the handle.
#include <errno.h>
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "common.h"
#include "../../include/sapphire_safetensors.h"

typedef struct {
    char *name;
    tensor_dtype_t dtype;
    int ndim;
    int shape[SAPPHIRE_ST_MAX_DIMS];
    uint64_t begin, end;
    tensor_t *view;
} st_entry;

struct sapphire_safetensors {
    int fd;
    uint8_t *map;
    size_t map_size;
    const uint8_t *data;      // start of the data section
    size_t data_size;
    st_entry *entries;
    int count;
};

// ------------------------------------------------------------ JSON reader --
// Just enough JSON for the header: objects, arrays, strings (with escapes),
// non-negative integers; other values are skipped.
typedef struct {
    const char *p, *end;
    int err;
} jcur;

static void jws(jcur *c) {
    while (c->p < c->end && (*c->p == ' ' || *c->p == '\t' || *c->p == '\n' || *c->p == '\r')) ++c->p;
}

static int jexpect(jcur *c, char ch) {
    jws(c);
    if (c->p < c->end && *c->p == ch) {
        ++c->p;
        return 1;
    }
    c->err = 1;
    return 0;
}

static int jpeek(jcur *c, char ch) {
    jws(c);
    return c->p < c->end && *c->p == ch;
}

// String into a malloc'd buffer (NULL on error).
static char *jstring(jcur *c) {
    if (!jexpect(c, '"')) return NULL;
    size_t cap = 32, n = 0;
    char *s = (char *)malloc(cap);
    if (!s) {
        c->err = 1;
        return NULL;
    }
    while (c->p < c->end && *c->p != '"') {
        char ch = *c->p++;
        if (ch == '\\') {
            if (c->p >= c->end) break;
            const char e = *c->p++;
            switch (e) {
                case 'n': ch = '\n'; break;
                case 't': ch = '\t'; break;
                case 'r': ch = '\r'; break;
                case 'b': ch = '\b'; break;
                case 'f': ch = '\f'; break;
                case 'u':
                    // Names are ASCII in practice; keep the escape's low byte.
                    if (c->end - c->p < 4) {
                        c->err = 1;
                        free(s);
                        return NULL;
                    }
                    ch = (char)strtol((char[5]){c->p[0], c->p[1], c->p[2], c->p[3], 0}, NULL, 16);
                    c->p += 4;
                    break;
                default: ch = e; break;
            }
        }
        if (n + 1 >= cap) {
            cap *= 2;
            char *t = (char *)realloc(s, cap);
            if (!t) {
                free(s);
                c->err = 1;
                return NULL;
            }
            s = t;
        }
        s[n++] = ch;
    }
    if (c->p >= c->end) {
        free(s);
        c->err = 1;
        return NULL;
    }
    ++c->p;   // closing quote
    s[n] = 0;
    return s;
}

static int juint(jcur *c, uint64_t *v) {
    jws(c);
    if (c->p >= c->end || *c->p < '0' || *c->p > '9') {
        c->err = 1;
        return 0;
    }
    uint64_t x = 0;
    while (c->p < c->end && *c->p >= '0' && *c->p <= '9') {
        const uint64_t d = (uint64_t)(*c->p++ - '0');
        if (x > (UINT64_MAX - d) / 10) {
            c->err = 1;
            return 0;
        }
        x = x * 10 + d;
    }
    *v = x;
    return 1;
}

// Skips any JSON value (depth-limited).
static void jskip(jcur *c, int depth) {
    jws(c);
    if (c->p >= c->end || depth > 32) {
        c->err = 1;
        return;
    }
    const char ch = *c->p;
    if (ch == '"') {
        free(jstring(c));
    } else if (ch == '{' || ch == '[') {
        const char close = ch == '{' ? '}' : ']';
        ++c->p;
        if (jpeek(c, close)) {
            ++c->p;
            return;
        }
        for (;;) {
            if (ch == '{') {
                free(jstring(c));
                if (!jexpect(c, ':')) return;
            }
            jskip(c, depth + 1);
            if (c->err) return;
            if (jpeek(c, ',')) {
                ++c->p;
                continue;
            }
            jexpect(c, close);
            return;
        }
    } else {
        while (c->p < c->end && *c->p != ',' && *c->p != '}' && *c->p != ']') ++c->p;
    }
}

static int dtype_of(const char *s, tensor_dtype_t *dt) {
    static const struct {
        const char *name;
        tensor_dtype_t dt;
    } tab[] = {{"F32", DTYPE_F32},   {"BF16", DTYPE_BF16}, {"F16", DTYPE_F16},
               {"Q4_0", DTYPE_Q4_0}, {"Q8_0", DTYPE_Q8_0}, {"TQ2_0", DTYPE_TQ2_0}};
    for (size_t i = 0; i < sizeof tab / sizeof tab[0]; ++i)
        if (strcmp(s, tab[i].name) == 0) {
            *dt = tab[i].dt;
            return 1;
        }
    return 0;
}

// One tensor's description: {"dtype": ..., "shape": [...], "data_offsets": [b, e]}.
static int parse_entry(jcur *c, st_entry *e) {
    int have_dtype = 0, have_shape = 0, have_off = 0;
    if (!jexpect(c, '{')) return 0;
    if (jpeek(c, '}')) {
        ++c->p;
        return 0;
    }
    for (;;) {
        char *key = jstring(c);
        if (!key || !jexpect(c, ':')) {
            free(key);
            return 0;
        }
        if (strcmp(key, "dtype") == 0) {
            char *v = jstring(c);
            const int ok = v && dtype_of(v, &e->dtype);
            if (!ok) LOG_ERROR("tensor '%s': dtype '%s' has no product in this library", e->name, v ? v : "?");
            free(v);
            if (!ok) {
                free(key);
                c->err = 1;
                return 0;
            }
            have_dtype = 1;
        } else if (strcmp(key, "shape") == 0) {
            if (!jexpect(c, '[')) {
                free(key);
                return 0;
            }
            e->ndim = 0;
            if (jpeek(c, ']')) {
                ++c->p;
            } else {
                for (;;) {
                    uint64_t d = 0;
                    if (!juint(c, &d) || d > 0x7fffffff || e->ndim >= SAPPHIRE_ST_MAX_DIMS) {
                        c->err = 1;
                        free(key);
                        return 0;
                    }
                    e->shape[e->ndim++] = (int)d;
                    if (jpeek(c, ',')) {
                        ++c->p;
                        continue;
                    }
                    if (!jexpect(c, ']')) {
                        free(key);
                        return 0;
                    }
                    break;
                }
            }
            have_shape = 1;
        } else if (strcmp(key, "data_offsets") == 0) {
            if (!jexpect(c, '[') || !juint(c, &e->begin) || !jexpect(c, ',') || !juint(c, &e->end) ||
                !jexpect(c, ']')) {
                free(key);
                return 0;
            }
            have_off = 1;
        } else {
            jskip(c, 1);
        }
        free(key);
        if (c->err) return 0;
        if (jpeek(c, ',')) {
            ++c->p;
            continue;
        }
        if (!jexpect(c, '}')) return 0;
        break;
    }
    if (!(have_dtype && have_shape && have_off)) {
        LOG_ERROR("tensor '%s': dtype, shape or data_offsets missing", e->name);
        c->err = 1;
        return 0;
    }
    return 1;
}

// Bytes the payload of a tensor must hold; 0 when the shape does not fit the
// dtype or its element count overflows (a file is untrusted input).
static int expected_bytes(const st_entry *e, uint64_t *bytes) {
    uint64_t n = 1;
    for (int i = 0; i < e->ndim; ++i) {
        const uint64_t d = (uint64_t)e->shape[i];
        if (d != 0 && n > (UINT64_MAX / 8) / d) return 0;
        n *= d;
    }
    switch (e->dtype) {
        case DTYPE_F32: *bytes = n * 4; return 1;
        case DTYPE_BF16:
        case DTYPE_F16: *bytes = n * 2; return 1;
        default:
            if (e->ndim != 2 || e->shape[0] <= 0 || e->shape[1] <= 0) return 0;
            *bytes = (uint64_t)e->shape[0] * sapphire_row_bytes(e->dtype, e->shape[1]);
            return 1;
    }
}

static void free_entries(sapphire_safetensors_t *st) {
    for (int i = 0; i < st->count; ++i) {
        free(st->entries[i].name);
        if (st->entries[i].view) tensor_release(st->entries[i].view);
    }
    free(st->entries);
    st->entries = NULL;
    st->count = 0;
}

SAPPHIRE_API void sapphire_safetensors_close(sapphire_safetensors_t *st) {
    if (!st) return;
    free_entries(st);
    if (st->map && st->map != MAP_FAILED) munmap(st->map, st->map_size);
    if (st->fd >= 0) close(st->fd);
    free(st);
}

SAPPHIRE_API sapphire_safetensors_t *sapphire_safetensors_open(const char *path) {
    if (!path) {
        LOG_ERROR("path is NULL");
        return NULL;
    }
    sapphire_safetensors_t *st = (sapphire_safetensors_t *)calloc(1, sizeof *st);
    if (!st) return NULL;
    st->fd = open(path, O_RDONLY);
    struct stat sb;
    if (st->fd < 0 || fstat(st->fd, &sb) != 0) {
        LOG_ERROR("cannot open '%s': %s", path, strerror(errno));
        sapphire_safetensors_close(st);
        return NULL;
    }
    st->map_size = (size_t)sb.st_size;
    if (st->map_size < 8) {
        LOG_ERROR("'%s' is too short for a safetensors header", path);
        sapphire_safetensors_close(st);
        return NULL;
    }
    st->map = (uint8_t *)mmap(NULL, st->map_size, PROT_READ, MAP_PRIVATE, st->fd, 0);
    if (st->map == MAP_FAILED) {
        LOG_ERROR("mmap of '%s' failed: %s", path, strerror(errno));
        st->map = NULL;
        sapphire_safetensors_close(st);
        return NULL;
    }
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | st->map[i];
    if (hlen > st->map_size - 8) {
        LOG_ERROR("'%s': header length %llu exceeds the file", path, (unsigned long long)hlen);
        sapphire_safetensors_close(st);
        return NULL;
    }
    st->data = st->map + 8 + hlen;
    st->data_size = st->map_size - 8 - (size_t)hlen;
    jcur c = {(const char *)st->map + 8, (const char *)st->map + 8 + hlen, 0};
    int cap = 0;
    if (!jexpect(&c, '{')) goto bad;
    if (jpeek(&c, '}')) {
        ++c.p;
        return st;
    }
    for (;;) {
        char *name = jstring(&c);
        if (!name || !jexpect(&c, ':')) {
            free(name);
            goto bad;
        }
        if (strcmp(name, "__metadata__") == 0) {
            free(name);
            jskip(&c, 1);
        } else {
            if (st->count == cap) {
                cap = cap ? 2 * cap : 64;
                st_entry *t = (st_entry *)realloc(st->entries, (size_t)cap * sizeof *t);
                if (!t) {
                    free(name);
                    goto bad;
                }
                st->entries = t;
            }
            st_entry *e = &st->entries[st->count];
            memset(e, 0, sizeof *e);
            e->name = name;
            ++st->count;
            if (!parse_entry(&c, e)) goto bad;
            uint64_t want = 0;
            if (!expected_bytes(e, &want)) {
                LOG_ERROR("tensor '%s': shape does not fit its dtype (a quantized tensor needs a positive 2-D "
                          "shape [rows, cols]; the element count must fit 64 bits)", e->name);
                goto bad;
            }
            if (e->end < e->begin || e->end > st->data_size || e->end - e->begin != want) {
                LOG_ERROR("tensor '%s': data_offsets [%llu, %llu) do not hold the %llu bytes its dtype and shape "
                          "need inside the %zu-byte data section",
                          e->name, (unsigned long long)e->begin, (unsigned long long)e->end,
                          (unsigned long long)want, st->data_size);
                goto bad;
            }
        }
        if (c.err) goto bad;
        if (jpeek(&c, ',')) {
            ++c.p;
            continue;
        }
        if (!jexpect(&c, '}')) goto bad;
        break;
    }
    return st;
bad:
    LOG_ERROR("'%s': malformed safetensors header", path);
    sapphire_safetensors_close(st);
    return NULL;
}

SAPPHIRE_API int sapphire_safetensors_count(const sapphire_safetensors_t *st) { return st ? st->count : -1; }

SAPPHIRE_API const char *sapphire_safetensors_name(const sapphire_safetensors_t *st, int index) {
    if (!st || index < 0 || index >= st->count) return NULL;
    return st->entries[index].name;
}

SAPPHIRE_API tensor_t *sapphire_safetensors_tensor(sapphire_safetensors_t *st, const char *name) {
    if (!st || !name) return NULL;
    for (int i = 0; i < st->count; ++i) {
        st_entry *e = &st->entries[i];
        if (strcmp(e->name, name) != 0) continue;
        if (!e->view) {
            // The view is read-only in practice: the mapping is private and
            // PROT_READ; the library only reads weight bytes.
            e->view = tensor_create_view(e->dtype, e->ndim, e->shape, (void *)(st->data + e->begin));
            if (!e->view) LOG_ERROR("tensor '%s': view creation failed", name);
        }
        return e->view;
    }
    return NULL;
}
