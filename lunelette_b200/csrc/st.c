#define _GNU_SOURCE
#include "st.h"

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

typedef struct {
    const unsigned char *at, *end;
} cursor;

static void blank(cursor *c)
{
    while (c->at < c->end && (*c->at == ' ' || *c->at == '\t' || *c->at == '\n' ||
            *c->at == '\r')) {
        c->at++;
    }
}

static int take(cursor *c, unsigned char want)
{
    blank(c);
    if (c->at < c->end && *c->at == want) {
        c->at++;
        return 1;
    }
    return 0;
}

static int hex_digit(unsigned char h)
{
    if (h >= '0' && h <= '9') {
        return h - '0';
    }
    if (h >= 'a' && h <= 'f') {
        return h - 'a' + 10;
    }
    if (h >= 'A' && h <= 'F') {
        return h - 'A' + 10;
    }
    return -1;
}

/* JSON string of printable ASCII; escapes \" \\ \/ and \uXXXX (printable only). */
static int string_value(cursor *c, char *out, size_t capacity)
{
    size_t n = 0;
    if (!take(c, '"')) {
        return 0;
    }
    while (c->at < c->end) {
        unsigned ch = *c->at++;
        if (ch == '"') {
            out[n] = 0;
            return 1;
        }
        if (ch == '\\') {
            if (c->at == c->end) {
                return 0;
            }
            ch = *c->at++;
            if (ch == 'u') {
                unsigned code = 0;
                for (int i = 0; i < 4; i++) {
                    int d = c->at < c->end ? hex_digit(*c->at++) : -1;
                    if (d < 0) {
                        return 0;
                    }
                    code = code * 16 + (unsigned)d;
                }
                ch = code;
            } else if (ch != '"' && ch != '\\' && ch != '/') {
                return 0;
            }
        }
        if (ch < 32 || ch > 126 || n + 1 >= capacity) {
            return 0;
        }
        out[n++] = (char)ch;
    }
    return 0;
}

/* Unsigned decimal without leading zeros, overflow-checked. */
static int number_value(cursor *c, uint64_t *out)
{
    blank(c);
    if (c->at == c->end || *c->at < '0' || *c->at > '9') {
        return 0;
    }
    if (*c->at == '0') {
        c->at++;
        if (c->at < c->end && *c->at >= '0' && *c->at <= '9') {
            return 0;
        }
        *out = 0;
        return 1;
    }
    uint64_t v = 0;
    while (c->at < c->end && *c->at >= '0' && *c->at <= '9') {
        unsigned d = (unsigned)(*c->at++ - '0');
        if (v > (UINT64_MAX - d) / 10) {
            return 0;
        }
        v = v * 10 + d;
    }
    *out = v;
    return 1;
}

static int number_list(cursor *c, uint64_t *values, size_t capacity, size_t *count)
{
    *count = 0;
    if (!take(c, '[')) {
        return 0;
    }
    if (take(c, ']')) {
        return 1;
    }
    do {
        if (*count == capacity || !number_value(c, &values[*count])) {
            return 0;
        }
        (*count)++;
    } while (take(c, ','));
    return take(c, ']');
}

static int tensor_entry(cursor *c, lun_tensor *t)
{
    unsigned seen = 0;
    if (!take(c, '{')) {
        return 0;
    }
    do {
        char key[32], dtype[16];
        unsigned bit;
        if (!string_value(c, key, sizeof key) || !take(c, ':')) {
            return 0;
        }
        if (!strcmp(key, "dtype")) {
            bit = 1;
            if (!string_value(c, dtype, sizeof dtype)) {
                return 0;
            }
            if (!strcmp(dtype, "F8_E4M3")) {
                t->dtype = LUN_F8_E4M3;
            } else if (!strcmp(dtype, "BF16")) {
                t->dtype = LUN_BF16;
            } else if (!strcmp(dtype, "F32")) {
                t->dtype = LUN_F32;
            } else if (!strcmp(dtype, "I64")) {
                t->dtype = LUN_I64;
            } else {
                return 0;
            }
        } else if (!strcmp(key, "shape")) {
            bit = 2;
            if (!number_list(c, t->shape, LUN_ST_MAX_DIMS, &t->rank)) {
                return 0;
            }
        } else if (!strcmp(key, "data_offsets")) {
            uint64_t range[2];
            size_t n;
            bit = 4;
            if (!number_list(c, range, 2, &n) || n != 2) {
                return 0;
            }
            t->begin = range[0];
            t->end = range[1];
        } else {
            return 0;
        }
        if (seen & bit) {
            return 0;
        }
        seen |= bit;
    } while (take(c, ','));
    return take(c, '}') && seen == 7;
}

static int metadata_entry(cursor *c)
{
    char keys[64][LUN_ST_MAX_NAME];
    char value[4096];
    size_t n = 0;
    if (!take(c, '{')) {
        return 0;
    }
    if (take(c, '}')) {
        return 1;
    }
    do {
        if (n == 64 || !string_value(c, keys[n], sizeof keys[n])) {
            return 0;
        }
        for (size_t i = 0; i < n; i++) {
            if (!strcmp(keys[i], keys[n])) {
                return 0;
            }
        }
        n++;
        if (!take(c, ':') || !string_value(c, value, sizeof value)) {
            return 0;
        }
    } while (take(c, ','));
    return take(c, '}');
}

static int parse_header(lun_st *s, const unsigned char *text, size_t length)
{
    cursor c = {text, text + length};
    int metadata = 0;
    if (length == 0 || text[0] != '{' || !take(&c, '{')) {
        return -1;
    }
    if (!take(&c, '}')) {
        do {
            char name[LUN_ST_MAX_NAME];
            if (!string_value(&c, name, sizeof name) || !name[0] || !take(&c, ':')) {
                return -1;
            }
            if (!strcmp(name, "__metadata__")) {
                if (metadata++ || !metadata_entry(&c)) {
                    return -1;
                }
                continue;
            }
            if (s->count == LUN_ST_MAX_TENSORS || lun_st_find(s, name)) {
                return -1;
            }
            lun_tensor *t = &s->tensors[s->count];
            memset(t, 0, sizeof *t);
            memcpy(t->name, name, strlen(name) + 1);
            if (!tensor_entry(&c, t)) {
                return -1;
            }
            s->count++;
        } while (take(&c, ','));
        if (!take(&c, '}')) {
            return -1;
        }
    }
    blank(&c);
    return c.at == c.end ? 0 : -1;
}

static int by_begin(const void *a, const void *b)
{
    const lun_tensor *x = *(const lun_tensor *const *)a, *y = *(const lun_tensor *const *)b;
    if (x->begin != y->begin) {
        return x->begin < y->begin ? -1 : 1;
    }
    return (x->end > x->begin) - (y->end > y->begin);
}

/* Sizes must match shapes; non-empty ranges must tile [0, data_bytes) exactly;
 * empty ranges may only sit on a boundary between tiles. */
static int check_layout(const lun_st *s, uint64_t data_bytes)
{
    for (size_t i = 0; i < s->count; i++) {
        const lun_tensor *t = &s->tensors[i];
        uint64_t elements = 1;
        int empty = 0;
        for (size_t k = 0; k < t->rank; k++) {
            if (t->shape[k] > INT64_MAX) {
                return -1;
            }
            empty |= t->shape[k] == 0;
        }
        if (empty) {
            elements = 0;
        } else {
            for (size_t k = 0; k < t->rank; k++) {
                if (elements > UINT64_MAX / t->shape[k]) {
                    return -1;
                }
                elements *= t->shape[k];
            }
        }
        if (elements > UINT64_MAX / (uint64_t)t->dtype || t->end < t->begin ||
            t->end > data_bytes || t->end - t->begin != elements * (uint64_t)t->dtype) {
            return -1;
        }
    }
    const lun_tensor **order = malloc((s->count ? s->count : 1) * sizeof *order);
    if (!order) {
        return -1;
    }
    for (size_t i = 0; i < s->count; i++) {
        order[i] = &s->tensors[i];
    }
    qsort(order, s->count, sizeof *order, by_begin);
    uint64_t cursor_at = 0;
    int status = 0;
    for (size_t i = 0; i < s->count && !status; i++) {
        const lun_tensor *t = order[i];
        if (t->end == t->begin) {
            /* must not fall strictly inside a non-empty tensor */
            for (size_t k = 0; k < s->count; k++) {
                if (s->tensors[k].begin < t->begin && t->begin < s->tensors[k].end) {
                    status = -1;
                }
            }
            continue;
        }
        if (t->begin != cursor_at) {
            status = -1;
        }
        cursor_at = t->end;
    }
    if (!status && cursor_at != data_bytes) {
        status = -1;
    }
    free(order);
    return status;
}

int lun_st_open(lun_st *s, const char *path, char *error, size_t capacity)
{
    const char *why = "invalid arguments";
    unsigned char *header = NULL;
    if (!s) {
        goto report;
    }
    memset(s, 0, sizeof *s);
    s->fd = -1;
    if (!path) {
        goto fail;
    }
    why = "cannot open/size file";
    s->fd = open(path, O_RDONLY | O_CLOEXEC);
    struct stat info;
    if (s->fd < 0 || fstat(s->fd, &info) != 0 || !S_ISREG(info.st_mode) || info.st_size < 8) {
        goto fail;
    }
    s->file_bytes = (uint64_t)info.st_size;
    unsigned char prefix[8];
    why = "invalid/truncated header length (limit 1 MiB)";
    if (pread(s->fd, prefix, 8, 0) != 8) {
        goto fail;
    }
    uint64_t n = 0;
    for (int i = 0; i < 8; i++) {
        n |= (uint64_t)prefix[i] << (8 * i);
    }
    if (n < 2 || n > LUN_ST_MAX_HEADER || n > s->file_bytes - 8) {
        goto fail;
    }
    s->data_base = 8 + n;
    why = "allocation failure";
    header = malloc((size_t)n);
    s->tensors = calloc(LUN_ST_MAX_TENSORS, sizeof *s->tensors);
    if (!header || !s->tensors) {
        goto fail;
    }
    why = "truncated header";
    if (pread(s->fd, header, (size_t)n, 8) != (ssize_t)n) {
        goto fail;
    }
    why = "invalid/unsupported header: require unique ASCII names, F8_E4M3/BF16/F32/I64, rank <=8";
    if (parse_header(s, header, (size_t)n)) {
        goto fail;
    }
    why = "invalid tensor shape/size/offsets or non-contiguous data";
    if (check_layout(s, s->file_bytes - s->data_base)) {
        goto fail;
    }
    free(header);
    if (error && capacity) {
        error[0] = 0;
    }
    return 0;
fail:
    free(header);
    lun_st_close(s);
report:
    if (error && capacity) {
        snprintf(error, capacity, "%s", why);
    }
    return -1;
}

void lun_st_close(lun_st *s)
{
    if (!s) {
        return;
    }
    if (s->fd >= 0) {
        close(s->fd);
    }
    free(s->tensors);
    memset(s, 0, sizeof *s);
    s->fd = -1;
}

const lun_tensor *lun_st_find(const lun_st *s, const char *name)
{
    if (!s || !name || !s->tensors) {
        return NULL;
    }
    for (size_t i = 0; i < s->count; i++) {
        if (!strcmp(s->tensors[i].name, name)) {
            return &s->tensors[i];
        }
    }
    return NULL;
}

int lun_st_read(const lun_st *s, const lun_tensor *t, uint64_t offset, void *out, size_t bytes)
{
    if (!s || s->fd < 0 || !t || (!out && bytes) || t < s->tensors ||
        t >= s->tensors + s->count) {
        return -1;
    }
    uint64_t size = t->end - t->begin;
    if (offset > size || bytes > size - offset) {
        return -1;
    }
    uint64_t position = s->data_base + t->begin + offset;
    unsigned char *dst = out;
    while (bytes) {
        ssize_t got = pread(s->fd, dst, bytes, (off_t)position);
        if (got < 0 && errno == EINTR) {
            continue;
        }
        if (got <= 0) {
            return -1;
        }
        dst += got;
        bytes -= (size_t)got;
        position += (uint64_t)got;
    }
    return 0;
}

float lun_bf16_to_f32(uint16_t bits)
{
    uint32_t word = (uint32_t)bits << 16;
    float value;
    memcpy(&value, &word, sizeof value);
    return value;
}

float lun_e4m3_to_f32(unsigned char code)
{
    unsigned magnitude = code & 0x7fu;
    if (magnitude == 0x7f) {
        return NAN;
    }
    unsigned exponent = magnitude >> 3, mantissa = magnitude & 7u;
    float value;
    if (exponent) {
        /* rebias 7 -> 127 and move the 3 mantissa bits to the top of FP32's 23 */
        uint32_t word = ((exponent + 120u) << 23) | (mantissa << 20);
        memcpy(&value, &word, sizeof value);
    } else {
        value = (float)mantissa * 0x1p-9f; /* subnormal: exact */
    }
    return (code & 0x80u) ? -value : value;
}
