/* Seeded synthetic checkpoint in the reference's tensor contract
 * (src/metal_weights.c:79-158): a random-init Ministral-3-3B-shaped model for
 * benchmarks and parity runs, since no real checkpoint is available.
 *
 *   linear W ~ N(0, 0.02); scale s = BF16_rne(max|W| / 448) (a BF16 scale is
 *   what compact admission requires); codes = E4M3 round-to-nearest-even of
 *   W / s, saturating at +-448 and never producing the NaN codes 0x7f/0xff;
 *   weight_scale_inv = s, activation_scale = 1.0 (both BF16 rank-0).
 *   embedding (tied head) ~ N(0, 0.02) in BF16; norm gains 1.0.
 *
 * Every tensor has its own counter-based stream (SplitMix64 keyed by seed and
 * tensor id, Box-Muller in double), so the file is identical for a seed on
 * every machine and thread count. Data are laid out large-first so every
 * matrix starts 256-byte aligned. */
#define _GNU_SOURCE
#include "weights.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define LUN_API __attribute__((visibility("default")))

static uint64_t mix64(uint64_t z)
{
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* Normal pair number k of tensor stream `key`. */
static void normal_pair(uint64_t key, uint64_t k, double *a, double *b)
{
    uint64_t z1 = mix64(key ^ mix64(2 * k)), z2 = mix64(key ^ mix64(2 * k + 1));
    double u1 = ((double)(z1 >> 11) + 0.5) * 0x1p-53;
    double u2 = (double)(z2 >> 11) * 0x1p-53;
    double r = sqrt(-2.0 * log(u1)), theta = 6.283185307179586 * u2;
    *a = r * cos(theta);
    *b = r * sin(theta);
}

static uint16_t bf16_rne(float v)
{
    uint32_t bits;
    memcpy(&bits, &v, 4);
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

/* FP32 -> E4M3FN, round to nearest even, saturating to +-448. */
LUN_API unsigned char lunelette_cuda_e4m3_encode(float v)
{
    unsigned char sign = signbit(v) ? 0x80 : 0;
    float a = fabsf(v);
    if (!(a < 448.0f)) {
        return sign | 0x7e;
    }
    if (a < 0x1p-6f) {
        /* subnormal grid 2^-9; q == 8 lands exactly on the smallest normal code */
        return sign | (unsigned char)nearbyintf(a * 512.0f);
    }
    int e2;
    frexpf(a, &e2);
    int exponent = e2 - 1; /* a in [2^exponent, 2^(exponent+1)) */
    float q = nearbyintf(ldexpf(a, 3 - exponent)); /* in [8, 16] */
    if (q == 16.0f) {
        exponent++;
        q = 8.0f;
    }
    int biased = exponent + 7, mantissa = (int)q - 8;
    if (biased > 15 || (biased == 15 && mantissa == 7)) {
        return sign | 0x7e;
    }
    return sign | (unsigned char)(biased << 3 | mantissa);
}

enum { FILL_NORMAL, FILL_BF16, FILL_E4M3 };

typedef struct {
    int mode;
    uint64_t key;
    size_t begin, end;    /* element range [begin, end) of the stream; begin even */
    size_t base;          /* stream index of values[0] / bytes[0] */
    float *values;
    unsigned char *bytes; /* FILL_BF16: 2 bytes per element; FILL_E4M3: 1 */
    float scale;
    float maxabs;
} fill_job;

static void *fill_worker(void *arg)
{
    fill_job *job = arg;
    float maxabs = 0;
    if (job->mode == FILL_E4M3) {
        for (size_t i = job->begin; i < job->end; i++) {
            job->bytes[i - job->base] = lunelette_cuda_e4m3_encode(job->values[i - job->base] /
                job->scale);
        }
        return NULL;
    }
    for (size_t i = job->begin; i < job->end; i += 2) {
        double a, b;
        normal_pair(job->key, i / 2, &a, &b);
        float pair[2] = {(float)(0.02 * a), (float)(0.02 * b)};
        for (size_t k = 0; k < 2 && i + k < job->end; k++) {
            size_t at = i + k - job->base;
            if (job->mode == FILL_NORMAL) {
                job->values[at] = pair[k];
                maxabs = fabsf(pair[k]) > maxabs ? fabsf(pair[k]) : maxabs;
            } else {
                uint16_t h = bf16_rne(pair[k]);
                job->bytes[2 * at] = (unsigned char)h;
                job->bytes[2 * at + 1] = (unsigned char)(h >> 8);
            }
        }
    }
    job->maxabs = maxabs;
    return NULL;
}

/* Run one pass over stream elements [begin, end) on `threads` threads;
 * returns max|value| for FILL_NORMAL. */
static float run_fill(fill_job proto, size_t begin, size_t end, int threads)
{
    pthread_t tid[64];
    fill_job jobs[64];
    int created[64] = {0};
    size_t n = end - begin, per = ((n + (size_t)threads - 1) / (size_t)threads + 1) & ~(size_t)1;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        size_t b = begin + (size_t)t * per;
        if (b >= end) {
            break;
        }
        jobs[t] = proto;
        jobs[t].begin = b;
        jobs[t].end = b + per < end ? b + per : end;
        jobs[t].base = begin;
        created[t] = pthread_create(&tid[t], NULL, fill_worker, &jobs[t]) == 0;
        if (!created[t]) {
            fill_worker(&jobs[t]);
        }
        started++;
    }
    float maxabs = 0;
    for (int t = 0; t < started; t++) {
        if (created[t]) {
            pthread_join(tid[t], NULL);
        }
        maxabs = jobs[t].maxabs > maxabs ? jobs[t].maxabs : maxabs;
    }
    return maxabs;
}

typedef struct {
    char name[LUN_ST_MAX_NAME + 32];
    const char *dtype;
    size_t rows, cols; /* cols 0: vector; rows 0: scalar */
    size_t bytes;
    int kind; /* 0 embedding, 1 linear, 2 norm, 3 weight scale, 4 activation scale */
    int linear; /* linear tensor id for kinds 1 and 3 */
} entry;

LUN_API int lunelette_cuda_synth_checkpoint(const char *path, uint64_t seed, char *error,
    size_t capacity)
{
    static const size_t linear_slots[7] = {1, 2, 3, 4, 6, 7, 8};
    const size_t count = 1 + LUN_LAYERS * 7 * 3 + 1 + LUN_LAYERS * 2;
    entry *e = calloc(count, sizeof *e);
    float *values = NULL;
    unsigned char *bytes = NULL;
    float *scales = calloc(LUN_LAYERS * 7, sizeof(float));
    FILE *file = NULL;
    char *header = NULL;
    int status = -1;
    long ncpu = sysconf(_SC_NPROCESSORS_ONLN);
    int threads = ncpu < 1 ? 1 : (ncpu > 64 ? 64 : (int)ncpu);
    if (!e || !scales || !path) {
        snprintf(error, capacity, "synth: bad arguments or allocation failure");
        goto done;
    }
    size_t n = 0;
    e[n++] = (entry){"language_model.model.embed_tokens.weight", "BF16", LUN_VOCAB, LUN_HIDDEN,
        (size_t)LUN_VOCAB * LUN_HIDDEN * 2, 0, 0};
    for (int layer = 0; layer < LUN_LAYERS; layer++) {
        for (int s = 0; s < 7; s++) {
            const lun_block_weight *b = &lun_block_weights[linear_slots[s]];
            entry *x = &e[n++];
            snprintf(x->name, sizeof x->name, "language_model.model.layers.%d.%s", layer, b->suffix);
            x->dtype = "F8_E4M3";
            x->rows = b->rows;
            x->cols = b->cols;
            x->bytes = b->rows * b->cols;
            x->kind = 1;
            x->linear = layer * 7 + s;
        }
    }
    e[n++] = (entry){"language_model.model.norm.weight", "BF16", LUN_HIDDEN, 0, LUN_HIDDEN * 2, 2, 0};
    for (int layer = 0; layer < LUN_LAYERS; layer++) {
        for (int s = 0; s < 2; s++) {
            entry *x = &e[n++];
            snprintf(x->name, sizeof x->name, "language_model.model.layers.%d.%s", layer,
                lun_block_weights[s ? 5 : 0].suffix);
            x->dtype = "BF16";
            x->rows = LUN_HIDDEN;
            x->bytes = LUN_HIDDEN * 2;
            x->kind = 2;
        }
    }
    for (int layer = 0; layer < LUN_LAYERS; layer++) {
        for (int s = 0; s < 7; s++) {
            for (int k = 0; k < 2; k++) {
                entry *x = &e[n++];
                snprintf(x->name, sizeof x->name, "language_model.model.layers.%d.%.*s%s", layer,
                    (int)strlen(lun_block_weights[linear_slots[s]].suffix) - 6,
                    lun_block_weights[linear_slots[s]].suffix,
                    k ? "activation_scale" : "weight_scale_inv");
                x->dtype = "BF16";
                x->bytes = 2;
                x->kind = 3 + k;
                x->linear = layer * 7 + s;
            }
        }
    }
    /* header: offsets in listed order, padded with spaces to a 256-byte data base */
    size_t header_capacity = count * 200 + 1024, used = 0, offset = 0;
    header = malloc(header_capacity);
    if (!header) {
        snprintf(error, capacity, "synth: allocation failure");
        goto done;
    }
    used += (size_t)snprintf(header + used, header_capacity - used,
        "{\"__metadata__\":{\"format\":\"pt\",\"generator\":\"lunelette_b200 synth seed %llu\"}",
        (unsigned long long)seed);
    for (size_t i = 0; i < n; i++) {
        char shape[64];
        if (e[i].kind == 3 || e[i].kind == 4) {
            snprintf(shape, sizeof shape, "[]");
        } else if (e[i].cols) {
            snprintf(shape, sizeof shape, "[%zu,%zu]", e[i].rows, e[i].cols);
        } else {
            snprintf(shape, sizeof shape, "[%zu]", e[i].rows);
        }
        used += (size_t)snprintf(header + used, header_capacity - used,
            ",\"%s\":{\"dtype\":\"%s\",\"shape\":%s,\"data_offsets\":[%zu,%zu]}", e[i].name,
            e[i].dtype, shape, offset, offset + e[i].bytes);
        offset += e[i].bytes;
    }
    header[used++] = '}';
    while ((8 + used) % 256) {
        header[used++] = ' ';
    }
    file = fopen(path, "wb");
    if (!file) {
        snprintf(error, capacity, "synth: cannot create %s", path);
        goto done;
    }
    unsigned char prefix[8];
    for (int i = 0; i < 8; i++) {
        prefix[i] = (unsigned char)((uint64_t)used >> (8 * i));
    }
    if (fwrite(prefix, 1, 8, file) != 8 || fwrite(header, 1, used, file) != used) {
        goto write_error;
    }
    const size_t chunk = (size_t)1 << 24;
    values = malloc(((size_t)LUN_INNER * LUN_HIDDEN > chunk ? (size_t)LUN_INNER * LUN_HIDDEN : chunk) *
        sizeof(float));
    bytes = malloc((size_t)LUN_INNER * LUN_HIDDEN > chunk * 2 ? (size_t)LUN_INNER * LUN_HIDDEN : chunk * 2);
    if (!values || !bytes) {
        snprintf(error, capacity, "synth: allocation failure");
        goto done;
    }
    uint64_t root = mix64(seed ^ 0x4c756e656c657474ull);
    for (size_t i = 0; i < n; i++) {
        if (e[i].kind == 0) {
            size_t total = e[i].rows * e[i].cols;
            uint64_t key = mix64(root ^ 0x1000000ull);
            for (size_t b = 0; b < total; b += chunk) {
                size_t m = total - b < chunk ? total - b : chunk;
                fill_job proto = {FILL_BF16, key, 0, 0, 0, NULL, bytes, 1.0f, 0};
                run_fill(proto, b, b + m, threads);
                if (fwrite(bytes, 1, 2 * m, file) != 2 * m) {
                    goto write_error;
                }
            }
        } else if (e[i].kind == 1) {
            size_t total = e[i].bytes;
            uint64_t key = mix64(root ^ (0x2000000ull + (uint64_t)e[i].linear));
            fill_job proto = {FILL_NORMAL, key, 0, 0, 0, values, bytes, 1.0f, 0};
            float maxabs = run_fill(proto, 0, total, threads);
            uint16_t scale_bits = bf16_rne(maxabs / 448.0f);
            float scale = lun_bf16_to_f32(scale_bits);
            scales[e[i].linear] = scale;
            proto.mode = FILL_E4M3;
            proto.scale = scale;
            run_fill(proto, 0, total, threads);
            if (fwrite(bytes, 1, total, file) != total) {
                goto write_error;
            }
        } else if (e[i].kind == 2) {
            for (size_t k = 0; k < LUN_HIDDEN; k++) {
                bytes[2 * k] = 0x80; /* BF16 1.0 = 0x3f80 */
                bytes[2 * k + 1] = 0x3f;
            }
            if (fwrite(bytes, 1, LUN_HIDDEN * 2, file) != LUN_HIDDEN * 2) {
                goto write_error;
            }
        } else {
            uint16_t h = e[i].kind == 3 ? bf16_rne(scales[e[i].linear]) : 0x3f80;
            unsigned char two[2] = {(unsigned char)h, (unsigned char)(h >> 8)};
            if (fwrite(two, 1, 2, file) != 2) {
                goto write_error;
            }
        }
    }
    if (fclose(file)) {
        file = NULL;
        goto write_error;
    }
    file = NULL;
    status = 0;
    goto done;
write_error:
    snprintf(error, capacity, "synth: write failed for %s", path);
done:
    if (file) {
        fclose(file);
    }
    free(e);
    free(values);
    free(bytes);
    free(scales);
    free(header);
    return status;
}
