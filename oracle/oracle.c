/* TEST INFRASTRUCTURE ONLY — CPU oracle for the Lunelette decoder hot path.
 * See oracle.h for the pinning story. Compiled with -ffp-contract=off and no
 * fast-math, matching the reference's "fp contract(off)" and precise math
 * (src/metal_kernels.metal:3, src/metal_runtime.m:114-116).
 *
 * A Metal SIMD-group of 32 lanes is modelled as 32 explicit partial sums; the
 * reference's simd_sum has an unspecified order, so this file fixes it as the
 * xor-butterfly (offsets 16, 8, 4, 2, 1) that a 32-lane shuffle reduction uses.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define LANES 32

/* Precision-study knobs (default 0 = the reference's FP32 everywhere). They let
 * tests measure what a narrower storage format for KV rows (kv_rounding) or for
 * projection inputs (input_rounding) does to per-layer drift: 1 rounds to BF16,
 * 2 to FP16, both round-to-nearest-even; for inputs, 3 and 4 write each row as
 * the sum of two or three scaled FP16 terms (round_inputs). Never used as a
 * reference result. */
static int kv_rounding, input_rounding;

void oracle_set_rounding(int kv, int input)
{
    kv_rounding = kv;
    input_rounding = input;
}

static float round_to(float v, int mode)
{
    if (mode == 1) {
        uint32_t bits;
        memcpy(&bits, &v, 4);
        bits = (bits + 0x7fffu + ((bits >> 16) & 1u)) & 0xffff0000u;
        memcpy(&v, &bits, 4);
    } else if (mode == 2) {
        _Float16 h = (_Float16)v;
        v = (float)h;
    }
    return v;
}

static void round_rows(float *v, size_t n, int mode)
{
    if (mode) {
        for (size_t i = 0; i < n; i++) {
            v[i] = round_to(v[i], mode);
        }
    }
}

/* Projection inputs as the CUDA kernels' tensor-core operands carry them
 * (input modes 3 and 4): each row scaled by the power of two that brings its
 * largest magnitude into [2^14, 2^15), then written as a sum of FP16 terms,
 * each the round-to-nearest-even of what the earlier terms left: two terms
 * (hi + lo, mode 3) or three (mode 4). Other modes round element by element. */
static void round_inputs(float *v, size_t count, size_t width, int mode)
{
    if (mode != 3 && mode != 4) {
        round_rows(v, count * width, mode);
        return;
    }
    for (size_t r = 0; r < count; r++) {
        float *row = v + r * width;
        float peak = 0.0f;
        for (size_t c = 0; c < width; c++) {
            peak = fmaxf(peak, fabsf(row[c]));
        }
        if (peak == 0.0f || !isfinite(peak)) {
            continue;
        }
        int e;
        frexpf(peak, &e);  /* peak = m * 2^e, m in [0.5, 1) */
        const int shift = 15 - e;  /* peak * 2^shift in [2^14, 2^15) */
        for (size_t c = 0; c < width; c++) {
            const float y = ldexpf(row[c], shift);
            float left = y, sum = 0.0f;
            for (int term = 0; term < mode - 1; term++) {
                const float part = (float)(_Float16)left;
                sum += part;
                left = y - sum;
            }
            row[c] = ldexpf(sum, -shift);
        }
    }
}

void oracle_set_threads(int threads)
{
#ifdef _OPENMP
    if (threads > 0) {
        omp_set_num_threads(threads);
    }
#else
    (void)threads;
#endif
}

int oracle_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* simd_sum over 32 lane values, fixed xor-butterfly order; lane 0's result. */
static float lane_sum(const float *values)
{
    float s[LANES];
    memcpy(s, values, sizeof s);
    for (int offset = LANES / 2; offset; offset >>= 1) {
        float t[LANES];
        for (int l = 0; l < LANES; l++) {
            t[l] = s[l] + s[l ^ offset];
        }
        memcpy(s, t, sizeof s);
    }
    return s[0];
}

/* E4M3FN byte -> FP32, restating weight() without the scale
 * (src/metal_kernels.metal:136-144; host twin st_f8_e4m3_to_f32,
 * src/safetensors.c:505-519). Codes 0x7f/0xff are NaN here (the host rejects
 * them before dispatch). */
float oracle_fp8_decode(unsigned char code)
{
    unsigned exponent = (code >> 3) & 15u;
    unsigned fraction = code & 7u;
    if (exponent == 15 && fraction == 7) {
        return NAN;
    }
    float value = exponent == 0 ? ldexpf((float)fraction, -9) :
        ldexpf(1.0f + (float)fraction / 8.0f, (int)exponent - 7);
    return (code & 128) ? -value : value;
}

/* YaRN cos/sin for one position: restates lunelette_metal_yarn
 * (src/metal_yarn.c:8-33) — ramp bounds from double maths, FP32 per-pair
 * inverse frequency blend, FP32 angle, split-half duplicated table, mscale 1. */
int oracle_yarn(uint32_t position, float cosine[128], float sine[128])
{
    if (position >= 262144u) {
        return -1;
    }
    const double pi = 3.14159265358979323846;
    const double head_dim = 128.0, original = 16384.0, theta = 1e6;
    float low = (float)floor(head_dim * log(original / (32.0 * 2.0 * pi)) /
        (2.0 * log(theta)));
    float high = (float)ceil(head_dim * log(original / (2.0 * pi)) / (2.0 * log(theta)));
    for (int pair = 0; pair < 64; pair++) {
        float frequency = powf(1000000.0f, (float)(2 * pair) / 128.0f);
        float ramp = fminf(1.0f, fmaxf(0.0f, ((float)pair - low) / (high - low)));
        float keep = 1.0f - ramp;
        float inverse = (1.0f / (16.0f * frequency)) * (1.0f - keep) +
            (1.0f / frequency) * keep;
        float angle = inverse * (float)position;
        float c = cosf(angle), s = sinf(angle);
        cosine[pair] = cosine[pair + 64] = c;
        sine[pair] = sine[pair + 64] = s;
    }
    return 0;
}

/* One output of `project` / `project_fp8`: lane-strided Kahan partials, then
 * simd_sum (src/metal_kernels.metal:7-27, 154-177). w holds already-scaled FP32
 * weights (weight(code, scale) in the FP8 case). */
/* The oracle's hot loops are compiled for several vector widths and the widest
 * the host supports is picked at load time; each lane's arithmetic is the same
 * scalar FP32 sequence whatever the width (no contraction: -ffp-contract=off). */
#if defined(__x86_64__) && defined(__GNUC__) && !defined(__clang__)
#define ORACLE_CLONES __attribute__((target_clones("avx512f", "avx2", "default")))
#else
#define ORACLE_CLONES
#endif

ORACLE_CLONES
static float kahan_dot(const float *w, const float *x, size_t cols)
{
    float sum[LANES] = {0}, correction[LANES] = {0};
    size_t full = cols / LANES * LANES;
    for (size_t c = 0; c < full; c += LANES) {
        for (int l = 0; l < LANES; l++) {
            float product = w[c + l] * x[c + l];
            float value = product - correction[l];
            float next = sum[l] + value;
            correction[l] = (next - sum[l]) - value;
            sum[l] = next;
        }
    }
    for (size_t l = 0; full + l < cols; l++) {
        float product = w[full + l] * x[full + l];
        float value = product - correction[l];
        float next = sum[l] + value;
        correction[l] = (next - sum[l]) - value;
        sum[l] = next;
    }
    return lane_sum(sum);
}

/* kahan_dot for four inputs over the same weights: four independent chains per
 * lane, each the exact operation sequence of kahan_dot, so each result equals
 * kahan_dot's bit for bit. The Kahan update is a chain of four dependent
 * additions per step; interleaving four inputs keeps the vector units busy
 * instead of waiting on that chain (and reads each weight once for all four). */
#define ORACLE_GROUP 4
ORACLE_CLONES
static void kahan_dot_group(const float *w, const float *x, size_t stride, size_t cols, float *out,
    size_t out_stride)
{
    float s[ORACLE_GROUP][LANES] = {{0}}, c[ORACLE_GROUP][LANES] = {{0}};
    size_t full = cols / LANES * LANES;
    for (size_t k = 0; k < full; k += LANES) {
        for (int g = 0; g < ORACLE_GROUP; g++) {
            const float *xg = x + g * stride + k;
            for (int l = 0; l < LANES; l++) {
                float product = w[k + l] * xg[l];
                float value = product - c[g][l];
                float next = s[g][l] + value;
                c[g][l] = (next - s[g][l]) - value;
                s[g][l] = next;
            }
        }
    }
    for (int g = 0; g < ORACLE_GROUP; g++) {
        const float *xg = x + g * stride;
        for (size_t l = 0; full + l < cols; l++) {
            float product = w[full + l] * xg[full + l];
            float value = product - c[g][l];
            float next = s[g][l] + value;
            c[g][l] = (next - s[g][l]) - value;
            s[g][l] = next;
        }
        out[g * out_stride] = lane_sum(s[g]);
    }
}

/* Precision-study knob (default 0: the Kahan lane sums above). A positive
 * value n models a tensor core's FP32 accumulation as measured on earlier
 * NVIDIA parts (Fasi, Higham, Mikaitis, Pranesh, "Numerical behavior of
 * NVIDIA tensor cores", PeerJ Computer Science 7:e330, 2021): products exact,
 * each block of 16 products added to the accumulator and the sum truncated
 * toward zero to FP32, over chains of n blocks (the kernels split K over CTAs
 * and accumulators) whose results are added in FP32. A model for studies
 * only, not a statement of how a B200 rounds. */
static int accumulation_study;

void oracle_set_accumulation(int mode)
{
    accumulation_study = mode;
}

static float toward_zero(double s)
{
    float f = (float)s;
    if (fabs((double)f) > fabs(s)) {
        f = nextafterf(f, 0.0f);
    }
    return f;
}

/* Chains of `chain` blocks of 16 products, each accumulated as above; the
 * chains' results added in FP32 (round to nearest) in order. */
static float truncated_dot(const float *w, const float *x, size_t cols, size_t chain)
{
    float total = 0.0f;
    const size_t span = 16 * chain;
    for (size_t k0 = 0; k0 < cols; k0 += span) {
        size_t k1 = k0 + span < cols ? k0 + span : cols;
        float acc = 0.0f;
        for (size_t c0 = k0; c0 < k1; c0 += 16) {
            size_t c1 = c0 + 16 < k1 ? c0 + 16 : k1;
            double s = acc;
            for (size_t c = c0; c < c1; c++) {
                s += (double)w[c] * (double)x[c];
            }
            acc = toward_zero(s);
        }
        total += acc;
    }
    return total;
}

void oracle_project(const float *weights, const float *input, float *output,
    size_t rows, size_t cols, size_t count)
{
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < rows; row++) {
        for (size_t token = 0; token < count; token++) {
            output[token * rows + row] = kahan_dot(weights + row * cols,
                input + token * cols, cols);
        }
    }
}

/* project_fp8 (src/metal_kernels.metal:154-177): weight(code, scale) * input.
 * Decoding a row once and reusing it for every token is value-identical. */
void oracle_project_fp8(const unsigned char *packed, float scale, const float *input,
    float *output, size_t rows, size_t cols, size_t count)
{
    float table[256];
    for (int code = 0; code < 256; code++) {
        table[code] = oracle_fp8_decode((unsigned char)code) * scale;
    }
    /* Blocks of ORACLE_ROWS decoded rows against blocks of ORACLE_TOKENS input
     * rows, so a block of inputs stays in cache while every row of the block
     * uses it (a long prompt's inputs are tens of MB). Each output is still one
     * kahan_dot sequence over all columns, so the results do not change. */
    enum { ORACLE_ROWS = 32, ORACLE_TOKENS = 32 };
    size_t blocks = (rows + ORACLE_ROWS - 1) / ORACLE_ROWS;
    #pragma omp parallel
    {
        float *row_values = malloc((size_t)ORACLE_ROWS * cols * sizeof(float));
        #pragma omp for schedule(dynamic, 1)
        for (size_t block = 0; block < blocks; block++) {
            size_t r0 = block * ORACLE_ROWS;
            size_t nr = rows - r0 < ORACLE_ROWS ? rows - r0 : ORACLE_ROWS;
            for (size_t r = 0; r < nr; r++) {
                const unsigned char *codes = packed + (r0 + r) * cols;
                for (size_t c = 0; c < cols; c++) {
                    row_values[r * cols + c] = table[codes[c]];
                }
            }
            for (size_t t0 = 0; t0 < count; t0 += ORACLE_TOKENS) {
                size_t t1 = t0 + ORACLE_TOKENS < count ? t0 + ORACLE_TOKENS : count;
                for (size_t r = 0; r < nr; r++) {
                    const float *w = row_values + r * cols;
                    size_t token = t0;
                    if (accumulation_study) {
                        for (; token < t1; token++) {
                            output[token * rows + r0 + r] = truncated_dot(w, input + token * cols, cols,
                                (size_t)accumulation_study);
                        }
                    }
                    for (; token + ORACLE_GROUP <= t1; token += ORACLE_GROUP) {
                        kahan_dot_group(w, input + token * cols, cols, cols, &output[token * rows + r0 + r], rows);
                    }
                    for (; token < t1; token++) {
                        output[token * rows + r0 + r] = kahan_dot(w, input + token * cols, cols);
                    }
                }
            }
        }
        free(row_values);
    }
}

/* Same lane loop over a BF16 matrix widened exactly to FP32: the tied head
 * reads the expanded FP32 embedding (src/metal_encode.m:207-210). */
static void project_bf16(const uint16_t *weights, const float *input, float *output,
    size_t rows, size_t cols)
{
    #pragma omp parallel
    {
        float *row_values = malloc(cols * sizeof(float));
        #pragma omp for schedule(static)
        for (size_t row = 0; row < rows; row++) {
            for (size_t c = 0; c < cols; c++) {
                uint32_t word = (uint32_t)weights[row * cols + c] << 16;
                memcpy(&row_values[c], &word, 4);
            }
            output[row] = kahan_dot(row_values, input, cols);
        }
        free(row_values);
    }
}

/* norm (src/metal_kernels.metal:29-44): w * (x * rsqrt(mean(x^2) + eps)). */
void oracle_norm(const float *weights, const float *input, float *output,
    size_t width, size_t count)
{
    for (size_t token = 0; token < count; token++) {
        const float *x = input + token * width;
        float lanes[LANES] = {0};
        for (size_t c = 0; c < width; c++) {
            lanes[c % LANES] += x[c] * x[c];
        }
        float scale = 1.0f / sqrtf(lane_sum(lanes) / (float)width + 1e-5f);
        for (size_t c = 0; c < width; c++) {
            output[token * width + c] = weights[c] * (x[c] * scale);
        }
    }
}

/* element (src/metal_kernels.metal:47-57): 0 residual add, 1 SiLU, 2 multiply. */
void oracle_element(const float *first, const float *second, float *output,
    size_t n, int mode)
{
    for (size_t i = 0; i < n; i++) {
        float value = first[i];
        output[i] = mode == 0 ? value + second[i] :
            (mode == 1 ? value / (1.0f + expf(-value)) : value * second[i]);
    }
}

/* rope (src/metal_kernels.metal:59-78): split-half rotation with the host
 * cos/sin table; queries also scale by 1 + 0.1*ln(1 + floor(pos/16384)). */
void oracle_rope(const float *input, const float *cosine, const float *sine,
    const uint32_t *positions, float *output, size_t width, size_t count, int query)
{
    for (size_t index = 0; index < width * count; index++) {
        size_t token = index / width;
        size_t column = index % 128;
        float rotated = column < 64 ? -input[index + 64] : input[index - 64];
        float value = input[index] * cosine[token * 128 + column] +
            rotated * sine[token * 128 + column];
        if (query) {
            value *= 1.0f + 0.1f * logf(1.0f + (float)(positions[token] / 16384u));
        }
        output[index] = value;
    }
}

/* scores + attend (src/metal_kernels.metal:81-132): causal GQA softmax over
 * positions 0..prefix+token, heads h -> h/4. query [count,4096]; keys/values
 * [prefix+count,1024]. probabilities: optional [count,32,prefix+count]. */
void oracle_attention(const float *query, const float *keys, const float *values,
    float *output, size_t count, size_t prefix, float *probabilities)
{
    size_t stride = prefix + count;
    #pragma omp parallel
    {
        float *row = malloc(stride * sizeof(float));
        #pragma omp for schedule(static)
        for (size_t group = 0; group < count * 32; group++) {
            size_t token = group / 32, head = group % 32;
            const float *q = query + token * 4096 + head * 128;
            float maximum = -INFINITY;
            size_t last = token + prefix;
            for (size_t position = 0; position <= last; position++) {
                const float *k = keys + position * 1024 + (head / 4) * 128;
                float lanes[LANES] = {0};
                for (size_t c = 0; c < 128; c++) {
                    lanes[c % LANES] += q[c] * k[c];
                }
                float score = lane_sum(lanes) * 0.08838834764831845f;
                row[position] = score;
                maximum = fmaxf(maximum, score);
            }
            float lanes[LANES] = {0};
            for (size_t position = 0; position <= last; position++) {
                float value = expf(row[position] - maximum);
                row[position] = value;
                lanes[position % LANES] += value;
            }
            float total = lane_sum(lanes);
            for (size_t position = 0; position < stride; position++) {
                row[position] = position <= last ? row[position] / total : 0.0f;
            }
            if (probabilities) {
                memcpy(probabilities + group * stride, row, stride * sizeof(float));
            }
            /* every column accumulates over positions in ascending order, as
             * the reference's per-column loop does; walking positions in the
             * outer loop reads each value row contiguously and gives the same
             * sums bit for bit */
            float sums[128] = {0};
            for (size_t position = 0; position <= last; position++) {
                const float p = row[position];
                const float *v = values + position * 1024 + (head / 4) * 128;
                for (size_t column = 0; column < 128; column++) {
                    sums[column] += p * v[column];
                }
            }
            memcpy(output + token * 4096 + head * 128, sums, sizeof sums);
        }
        free(row);
    }
}

/* ------------------------------------------------------------------------- */
/* Model: reads a safetensors checkpoint in the reference's tensor contract
 * (src/metal_weights.c:79-128) through a read-only mapping. Minimal header
 * scanner: this checker only reads files the test suite writes or the
 * reference format admits; the product has its own validating reader. */

typedef struct {
    const unsigned char *data;
    char dtype[16];
    uint64_t shape[4];
    int rank;
    uint64_t bytes;
} oracle_tensor;

struct oracle_model {
    void *map;
    size_t map_bytes;
    const unsigned char *base;
    const uint16_t *embedding;
    float final_norm[ORACLE_HIDDEN];
    float norms[ORACLE_LAYERS][2][ORACLE_HIDDEN];
    const unsigned char *linear[ORACLE_LAYERS][7];
    float scale[ORACLE_LAYERS][7];
    float *keys, *values; /* [26][context][1024] FP32 */
    size_t context, length;
};

static const char *block_names[9] = {
    "input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
    "self_attn.v_proj.weight", "self_attn.o_proj.weight", "post_attention_layernorm.weight",
    "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"};

static const char *skip_space(const char *p, const char *end)
{
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) {
        p++;
    }
    return p;
}

/* Find tensor `name` in the JSON header; fills dtype/shape/offsets. */
static int find_tensor(const oracle_model *m, const char *header, size_t header_bytes,
    const char *name, oracle_tensor *out)
{
    char key[320];
    snprintf(key, sizeof key, "\"%s\"", name);
    const char *end = header + header_bytes;
    const char *p = memmem(header, header_bytes, key, strlen(key));
    while (p) {
        const char *q = skip_space(p + strlen(key), end);
        if (q < end && *q == ':') {
            break;
        }
        p = memmem(p + 1, (size_t)(end - p - 1), key, strlen(key));
    }
    if (!p) {
        return -1;
    }
    const char *object_end = memchr(p, '}', (size_t)(end - p));
    if (!object_end) {
        return -1;
    }
    size_t span = (size_t)(object_end - p);
    const char *d = memmem(p, span, "\"dtype\"", 7);
    const char *s = memmem(p, span, "\"shape\"", 7);
    const char *o = memmem(p, span, "\"data_offsets\"", 14);
    if (!d || !s || !o) {
        return -1;
    }
    d = memchr(d + 7, '"', (size_t)(object_end - d - 7));
    if (!d) {
        return -1;
    }
    size_t n = 0;
    d++;
    while (d < object_end && *d != '"' && n + 1 < sizeof out->dtype) {
        out->dtype[n++] = *d++;
    }
    out->dtype[n] = 0;
    s = memchr(s, '[', (size_t)(object_end - s));
    out->rank = 0;
    if (!s) {
        return -1;
    }
    s++;
    for (;;) {
        s = skip_space(s, object_end);
        if (*s == ']') {
            break;
        }
        if (out->rank == 4) {
            return -1;
        }
        out->shape[out->rank++] = strtoull(s, (char **)&s, 10);
        s = skip_space(s, object_end);
        if (*s == ',') {
            s++;
        }
    }
    o = memchr(o, '[', (size_t)(object_end - o));
    if (!o) {
        return -1;
    }
    uint64_t begin = strtoull(o + 1, (char **)&o, 10);
    o = memchr(o, ',', (size_t)(object_end - o));
    if (!o) {
        return -1;
    }
    uint64_t finish = strtoull(o + 1, NULL, 10);
    if (finish < begin || (size_t)(m->base - (const unsigned char *)m->map) + finish >
            m->map_bytes) {
        return -1;
    }
    out->data = m->base + begin;
    out->bytes = finish - begin;
    return 0;
}

static float bf16_value(const unsigned char *p)
{
    uint32_t word = ((uint32_t)p[0] | (uint32_t)p[1] << 8) << 16;
    float value;
    memcpy(&value, &word, 4);
    return value;
}

oracle_model *oracle_open(const char *path, size_t context, char *error, size_t capacity)
{
    oracle_model *m = calloc(1, sizeof *m);
    int fd = -1;
    char *header = NULL;
    if (!m || !path || (context != 256 && context != 4352)) {
        snprintf(error, capacity, "oracle: bad arguments");
        free(m);
        return NULL;
    }
    fd = open(path, O_RDONLY);
    struct stat st;
    if (fd < 0 || fstat(fd, &st) != 0 || st.st_size < 8) {
        snprintf(error, capacity, "oracle: cannot open %s", path);
        goto fail;
    }
    m->map_bytes = (size_t)st.st_size;
    m->map = mmap(NULL, m->map_bytes, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    fd = -1;
    if (m->map == MAP_FAILED) {
        m->map = NULL;
        snprintf(error, capacity, "oracle: mmap failed");
        goto fail;
    }
    const unsigned char *bytes = m->map;
    uint64_t header_bytes = 0;
    for (int i = 0; i < 8; i++) {
        header_bytes |= (uint64_t)bytes[i] << (8 * i);
    }
    if (header_bytes > m->map_bytes - 8) {
        snprintf(error, capacity, "oracle: bad header");
        goto fail;
    }
    header = malloc(header_bytes + 1);
    memcpy(header, bytes + 8, header_bytes);
    header[header_bytes] = 0;
    m->base = bytes + 8 + header_bytes;
    oracle_tensor t;
    if (find_tensor(m, header, header_bytes, "language_model.model.embed_tokens.weight", &t) ||
        strcmp(t.dtype, "BF16") || t.bytes != (uint64_t)ORACLE_VOCAB * ORACLE_HIDDEN * 2) {
        snprintf(error, capacity, "oracle: embedding missing");
        goto fail;
    }
    m->embedding = (const uint16_t *)t.data;
    if (find_tensor(m, header, header_bytes, "language_model.model.norm.weight", &t) ||
        strcmp(t.dtype, "BF16") || t.bytes != ORACLE_HIDDEN * 2) {
        snprintf(error, capacity, "oracle: final norm missing");
        goto fail;
    }
    for (size_t c = 0; c < ORACLE_HIDDEN; c++) {
        m->final_norm[c] = bf16_value(t.data + 2 * c);
    }
    for (int layer = 0; layer < ORACLE_LAYERS; layer++) {
        int linear = 0, norm = 0;
        for (int slot = 0; slot < 9; slot++) {
            char name[256];
            snprintf(name, sizeof name, "language_model.model.layers.%d.%s", layer,
                block_names[slot]);
            if (find_tensor(m, header, header_bytes, name, &t)) {
                snprintf(error, capacity, "oracle: missing %s", name);
                goto fail;
            }
            if (slot == 0 || slot == 5) {
                for (size_t c = 0; c < ORACLE_HIDDEN; c++) {
                    m->norms[layer][norm][c] = bf16_value(t.data + 2 * c);
                }
                norm++;
                continue;
            }
            if (strcmp(t.dtype, "F8_E4M3") || t.rank != 2 ||
                t.bytes != t.shape[0] * t.shape[1]) {
                snprintf(error, capacity, "oracle: bad linear %s", name);
                goto fail;
            }
            m->linear[layer][linear] = t.data;
            char scale_name[300];
            snprintf(scale_name, sizeof scale_name, "%.*sweight_scale_inv",
                (int)strlen(name) - 6, name);
            oracle_tensor s;
            if (find_tensor(m, header, header_bytes, scale_name, &s) || s.bytes != 2) {
                snprintf(error, capacity, "oracle: missing %s", scale_name);
                goto fail;
            }
            m->scale[layer][linear] = bf16_value(s.data);
            linear++;
        }
    }
    m->context = context;
    size_t kv = (size_t)ORACLE_LAYERS * context * ORACLE_KV;
    m->keys = calloc(kv, sizeof(float));
    m->values = calloc(kv, sizeof(float));
    if (!m->keys || !m->values) {
        snprintf(error, capacity, "oracle: KV allocation failed");
        goto fail;
    }
    free(header);
    return m;
fail:
    free(header);
    if (fd >= 0) {
        close(fd);
    }
    oracle_close(m);
    return NULL;
}

void oracle_close(oracle_model *m)
{
    if (!m) {
        return;
    }
    if (m->map) {
        munmap(m->map, m->map_bytes);
    }
    free(m->keys);
    free(m->values);
    free(m);
}

void oracle_reset(oracle_model *m)
{
    m->length = 0;
}

size_t oracle_length(const oracle_model *m)
{
    return m->length;
}

int oracle_rewind(oracle_model *m, size_t length)
{
    if (length > m->length) {
        return -1;
    }
    m->length = length;
    return 0;
}

/* One call of the reference graph: host gather + YaRN table
 * (src/metal_runtime.m:388-402), 26 x encode_layer (src/metal_encode.m:124-187),
 * final norm and tied head on the last row (src/metal_encode.m:204-210). */
int oracle_forward(oracle_model *m, const int64_t *ids, size_t count, float *logits,
    float *trace, float *final_norm, char *error, size_t capacity)
{
    if (!m || !ids || !count || !logits || m->length + count > m->context) {
        snprintf(error, capacity, "oracle: bad forward arguments");
        return -1;
    }
    for (size_t i = 0; i < count; i++) {
        if (ids[i] < 0 || ids[i] >= ORACLE_VOCAB) {
            snprintf(error, capacity, "oracle: bad token id");
            return -1;
        }
    }
    const size_t H = ORACLE_HIDDEN, Q = ORACLE_QUERY, KV = ORACLE_KV, F = ORACLE_INNER;
    float *x = malloc(count * H * sizeof(float));
    float *normed = malloc(count * H * sizeof(float));
    float *q = malloc(count * Q * sizeof(float));
    float *rq = malloc(count * Q * sizeof(float));
    float *k = malloc(count * KV * sizeof(float));
    float *v = malloc(count * KV * sizeof(float));
    float *attn = malloc(count * Q * sizeof(float));
    float *o = malloc(count * H * sizeof(float));
    float *residual = malloc(count * H * sizeof(float));
    float *gate = malloc(count * F * sizeof(float));
    float *up = malloc(count * F * sizeof(float));
    float *gated = malloc(count * F * sizeof(float));
    float *down = malloc(count * H * sizeof(float));
    float *cosine = malloc(count * 128 * sizeof(float));
    float *sine = malloc(count * 128 * sizeof(float));
    uint32_t *positions = malloc(count * sizeof(uint32_t));
    int status = -1;
    if (!x || !normed || !q || !rq || !k || !v || !attn || !o || !residual || !gate ||
        !up || !gated || !down || !cosine || !sine || !positions) {
        snprintf(error, capacity, "oracle: allocation failed");
        goto done;
    }
    for (size_t i = 0; i < count; i++) {
        for (size_t c = 0; c < H; c++) {
            uint32_t word = (uint32_t)m->embedding[(size_t)ids[i] * H + c] << 16;
            memcpy(&x[i * H + c], &word, 4);
        }
        positions[i] = (uint32_t)(m->length + i);
        oracle_yarn(positions[i], cosine + i * 128, sine + i * 128);
    }
    for (int layer = 0; layer < ORACLE_LAYERS; layer++) {
        float *keys = m->keys + (size_t)layer * m->context * KV;
        float *values = m->values + (size_t)layer * m->context * KV;
        oracle_norm(m->norms[layer][0], x, normed, H, count);
        round_inputs(normed, count, H, input_rounding);
        oracle_project_fp8(m->linear[layer][0], m->scale[layer][0], normed, q, Q, H, count);
        oracle_project_fp8(m->linear[layer][1], m->scale[layer][1], normed, k, KV, H, count);
        oracle_project_fp8(m->linear[layer][2], m->scale[layer][2], normed, v, KV, H, count);
        oracle_rope(q, cosine, sine, positions, rq, Q, count, 1);
        oracle_rope(k, cosine, sine, positions, keys + m->length * KV, KV, count, 0);
        memcpy(values + m->length * KV, v, count * KV * sizeof(float));
        round_rows(keys + m->length * KV, count * KV, kv_rounding);
        round_rows(values + m->length * KV, count * KV, kv_rounding);
        oracle_attention(rq, keys, values, attn, count, m->length, NULL);
        round_inputs(attn, count, Q, input_rounding);
        oracle_project_fp8(m->linear[layer][3], m->scale[layer][3], attn, o, H, Q, count);
        oracle_element(x, o, residual, count * H, 0);
        oracle_norm(m->norms[layer][1], residual, normed, H, count);
        round_inputs(normed, count, H, input_rounding);
        oracle_project_fp8(m->linear[layer][4], m->scale[layer][4], normed, gate, F, H, count);
        oracle_project_fp8(m->linear[layer][5], m->scale[layer][5], normed, up, F, H, count);
        oracle_element(gate, gate, gated, count * F, 1);
        oracle_element(gated, up, gated, count * F, 2);
        round_inputs(gated, count, F, input_rounding);
        oracle_project_fp8(m->linear[layer][6], m->scale[layer][6], gated, down, H, F, count);
        oracle_element(residual, down, x, count * H, 0);
        if (trace) {
            memcpy(trace + (size_t)layer * count * H, x, count * H * sizeof(float));
        }
    }
    oracle_norm(m->final_norm, x, normed, H, count);
    if (final_norm) {
        memcpy(final_norm, normed, count * H * sizeof(float));
    }
    project_bf16(m->embedding, normed + (count - 1) * H, logits, ORACLE_VOCAB, H);
    for (size_t i = 0; i < ORACLE_VOCAB; i++) {
        if (!isfinite(logits[i])) {
            snprintf(error, capacity, "oracle: nonfinite logit %zu", i);
            goto done;
        }
    }
    m->length += count;
    status = 0;
done:
    free(x); free(normed); free(q); free(rq); free(k); free(v); free(attn); free(o);
    free(residual); free(gate); free(up); free(gated); free(down); free(cosine);
    free(sine); free(positions);
    return status;
}
