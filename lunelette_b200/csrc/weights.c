#define _GNU_SOURCE
#include "weights.h"

#include <math.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

const lun_block_weight lun_block_weights[LUN_BLOCK_WEIGHTS] = {
    {"input_layernorm.weight", LUN_HIDDEN, 0},
    {"self_attn.q_proj.weight", LUN_QUERY, LUN_HIDDEN},
    {"self_attn.k_proj.weight", LUN_KV, LUN_HIDDEN},
    {"self_attn.v_proj.weight", LUN_KV, LUN_HIDDEN},
    {"self_attn.o_proj.weight", LUN_HIDDEN, LUN_QUERY},
    {"post_attention_layernorm.weight", LUN_HIDDEN, 0},
    {"mlp.gate_proj.weight", LUN_INNER, LUN_HIDDEN},
    {"mlp.up_proj.weight", LUN_INNER, LUN_HIDDEN},
    {"mlp.down_proj.weight", LUN_HIDDEN, LUN_INNER},
};

/* The checkpoint contract as a catalogue: every tensor the decoder reads
 * (embedding, final norm, 26 x 9 block tensors) and the two rank-0 BF16 scalars
 * beside each FP8 linear ("<stem>.weight_scale_inv", "<stem>.activation_scale"),
 * each with its dtype and shape, listed in the order failures are reported:
 * the embedding, the final norm, then layer by layer each tensor followed by its
 * scalars. One pass over the file's "language_model." tensors finds every
 * entry by binary search over the names and remembers the first tensor the
 * contract does not list; tensors outside "language_model." (a vision tower,
 * a projector) are not this backend's concern. */
enum { ENTRY_TENSOR, ENTRY_SCALE, ENTRY_ACTIVATION_SCALE };
enum { CONTRACT_ENTRIES = LUN_WEIGHT_COUNT + 2 * LUN_LAYERS * 7 };  /* 7 FP8 linears a layer */

typedef struct {
    char name[LUN_ST_MAX_NAME + 32];
    lun_dtype dtype;
    size_t rows, cols;  /* cols == 0: a vector of rows elements */
    int kind;           /* ENTRY_* */
    size_t weight;      /* index into lun_weights.w (of the owning tensor for a scalar) */
    const lun_tensor *found;
} contract_entry;

static const char *dtype_name(lun_dtype dtype)
{
    return dtype == LUN_F8_E4M3 ? "F8_E4M3" : "BF16";
}

static size_t contract_add(contract_entry *c, size_t n, const char *name, lun_dtype dtype, size_t rows,
    size_t cols, int kind, size_t weight)
{
    snprintf(c[n].name, sizeof c[n].name, "%s", name);
    c[n].dtype = dtype;
    c[n].rows = rows;
    c[n].cols = cols;
    c[n].kind = kind;
    c[n].weight = weight;
    c[n].found = NULL;
    return n + 1;
}

static size_t contract_build(contract_entry *c)
{
    size_t n = 0;
    n = contract_add(c, n, "language_model.model.embed_tokens.weight", LUN_BF16, LUN_VOCAB, LUN_HIDDEN,
        ENTRY_TENSOR, 0);
    n = contract_add(c, n, "language_model.model.norm.weight", LUN_BF16, LUN_HIDDEN, 0, ENTRY_TENSOR, 1);
    for (size_t layer = 0; layer < LUN_LAYERS; layer++) {
        for (size_t slot = 0; slot < LUN_BLOCK_WEIGHTS; slot++) {
            const lun_block_weight *b = &lun_block_weights[slot];
            const size_t index = 2 + layer * LUN_BLOCK_WEIGHTS + slot;
            char name[LUN_ST_MAX_NAME];
            snprintf(name, sizeof name, "language_model.model.layers.%zu.%s", layer, b->suffix);
            const int fp8 = b->cols != 0;  /* linears are FP8, norm gains BF16 */
            n = contract_add(c, n, name, fp8 ? LUN_F8_E4M3 : LUN_BF16, b->rows, b->cols, ENTRY_TENSOR, index);
            if (fp8) {
                /* "<stem>.weight" -> "<stem>.weight_scale_inv" / "<stem>.activation_scale" */
                const int stem = (int)(strlen(name) - strlen("weight"));
                char scalar[LUN_ST_MAX_NAME + 32];
                snprintf(scalar, sizeof scalar, "%.*sweight_scale_inv", stem, name);
                n = contract_add(c, n, scalar, LUN_BF16, 0, 0, ENTRY_SCALE, index);
                snprintf(scalar, sizeof scalar, "%.*sactivation_scale", stem, name);
                n = contract_add(c, n, scalar, LUN_BF16, 0, 0, ENTRY_ACTIVATION_SCALE, index);
            }
        }
    }
    return n;
}

static int entry_by_name(const void *a, const void *b)
{
    return strcmp((*(contract_entry *const *)a)->name, (*(contract_entry *const *)b)->name);
}

static int name_to_entry(const void *key, const void *item)
{
    return strcmp((const char *)key, (*(contract_entry *const *)item)->name);
}

/* 0 when the file's tensor matches the entry, else -1 with the reason. */
static int entry_check(const contract_entry *e, char *error, size_t capacity)
{
    const lun_tensor *t = e->found;
    if (e->kind != ENTRY_TENSOR) {
        if (!t || t->dtype != LUN_BF16 || t->rank != 0 || t->end - t->begin != 2) {
            snprintf(error, capacity, "scalar %s: an FP8 tensor needs this rank-0 BF16 value beside it", e->name);
            return -1;
        }
        return 0;
    }
    char want[64];
    if (e->cols) {
        snprintf(want, sizeof want, "%s [%zu,%zu]", dtype_name(e->dtype), e->rows, e->cols);
    } else {
        snprintf(want, sizeof want, "%s [%zu]", dtype_name(e->dtype), e->rows);
    }
    if (!t) {
        snprintf(error, capacity, "tensor %s: not in the checkpoint (the decoder reads %s)", e->name, want);
        return -1;
    }
    const unsigned rank = e->cols ? 2u : 1u;
    if (t->dtype != e->dtype || t->rank != rank || t->shape[0] != e->rows || (e->cols && t->shape[1] != e->cols)) {
        snprintf(error, capacity, "tensor %s: the decoder reads %s here", e->name, want);
        return -1;
    }
    return 0;
}

static int validate(lun_weights *weights, char *error, size_t capacity)
{
    contract_entry *contract = calloc(CONTRACT_ENTRIES, sizeof *contract);
    contract_entry **sorted = calloc(CONTRACT_ENTRIES, sizeof *sorted);
    if (!contract || !sorted) {
        free(contract);
        free(sorted);
        snprintf(error, capacity, "checkpoint contract: out of host memory");
        return -1;
    }
    const size_t n = contract_build(contract);
    for (size_t i = 0; i < n; i++) {
        sorted[i] = &contract[i];
    }
    qsort(sorted, n, sizeof *sorted, entry_by_name);
    const char *stranger = NULL;
    for (size_t i = 0; i < weights->file.count; i++) {
        const lun_tensor *t = &weights->file.tensors[i];
        if (strncmp(t->name, "language_model.", 15) != 0) {
            continue;
        }
        contract_entry **hit = bsearch(t->name, sorted, n, sizeof *sorted, name_to_entry);
        if (hit) {
            (*hit)->found = t;
        } else if (!stranger) {
            stranger = t->name;
        }
    }
    int status = 0;
    for (size_t i = 0; i < n && !status; i++) {
        status = entry_check(&contract[i], error, capacity);
    }
    if (!status && stranger) {
        snprintf(error, capacity, "tensor %s: not part of the text model this backend runs", stranger);
        status = -1;
    }
    for (size_t i = 0; i < n && !status; i++) {
        const contract_entry *e = &contract[i];
        if (e->kind == ENTRY_TENSOR) {
            weights->w[e->weight].tensor = e->found;
            weights->w[e->weight].scale = 1.0f;
            weights->w[e->weight].elements = e->rows * (e->cols ? e->cols : 1);
        } else if (e->kind == ENTRY_SCALE) {
            weights->w[e->weight].scale_tensor = e->found;
        } else {
            weights->w[e->weight].activation_tensor = e->found;
        }
    }
    free(sorted);
    free(contract);
    return status;
}

/* Both scalars of every FP8 tensor must be positive and finite; the weight
 * scale becomes the tensor's dequantisation factor. The activation scale is
 * only checked: activations are never quantised statically here. */
static int read_scales(lun_weights *weights, char *error, size_t capacity)
{
    for (size_t i = 0; i < LUN_WEIGHT_COUNT; i++) {
        const lun_tensor *pair[2] = {weights->w[i].scale_tensor, weights->w[i].activation_tensor};
        if (weights->w[i].tensor->dtype != LUN_F8_E4M3) {
            continue;
        }
        for (int k = 0; k < 2; k++) {
            unsigned char raw[2];
            if (lun_st_read(&weights->file, pair[k], 0, raw, 2)) {
                snprintf(error, capacity, "scalar %s: read failed", pair[k]->name);
                return -1;
            }
            const float value = lun_bf16_to_f32((uint16_t)(raw[0] | raw[1] << 8));
            if (!isfinite(value) || value <= 0) {
                snprintf(error, capacity, "scalar %s: holds %g, where an FP8 tensor's scalars must be positive finite BF16",
                    pair[k]->name, value);
                return -1;
            }
            if (k == 0) {
                weights->w[i].scale = value;
            }
        }
    }
    return 0;
}

int lun_weights_open(lun_weights *weights, const char *path, char *error, size_t capacity)
{
    memset(weights, 0, sizeof *weights);
    weights->file.fd = -1;
    if (!path) {
        snprintf(error, capacity, "requires one explicit FP8 safetensors path");
        return -1;
    }
    if (lun_st_open(&weights->file, path, error, capacity) || validate(weights, error, capacity) ||
        read_scales(weights, error, capacity)) {
        lun_weights_close(weights);
        return -1;
    }
    return 0;
}

void lun_weights_close(lun_weights *weights)
{
    lun_st_close(&weights->file);
    memset(weights->w, 0, sizeof weights->w);
}

int lun_weights_admission(const lun_weights *weights, size_t index, int compact,
    lun_admission *table, char *error, size_t capacity)
{
    const lun_tensor *t = index < LUN_WEIGHT_COUNT ? weights->w[index].tensor : NULL;
    if (!t || t->dtype != LUN_F8_E4M3) {
        snprintf(error, capacity, "tensor %s: code admission applies to F8_E4M3 tensors only",
            t ? t->name : "(invalid index)");
        return -1;
    }
    float scale = weights->w[index].scale;
    if (compact) {
        uint32_t bits;
        memcpy(&bits, &scale, sizeof bits);
        if (!(scale > 0) || !isnormal(scale) || (bits & 0xffffu)) {
            snprintf(error, capacity,
                "tensor %s: the compact strategies need a positive scale that is an FP32-normal widened BF16 "
                "(got %g)", t->name, scale);
            return -1;
        }
    }
    table->nan_only = 1;
    for (unsigned code = 0; code < 256; code++) {
        float decoded = lun_e4m3_to_f32((unsigned char)code);
        float product = decoded * scale;
        table->allowed[code] = compact ? (isfinite(product) && (decoded == 0 || isnormal(product)))
                                       : isfinite(product);
        table->nan_only &= table->allowed[code] == ((code & 0x7Fu) != 0x7Fu);
    }
    return 0;
}

/* Whether any byte has its low seven bits all ones (an E4M3 NaN code), eight
 * bytes at a time: a byte of y = (w & 0x7F..) ^ 0x7F.. is zero exactly for such
 * a code, and (y - 0x01..) & ~y & 0x80.. is nonzero exactly when some byte of y
 * is zero (no byte of y has its top bit set). Branch-free, so it vectorizes. */
static int has_nan_code(const unsigned char *p, size_t n)
{
    const uint64_t low7 = 0x7F7F7F7F7F7F7F7Full, ones = 0x0101010101010101ull, tops = 0x8080808080808080ull;
    uint64_t found = 0;
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t w;
        memcpy(&w, p + i, 8);
        const uint64_t y = (w & low7) ^ low7;
        found |= (y - ones) & ~y & tops;
    }
    for (; i < n; i++) {
        found |= (p[i] & 0x7Fu) == 0x7Fu;
    }
    return found != 0;
}

int lun_admit_codes(const lun_weights *weights, size_t index, const lun_admission *table,
    const unsigned char *codes, size_t count, uint64_t offset, float scale,
    char *error, size_t capacity)
{
    /* the usual table (only NaN codes rejected): a word-wide scan, and the byte
     * loop below only to name the first rejected byte */
    if (table->nan_only && !has_nan_code(codes, count)) {
        return 0;
    }
    for (size_t i = 0; i < count; i++) {
        if (!table->allowed[codes[i]]) {
            snprintf(error, capacity, "tensor %s byte %llu code 0x%02x: code x scale %.9g is not admitted "
                "(NaN, an overflow or a non-normal product)",
                weights->w[index].tensor->name, (unsigned long long)(offset + i), codes[i], scale);
            return -1;
        }
    }
    return 0;
}

/* YaRN (rope_type "yarn", mscale 1): pair j blends the extrapolated frequency
 * theta^(-2j/128) with the interpolated one (divided by factor 16) through a
 * linear ramp between the correction dims of beta_fast 32 and beta_slow 1 at
 * original context 16384. Ramp bounds use double maths, everything else FP32,
 * exactly as the reference's table builder (src/metal_yarn.c:8-33). */
int lun_yarn(uint32_t position, float cosine[128], float sine[128])
{
    if (position >= 262144u) {
        return -1;
    }
    const double two_pi = 2.0 * 3.14159265358979323846;
    const double log_theta2 = 2.0 * log(1e6);
    float low = (float)floor(128.0 * log(16384.0 / (32.0 * two_pi)) / log_theta2);
    float high = (float)ceil(128.0 * log(16384.0 / two_pi) / log_theta2);
    for (int j = 0; j < 64; j++) {
        float frequency = powf(1000000.0f, (float)(2 * j) / 128.0f);
        float ramp = fminf(1.0f, fmaxf(0.0f, ((float)j - low) / (high - low)));
        float extrapolated = 1.0f - ramp;
        float inverse = (1.0f / (16.0f * frequency)) * (1.0f - extrapolated) +
            (1.0f / frequency) * extrapolated;
        float angle = inverse * (float)position;
        float c = cosf(angle), s = sinf(angle);
        cosine[j] = c;
        cosine[j + 64] = c;
        sine[j] = s;
        sine[j + 64] = s;
    }
    return 0;
}
