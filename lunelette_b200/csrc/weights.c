#define _GNU_SOURCE
#include "weights.h"

#include <math.h>
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

static const char *companions[2] = {"weight_scale_inv", "activation_scale"};

/* "<prefix>.weight" -> "<prefix>.<suffix>" */
static void companion_name(char *out, size_t capacity, const char *name, const char *suffix)
{
    size_t stem = strlen(name) - strlen("weight");
    snprintf(out, capacity, "%.*s%s", (int)stem, name, suffix);
}

static int expect(lun_weights *weights, size_t index, const char *name, size_t rows,
    size_t cols, char *error, size_t capacity)
{
    const lun_tensor *t = lun_st_find(&weights->file, name);
    lun_dtype want = (cols && index != 0) ? LUN_F8_E4M3 : LUN_BF16;
    if (!t || t->dtype != want || t->rank != (cols ? 2u : 1u) || t->shape[0] != rows ||
        (cols && t->shape[1] != cols)) {
        if (cols) {
            snprintf(error, capacity, "tensor %s: expected %s [%zu,%zu]", name,
                want == LUN_BF16 ? "BF16" : "F8_E4M3", rows, cols);
        } else {
            snprintf(error, capacity, "tensor %s: expected BF16 [%zu]", name, rows);
        }
        return -1;
    }
    if (want == LUN_F8_E4M3) {
        for (int i = 0; i < 2; i++) {
            char scalar[LUN_ST_MAX_NAME + 32];
            companion_name(scalar, sizeof scalar, name, companions[i]);
            const lun_tensor *s = lun_st_find(&weights->file, scalar);
            if (!s || s->dtype != LUN_BF16 || s->rank != 0 || s->end - s->begin != 2) {
                snprintf(error, capacity, "scalar %s: expected BF16 rank0", scalar);
                return -1;
            }
        }
    }
    weights->w[index].tensor = t;
    weights->w[index].scale = 1.0f;
    weights->w[index].elements = rows * (cols ? cols : 1);
    return 0;
}

static int validate(lun_weights *weights, char *error, size_t capacity)
{
    if (expect(weights, 0, "language_model.model.embed_tokens.weight", LUN_VOCAB, LUN_HIDDEN,
            error, capacity) ||
        expect(weights, 1, "language_model.model.norm.weight", LUN_HIDDEN, 0, error, capacity)) {
        return -1;
    }
    for (size_t layer = 0; layer < LUN_LAYERS; layer++) {
        for (size_t slot = 0; slot < LUN_BLOCK_WEIGHTS; slot++) {
            char name[LUN_ST_MAX_NAME];
            const lun_block_weight *b = &lun_block_weights[slot];
            snprintf(name, sizeof name, "language_model.model.layers.%zu.%s", layer, b->suffix);
            if (expect(weights, 2 + layer * LUN_BLOCK_WEIGHTS + slot, name, b->rows, b->cols,
                    error, capacity)) {
                return -1;
            }
        }
    }
    /* Every "language_model." tensor must be a known weight or companion;
     * other prefixes (vision, projector) are left alone. */
    for (size_t i = 0; i < weights->file.count; i++) {
        const char *name = weights->file.tensors[i].name;
        if (strncmp(name, "language_model.", 15) != 0) {
            continue;
        }
        int known = 0;
        for (size_t j = 0; j < LUN_WEIGHT_COUNT && !known; j++) {
            const lun_tensor *t = weights->w[j].tensor;
            known = !strcmp(name, t->name);
            if (!known && t->dtype == LUN_F8_E4M3) {
                for (int k = 0; k < 2 && !known; k++) {
                    char scalar[LUN_ST_MAX_NAME + 32];
                    companion_name(scalar, sizeof scalar, t->name, companions[k]);
                    known = !strcmp(name, scalar);
                }
            }
        }
        if (!known) {
            snprintf(error, capacity, "Unexpected text tensor: %s", name);
            return -1;
        }
    }
    return 0;
}

static int read_scales(lun_weights *weights, char *error, size_t capacity)
{
    for (size_t i = 0; i < LUN_WEIGHT_COUNT; i++) {
        const lun_tensor *t = weights->w[i].tensor;
        if (t->dtype != LUN_F8_E4M3) {
            continue;
        }
        for (int k = 0; k < 2; k++) {
            char scalar[LUN_ST_MAX_NAME + 32];
            companion_name(scalar, sizeof scalar, t->name, companions[k]);
            const lun_tensor *s = lun_st_find(&weights->file, scalar);
            unsigned char raw[2];
            if (lun_st_read(&weights->file, s, 0, raw, 2)) {
                snprintf(error, capacity, "scalar %s: read failed", scalar);
                return -1;
            }
            float value = lun_bf16_to_f32((uint16_t)(raw[0] | raw[1] << 8));
            if (!isfinite(value) || value <= 0) {
                snprintf(error, capacity, "scalar %s: expected positive finite BF16", scalar);
                return -1;
            }
            /* activation_scale is checked and then unused: weights are
             * dequantised, activations are never statically quantised. */
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
        snprintf(error, capacity, "compact tensor %s: expected exact compact F8 element count",
            t ? t->name : "(invalid index)");
        return -1;
    }
    float scale = weights->w[index].scale;
    if (compact) {
        uint32_t bits;
        memcpy(&bits, &scale, sizeof bits);
        if (!(scale > 0) || !isnormal(scale) || (bits & 0xffffu)) {
            snprintf(error, capacity,
                "compact tensor %s: compact scale must be positive FP32-normal widened BF16",
                t->name);
            return -1;
        }
    }
    for (unsigned code = 0; code < 256; code++) {
        float decoded = lun_e4m3_to_f32((unsigned char)code);
        float product = decoded * scale;
        table->allowed[code] = compact ? (isfinite(product) && (decoded == 0 || isnormal(product)))
                                       : isfinite(product);
    }
    return 0;
}

int lun_admit_codes(const lun_weights *weights, size_t index, const lun_admission *table,
    const unsigned char *codes, size_t count, uint64_t offset, float scale,
    char *error, size_t capacity)
{
    for (size_t i = 0; i < count; i++) {
        if (!table->allowed[codes[i]]) {
            snprintf(error, capacity, "compact tensor %s byte %llu code 0x%02x: "
                "NaN or non-normal/overflow reconstructed product (scale %.9g)",
                weights->w[index].tensor->name, (unsigned long long)(offset + i), codes[i],
                scale);
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
