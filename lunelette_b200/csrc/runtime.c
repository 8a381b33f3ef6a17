/* Host runtime (C11) behind include/metal.h for the B200 backend.
 *
 * Same contract and state machine as the reference's src/metal_runtime.m:
 * argument errors are rejected before any mutation; an execution, allocation or
 * non-finite failure leaves the sequence invalid until reset; checkpoints hold
 * host logits plus a length, guarded by a never-recycled context identity and a
 * per-context epoch. The device work goes through device.h.
 */
#include "metal.h"

#include "device.h"
#include "weights.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <stdatomic.h>
#include <stdbool.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define LUN_API __attribute__((visibility("default")))

struct lunelette_metal {
    lun_device *device;
    lunelette_metal_limits limits;
    lunelette_metal_prefill_mode prefill;
    lunelette_metal_strategy strategy;
    size_t length;
    bool valid, endpoint_valid;
    uint64_t identity, epoch;
    lunelette_metal_checkpoint *active; /* borrowed; the caller owns handles */
    float *logits;                      /* pinned host logits owned by the device layer */
};

struct lunelette_metal_checkpoint {
    lunelette_metal *owner;
    uint64_t identity, epoch;
    size_t length;
    float logits[LUN_VOCAB];
};

/* Saturating process-wide identity: address reuse never revives a handle. */
static _Atomic uint64_t last_identity;

static uint64_t next_identity(void)
{
    uint64_t previous = atomic_load(&last_identity);
    while (previous != UINT64_MAX) {
        if (atomic_compare_exchange_weak(&last_identity, &previous, previous + 1)) {
            return previous + 1;
        }
    }
    return 0;
}

static int profile_supported(lunelette_metal_limits l)
{
    return (l.context == 256 && l.block == 256) ||
        (l.context == 4352 && (l.block == 256 || l.block == 128));
}

static int resolve_options(const lunelette_metal_options *options, lunelette_metal_options *out,
    char *error, size_t capacity)
{
    lunelette_metal_options selected = LUNELETTE_METAL_OPTIONS_DEFAULT;
    if (options) {
        selected = *options;
    }
    if (selected.prefill != LUNELETTE_METAL_PREFILL_MPS &&
        selected.prefill != LUNELETTE_METAL_PREFILL_CUSTOM) {
        snprintf(error, capacity, "invalid prefill option; select MPS or CUSTOM");
        return -1;
    }
    if (selected.strategy != LUNELETTE_METAL_RESIDENT_FP32 &&
        selected.strategy != LUNELETTE_METAL_COMPACT_FP8_ARITHMETIC &&
        selected.strategy != LUNELETTE_METAL_COMPACT_FP8_LOOKUP) {
        snprintf(error, capacity,
            "invalid strategy; select resident-fp32, compact-fp8-arithmetic or compact-fp8-lookup");
        return -1;
    }
    *out = selected;
    return 0;
}

/* Stream every tensor into device memory through the two pinned staging
 * buffers, checking FP8 admission on the bytes as they pass. */
static int upload(lun_device *device, lun_weights *w, int compact, char *error, size_t capacity)
{
    size_t staging = lun_device_staging_bytes();
    int buffer = 0;
    for (size_t layer = 0; layer < LUN_LAYERS; layer++) {
        static const int slot_of[LUN_BLOCK_WEIGHTS] = {-1, LUN_SLOT_Q, LUN_SLOT_K, LUN_SLOT_V,
            LUN_SLOT_O, -1, LUN_SLOT_GATE, LUN_SLOT_UP, LUN_SLOT_DOWN};
        for (size_t b = 0; b < LUN_BLOCK_WEIGHTS; b++) {
            if (slot_of[b] < 0) {
                continue;
            }
            size_t index = 2 + layer * LUN_BLOCK_WEIGHTS + b;
            const lun_tensor *t = w->w[index].tensor;
            size_t bytes = w->w[index].elements;
            lun_admission table;
            if (bytes > staging || lun_weights_admission(w, index, compact, &table, error, capacity) ||
                lun_device_staging_wait(device, buffer)) {
                if (bytes > staging) {
                    snprintf(error, capacity, "tensor %s exceeds staging", t->name);
                }
                return -1;
            }
            unsigned char *dst = lun_device_staging(device, buffer);
            if (lun_st_read(&w->file, t, 0, dst, bytes)) {
                snprintf(error, capacity, "compact tensor %s: compact bounded payload read failed",
                    t->name);
                return -1;
            }
            if (lun_admit_codes(w, index, &table, dst, bytes, 0, w->w[index].scale, error,
                    capacity) ||
                lun_device_upload_linear(device, buffer, (int)layer, slot_of[b],
                    lun_block_weights[b].rows, lun_block_weights[b].cols, w->w[index].scale)) {
                if (!error[0]) {
                    snprintf(error, capacity, "weight upload failed: %s", t->name);
                }
                return -1;
            }
            buffer ^= 1;
        }
    }
    const lun_tensor *embedding = w->w[0].tensor;
    size_t total = w->w[0].elements * 2;
    for (size_t offset = 0; offset < total; offset += staging) {
        size_t bytes = total - offset < staging ? total - offset : staging;
        if (lun_device_staging_wait(device, buffer) ||
            lun_st_read(&w->file, embedding, offset, lun_device_staging(device, buffer), bytes) ||
            lun_device_upload_embedding(device, buffer, offset, bytes)) {
            snprintf(error, capacity, "weight decode/read failed: %s", embedding->name);
            return -1;
        }
        buffer ^= 1;
    }
    float *norms = malloc((size_t)2 * LUN_LAYERS * LUN_HIDDEN * sizeof(float));
    float *final_norm = malloc(LUN_HIDDEN * sizeof(float));
    unsigned char *raw = malloc(LUN_HIDDEN * 2);
    int status = norms && final_norm && raw ? 0 : -1;
    for (size_t i = 0; !status && i < 1 + 2 * LUN_LAYERS; i++) {
        size_t index = i == 0 ? 1 : 2 + ((i - 1) / 2) * LUN_BLOCK_WEIGHTS + ((i - 1) % 2) * 5;
        float *out = i == 0 ? final_norm : norms + (i - 1) * LUN_HIDDEN;
        status = lun_st_read(&w->file, w->w[index].tensor, 0, raw, LUN_HIDDEN * 2);
        for (size_t c = 0; !status && c < LUN_HIDDEN; c++) {
            out[c] = lun_bf16_to_f32((uint16_t)(raw[2 * c] | raw[2 * c + 1] << 8));
        }
    }
    if (!status) {
        status = lun_device_upload_norms(device, norms, final_norm);
    }
    free(norms);
    free(final_norm);
    free(raw);
    if (status) {
        snprintf(error, capacity, "norm weight read/upload failed");
        return -1;
    }
    return 0;
}

static int upload_rope(lun_device *device, size_t context)
{
    float *cosine = malloc(context * LUN_HEAD_DIM * sizeof(float));
    float *sine = malloc(context * LUN_HEAD_DIM * sizeof(float));
    int status = cosine && sine ? 0 : -1;
    for (size_t p = 0; !status && p < context; p++) {
        status = lun_yarn((uint32_t)p, cosine + p * LUN_HEAD_DIM, sine + p * LUN_HEAD_DIM);
    }
    if (!status) {
        status = lun_device_upload_rope(device, cosine, sine, context);
    }
    free(cosine);
    free(sine);
    return status;
}

/* Checkpoint -> device (FP8 compact admission), the YaRN table for
 * rope_positions positions, then the upload's end; shared with batch.c. */
int lun_runtime_load(lun_device *device, const char *path, size_t rope_positions, char *error, size_t capacity)
{
    lun_weights weights;
    if (lun_weights_open(&weights, path, error, capacity)) {
        return -1;
    }
    int status = upload(device, &weights, 1, error, capacity) || upload_rope(device, rope_positions) ||
        lun_device_upload_finish(device, error, capacity);
    if (status && !error[0]) {
        snprintf(error, capacity, "weight upload failed");
    }
    lun_weights_close(&weights);
    return status ? -1 : 0;
}

LUN_API lunelette_metal *lunelette_metal_create_configured(const char *path,
    const lunelette_metal_options *options, const lunelette_metal_limits *limits,
    char *error, size_t capacity)
{
    char fallback[512];
    if (!error || !capacity) {
        error = fallback;
        capacity = sizeof fallback;
    }
    error[0] = 0;
    lunelette_metal_limits resolved = limits ? *limits : (lunelette_metal_limits){256, 256};
    if (!profile_supported(resolved)) {
        snprintf(error, capacity, "unsupported context/block profile");
        return NULL;
    }
    lunelette_metal_options selected;
    if (resolve_options(options, &selected, error, capacity)) {
        return NULL;
    }
    lun_weights weights;
    if (lun_weights_open(&weights, path, error, capacity)) {
        return NULL;
    }
    lunelette_metal *context = calloc(1, sizeof *context);
    lun_device *device = NULL;
    if (!context) {
        snprintf(error, capacity, "context allocation failed");
        goto fail;
    }
    context->identity = next_identity();
    if (!context->identity) {
        snprintf(error, capacity, "context identity exhausted");
        goto fail;
    }
    device = lun_device_create(resolved.context, resolved.block, error, capacity);
    if (!device) {
        goto fail;
    }
    int compact = selected.strategy != LUNELETTE_METAL_RESIDENT_FP32;
    if (upload(device, &weights, compact, error, capacity) || upload_rope(device, resolved.context) ||
        lun_device_upload_finish(device, error, capacity)) {
        if (!error[0]) {
            snprintf(error, capacity, "weight upload failed");
        }
        goto fail;
    }
    lun_weights_close(&weights);
    context->device = device;
    context->limits = resolved;
    context->prefill = selected.prefill;
    context->strategy = selected.strategy;
    context->valid = true;
    context->logits = lun_device_host_logits(device);
    return context;
fail:
    lun_device_destroy(device);
    lun_weights_close(&weights);
    free(context);
    return NULL;
}

LUN_API lunelette_metal *lunelette_metal_create_with_options(const char *path,
    const lunelette_metal_options *options, char *error, size_t capacity)
{
    return lunelette_metal_create_configured(path, options, NULL, error, capacity);
}

LUN_API lunelette_metal *lunelette_metal_create(const char *path, char *error, size_t capacity)
{
    return lunelette_metal_create_with_options(path, NULL, error, capacity);
}

LUN_API int lunelette_metal_get_limits(const lunelette_metal *context,
    lunelette_metal_limits *limits)
{
    if (!context || !limits) {
        return -1;
    }
    *limits = context->limits;
    return 0;
}

LUN_API int lunelette_metal_get_memory(const lunelette_metal *context,
    lunelette_metal_memory *memory)
{
    if (!context || !context->device || !memory) {
        return -1;
    }
    lun_device_bytes bytes;
    lun_device_bytes_owned(context->device, &bytes);
    lunelette_metal_memory result = {0};
    result.strategy = context->strategy;
    result.weight_bytes = bytes.weight_bytes;
    result.conversion_stage_bytes = 0;
    result.scratch_bytes = bytes.scratch_bytes;
    result.kv_bytes = bytes.kv_bytes;
    result.total_bytes = bytes.weight_bytes + bytes.scratch_bytes + bytes.kv_bytes;
    *memory = result;
    return 0;
}

LUN_API void lunelette_metal_destroy(lunelette_metal *context)
{
    if (!context) {
        return;
    }
    if (context->device) {
        cudaSetDevice(lun_device_ordinal(context->device));
    }
    lun_device_destroy(context->device);
    free(context);
}

LUN_API int lunelette_metal_reset(lunelette_metal *context, char *error, size_t capacity)
{
    if (!context) {
        if (error && capacity) {
            snprintf(error, capacity, "reset requires a context");
        }
        return -1;
    }
    context->active = NULL;
    context->endpoint_valid = false;
    context->length = 0;
    context->valid = true;
    return 0;
}

static int execute(lunelette_metal *context, const int64_t *ids, size_t count, bool prefill,
    const float **logits, char *error, size_t capacity)
{
    char fallback[512];
    if (!error || !capacity) {
        error = fallback;
        capacity = sizeof fallback;
    }
    if (logits) {
        *logits = NULL;
    }
    if (!context || !logits || !ids || !count || count > context->limits.block ||
        count > context->limits.context || !context->valid ||
        context->length > context->limits.context - count ||
        (prefill ? context->length != 0 : context->length == 0)) {
        snprintf(error, capacity, "sequence rejected: require reset/valid IDs and "
            "configured block/context capacity");
        return -1;
    }
    for (size_t i = 0; i < count; i++) {
        if (ids[i] < 0 || ids[i] >= LUN_VOCAB) {
            snprintf(error, capacity, "invalid token ID at position %zu", i);
            return -1;
        }
    }
    /* Nothing is published until the device work and the finite check succeed;
     * a failure also drops the checkpoint, a success keeps it. */
    lunelette_metal_checkpoint *checkpoint = context->active;
    context->active = NULL;
    context->endpoint_valid = false;
    context->valid = false;
    const float *output = NULL;
    int nonfinite = 0;
    error[0] = 0;
    if (lun_device_run(context->device, ids, count, context->length, &output, &nonfinite, error,
            capacity)) {
        size_t used = strlen(error);
        snprintf(error + used, capacity - used, "; reset required");
        return -1;
    }
    if (nonfinite) {
        for (size_t i = 0; i < LUN_VOCAB; i++) {
            if (!isfinite(output[i])) {
                snprintf(error, capacity, "nonfinite logit %zu; reset required", i);
                return -1;
            }
        }
        snprintf(error, capacity, "nonfinite logit; reset required");
        return -1;
    }
    context->length += count;
    context->valid = true;
    context->endpoint_valid = true;
    context->active = checkpoint;
    *logits = output;
    return 0;
}

LUN_API int lunelette_metal_prefill(lunelette_metal *context, const int64_t *ids, size_t count,
    const float **logits, char *error, size_t capacity)
{
    return execute(context, ids, count, true, logits, error, capacity);
}

LUN_API int lunelette_metal_decode(lunelette_metal *context, int64_t token,
    const float **logits, char *error, size_t capacity)
{
    return execute(context, &token, 1, false, logits, error, capacity);
}

LUN_API int lunelette_metal_append(lunelette_metal *context, const int64_t *ids, size_t count,
    const float **logits, char *error, size_t capacity)
{
    return execute(context, ids, count, false, logits, error, capacity);
}

LUN_API int lunelette_metal_checkpoint_create(lunelette_metal *context,
    lunelette_metal_checkpoint **checkpoint, char *error, size_t capacity)
{
    if (checkpoint) {
        *checkpoint = NULL;
    }
    if (!context || !checkpoint || !context->identity || !context->valid ||
        !context->endpoint_valid || !context->length ||
        context->length > context->limits.context || context->epoch == UINT64_MAX) {
        if (error && capacity) {
            snprintf(error, capacity, "checkpoint requires valid endpoint/available epoch");
        }
        return -1;
    }
    for (size_t i = 0; i < LUN_VOCAB; i++) {
        if (!isfinite(context->logits[i])) {
            if (error && capacity) {
                snprintf(error, capacity, "checkpoint nonfinite logit %zu", i);
            }
            context->valid = false;
            context->endpoint_valid = false;
            context->active = NULL;
            return -1;
        }
    }
    lunelette_metal_checkpoint *saved = malloc(sizeof *saved);
    if (!saved) {
        if (error && capacity) {
            snprintf(error, capacity, "checkpoint allocation failed");
        }
        return -1;
    }
    saved->owner = context;
    saved->identity = context->identity;
    saved->epoch = context->epoch + 1;
    saved->length = context->length;
    memcpy(saved->logits, context->logits, sizeof saved->logits);
    context->epoch = saved->epoch;
    context->active = saved;
    *checkpoint = saved;
    return 0;
}

LUN_API int lunelette_metal_checkpoint_restore(lunelette_metal *context,
    const lunelette_metal_checkpoint *checkpoint, const float **logits,
    char *error, size_t capacity)
{
    if (logits) {
        *logits = NULL;
    }
    if (!context || !logits || !checkpoint || context->active != checkpoint ||
        checkpoint->identity != context->identity || checkpoint->epoch != context->epoch ||
        !context->valid || context->length > context->limits.context || !checkpoint->length ||
        checkpoint->length > context->limits.context || checkpoint->length > context->length) {
        if (error && capacity) {
            snprintf(error, capacity, "checkpoint stale, invalid or wrong context");
        }
        return -1;
    }
    memcpy(context->logits, checkpoint->logits, sizeof checkpoint->logits);
    context->length = checkpoint->length;
    context->endpoint_valid = true;
    *logits = context->logits;
    return 0;
}

LUN_API void lunelette_metal_checkpoint_destroy(lunelette_metal_checkpoint *checkpoint)
{
    if (!checkpoint) {
        return;
    }
    if (checkpoint->owner->active == checkpoint) {
        checkpoint->owner->active = NULL;
    }
    free(checkpoint);
}

/* ---- additive entry points (include/lunelette_cuda.h) ---- */

LUN_API int lunelette_cuda_validate_checkpoint(const char *path,
    lunelette_metal_strategy strategy, char *error, size_t capacity)
{
    char fallback[512];
    if (!error || !capacity) {
        error = fallback;
        capacity = sizeof fallback;
    }
    error[0] = 0;
    if (strategy != LUNELETTE_METAL_RESIDENT_FP32 &&
        strategy != LUNELETTE_METAL_COMPACT_FP8_ARITHMETIC &&
        strategy != LUNELETTE_METAL_COMPACT_FP8_LOOKUP) {
        snprintf(error, capacity, "invalid strategy");
        return -1;
    }
    lun_weights weights;
    if (lun_weights_open(&weights, path, error, capacity)) {
        return -1;
    }
    enum { CHUNK = 1 << 20 };
    unsigned char *buffer = malloc(CHUNK);
    int status = buffer ? 0 : -1;
    for (size_t index = 0; !status && index < LUN_WEIGHT_COUNT; index++) {
        if (weights.w[index].tensor->dtype != LUN_F8_E4M3) {
            continue;
        }
        lun_admission table;
        status = lun_weights_admission(&weights, index, strategy != LUNELETTE_METAL_RESIDENT_FP32,
            &table, error, capacity);
        size_t total = weights.w[index].elements;
        for (size_t offset = 0; !status && offset < total; offset += CHUNK) {
            size_t n = total - offset < CHUNK ? total - offset : CHUNK;
            if (lun_st_read(&weights.file, weights.w[index].tensor, offset, buffer, n)) {
                snprintf(error, capacity, "compact tensor %s: compact bounded payload read failed",
                    weights.w[index].tensor->name);
                status = -1;
            } else {
                status = lun_admit_codes(&weights, index, &table, buffer, n, offset,
                    weights.w[index].scale, error, capacity);
            }
        }
    }
    free(buffer);
    lun_weights_close(&weights);
    return status;
}

LUN_API int lunelette_cuda_trace(lunelette_metal *context, int enable)
{
    return context && context->device ? lun_device_trace(context->device, enable) : -1;
}

LUN_API int lunelette_cuda_trace_copy(lunelette_metal *context, int which, float *out,
    size_t floats)
{
    return context && context->device && out ?
        lun_device_trace_copy(context->device, which, out, floats) : -1;
}

LUN_API size_t lunelette_cuda_length(const lunelette_metal *context)
{
    return context ? context->length : 0;
}

LUN_API int lunelette_cuda_decode_loop(lunelette_metal *context, int64_t first_token, size_t steps,
    int64_t *tokens, float *milliseconds, int *launches, char *error, size_t capacity)
{
    char fallback[512];
    if (!error || !capacity) {
        error = fallback;
        capacity = sizeof fallback;
    }
    if (!context || !tokens || !steps || !context->valid || !context->length ||
        context->length > context->limits.context - steps || first_token < 0 ||
        first_token >= LUN_VOCAB) {
        snprintf(error, capacity, "decode loop rejected: require a valid non-empty sequence, "
            "a valid token and room for every step");
        return -1;
    }
    lunelette_metal_checkpoint *checkpoint = context->active;
    context->active = NULL;
    context->endpoint_valid = false;
    context->valid = false;
    if (lun_device_decode_loop(context->device, first_token, context->length, steps, tokens,
            milliseconds, launches, error, capacity)) {
        return -1;
    }
    /* The KV cache now holds `steps` more positions; the host logits were not
     * refreshed, so there is no published endpoint until the next call. */
    context->length += steps;
    context->valid = true;
    context->active = checkpoint;
    return 0;
}

LUN_API int lunelette_cuda_timeline(lunelette_metal *context, int enable)
{
    return context && context->device ? lun_device_timeline(context->device, enable) : -1;
}

LUN_API int lunelette_cuda_timeline_copy(lunelette_metal *context, unsigned long long *out,
    size_t entries)
{
    return context && context->device && out ?
        lun_device_timeline_copy(context->device, out, entries) : -1;
}

LUN_API int lunelette_cuda_yarn(uint32_t position, float *cosine, float *sine)
{
    return cosine && sine ? lun_yarn(position, cosine, sine) : -1;
}
