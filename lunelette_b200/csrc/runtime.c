/* Host runtime (C11) behind include/metal.h for the B200 backend.
 *
 * It serves the contract that include/metal.h states (the reference's
 * include/metal.h:74-120, implemented there by src/metal_runtime.m:349-575):
 * arguments are checked before anything changes; a failed or non-finite
 * device step leaves the sequence unusable until reset; a checkpoint is the
 * published length plus a host copy of its logits, accepted back only by the
 * context and epoch that made it. The sequence is one state value (seq_state)
 * and the device work goes through device.h.
 */
#include "metal.h"

#include "device.h"
#include "weights.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdbool.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define LUN_API __attribute__((visibility("default")))

/* Where a context's sequence stands. The contract in include/metal.h is a small
 * state machine; keeping it as one explicit value (instead of separate flags)
 * makes every transition visible at the place it happens:
 *   SEQ_EMPTY        after create/reset: length 0, prefill allowed
 *   SEQ_PUBLISHED    length > 0 and the host logits belong to the last position
 *   SEQ_UNPUBLISHED  length > 0, KV valid, but the host logits are not the
 *                    endpoint's (after lunelette_cuda_decode_loop)
 *   SEQ_BROKEN       a device step failed or produced a non-finite logit; only
 *                    reset leaves this state */
typedef enum { SEQ_EMPTY, SEQ_PUBLISHED, SEQ_UNPUBLISHED, SEQ_BROKEN } seq_state;

struct lunelette_metal {
    lun_device *device;
    lunelette_metal_limits limits;
    lunelette_metal_prefill_mode prefill;
    lunelette_metal_strategy strategy;
    seq_state state;
    size_t length;
    uint64_t identity;  /* never reused within the process; 0 = exhausted */
    uint64_t epoch;     /* bumped by every successful checkpoint create */
    lunelette_metal_checkpoint *current; /* caller-owned; the only handle restore accepts */
    float *logits;      /* pinned host logits owned by the device layer */
    float *snapshot[2]; /* lunelette_cuda_snapshot: last block's layer-25 / final-norm rows */
};

struct lunelette_metal_checkpoint {
    lunelette_metal *context;
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

/* Parallel read (and FP8 admission scan) of one tensor's bytes into pinned
 * staging: the range is cut into chunks that worker threads pread and scan at
 * the same time, so a 3.8 GB checkpoint in the page cache loads at memory
 * speed rather than one thread's copy rate. The first failing chunk (in file
 * order) supplies the diagnostic. */
enum { READ_CHUNK = 4 << 20, READ_MAX_THREADS = 16 };

typedef struct {
    const lun_weights *w;
    const lun_tensor *tensor;
    size_t index;              /* weight index, for the admission scan */
    const lun_admission *table; /* NULL: no scan (BF16 payloads) */
    uint64_t offset;           /* byte offset of dst[0] within the tensor */
    unsigned char *dst;
    size_t bytes;
    _Atomic size_t next_chunk;
    size_t failed_chunk;       /* lowest failing chunk, SIZE_MAX if none */
    pthread_mutex_t lock;
    char error[512];
} read_job;

static void *read_worker(void *arg)
{
    read_job *job = arg;
    size_t chunks = (job->bytes + READ_CHUNK - 1) / READ_CHUNK;
    for (;;) {
        size_t c = atomic_fetch_add(&job->next_chunk, 1);
        if (c >= chunks) {
            break;
        }
        size_t at = c * (size_t)READ_CHUNK, n = job->bytes - at < READ_CHUNK ? job->bytes - at : READ_CHUNK;
        char message[512] = "";
        int bad = lun_st_read(&job->w->file, job->tensor, job->offset + at, job->dst + at, n);
        if (bad) {
            snprintf(message, sizeof message, "tensor %s: bounded payload read failed", job->tensor->name);
        } else if (job->table) {
            bad = lun_admit_codes(job->w, job->index, job->table, job->dst + at, n, job->offset + at,
                job->w->w[job->index].scale, message, sizeof message);
        }
        if (bad) {
            pthread_mutex_lock(&job->lock);
            if (c < job->failed_chunk) {
                job->failed_chunk = c;
                snprintf(job->error, sizeof job->error, "%s", message);
            }
            pthread_mutex_unlock(&job->lock);
        }
    }
    return NULL;
}

static int read_threads(void)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n < 1 ? 1 : (n > READ_MAX_THREADS ? READ_MAX_THREADS : (int)n);
}

static int parallel_read(const lun_weights *w, size_t index, const lun_admission *table, uint64_t offset,
    unsigned char *dst, size_t bytes, char *error, size_t capacity)
{
    read_job job = {w, w->w[index].tensor, index, table, offset, dst, bytes, 0, SIZE_MAX,
        PTHREAD_MUTEX_INITIALIZER, ""};
    size_t chunks = (bytes + READ_CHUNK - 1) / READ_CHUNK;
    int threads = read_threads();
    if ((size_t)threads > chunks) {
        threads = (int)chunks;
    }
    pthread_t tid[READ_MAX_THREADS];
    int started = 0;
    for (int t = 1; t < threads; t++) {
        if (pthread_create(&tid[started], NULL, read_worker, &job) == 0) {
            started++;
        }
    }
    read_worker(&job); /* the calling thread works too; it finishes what others did not take */
    for (int t = 0; t < started; t++) {
        pthread_join(tid[t], NULL);
    }
    pthread_mutex_destroy(&job.lock);
    if (job.failed_chunk != SIZE_MAX) {
        snprintf(error, capacity, "%s", job.error);
        return -1;
    }
    return 0;
}

/* Stream every tensor into device memory through the two pinned staging
 * buffers, checking FP8 admission on the bytes as they pass (parallel_read);
 * the device copies and tiling of one buffer overlap the reads of the next. */
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
            if (parallel_read(w, index, &table, 0, dst, bytes, error, capacity) ||
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
            parallel_read(w, 0, NULL, offset, lun_device_staging(device, buffer), bytes, error, capacity) ||
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
    char local[512];
    if (!error || !capacity) {
        error = local;
        capacity = sizeof local;
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
    /* test support: LUNELETTE_CUDA_TRACE=1 keeps every call's layer outputs
     * (lunelette_cuda_snapshot), for harnesses that cannot call
     * lunelette_cuda_trace between create and their first step */
    const char *trace = getenv("LUNELETTE_CUDA_TRACE");
    if (trace && trace[0] && strcmp(trace, "0") != 0 && lun_device_trace(device, 1)) {
        snprintf(error, capacity, "trace buffer allocation failed");
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
    context->state = SEQ_EMPTY;
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
    free(context->snapshot[0]);
    free(context->snapshot[1]);
    free(context);
}

LUN_API int lunelette_metal_reset(lunelette_metal *context, char *error, size_t capacity)
{
    if (!context) {
        if (error && capacity) {
            snprintf(error, capacity, "lunelette: reset needs a context");
        }
        return -1;
    }
    /* Old KV rows stay in device memory but length 0 makes them unreachable;
     * the current checkpoint no longer describes this sequence. */
    context->state = SEQ_EMPTY;
    context->length = 0;
    context->current = NULL;
    return 0;
}

/* Kinds of model call; they differ only in which sequence states admit them. */
typedef enum { CALL_PREFILL, CALL_APPEND } call_kind;

/* Argument and state check of one model call. Returns NULL when the call may
 * run, else the reason, written into `buffer`. Nothing is changed here: a
 * rejected call leaves the context exactly as it was. */
static const char *check_call(const lunelette_metal *context, const int64_t *ids, size_t count,
    call_kind kind, const float *const *logits, char *buffer, size_t size)
{
    if (!context || !ids || !logits) {
        return "lunelette: context, ids and logits output are required";
    }
    if (context->state == SEQ_BROKEN) {
        return "lunelette: sequence is invalid after a failed call; reset required";
    }
    if (count == 0 || count > context->limits.block) {
        snprintf(buffer, size, "lunelette: %zu ids in one call; the profile allows 1..%zu", count,
            context->limits.block);
        return buffer;
    }
    if (kind == CALL_PREFILL && context->state != SEQ_EMPTY) {
        snprintf(buffer, size, "lunelette: prefill needs an empty sequence (length is %zu); reset first",
            context->length);
        return buffer;
    }
    if (kind == CALL_APPEND && context->state == SEQ_EMPTY) {
        return "lunelette: append/decode needs a prefilled sequence";
    }
    if (count > context->limits.context || context->length > context->limits.context - count) {
        snprintf(buffer, size, "lunelette: %zu + %zu positions exceed the context of %zu",
            context->length, count, context->limits.context);
        return buffer;
    }
    for (size_t i = 0; i < count; i++) {
        if (ids[i] < 0 || ids[i] >= LUN_VOCAB) {
            snprintf(buffer, size, "lunelette: token id %lld at index %zu is outside [0, %d)",
                (long long)ids[i], i, LUN_VOCAB);
            return buffer;
        }
    }
    return NULL;
}

/* One model call (prefill, append or decode). The sequence is marked broken
 * before the device runs, so every failure path below leaves it broken; only a
 * finished step with finite logits moves it to SEQ_PUBLISHED. The current
 * checkpoint survives a successful call (restore rewinds to it) and is dropped
 * by a failed one. */
static int run_call(lunelette_metal *context, const int64_t *ids, size_t count, call_kind kind,
    const float **logits, char *error, size_t capacity)
{
    char local[512];
    if (!error || !capacity) {
        error = local;
        capacity = sizeof local;
    }
    error[0] = 0;
    if (logits) {
        *logits = NULL;
    }
    char reason[256];
    const char *rejected = check_call(context, ids, count, kind, logits, reason, sizeof reason);
    if (rejected) {
        snprintf(error, capacity, "%s", rejected);
        return -1;
    }
    lunelette_metal_checkpoint *keep = context->current;
    context->current = NULL;
    context->state = SEQ_BROKEN;
    const float *output = NULL;
    int flagged = 0;
    if (lun_device_run(context->device, ids, count, context->length, &output, &flagged, error,
            capacity)) {
        size_t used = strlen(error);
        if (used + 1 < capacity) {
            snprintf(error + used, capacity - used, "%sreset required", used ? "; " : "");
        }
        return -1;
    }
    if (flagged) {
        size_t bad = 0;
        while (bad < LUN_VOCAB && isfinite(output[bad])) {
            bad++;
        }
        if (bad < LUN_VOCAB) {
            snprintf(error, capacity, "lunelette: logit %zu is not finite; reset required", bad);
        } else {
            snprintf(error, capacity, "lunelette: the head reported a non-finite value; reset required");
        }
        return -1;
    }
    context->length += count;
    context->state = SEQ_PUBLISHED;
    context->current = keep;
    *logits = output;
    return 0;
}

LUN_API int lunelette_metal_prefill(lunelette_metal *context, const int64_t *ids, size_t count,
    const float **logits, char *error, size_t capacity)
{
    return run_call(context, ids, count, CALL_PREFILL, logits, error, capacity);
}

LUN_API int lunelette_metal_decode(lunelette_metal *context, int64_t token,
    const float **logits, char *error, size_t capacity)
{
    return run_call(context, &token, 1, CALL_APPEND, logits, error, capacity);
}

LUN_API int lunelette_metal_append(lunelette_metal *context, const int64_t *ids, size_t count,
    const float **logits, char *error, size_t capacity)
{
    return run_call(context, ids, count, CALL_APPEND, logits, error, capacity);
}

static void put_error(char *error, size_t capacity, const char *message)
{
    if (error && capacity) {
        snprintf(error, capacity, "%s", message);
    }
}

/* A checkpoint is the published endpoint: its length and a copy of its logits.
 * No KV is copied, because a later restore only shortens the sequence, and the
 * rows below the saved length are never rewritten while this handle is current
 * (appends write at the end; reset drops the handle). */
LUN_API int lunelette_metal_checkpoint_create(lunelette_metal *context,
    lunelette_metal_checkpoint **checkpoint, char *error, size_t capacity)
{
    if (checkpoint) {
        *checkpoint = NULL;
    }
    if (!context || !checkpoint) {
        put_error(error, capacity, "checkpoint: context and output handle are required");
        return -1;
    }
    if (context->state != SEQ_PUBLISHED || context->length == 0 ||
        context->length > context->limits.context || context->identity == 0) {
        put_error(error, capacity, "checkpoint: needs a valid sequence with published logits");
        return -1;
    }
    if (context->epoch == UINT64_MAX) {
        put_error(error, capacity, "checkpoint: epoch counter exhausted; handle not replaced");
        return -1;
    }
    for (size_t i = 0; i < LUN_VOCAB; i++) {
        if (!isfinite(context->logits[i])) {
            if (error && capacity) {
                snprintf(error, capacity, "checkpoint: endpoint logit %zu is not finite; reset required",
                    i);
            }
            context->state = SEQ_BROKEN;
            context->current = NULL;
            return -1;
        }
    }
    lunelette_metal_checkpoint *handle = malloc(sizeof *handle);
    if (!handle) {
        put_error(error, capacity, "checkpoint: out of host memory; previous handle kept");
        return -1;
    }
    handle->context = context;
    handle->identity = context->identity;
    handle->epoch = ++context->epoch;
    handle->length = context->length;
    memcpy(handle->logits, context->logits, sizeof handle->logits);
    context->current = handle;
    *checkpoint = handle;
    return 0;
}

LUN_API int lunelette_metal_checkpoint_restore(lunelette_metal *context,
    const lunelette_metal_checkpoint *checkpoint, const float **logits,
    char *error, size_t capacity)
{
    if (logits) {
        *logits = NULL;
    }
    const char *why = NULL;
    if (!context || !checkpoint || !logits) {
        why = "checkpoint: context, handle and logits output are required";
    } else if (context->current != checkpoint || checkpoint->identity != context->identity ||
        checkpoint->epoch != context->epoch) {
        why = "checkpoint: handle is not this context's current checkpoint";
    } else if (context->state == SEQ_BROKEN || context->state == SEQ_EMPTY) {
        why = "checkpoint: sequence was reset or invalidated since the handle was made";
    } else if (checkpoint->length == 0 || checkpoint->length > context->length ||
        checkpoint->length > context->limits.context) {
        why = "checkpoint: saved length does not fit the current sequence";
    }
    if (why) {
        put_error(error, capacity, why);
        return -1;
    }
    memcpy(context->logits, checkpoint->logits, sizeof checkpoint->logits);
    context->length = checkpoint->length;
    context->state = SEQ_PUBLISHED;
    *logits = context->logits;
    return 0;
}

LUN_API void lunelette_metal_checkpoint_destroy(lunelette_metal_checkpoint *checkpoint)
{
    if (!checkpoint) {
        return;
    }
    if (checkpoint->context && checkpoint->context->current == checkpoint) {
        checkpoint->context->current = NULL;
    }
    free(checkpoint);
}

/* ---- additive entry points (include/lunelette_cuda.h) ---- */

LUN_API int lunelette_cuda_validate_checkpoint(const char *path,
    lunelette_metal_strategy strategy, char *error, size_t capacity)
{
    char local[512];
    if (!error || !capacity) {
        error = local;
        capacity = sizeof local;
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
    /* every FP8 tensor read and scanned whole, by the same parallel reader
     * the upload uses (the largest tensor is 9216 x 3072 bytes) */
    size_t largest = 0;
    for (size_t index = 0; index < LUN_WEIGHT_COUNT; index++) {
        if (weights.w[index].tensor->dtype == LUN_F8_E4M3 && weights.w[index].elements > largest) {
            largest = weights.w[index].elements;
        }
    }
    unsigned char *buffer = malloc(largest ? largest : 1);
    int status = buffer ? 0 : -1;
    if (!buffer) {
        snprintf(error, capacity, "validate: out of host memory");
    }
    for (size_t index = 0; !status && index < LUN_WEIGHT_COUNT; index++) {
        if (weights.w[index].tensor->dtype != LUN_F8_E4M3) {
            continue;
        }
        lun_admission table;
        status = lun_weights_admission(&weights, index, strategy != LUNELETTE_METAL_RESIDENT_FP32,
            &table, error, capacity) ||
            parallel_read(&weights, index, &table, 0, buffer, weights.w[index].elements, error, capacity);
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

LUN_API const float *lunelette_cuda_snapshot(lunelette_metal *context, int normalized)
{
    if (!context || !context->device || context->state != SEQ_PUBLISHED) {
        return NULL;
    }
    const size_t rows = lun_device_trace_rows(context->device);
    const int kind = normalized != 0;
    if (!rows) {
        return NULL;
    }
    if (!context->snapshot[kind] &&
        !(context->snapshot[kind] = malloc(context->limits.block * (size_t)LUN_HIDDEN * sizeof(float)))) {
        return NULL;
    }
    if (lun_device_trace_copy(context->device, kind ? LUN_LAYERS : LUN_LAYERS - 1, context->snapshot[kind],
            rows * (size_t)LUN_HIDDEN)) {
        return NULL;
    }
    return context->snapshot[kind];
}

LUN_API size_t lunelette_cuda_length(const lunelette_metal *context)
{
    return context ? context->length : 0;
}

LUN_API int lunelette_cuda_decode_loop(lunelette_metal *context, int64_t first_token, size_t steps,
    int64_t *tokens, float *milliseconds, int *launches, char *error, size_t capacity)
{
    char local[512];
    if (!error || !capacity) {
        error = local;
        capacity = sizeof local;
    }
    error[0] = 0;
    if (!context || !tokens || !steps || first_token < 0 || first_token >= LUN_VOCAB ||
        (context->state != SEQ_PUBLISHED && context->state != SEQ_UNPUBLISHED) ||
        steps > context->limits.context - context->length) {
        snprintf(error, capacity, "decode loop: needs a prefilled valid sequence, a token id in "
            "[0, %d) and room for %zu more positions", LUN_VOCAB, steps);
        return -1;
    }
    lunelette_metal_checkpoint *keep = context->current;
    context->current = NULL;
    context->state = SEQ_BROKEN;
    if (lun_device_decode_loop(context->device, first_token, context->length, steps, tokens,
            milliseconds, launches, error, capacity)) {
        return -1;
    }
    /* The KV cache holds `steps` more positions; the host logits were not
     * refreshed, so no endpoint is published until the next model call. */
    context->length += steps;
    context->state = SEQ_UNPUBLISHED;
    context->current = keep;
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
