/* A CPU stand-in for the CUDA layer behind lunelette_b200/csrc/device.h, so that
 * the host runtime (runtime.c: the metal.h state machine and checkpoints),
 * the batch manager (batch.c: pages, forks) and the upload path can be built
 * and tested without a GPU, under sanitizers (tests/test_fake_device.py).
 *
 * The "model" is a deterministic function of the whole token history: the
 * KV pool stores the token id written at each position (pages of 64 positions
 * reached through a session's page table, as on the device), and the logits
 * of a position are a hash of every id at positions 0..p read back through
 * that table. So a wrong page table, a page shared or copied wrongly, a stale
 * row read past the length, or a restore that leaves the wrong length all show
 * up as different logits than a fresh sequence with the same ids. Token id
 * FAKE_NAN_ID in a block makes that block's logits non-finite.
 *
 * The upload path records, per FP8 tensor (layer, slot), a digest of the bytes
 * and the scale it was given, and a digest of the embedding, so a test can
 * check that every checkpoint tensor reached its slot. Test hooks: the
 * fake_device_* functions at the end. */
#include "device.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define FAKE_VOCAB 131072
#define FAKE_HIDDEN 3072
#define FAKE_LAYERS 26
#define FAKE_PAGE 64
#define FAKE_STAGING ((size_t)32 << 20)
#define FAKE_NAN_ID 131071

struct lun_device {
    size_t context, block, pool_pages, row_pages, sessions;
    int64_t *pool;        /* [pool_pages][64] token ids */
    int *tables;          /* [sessions][row_pages] page ids, -1 unset */
    int current;          /* session of single-sequence calls */
    float *logits;        /* host logits of the last call */
    unsigned char *staging[2];
    int trace;
    size_t trace_rows;
    uint64_t trace_hash;  /* history hash of the last traced call */
    uint64_t digest[FAKE_LAYERS][LUN_SLOT_COUNT];
    float scale[FAKE_LAYERS][LUN_SLOT_COUNT];
    uint64_t embedding_digest;
    size_t embedding_bytes;
    int finished;
};

static lun_device *last_device;

/* Weighted sum of the little-endian 64-bit words (word i weighted 2 i + 1,
 * counted from `first_word`), modulo 2^64; bytes past the last whole word
 * count as a zero-padded word. */
static uint64_t digest_words(const unsigned char *p, size_t bytes, uint64_t first_word)
{
    uint64_t sum = 0;
    size_t words = bytes / 8;
    for (size_t i = 0; i < words; i++) {
        uint64_t w;
        memcpy(&w, p + 8 * i, 8);
        sum += w * (2 * (first_word + i) + 1);
    }
    if (bytes % 8) {
        uint64_t w = 0;
        memcpy(&w, p + 8 * words, bytes % 8);
        sum += w * (2 * (first_word + words) + 1);
    }
    return sum;
}

static int set_error(char *error, size_t capacity, const char *what)
{
    if (error && capacity) {
        snprintf(error, capacity, "%s", what);
    }
    return -1;
}

static lun_device *make(size_t pool_pages, size_t context, size_t block, size_t sessions, char *error,
    size_t capacity)
{
    lun_device *d = calloc(1, sizeof *d);
    if (!d) {
        set_error(error, capacity, "fake device: out of host memory");
        return NULL;
    }
    d->context = context;
    d->block = block;
    d->pool_pages = pool_pages;
    d->row_pages = (context + FAKE_PAGE - 1) / FAKE_PAGE;
    d->sessions = sessions;
    d->pool = calloc(pool_pages * FAKE_PAGE, sizeof *d->pool);
    d->tables = malloc(sessions * d->row_pages * sizeof *d->tables);
    d->logits = calloc(FAKE_VOCAB, sizeof *d->logits);
    d->staging[0] = malloc(FAKE_STAGING);
    d->staging[1] = malloc(FAKE_STAGING);
    if (!d->pool || !d->tables || !d->logits || !d->staging[0] || !d->staging[1]) {
        lun_device_destroy(d);
        set_error(error, capacity, "fake device: out of host memory");
        return NULL;
    }
    for (size_t i = 0; i < sessions * d->row_pages; i++) {
        d->tables[i] = -1;
    }
    last_device = d;
    return d;
}

lun_device *lun_device_create(size_t context, size_t block, char *error, size_t capacity)
{
    size_t pages = (context + FAKE_PAGE - 1) / FAKE_PAGE;
    lun_device *d = make(pages, context, block, 1, error, capacity);
    if (d) {
        for (size_t i = 0; i < pages; i++) {
            d->tables[i] = (int)i;
        }
    }
    return d;
}

lun_device *lun_device_create_batch(size_t pool_pages, size_t session_context, size_t block,
    size_t max_sessions, char *error, size_t capacity)
{
    return make(pool_pages, session_context, block, max_sessions, error, capacity);
}

void lun_device_destroy(lun_device *d)
{
    if (!d) {
        return;
    }
    if (last_device == d) {
        last_device = NULL;
    }
    free(d->pool);
    free(d->tables);
    free(d->logits);
    free(d->staging[0]);
    free(d->staging[1]);
    free(d);
}

int lun_device_ordinal(const lun_device *d)
{
    (void)d;
    return 0;
}

void lun_device_bytes_owned(const lun_device *d, lun_device_bytes *bytes)
{
    bytes->weight_bytes = 0;
    bytes->scratch_bytes = FAKE_VOCAB * sizeof(float);
    bytes->kv_bytes = d->pool_pages * FAKE_PAGE * sizeof(int64_t);
}

size_t lun_device_staging_bytes(void) { return FAKE_STAGING; }

void *lun_device_staging(lun_device *d, int index) { return d->staging[index & 1]; }

int lun_device_staging_wait(lun_device *d, int index)
{
    (void)d;
    (void)index;
    return 0;
}

int lun_device_upload_linear(lun_device *d, int index, int layer, int slot, size_t rows, size_t cols,
    float scale)
{
    if (layer < 0 || layer >= FAKE_LAYERS || slot < 0 || slot >= LUN_SLOT_COUNT || rows * cols > FAKE_STAGING) {
        return -1;
    }
    d->digest[layer][slot] = digest_words(d->staging[index & 1], rows * cols, 0);
    d->scale[layer][slot] = scale;
    return 0;
}

int lun_device_upload_embedding(lun_device *d, int index, size_t offset, size_t bytes)
{
    if ((offset % 8) || bytes > FAKE_STAGING) {
        return -1;
    }
    d->embedding_digest += digest_words(d->staging[index & 1], bytes, offset / 8);
    d->embedding_bytes += bytes;
    return 0;
}

int lun_device_upload_norms(lun_device *d, const float *norms, const float *final_norm)
{
    (void)d;
    return norms && final_norm ? 0 : -1;
}

int lun_device_upload_rope(lun_device *d, const float *cosine, const float *sine, size_t positions)
{
    return cosine && sine && positions >= d->context ? 0 : -1;
}

int lun_device_upload_finish(lun_device *d, char *error, size_t capacity)
{
    (void)error;
    (void)capacity;
    d->finished = 1;
    return 0;
}

/* ---- the deterministic "model" ---------------------------------------------- */

static uint64_t mix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* Slot of position `position` of session `session`, or NULL past its pages. */
static int64_t *slot(lun_device *d, int session, size_t position)
{
    size_t index = position / FAKE_PAGE;
    if (session < 0 || (size_t)session >= d->sessions || index >= d->row_pages) {
        return NULL;
    }
    int page = d->tables[(size_t)session * d->row_pages + index];
    if (page < 0 || (size_t)page >= d->pool_pages) {
        return NULL;
    }
    return &d->pool[(size_t)page * FAKE_PAGE + position % FAKE_PAGE];
}

/* Hash of the ids at positions 0..last of a session, or 0 if a page is missing. */
static uint64_t history(lun_device *d, int session, size_t last)
{
    uint64_t h = 1469598103934665603ull;
    for (size_t p = 0; p <= last; p++) {
        int64_t *s = slot(d, session, p);
        if (!s) {
            return 0;
        }
        h = (h ^ (uint64_t)(*s + 1)) * 1099511628211ull;
    }
    return h;
}

static void logits_of(uint64_t h, int nan, float *out)
{
    for (int v = 0; v < FAKE_VOCAB; v++) {
        out[v] = (float)((double)(mix64(h + (uint64_t)v) >> 11) * 0x1p-53 * 8.0 - 4.0);
    }
    if (nan) {
        out[7] = NAN;
    }
}

static int64_t argmax(const float *x)
{
    int64_t best = 0;
    for (int v = 1; v < FAKE_VOCAB; v++) {
        if (x[v] > x[best]) {
            best = v;
        }
    }
    return best;
}

/* Write the block's ids at positions length.., then the logits of its last position. */
static int step(lun_device *d, int session, const int64_t *ids, size_t count, size_t length, float *out,
    int *nonfinite)
{
    int nan = 0;
    for (size_t i = 0; i < count; i++) {
        int64_t *s = slot(d, session, length + i);
        if (!s || ids[i] < 0 || ids[i] >= FAKE_VOCAB) {
            return -1;
        }
        *s = ids[i];
        nan |= ids[i] == FAKE_NAN_ID;
    }
    uint64_t h = history(d, session, length + count - 1);
    if (!h) {
        return -1;
    }
    logits_of(h, nan, out);
    *nonfinite = nan;
    if (d->trace) {
        d->trace_rows = count;
        d->trace_hash = h;
    }
    return 0;
}

int lun_device_run(lun_device *d, const int64_t *ids, size_t count, size_t length, const float **logits,
    int *nonfinite, char *error, size_t capacity)
{
    if (!d->finished || !count || count > d->block || length + count > d->context) {
        return set_error(error, capacity, "fake device run: block/context exceeded");
    }
    if (step(d, d->current, ids, count, length, d->logits, nonfinite)) {
        return set_error(error, capacity, "fake device run: no page for a position");
    }
    if (logits) {
        *logits = d->logits;
    }
    return 0;
}

float *lun_device_host_logits(lun_device *d) { return d->logits; }

int lun_device_decode_loop(lun_device *d, int64_t first_token, size_t length, size_t steps, int64_t *tokens,
    float *milliseconds, int *launches, char *error, size_t capacity)
{
    int64_t tok = first_token;
    int nonfinite = 0;
    for (size_t i = 0; i < steps; i++) {
        if (length + i >= d->context || step(d, d->current, &tok, 1, length + i, d->logits, &nonfinite)) {
            return set_error(error, capacity, "fake device decode loop: context exceeded");
        }
        tok = argmax(d->logits);
        tokens[i] = tok;
    }
    if (milliseconds) {
        *milliseconds = 0.0f;
    }
    if (launches) {
        *launches = 1;
    }
    return 0;
}

int lun_device_session_table(lun_device *d, int session, const int *pages, size_t n)
{
    if (session < 0 || (size_t)session >= d->sessions || n > d->row_pages) {
        return -1;
    }
    for (size_t i = 0; i < d->row_pages; i++) {
        d->tables[(size_t)session * d->row_pages + i] = i < n ? pages[i] : -1;
    }
    return 0;
}

int lun_device_use_session(lun_device *d, int session)
{
    if (session < 0 || (size_t)session >= d->sessions) {
        return -1;
    }
    d->current = session;
    return 0;
}

int lun_device_copy_page(lun_device *d, int src_page, int dst_page, int slots)
{
    if (src_page < 0 || dst_page < 0 || (size_t)src_page >= d->pool_pages || (size_t)dst_page >= d->pool_pages ||
        slots < 1 || slots > FAKE_PAGE) {
        return -1;
    }
    memcpy(&d->pool[(size_t)dst_page * FAKE_PAGE], &d->pool[(size_t)src_page * FAKE_PAGE],
        (size_t)slots * sizeof *d->pool);
    return 0;
}

int lun_device_batch_decode(lun_device *d, const int *sessions, const int64_t *ids, const int *positions,
    size_t n, float *logits, int64_t *next, int *nonfinite, char *error, size_t capacity)
{
    float *row = d->logits;
    *nonfinite = 0;
    for (size_t i = 0; i < n; i++) {
        float *out = logits ? logits + i * FAKE_VOCAB : row;
        int bad = 0;
        if (positions[i] < 0 || step(d, sessions[i], &ids[i], 1, (size_t)positions[i], out, &bad)) {
            return set_error(error, capacity, "fake device batch decode: no page for a position");
        }
        next[i] = argmax(out);
        *nonfinite |= bad;
    }
    return 0;
}

int lun_device_timeline(lun_device *d, int enable)
{
    (void)d;
    (void)enable;
    return -1;
}

int lun_device_timeline_copy(lun_device *d, unsigned long long *out, size_t entries)
{
    (void)d;
    (void)out;
    (void)entries;
    return -1;
}

int lun_device_trace(lun_device *d, int enable)
{
    d->trace = enable != 0;
    d->trace_rows = 0;
    return 0;
}

/* Traced rows: element (row r, column c) of layer `which` is a value derived
 * from the traced call's history hash, so a copy of the wrong layer, row or
 * call is visible. */
int lun_device_trace_copy(lun_device *d, int which, float *out, size_t floats)
{
    if (which < 0 || which > FAKE_LAYERS || floats > d->trace_rows * FAKE_HIDDEN) {
        return -1;
    }
    for (size_t i = 0; i < floats; i++) {
        out[i] = (float)((double)(mix64(d->trace_hash ^ ((uint64_t)which << 40) ^ i) >> 40) * 0x1p-24);
    }
    return 0;
}

size_t lun_device_trace_rows(const lun_device *d) { return d->trace ? d->trace_rows : 0; }

cudaError_t cudaSetDevice(int device)
{
    (void)device;
    return cudaSuccess;
}

/* ---- test hooks (ctypes) ------------------------------------------------------ */

/* Digest and scale of the FP8 tensor uploaded to (layer, slot) of the most
 * recently created device; the embedding's digest and byte count. */
uint64_t fake_device_linear_digest(int layer, int slot, float *scale)
{
    if (!last_device || layer < 0 || layer >= FAKE_LAYERS || slot < 0 || slot >= LUN_SLOT_COUNT) {
        return 0;
    }
    *scale = last_device->scale[layer][slot];
    return last_device->digest[layer][slot];
}

uint64_t fake_device_embedding_digest(size_t *bytes)
{
    if (!last_device) {
        return 0;
    }
    *bytes = last_device->embedding_bytes;
    return last_device->embedding_digest;
}

/* The logits a fresh sequence of these ids gives at its last position. */
void fake_device_reference_logits(const int64_t *ids, size_t count, float *out)
{
    uint64_t h = 1469598103934665603ull;
    int nan = 0;
    for (size_t p = 0; p < count; p++) {
        h = (h ^ (uint64_t)(ids[p] + 1)) * 1099511628211ull;
        nan |= ids[p] == FAKE_NAN_ID;
    }
    logits_of(h, nan, out);
}
