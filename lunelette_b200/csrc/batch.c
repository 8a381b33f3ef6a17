/* Batched decode over many independent sessions sharing one weight replica
 * (lunelette_cuda_batch_* in include/lunelette_cuda.h).
 *
 * The reference's context is one set of weights with one sequence
 * (src/metal_internal.h:29-50); a service serving many users opens one context
 * per user. Here one device context holds the weights once and a paged FP32 KV
 * pool: every session owns pages (64 positions each) through its row of a page
 * table, taken from a free list as it grows and returned when it closes.
 * Appends run one session at a time through the single-sequence path (the
 * tcgen05 GEMMs for blocks, the persistent kernel for one token); a decode step
 * takes one token of each of n sessions and runs the projections once for all
 * of them. A session can be forked from a prefix of another: the new session
 * shares the prefix's full pages (reference-counted; no session ever rewrites
 * a position below its length) and gets its own copy of a partial last page.
 * Single caller per batch context, like lunelette_metal.
 */
#include "lunelette_cuda.h"

#include "device.h"
#include "weights.h"

#include <cuda_runtime_api.h>
#include <stdbool.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define LUN_API __attribute__((visibility("default")))
#define LUN_PAGE 64

int lun_runtime_load(lun_device *device, const char *path, size_t rope_positions, char *error, size_t capacity);

typedef struct {
    bool open;
    size_t length;
    int *pages;
    size_t npages;
} lun_session;

struct lunelette_cuda_batch {
    lun_device *device;
    size_t context, block, max_sessions, pool_pages, row_pages;
    int *free_pages;
    size_t free_count;
    unsigned *page_refs; /* sessions holding each pool page; 0 = on the free list */
    lun_session *sessions;
    int *meta_sessions, *meta_positions; /* per decode call */
};

static int set_error(char *error, size_t capacity, const char *what)
{
    if (error && capacity) {
        snprintf(error, capacity, "%s", what);
    }
    return -1;
}

LUN_API void lunelette_cuda_batch_destroy(lunelette_cuda_batch *b)
{
    if (!b) {
        return;
    }
    if (b->device) {
        cudaSetDevice(lun_device_ordinal(b->device));
        lun_device_destroy(b->device);
    }
    if (b->sessions) {
        for (size_t s = 0; s < b->max_sessions; s++) {
            free(b->sessions[s].pages);
        }
    }
    free(b->sessions);
    free(b->free_pages);
    free(b->page_refs);
    free(b->meta_sessions);
    free(b->meta_positions);
    free(b);
}

LUN_API lunelette_cuda_batch *lunelette_cuda_batch_create(const char *path, size_t max_sessions, size_t context,
    size_t pool_positions, size_t block, char *error, size_t capacity)
{
    char local[512];
    if (!error || !capacity) {
        error = local;
        capacity = sizeof local;
    }
    error[0] = 0;
    if (!path || !max_sessions || max_sessions > 65536 || !context || context > 4352 || block < 8 ||
        block > 256 || pool_positions < LUN_PAGE) {
        set_error(error, capacity, "batch: invalid sessions, context (<= 4352), pool or block (8..256)");
        return NULL;
    }
    lunelette_cuda_batch *b = calloc(1, sizeof *b);
    if (!b) {
        set_error(error, capacity, "batch: allocation failed");
        return NULL;
    }
    b->context = context;
    b->block = block;
    b->max_sessions = max_sessions;
    b->pool_pages = (pool_positions + LUN_PAGE - 1) / LUN_PAGE;
    b->row_pages = (context + LUN_PAGE - 1) / LUN_PAGE;
    b->free_pages = malloc(b->pool_pages * sizeof(int));
    b->page_refs = calloc(b->pool_pages, sizeof(unsigned));
    b->sessions = calloc(max_sessions, sizeof(lun_session));
    b->meta_sessions = malloc(block * sizeof(int));
    b->meta_positions = malloc(block * sizeof(int));
    if (!b->free_pages || !b->page_refs || !b->sessions || !b->meta_sessions || !b->meta_positions) {
        set_error(error, capacity, "batch: allocation failed");
        lunelette_cuda_batch_destroy(b);
        return NULL;
    }
    for (size_t s = 0; s < max_sessions; s++) {
        b->sessions[s].pages = malloc(b->row_pages * sizeof(int));
        if (!b->sessions[s].pages) {
            set_error(error, capacity, "batch: allocation failed");
            lunelette_cuda_batch_destroy(b);
            return NULL;
        }
    }
    /* lowest page ids are handed out first */
    for (size_t i = 0; i < b->pool_pages; i++) {
        b->free_pages[i] = (int)(b->pool_pages - 1 - i);
    }
    b->free_count = b->pool_pages;
    b->device = lun_device_create_batch(b->pool_pages, context, block, max_sessions, error, capacity);
    if (!b->device || lun_runtime_load(b->device, path, context, error, capacity)) {
        lunelette_cuda_batch_destroy(b);
        return NULL;
    }
    return b;
}

LUN_API int lunelette_cuda_batch_open(lunelette_cuda_batch *b, int *session, char *error, size_t capacity)
{
    if (!b || !session) {
        return set_error(error, capacity, "batch open: invalid arguments");
    }
    for (size_t s = 0; s < b->max_sessions; s++) {
        if (!b->sessions[s].open) {
            b->sessions[s].open = true;
            b->sessions[s].length = 0;
            b->sessions[s].npages = 0;
            *session = (int)s;
            return 0;
        }
    }
    return set_error(error, capacity, "batch open: every session is in use");
}

LUN_API int lunelette_cuda_batch_close(lunelette_cuda_batch *b, int session)
{
    if (!b || session < 0 || (size_t)session >= b->max_sessions || !b->sessions[session].open) {
        return -1;
    }
    lun_session *s = &b->sessions[session];
    for (size_t i = s->npages; i > 0; i--) {
        int page = s->pages[i - 1];
        if (--b->page_refs[page] == 0) {
            b->free_pages[b->free_count++] = page;
        }
    }
    s->npages = 0;
    s->length = 0;
    s->open = false;
    return 0;
}

LUN_API size_t lunelette_cuda_batch_length(const lunelette_cuda_batch *b, int session)
{
    if (!b || session < 0 || (size_t)session >= b->max_sessions || !b->sessions[session].open) {
        return 0;
    }
    return b->sessions[session].length;
}

LUN_API size_t lunelette_cuda_batch_free_positions(const lunelette_cuda_batch *b)
{
    return b ? b->free_count * LUN_PAGE : 0;
}

/* Pages so that session s holds `positions` positions; the device row follows. */
static int reserve(lunelette_cuda_batch *b, int session, size_t positions, char *error, size_t capacity)
{
    lun_session *s = &b->sessions[session];
    size_t need = (positions + LUN_PAGE - 1) / LUN_PAGE;
    if (need <= s->npages) {
        return 0;
    }
    if (need - s->npages > b->free_count) {
        return set_error(error, capacity, "batch: KV pool exhausted");
    }
    while (s->npages < need) {
        int page = b->free_pages[--b->free_count];
        b->page_refs[page] = 1;
        s->pages[s->npages++] = page;
    }
    if (lun_device_session_table(b->device, session, s->pages, s->npages)) {
        return set_error(error, capacity, "batch: page table upload failed");
    }
    return 0;
}

LUN_API int lunelette_cuda_batch_fork(lunelette_cuda_batch *b, int source, size_t length, int *session,
    char *error, size_t capacity)
{
    if (!b || !session || source < 0 || (size_t)source >= b->max_sessions || !b->sessions[source].open ||
        length == 0 || length > b->sessions[source].length) {
        return set_error(error, capacity, "batch fork: needs an open source session and 1..its length positions");
    }
    size_t slot = 0;
    while (slot < b->max_sessions && b->sessions[slot].open) {
        slot++;
    }
    if (slot == b->max_sessions) {
        return set_error(error, capacity, "batch fork: every session is in use");
    }
    const lun_session *src = &b->sessions[source];
    size_t shared = length / LUN_PAGE, partial = length % LUN_PAGE;
    if (partial && b->free_count == 0) {
        return set_error(error, capacity, "batch fork: KV pool exhausted");
    }
    lun_session *s = &b->sessions[slot];
    for (size_t i = 0; i < shared; i++) {
        s->pages[i] = src->pages[i];
        b->page_refs[src->pages[i]]++;
    }
    s->npages = shared;
    if (partial) {
        int page = b->free_pages[--b->free_count];
        b->page_refs[page] = 1;
        s->pages[s->npages++] = page;
        if (lun_device_copy_page(b->device, src->pages[shared], page, (int)partial)) {
            s->open = true; /* let close return every page taken above */
            lunelette_cuda_batch_close(b, (int)slot);
            return set_error(error, capacity, "batch fork: partial page copy failed");
        }
    }
    if (lun_device_session_table(b->device, (int)slot, s->pages, s->npages)) {
        s->open = true;
        lunelette_cuda_batch_close(b, (int)slot);
        return set_error(error, capacity, "batch fork: page table upload failed");
    }
    s->open = true;
    s->length = length;
    *session = (int)slot;
    return 0;
}

LUN_API int lunelette_cuda_batch_append(lunelette_cuda_batch *b, int session, const int64_t *ids, size_t count,
    const float **logits, char *error, size_t capacity)
{
    if (!b || session < 0 || (size_t)session >= b->max_sessions || !b->sessions[session].open || !ids || !count ||
        count > b->block || !logits) {
        return set_error(error, capacity, "batch append: invalid arguments");
    }
    lun_session *s = &b->sessions[session];
    if (s->length + count > b->context) {
        return set_error(error, capacity, "batch append: context exceeded");
    }
    for (size_t i = 0; i < count; i++) {
        if (ids[i] < 0 || ids[i] >= LUN_VOCAB) {
            return set_error(error, capacity, "batch append: token id out of range");
        }
    }
    if (reserve(b, session, s->length + count, error, capacity) || lun_device_use_session(b->device, session)) {
        return -1;
    }
    int nonfinite = 0;
    if (lun_device_run(b->device, ids, count, s->length, logits, &nonfinite, error, capacity)) {
        return -1;
    }
    s->length += count;
    if (nonfinite) {
        return set_error(error, capacity, "batch append: non-finite logits");
    }
    return 0;
}

LUN_API int lunelette_cuda_batch_decode(lunelette_cuda_batch *b, const int *sessions, const int64_t *ids, size_t n,
    float *logits, int64_t *next, char *error, size_t capacity)
{
    if (!b || !sessions || !ids || !n || n > b->block || !next) {
        return set_error(error, capacity, "batch decode: invalid arguments");
    }
    for (size_t i = 0; i < n; i++) {
        int s = sessions[i];
        if (s < 0 || (size_t)s >= b->max_sessions || !b->sessions[s].open || b->sessions[s].length == 0 ||
            b->sessions[s].length >= b->context || ids[i] < 0 || ids[i] >= LUN_VOCAB) {
            return set_error(error, capacity, "batch decode: invalid session, length or id");
        }
        for (size_t j = 0; j < i; j++) {
            if (sessions[j] == s) {
                return set_error(error, capacity, "batch decode: a session appears twice");
            }
        }
    }
    for (size_t i = 0; i < n; i++) {
        if (reserve(b, sessions[i], b->sessions[sessions[i]].length + 1, error, capacity)) {
            return -1;
        }
        b->meta_positions[i] = (int)b->sessions[sessions[i]].length;
    }
    int nonfinite = 0;
    if (lun_device_batch_decode(b->device, sessions, ids, b->meta_positions, n, logits, next, &nonfinite, error,
            capacity)) {
        return -1;
    }
    for (size_t i = 0; i < n; i++) {
        b->sessions[sessions[i]].length++;
    }
    if (nonfinite) {
        return set_error(error, capacity, "batch decode: non-finite logits");
    }
    return 0;
}
