/* Thin C-ABI between the plain-C host runtime (runtime.c) and the CUDA layer
 * (device.cu). Plain pointers and sizes only. This is the seam that takes the
 * place of the reference's Objective-C owner and encoder
 * (src/metal_internal.h:412-457, src/metal_encode.m). */
#ifndef LUN_DEVICE_H
#define LUN_DEVICE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lun_device lun_device;

/* Linear slots within a layer (storage order on the device). */
enum { LUN_SLOT_Q, LUN_SLOT_K, LUN_SLOT_V, LUN_SLOT_O, LUN_SLOT_GATE, LUN_SLOT_UP,
    LUN_SLOT_DOWN, LUN_SLOT_COUNT };

/* Byte sizes of what lun_device_create would allocate for a (context, block)
 * profile; used for preflight and get_memory. */
typedef struct {
    uint64_t weight_bytes, scratch_bytes, kv_bytes;
} lun_device_bytes;
void lun_device_plan(size_t context, size_t block, lun_device_bytes *bytes);

/* Allocates weights, KV, scratch, tables and pinned staging on the current
 * device. Fails (NULL + diagnostic) before allocating when cudaMemGetInfo shows
 * too little free memory. */
lun_device *lun_device_create(size_t context, size_t block, char *error, size_t capacity);
void lun_device_destroy(lun_device *d);
int lun_device_ordinal(const lun_device *d);
void lun_device_bytes_owned(const lun_device *d, lun_device_bytes *bytes);

/* Upload path. Two pinned staging buffers of lun_device_staging_bytes() each;
 * wait before refilling a buffer that an earlier upload may still read. */
size_t lun_device_staging_bytes(void);
void *lun_device_staging(lun_device *d, int index);
int lun_device_staging_wait(lun_device *d, int index);
/* A whole FP8 tensor from staging buffer `index` (rows*cols bytes). */
int lun_device_upload_linear(lun_device *d, int index, int layer, int slot, size_t rows,
    size_t cols, float scale);
/* Bytes [offset, offset+bytes) of the BF16 embedding from staging buffer `index`. */
int lun_device_upload_embedding(lun_device *d, int index, size_t offset, size_t bytes);
/* norms: [26][2][3072] FP32 (input, post-attention), final: [3072] FP32. */
int lun_device_upload_norms(lun_device *d, const float *norms, const float *final_norm);
int lun_device_upload_rope(lun_device *d, const float *cosine, const float *sine,
    size_t positions);
int lun_device_upload_finish(lun_device *d, char *error, size_t capacity);

/* One prefill/append/decode block at sequence length `length`. On success
 * *logits points to the context's pinned host copy of the 131072 logits and
 * *nonfinite is 1 when the device saw a NaN/Inf logit. */
int lun_device_run(lun_device *d, const int64_t *ids, size_t count, size_t length,
    const float **logits, int *nonfinite, char *error, size_t capacity);
float *lun_device_host_logits(lun_device *d);

/* Device-resident greedy decode: `steps` decode steps starting from token
 * `first_token` at sequence length `length` (a valid prefix must already be in
 * the KV cache), each step one replay of a captured CUDA graph whose last
 * kernels pick the argmax and feed it to the next step. Writes the generated
 * ids, the CUDA-event time of the call and the kernel launches it made. */
int lun_device_decode_loop(lun_device *d, int64_t first_token, size_t length, size_t steps,
    int64_t *tokens, float *milliseconds, int *launches, char *error, size_t capacity);

/* Batched decode over independent sessions. The KV pool has pool_pages pages
 * of 64 positions; each of max_sessions sessions owns up to
 * ceil(session_context / 64) of them through its row of a page-table array.
 * block (8..256) bounds the tokens of one call. */
lun_device *lun_device_create_batch(size_t pool_pages, size_t session_context, size_t block,
    size_t max_sessions, char *error, size_t capacity);
/* Write session `session`'s page ids (n <= its row length). */
int lun_device_session_table(lun_device *d, int session, const int *pages, size_t n);
/* Single-sequence calls (lun_device_run) run on this session's pages. */
int lun_device_use_session(lun_device *d, int session);
/* Copy the first `slots` (1..64) positions of pool page src_page to dst_page,
 * K and V of every layer (copy-on-write of a partial page when a session is
 * forked from another's prefix). Synchronous. */
int lun_device_copy_page(lun_device *d, int src_page, int dst_page, int slots);
/* One decode step for n tokens of n sessions at their positions; greedy ids
 * into next, logits (n x 131072) when not NULL. */
int lun_device_batch_decode(lun_device *d, const int *sessions, const int64_t *ids, const int *positions,
    size_t n, float *logits, int64_t *next, int *nonfinite, char *error, size_t capacity);

/* Measurement: record %globaltimer at the start and after every grid barrier of
 * the first step of each persistent-kernel launch (133 entries). */
int lun_device_timeline(lun_device *d, int enable);
int lun_device_timeline_copy(lun_device *d, unsigned long long *out, size_t entries);

/* Test support: keep each layer's output hidden rows and the final-norm rows of
 * the most recent call (eager launches while enabled). */
int lun_device_trace(lun_device *d, int enable);
/* which: 0..25 = layer output [count][3072]; 26 = final norm [count][3072]. */
int lun_device_trace_copy(lun_device *d, int which, float *out, size_t floats);
/* Rows the most recent traced call kept (0 while tracing is off). */
size_t lun_device_trace_rows(const lun_device *d);

#ifdef __cplusplus
}
#endif

#endif
