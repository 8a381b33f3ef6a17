/* Additive C-ABI of the B200 backend (lunelette_b200/liblunelette_cuda.so),
 * next to the drop-in contract in metal.h. Nothing here is needed by callers of
 * metal.h. Device pointers are CUDA global memory of the current device;
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * All functions return 0 on success and -1 on invalid arguments or a CUDA
 * launch error; they launch asynchronously on `stream` unless noted.
 */
#ifndef LUNELETTE_CUDA_H
#define LUNELETTE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#include "metal.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- kernel-level entry points (parity tests, microbenchmarks) */

/* Set per-device kernel attributes; the model runtime does this itself. */
int lunelette_cuda_kernels_init(void);

/* out[i] = decode_e4m3(codes[i]) * scale, through the GEMV's in-register
 * conversion. Replaces convert_fp8 (src/metal_kernels.metal:145-152); the
 * decode itself restates st_f8_e4m3_to_f32 (src/safetensors.c:505-519). */
int lunelette_cuda_fp8_decode(const uint8_t *codes, size_t n, float scale, float *out,
    void *stream);

/* Row-major E4M3 codes [rows][cols] (cols % 16 == 0) -> the tiled layout that
 * the GEMV entry points below read: 8-row tiles of 1 KB blocks (8 rows x 128
 * columns) in tensor-core fragment order, rows padded to 8 and columns to 128
 * with zeros; dst holds ceil(rows/8)*8 * ceil(cols/128)*128 bytes. order 0 keeps
 * the row order; 1 takes q|k|v rows (rows % 128 == 0) and stores the RoPE pair
 * rows (j, j + 64) of each 128-row head adjacently (2j, 2j + 1); 2 takes the gate
 * rows followed by the up rows (rows even) and interleaves them (gate f at 2f,
 * up f at 2f + 1). The runtime stores its weights this way at upload, in place
 * of the reference's row-major MTLBuffers (src/metal_weights.c:150-231). */
int lunelette_cuda_tile_fp8(const uint8_t *src, size_t rows, size_t cols, int order, uint8_t *dst,
    void *stream);

/* y[t][r] = scale * sum_c decode(W[r][c]) * x[t][c]  (+ res[t][r] when res).
 * W tiled (order 0) from [rows][cols] E4M3, cols % 16 == 0, cols <= 9216; any
 * count. FP32 activations enter the tensor core as FP16 hi + lo halves after an
 * exact power-of-two scaling; products are exact and accumulate in FP32.
 * Replaces project_fp8 / project_fp8_lookup (src/metal_kernels.metal:154-177,
 * 249-272) and, with res, the residual element op (:47-57). */
int lunelette_cuda_gemv_fp8(const uint8_t *W, size_t rows, size_t cols, float scale,
    const float *x, const float *res, size_t count, float *y, void *stream);

/* Fused input RMSNorm + q/k/v projection + YaRN RoPE (+ query scale) + KV store
 * for `count` tokens at positions length..length+count-1. W is the [6144][3072]
 * q|k|v matrix tiled with order 1 (RoPE pairs adjacent); scales is a HOST array
 * {q, k, v}; q_out [count][4096] in the checkpoint's (unpermuted) order;
 * kv_pool is the paged FP32 pool [layer][page][K|V][8 heads][64 slots][128].
 * Replaces norm + 3x project_fp8 + 2x rope + the KV blit
 * (src/metal_encode.m:129-153, src/metal_kernels.metal:29-78). */
int lunelette_cuda_qkv_rope(const uint8_t *W, const float *scales, const float *gain,
    const float *x, size_t count, size_t length, const float *rope_cos, const float *rope_sin,
    float *q_out, float *kv_pool, const int *page_table, size_t num_pages, size_t layer,
    void *stream);

/* Fused post-attention RMSNorm + gate/up projection + SwiGLU. W is the gate
 * rows followed by the up rows ([18432][3072]) tiled with order 2; act
 * [count][9216].
 * Replaces norm + 2x project_fp8 + SiLU + multiply (src/metal_encode.m:162-172). */
int lunelette_cuda_gateup_swiglu(const uint8_t *W, float scale_gate, float scale_up,
    const float *gain, const float *x, size_t count, float *act, void *stream);

/* The same three projections on the tcgen05 tensor cores, the runtime's path
 * for blocks of more than four tokens (prefill, append): activations split
 * into FP16 hi + lo parts as above, FP8 weights converted to FP16 in shared
 * memory, tcgen05.mma (M = 128 tokens, N = 256 rows, K = 16) accumulating both
 * parts in TMEM (FP32), K ranges added in a fixed order. Same arguments and
 * results as lunelette_cuda_gemv_fp8 / _qkv_rope / _gateup_swiglu (rows % 8 == 0
 * here, cols <= 16384); each call allocates its workspace on the stream and synchronises it.
 * Replaces the MPS prefill GEMMs (src/metal_mps.m:26-111). */
int lunelette_cuda_gemm_fp8(const uint8_t *W, size_t rows, size_t cols, float scale,
    const float *x, const float *res, size_t count, float *y, void *stream);
int lunelette_cuda_gemm_qkv_rope(const uint8_t *W, const float *scales, const float *gain,
    const float *x, size_t count, size_t length, const float *rope_cos, const float *rope_sin,
    float *q_out, float *kv_pool, const int *page_table, size_t num_pages, size_t layer,
    void *stream);
int lunelette_cuda_gemm_gateup_swiglu(const uint8_t *W, float scale_gate, float scale_up,
    const float *gain, const float *x, size_t count, float *act, void *stream);

/* Microbenchmark of the tensor-core path: runs lunelette_cuda_gemm_fp8 (no
 * residual) `reps` times back to back, run r on the tiled matrix copy r % copies
 * of `copies` consecutive ones at W, and writes the mean device time in ms of
 * its three kernels from CUDA events on the stream: ms[0] activation split,
 * ms[1] the tcgen05 GEMM, ms[2] the ordered K-range finish. */
int lunelette_cuda_gemm_fp8_timed(const uint8_t *W, size_t copies, size_t rows, size_t cols, float scale,
    const float *x, size_t count, float *y, int reps, float *ms, void *stream);

/* out = gain * (x * rsqrt(mean(x^2) + 1e-5)) per row (src/metal_kernels.metal:29-44). */
int lunelette_cuda_rmsnorm(const float *gain, const float *x, size_t width, size_t count,
    float *out, void *stream);

/* Final RMSNorm + tied BF16 head over one hidden row: logits[rows]; *nonfinite
 * (device int) is OR-ed with 1 when a logit is NaN/Inf. cols % 8 == 0.
 * Replaces norm + project on the last row (src/metal_encode.m:204-210). */
int lunelette_cuda_head_bf16(const uint16_t *W, size_t rows, size_t cols, const float *x,
    const float *gain, float *logits, int *nonfinite, void *stream);

/* Causal GQA attention (32 query heads over 8 KV heads, head dim 128) of `count`
 * query rows at positions length..length+count-1 against KV layer `layer` of the
 * paged pool; out [count][4096]. part_acc (slots*128 floats) and part_ml
 * (slots*2 floats) are caller scratch, slots >= 32*count.
 * Replaces scores + attend (src/metal_kernels.metal:81-132). */
int lunelette_cuda_attention(const float *q, const float *kv_pool, const int *page_table,
    size_t num_pages, size_t layer, size_t length, size_t count, float *out, float *part_acc,
    float *part_ml, size_t slots, void *stream);

/* Same attention as lunelette_cuda_attention, for callers that cannot allocate
 * device memory (an engine that has already reserved the whole device for its
 * own pool, or a latency-critical loop where cudaMalloc/cudaFree would
 * synchronise the device). It allocates nothing: its partial results live in a
 * fixed array inside the library, 4096 slots (2,129,920 bytes) per GPU, held
 * until the process exits, so count may be at most 128; larger counts are
 * rejected with a message in error[0..capacity). The first call on a device
 * looks up that array's device address, so make it before any stream capture.
 * Every call shares the array: calls that overlap on the GPU (other streams,
 * other threads) race and must be serialised by the caller.
 * No counterpart in the reference (its Metal runtime owns all scratch). */
int lunelette_cuda_attention_noalloc(const float *q, const float *kv_pool, const int *page_table,
    size_t num_pages, size_t layer, size_t length, size_t count, float *out, void *stream,
    char *error, size_t capacity);

/* ---------------- batched decode over many sessions (one weight replica) */

/* One set of weights and a paged FP32 KV pool of pool_positions positions
 * (rounded up to pages of 64) shared by up to max_sessions independent
 * sessions of up to `context` (<= 4352) positions each; `block` (8..256)
 * bounds the tokens of one append and the sessions of one decode step. The
 * reference serves one sequence per context (src/metal_internal.h:29-50); this
 * is the multi-session engine the service's many users share. Returns NULL
 * with a diagnostic on failure. Single caller per batch context. */
typedef struct lunelette_cuda_batch lunelette_cuda_batch;
lunelette_cuda_batch *lunelette_cuda_batch_create(const char *path, size_t max_sessions, size_t context,
    size_t pool_positions, size_t block, char *error, size_t capacity);
void lunelette_cuda_batch_destroy(lunelette_cuda_batch *batch);
/* A new empty session (its id into *session); -1 when all are in use. */
int lunelette_cuda_batch_open(lunelette_cuda_batch *batch, int *session, char *error, size_t capacity);
/* Return the session's pages to the pool. */
int lunelette_cuda_batch_close(lunelette_cuda_batch *batch, int session);
/* Prefill or extend one session by count (1..block) tokens, as
 * lunelette_metal_prefill/append; *logits borrows the last token's 131072
 * host logits until the next call. */
int lunelette_cuda_batch_append(lunelette_cuda_batch *batch, int session, const int64_t *ids, size_t count,
    const float **logits, char *error, size_t capacity);
/* One greedy decode step for n (1..block) distinct non-empty sessions, token
 * ids[i] of session sessions[i] at its current length: the projections run
 * once for all n tokens (tcgen05 GEMMs), attention per token over its own
 * pages. next[i] receives the greedy id (strict '>', lowest id on ties); when
 * logits is not NULL it receives the n x 131072 logits. */
int lunelette_cuda_batch_decode(lunelette_cuda_batch *batch, const int *sessions, const int64_t *ids, size_t n,
    float *logits, int64_t *next, char *error, size_t capacity);
/* Positions held by an open session (0 otherwise), and free pool positions. */
/* Open a new session whose first `length` positions (1..the source's length)
 * are the source session's: its full pages are shared (a page returns to the
 * pool when its last session closes) and a partial last page is copied, so
 * either session may append afterwards without affecting the other. Replaces
 * re-prefilling a shared prefix; the reference reuses a prefix only within its
 * one sequence, by rewinding (src/metal_runtime.m:494-575). */
int lunelette_cuda_batch_fork(lunelette_cuda_batch *batch, int source, size_t length, int *session,
    char *error, size_t capacity);
size_t lunelette_cuda_batch_length(const lunelette_cuda_batch *batch, int session);
size_t lunelette_cuda_batch_free_positions(const lunelette_cuda_batch *batch);

/* KV prefix reuse across sequences: copies pages of the paged FP32 pool
 * [layer][page][K|V][8 heads][64 slots][128]. For i < pairs, every layer's
 * K and V of page src_pages[i] go to page dst_pages[i] (device int arrays);
 * the last pair copies only its first last_slots (1..64) positions. A sequence
 * forked from another's prefix shares the full pages through its page table
 * and copies only the partial last page (copy on write), or copies the whole
 * prefix. The reference keeps one sequence per context and restores a prefix
 * by rewinding its length (src/metal_runtime.m:494-575); this is the device
 * side of reusing that prefix in another sequence. */
int lunelette_cuda_kv_copy(float *kv_pool, size_t num_pages, size_t layers, const int *src_pages,
    const int *dst_pages, size_t pairs, size_t last_slots, void *stream);

/* ---------------- model-level test support */

/* Keep every layer's output rows (which 0..25) and the final-norm rows (26) of
 * the most recent call; host copy of count*3072 floats. Host-synchronous.
 * While enabled, calls run the per-projection kernels (not the persistent
 * decode kernel). Setting LUNELETTE_CUDA_TRACE=1 in the environment enables it
 * for every context created afterwards. */
int lunelette_cuda_trace(lunelette_metal *context, int enable);
int lunelette_cuda_trace_copy(lunelette_metal *context, int which, float *out, size_t floats);
/* Borrowed host rows of the most recent successful call while tracing: the
 * layer-25 output (normalized 0) or the final-norm rows (normalized 1), one row
 * per token of that call, valid until the next call on the context; NULL when
 * tracing is off or the sequence holds no published result. The reference's
 * test hook test_metal_snapshot (tests/metal_snapshot.m:5-8) returns the same
 * two buffers of its Metal runtime; tests/c_drivers/metal_snapshot_cuda.c
 * defines that hook on this function so tests/compare_metal.c links unchanged. */
const float *lunelette_cuda_snapshot(lunelette_metal *context, int normalized);
/* Device-resident greedy decode for throughput measurement: decode `first_token`
 * and then keep feeding each step's argmax (strict '>', lowest id on ties, as
 * src/generation.c:8-34) back on the GPU, `steps` steps in all, with no host
 * round trip between steps: one launch of the persistent decode kernel for all
 * steps, or (LUNELETTE_MEGA=0) one replay of a captured CUDA graph per step.
 * On success the sequence length grows by `steps`, tokens[0..steps) holds the
 * generated ids, *milliseconds the CUDA-event time of the call's device work
 * and *launches the kernel launches it made. Host logits are not refreshed, so
 * no endpoint is published (checkpoint_create needs another prefill/append/decode
 * first). */
int lunelette_cuda_decode_loop(lunelette_metal *context, int64_t first_token, size_t steps,
    int64_t *tokens, float *milliseconds, int *launches, char *error, size_t capacity);

/* Phase timing of the persistent decode kernel: while enabled, the first step of
 * each launch records %globaltimer (ns) at its start (entry 0) and as CTA 0
 * leaves each of its 79 grid barriers (entry 1 + k; per layer one after the o
 * projection, one after gate/up and one after down, then one after the greedy
 * pick). From entry 80, CTA b's marks m at 80 + m * ctas + b (ctas = the
 * device's SM count): per layer L at 13L + 0 qkv row staged, 1 qkv items done,
 * 2 q/k/v published, 3 attention published (CTAs that own one, else 0), 4 o row
 * staged, 5 o items done, 6 arrival at the o barrier, 7-9 the same three for
 * gate/up, 10-12 for down; mark 338 the arrival at the last barrier. Copy up
 * to 80 + 339 * ctas entries. */
int lunelette_cuda_timeline(lunelette_metal *context, int enable);
int lunelette_cuda_timeline_copy(lunelette_metal *context, unsigned long long *out, size_t entries);

/* Current sequence length (0 for NULL). */
size_t lunelette_cuda_length(const lunelette_metal *context);

/* The host YaRN table row the runtime uploads for `position` (128 cos, 128
 * sin, split-half duplicated); -1 for position >= 262144. Restates
 * lunelette_metal_yarn (src/metal_yarn.c:8-33). */
int lunelette_cuda_yarn(uint32_t position, float *cosine, float *sine);

/* Host-only admission of a checkpoint: the same name/dtype/shape/companion
 * validation and FP8 payload admission that create() applies for `strategy`,
 * without touching a GPU (src/metal_weights.c:51-231). */
int lunelette_cuda_validate_checkpoint(const char *path, lunelette_metal_strategy strategy,
    char *error, size_t capacity);

/* ---------------- synthetic checkpoint */

/* Write a seeded random-init checkpoint in the reference's tensor contract
 * (3.8 GB): FP8 linears N(0,0.02) with BF16 per-tensor scales, BF16 embedding,
 * unit norm gains. Host-only; deterministic for a seed. */
int lunelette_cuda_synth_checkpoint(const char *path, uint64_t seed, char *error,
    size_t capacity);
/* FP32 -> E4M3FN code, round-to-nearest-even, saturating at +-448. */
unsigned char lunelette_cuda_e4m3_encode(float value);

#ifdef __cplusplus
}
#endif

#endif
