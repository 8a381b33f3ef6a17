/* Lunelette runtime contract, served by the B200 (sm_100a) backend in
 * lunelette_b200/liblunelette_cuda.so.
 *
 * This header declares the same 13 C entry points, enum values and struct
 * layouts as the reference's include/metal.h:11-120, so callers written against
 * that contract (src/generation.c via src/main.c:48-67, service/native.c,
 * tests/compare_native.c) link against this library unchanged. The names keep
 * the reference's "metal" prefix because they are the ABI; nothing here uses
 * Metal. No CUDA types cross this boundary.
 *
 * Each entry point replaces the Objective-C implementation at the cited
 * reference location (src/metal_runtime.m unless noted).
 *
 * Threading: one caller per context, including reset and destroy. A context is
 * bound to the CUDA device that was current when it was created and re-selects
 * that device on every call.
 */
#ifndef LUNELETTE_METAL_H
#define LUNELETTE_METAL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lunelette_metal lunelette_metal;
typedef struct lunelette_metal_checkpoint lunelette_metal_checkpoint;

/* Prefill engine selector. Both values run the same tensor-core path here; the
 * value is validated and kept only so that callers' option handling is intact. */
typedef enum {
    LUNELETTE_METAL_PREFILL_MPS = 0,
    LUNELETTE_METAL_PREFILL_CUSTOM = 1
} lunelette_metal_prefill_mode;

/* Weight residency strategy. All three run the one FP8 path on the B200; the
 * requested value is echoed by lunelette_metal_get_memory() because callers
 * (service/native.c:552-556, tests/compare_native.c:411) check the echo. */
typedef enum {
    LUNELETTE_METAL_RESIDENT_FP32 = 0,
    LUNELETTE_METAL_COMPACT_FP8_ARITHMETIC = 1,
    LUNELETTE_METAL_COMPACT_FP8_LOOKUP = 2
} lunelette_metal_strategy;

typedef struct {
    lunelette_metal_prefill_mode prefill;
    lunelette_metal_strategy strategy;
} lunelette_metal_options;

#define LUNELETTE_METAL_OPTIONS_DEFAULT \
    { LUNELETTE_METAL_PREFILL_MPS, LUNELETTE_METAL_COMPACT_FP8_ARITHMETIC }

/* Capacity profile: total KV positions C and largest single call B.
 * Accepted pairs: (256,256), (4352,256), (4352,128); NULL means (256,256). */
typedef struct {
    size_t context, block;
} lunelette_metal_limits;

/* Device bytes this context owns (not driver or process overhead). */
typedef struct {
    lunelette_metal_strategy strategy;
    uint64_t weight_bytes, conversion_stage_bytes, scratch_bytes, kv_bytes, total_bytes;
} lunelette_metal_memory;

/* Open one mixed FP8/BF16 model.safetensors, validate every text tensor's name,
 * dtype and shape and the FP8 payload admission rules before any device
 * allocation, upload, and allocate scratch and KV. NULL on failure with a
 * diagnostic in error[0..capacity) when given (NULL/0 is allowed).
 * Replaces lunelette_metal_create / _with_options / _create_configured
 * (src/metal_runtime.m:187-320). NULL options selects the product default
 * (LUNELETTE_METAL_OPTIONS_DEFAULT); invalid enum values and unsupported
 * limits fail before the file is opened. */
lunelette_metal *lunelette_metal_create(const char *path, char *error, size_t capacity);
lunelette_metal *lunelette_metal_create_with_options(const char *path,
    const lunelette_metal_options *options, char *error, size_t capacity);
lunelette_metal *lunelette_metal_create_configured(const char *path,
    const lunelette_metal_options *options, const lunelette_metal_limits *limits,
    char *error, size_t capacity);

/* Non-mutating queries (src/metal_runtime.m:577-585, 446-486). NULL arguments
 * return -1 and leave the output untouched; borrowed logits stay valid. */
int lunelette_metal_get_limits(const lunelette_metal *context, lunelette_metal_limits *limits);
int lunelette_metal_get_memory(const lunelette_metal *context, lunelette_metal_memory *memory);

/* Release everything the context owns; NULL is allowed (src/metal_runtime.m:322-331).
 * Destroy every checkpoint handle of this context first. */
void lunelette_metal_destroy(lunelette_metal *context);

/* Empty the sequence and revalidate it without device work or reload
 * (src/metal_runtime.m:333-347). Invalidates the active checkpoint. */
int lunelette_metal_reset(lunelette_metal *context, char *error, size_t capacity);

/* Run one block of token ids (src/metal_runtime.m:349-444, 488-492).
 *   prefill: sequence empty, 1 <= count <= B, count <= C
 *   append:  sequence non-empty, 1 <= count <= B, length + count <= C
 *   decode:  sequence non-empty, length < C
 * ids must lie in [0, 131072). On success *logits points at 131072 FP32 values in
 * host memory owned by the context, valid until the next mutating call on it
 * (get_limits/get_memory and checkpoint create/destroy do not end the borrow).
 * On failure *logits is NULL. Argument errors are rejected before any state or
 * device change; an execution, allocation or non-finite failure invalidates the
 * sequence (and its checkpoint) until reset. */
int lunelette_metal_prefill(lunelette_metal *context, const int64_t *ids, size_t count,
    const float **logits, char *error, size_t capacity);
int lunelette_metal_decode(lunelette_metal *context, int64_t token,
    const float **logits, char *error, size_t capacity);
int lunelette_metal_append(lunelette_metal *context, const int64_t *ids, size_t count,
    const float **logits, char *error, size_t capacity);

/* Checkpoints (src/metal_runtime.m:494-575): a handle holds a copy of the
 * finite endpoint logits (524288 host bytes) and the sequence length, not KV.
 * Only the newest handle of a context restores; restore rewinds the length and
 * republishes the saved logits with no device work (KV rows past the restored
 * length are masked by the length and overwritten by the next call). The caller
 * owns handles and destroys them before the context. */
int lunelette_metal_checkpoint_create(lunelette_metal *context,
    lunelette_metal_checkpoint **checkpoint, char *error, size_t capacity);
int lunelette_metal_checkpoint_restore(lunelette_metal *context,
    const lunelette_metal_checkpoint *checkpoint, const float **logits,
    char *error, size_t capacity);
void lunelette_metal_checkpoint_destroy(lunelette_metal_checkpoint *checkpoint);

#ifdef __cplusplus
}
#endif

#endif
