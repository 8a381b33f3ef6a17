/* TEST INFRASTRUCTURE ONLY — the CPU oracle for the Lunelette decoder hot path.
 *
 * Plain C restatement of the reference's Metal kernels (src/metal_kernels.metal)
 * and of its per-layer graph (src/metal_encode.m:124-215), in FP32 with FP32 KV,
 * exactly as the reference executes it. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load this library; the
 * product path (lunelette_b200/) never links or calls it.
 *
 * Pinning: FP8 decode is checked bit-for-bit against the reference's frozen
 * PyTorch table (tests/fp8_golden.h, all 256 codes); the YaRN table against the
 * reference's Transformers golden values (tests/rope_golden.h) and bit-for-bit
 * against the reference's own lunelette_metal_yarn compiled from its sources
 * (oracle/_ref). Kernel arithmetic follows the reference's analytic tests
 * (tests/test_metal.m:169-627, 956-997). Full-model outputs have no reference
 * capture (the Metal runtime cannot run here), so model-level parity rests on
 * this restatement.
 */
#ifndef LUNELETTE_ORACLE_H
#define LUNELETTE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define ORACLE_HIDDEN 3072
#define ORACLE_QUERY 4096
#define ORACLE_KV 1024
#define ORACLE_INNER 9216
#define ORACLE_LAYERS 26
#define ORACLE_VOCAB 131072
#define ORACLE_HEAD_DIM 128
#define ORACLE_QUERY_HEADS 32
#define ORACLE_KV_HEADS 8

/* ---- operator level (one function per reference kernel) ---- */
float oracle_fp8_decode(unsigned char code);
int oracle_yarn(uint32_t position, float cosine[128], float sine[128]);
void oracle_project(const float *weights, const float *input, float *output,
    size_t rows, size_t cols, size_t count);
void oracle_project_fp8(const unsigned char *packed, float scale, const float *input,
    float *output, size_t rows, size_t cols, size_t count);
void oracle_norm(const float *weights, const float *input, float *output,
    size_t width, size_t count);
void oracle_element(const float *first, const float *second, float *output,
    size_t n, int mode);
void oracle_rope(const float *input, const float *cosine, const float *sine,
    const uint32_t *positions, float *output, size_t width, size_t count, int query);
void oracle_attention(const float *query, const float *keys, const float *values,
    float *output, size_t count, size_t prefix, float *probabilities);
void oracle_set_threads(int threads);
int oracle_threads(void);
/* Precision study only (default 0,0 = FP32 as the reference): round stored KV
 * rows and/or projection inputs to 1 = BF16 or 2 = FP16 to measure drift. */
void oracle_set_rounding(int kv, int input);
void oracle_set_accumulation(int mode);

/* ---- model level ---- */
typedef struct oracle_model oracle_model;
oracle_model *oracle_open(const char *path, size_t context, char *error, size_t capacity);
void oracle_close(oracle_model *model);
void oracle_reset(oracle_model *model);
size_t oracle_length(const oracle_model *model);
int oracle_rewind(oracle_model *model, size_t length);
/* One prefill/append/decode call: count ids at positions length..length+count-1.
 * logits: 131072 FP32 for the last row. trace: NULL or [26][count][3072] (each
 * layer's output hidden state). final_norm: NULL or [count][3072]. */
int oracle_forward(oracle_model *model, const int64_t *ids, size_t count, float *logits,
    float *trace, float *final_norm, char *error, size_t capacity);

#endif
