/* Model tensor contract for the fixed Ministral-3-3B text decoder.
 *
 * Index order follows the reference's weight table (src/metal_weights.c:79-100,
 * include/model_facts.h:28-34): 0 = tied embedding/head, 1 = final norm, then
 * nine tensors per layer (input norm, q, k, v, o, post-attention norm, gate, up,
 * down). Validation and payload admission restate the reference's rules
 * (src/metal_weights.c:14-231) in this file's own code.
 */
#ifndef LUN_WEIGHTS_H
#define LUN_WEIGHTS_H

#include "st.h"

#define LUN_HIDDEN 3072
#define LUN_QUERY 4096
#define LUN_KV 1024
#define LUN_INNER 9216
#define LUN_LAYERS 26
#define LUN_VOCAB 131072
#define LUN_HEAD_DIM 128
#define LUN_QUERY_HEADS 32
#define LUN_KV_HEADS 8
#define LUN_BLOCK_WEIGHTS 9
#define LUN_WEIGHT_COUNT (2 + LUN_LAYERS * LUN_BLOCK_WEIGHTS)

typedef struct {
    const char *suffix;
    size_t rows, cols; /* cols == 0: a norm vector */
} lun_block_weight;
extern const lun_block_weight lun_block_weights[LUN_BLOCK_WEIGHTS];

typedef struct {
    lun_st file;
    struct {
        const lun_tensor *tensor;
        float scale; /* widened BF16 weight_scale_inv; 1 for BF16 tensors */
        size_t elements;
        /* FP8 tensors: their rank-0 BF16 companions weight_scale_inv and
         * activation_scale (NULL for BF16 tensors) */
        const lun_tensor *scale_tensor, *activation_tensor;
    } w[LUN_WEIGHT_COUNT];
} lun_weights;

/* Open, validate names/dtypes/shapes/companions, reject unexpected text tensors,
 * read and check both scalar companions of every FP8 tensor. */
int lun_weights_open(lun_weights *weights, const char *path, char *error, size_t capacity);
void lun_weights_close(lun_weights *weights);

/* Admission of FP8 payload codes for tensor `index`.
 * compact != 0: the scale must be a positive, FP32-normal, BF16-exact value and
 *   every code's decoded*scale must be finite and either exactly zero-coded or
 *   normal (src/metal_weights.c:188-200).
 * compact == 0: every decoded*scale must be finite (src/safetensors.c:537-542).
 * Builds the 256-entry table once per call of lun_weights_admission(). */
typedef struct {
    unsigned char allowed[256];
    int nan_only; /* the rejected codes are exactly the two NaN codes 0x7F and 0xFF */
} lun_admission;
int lun_weights_admission(const lun_weights *weights, size_t index, int compact,
    lun_admission *table, char *error, size_t capacity);
/* Scan codes[0..count) (which start at byte `offset` of the tensor). */
int lun_admit_codes(const lun_weights *weights, size_t index, const lun_admission *table,
    const unsigned char *codes, size_t count, uint64_t offset, float scale,
    char *error, size_t capacity);

/* YaRN cos/sin for one position (split-half duplicated, 128 entries each). */
int lun_yarn(uint32_t position, float cosine[128], float sine[128]);

#endif
