// Parameters of the persistent decode kernel (decode_mega.cuh), shared with
// the host code that fills them (device.cu).
#pragma once
#include "common.cuh"

namespace lun {

constexpr int kMegaBarriersPerStep = kLayers * 5 + 2;
constexpr int kMegaTimelineEntries = 1 + kMegaBarriersPerStep;

struct MegaParams {
    const uint8_t *w8;       // [26][qkv | o | gate/up | down]
    const float *scales;     // [26][7]: q k v o gate up down
    const uint16_t *embedding;
    const float *norms;      // [26][2][3072]
    const float *final_norm;
    float *kv;
    const int *page_table;
    int num_pages;
    const float *rope_cos, *rope_sin;
    StepParams *step;        // length and ids[0] advance on the device each step
    float *x, *h, *q, *attn, *act;
    float *part_acc, *part_ml;  // [32 heads][splits][128] and [..][2]
    unsigned *attn_count;       // [8] self-resetting arrival counters
    int split_len, splits;
    float *logits;
    int *nonfinite;
    float *arg_val;
    int *arg_idx;               // [gridDim.x] per-CTA argmax partials
    int *tokens;                // generated ids
    unsigned *barrier;          // [0] arrivals, [1] generation; zero at launch
    int *error;
    int steps;
    // optional: CTA 0 records %globaltimer (ns) at kernel start and after every
    // grid barrier of the first step ([1 + barriers per step] entries)
    unsigned long long *timeline;
    int prefetch;  // 0 disables the next-matrix L2 prefetch (measurement only)
};

}  // namespace lun
