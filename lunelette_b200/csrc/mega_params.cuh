// Parameters of the persistent decode kernel (decode_mega.cuh), shared with
// the host code that fills them (device.cu).
#pragma once
#include "common.cuh"

namespace lun {

// grid barriers per decode step: 5 per layer, one after the head and the pick
constexpr int kMegaBarriersPerStep = kLayers * 5 + 1;
// Timeline of the first step of a launch: [0] start, [1 + k] CTA 0 leaving
// barrier k (k = 0..130), then from kMegaTimelineHead every CTA b's arrival at
// barrier k in entry kMegaTimelineHead + k * gridDim.x + b.
constexpr int kMegaTimelineHead = 1 + kMegaBarriersPerStep;

// Synchronisation words of one launch, each on its own 128-byte line, zero at
// launch and only ever increased:
//   kSyncBarrier        grid barrier arrivals (gridDim per barrier)
//   kSyncTicket + kvh   attention ranges of KV head kvh finished
//   kSyncPick           CTAs done with the head (gridDim per step)
constexpr int kSyncStride = 32;
enum : int {
    kSyncBarrier = 0,
    kSyncTicket = 1,
    kSyncPick = kSyncTicket + kKVHeads,
    kSyncWords = kSyncPick + 1,
};

struct MegaParams {
    const uint8_t *w8;       // [26][qkv | o | gate/up | down], tiled (gemv.cuh)
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
    float *part_acc, *part_ml;  // [8 KV heads][ranges][4 query heads][128] and [..][2]
    float *logits;
    int *nonfinite;
    float *arg_val;
    int *arg_idx;               // [gridDim.x] per-CTA argmax partials
    int *tokens;                // generated ids
    unsigned *sync;             // kSyncWords * kSyncStride words, zero at launch
    int *error;
    int steps;
    unsigned l2_ahead;          // bytes of a CTA's weight stream kept prefetched into L2 ahead of its ring
    unsigned long long *timeline;  // optional %globaltimer (ns) record, layout above
};

}  // namespace lun
