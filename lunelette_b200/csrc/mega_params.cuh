// Parameters of the persistent decode kernel (decode_mega.cuh), shared with
// the host code that fills them (device.cu).
#pragma once
#include "common.cuh"

namespace lun {

// Grid barriers per decode step: two per layer (after o, once h is whole;
// after the FFN, once every act slice's down output is added into xfix) and
// one after the head and the pick. qkv -> attention goes through tagged words
// (the attention CTAs poll the q, k and v values themselves), attention -> o
// through a counter (kSyncAttn); gate/up -> down stays inside each CTA.
constexpr int kMegaBarriersPerStep = kLayers * 2 + 1;
// Timeline of the first step of a launch: [0] start, [1 + k] CTA 0 leaving
// barrier k, then from kMegaTimelineHead one entry per CTA b for each mark m at
// kMegaTimelineHead + m * gridDim.x + b. Marks per layer L, at 13L + :
//   0 qkv row staged, 1 qkv items done, 2 q/k/v stored (tagged),
//   3 attention published (CTAs that own a unit, else 0),
//   4 o row staged, 5 o items done, 6 arrival at the o barrier,
//   7 gate/up row staged, 8 gate/up items done, 9 act slice stored,
//   10 (unused), 11 down items done, 12 arrival at the FFN barrier;
// mark 13 * 26 is the arrival at the barrier after the pick.
constexpr int kMarksPerLayer = 13;
constexpr int kMegaMarksPerStep = kLayers * kMarksPerLayer + 1;
constexpr int kMegaTimelineHead = 1 + kMegaBarriersPerStep;

// Synchronisation words of one launch, each on its own 128-byte line, zero at
// launch and only ever increased (targets grow with the layers the launch ran):
//   kSyncBarrier        grid barrier arrivals (gridDim per barrier)
//   kSyncAttn           attention units whose output is stored (8 per layer, or 32 when
//                       each query head has its own unit)
//   kSyncTicket + kvh   attention ranges of KV head kvh finished
//   kSyncPick           CTAs done with the head (gridDim per step)
constexpr int kSyncStride = 32;
enum : int {
    kSyncBarrier = 0,
    kSyncAttn = 1,
    kSyncTicket = kSyncAttn + 1,
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
    float *x;                // the step's final residual stream (written before the head)
    float *attn;
    float *hbuf;             // [2][3072]: layer L's h (x + o) in hbuf[L & 1]
    long long *xfix;         // [2][3072]: layer L's output x in xfix[L & 1], 64-bit fixed point (2^-32):
                             // its o epilogue stores h, then every act slice adds its down rows
    unsigned long long *qkvt;  // the step's q (4096) and k, v (1024 each) of the current layer, tagged
    unsigned tag_base;         // tag of this launch's first layer (step s, layer L: tag_base + 26 s + L)
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
    unsigned l2_ahead_ffn;      // the same while the ring is filled with FFN (gate/up, down) items
    unsigned l2_hints;          // bit 0: ring copies mark their lines evict_first (read once per step);
                                // bit 1: L2 prefetches mark theirs evict_last (kept until the copy)
    unsigned attn_rows;         // range-mode attention with lanes = dims (row-coalesced K loads)
    unsigned kv_early;          // long contexts: prefetch layer L + 1's K/V rows into L2 during layer L's FFN
    unsigned long long *timeline;  // optional %globaltimer (ns) record, layout above
};

}  // namespace lun
