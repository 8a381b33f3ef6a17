// Persistent cooperative decode kernel: one CTA per SM runs whole batch-1
// decode steps (26 layers, final norm, tied head, greedy pick) of the
// reference's layer graph (src/metal_encode.m:124-215).
//
// Warp roles per CTA (256 threads):
//   producers (lanes 0-6 of warp 7, lane w serving consumer warp w): walk this
//     CTA's share of every weight matrix in the order the step consumes it and
//     copy it, 8-12 KB items at a time, into shared-memory slots with bulk async
//     copies (cp.async.bulk + mbarrier complete_tx). Weights never depend on
//     activations, so the producers run ahead across phases and grid barriers,
//     bounded by free slots; they also keep a short stretch of the stream
//     (p.l2_ahead bytes) prefetched into L2 while the layers run.
//   consumers (warps 0-6): per phase, wait at a grid barrier for the previous
//     phase's activations, stage the activation row as FP16 hi/lo MMA fragments
//     (and the epilogue's residual rows), then take items (8 rows x 1024 or
//     1536 columns of the tiled layout of gemv.cuh), run the tensor-core dot
//     products, leave 8 partial row sums per item in shared memory, and
//     finally add each tile's partials in a fixed order and run the fused
//     epilogue. Attention and the greedy pick run on consumers only.
// Item i of the CTA's stream goes to consumer warp i mod 7, which owns
// kSlotsPerWarp private slots and takes its items strictly in order, so every
// slot's full and empty barriers are waited on in phase order by one waiter.
// Phases per layer: qkv (norm + q/k/v + RoPE + KV store; the epilogue also
// writes q and the new k/v as 64-bit words tagged with the layer's tag),
// attention (one CTA per KV head and position range, started when the tagged
// q/k/v words it polls carry the current tag), o (+ residual; starts once the
// eight attention results are counted, ends at a grid barrier), gate/up
// (norm + SwiGLU), down (+ residual); then the head (final norm + tied BF16
// GEMV) with a per-CTA argmax whose last CTA picks the token.
//
// Every wait is bounded (kSpinLimit polls): a CTA that gives up sets *error and
// later waits return at once, so a failed launch ends and the host reports it.
#pragma once
#include <cuda.h>

#include "async.cuh"
#include "attention.cuh"
#include "gemv.cuh"
#include "mega_params.cuh"

namespace lun {

constexpr int kMegaConsumerWarps = 7;
constexpr int kMegaConsumers = kMegaConsumerWarps * 32;
constexpr int kMegaThreads = kMegaConsumers + 32;
constexpr int kSlotsPerWarp = 2;
constexpr int kRingSlots = kMegaConsumerWarps * kSlotsPerWarp;
constexpr int kSlotBytes = 12288;
constexpr int kFragBytes = (kInner / 64) * 256;          // hi/lo fragments of a 9216-column row
constexpr int kMegaMaxItems = 48;                         // FP8 items of one phase per CTA
constexpr int kMegaMaxTiles = 16;                         // tiles of one phase per CTA
constexpr int kMegaSmemBytes =
    kRingSlots * kSlotBytes + kFragBytes + kMegaMaxItems * 16 * 4 + 2 * kRingSlots * 8;
constexpr unsigned kSpinLimit = 1u << 22;
constexpr int kPhasesPerStep = kLayers * 4 + 1;  // 4 FP8 phases per layer, then the head
constexpr int kAttnMaxRanges = 18;               // position ranges per KV head (8 x 18 <= CTAs)
constexpr int kHeadModeMax = 112;                // positions up to which each query head gets a CTA
constexpr int kQStride = 36;                     // floats per staged query quarter (32 + pad)
constexpr int kCmbStride = 132;                  // floats per (warp, head) attention partial
// FFN in act slices: slice s (64 SwiGLU features, CTA s) takes the 16 gate/up
// tiles that produce it, then the slice's 64 columns of down for all 3072 rows
// as 16 items of 24 tile pieces (8 rows x 64 columns, 512 bytes each): items
// as large as a slot, so the ring holds most of the slice's down before act
// is ready (smaller items measured slower: fewer bytes in flight per warp).
constexpr int kFfnSlices = kInner / 64;
constexpr int kSliceTiles = kGateUpRows / kTileRows / kFfnSlices;
constexpr int kDownItemTiles = 24;
constexpr int kDownItems = kHidden / kTileRows / kDownItemTiles;
constexpr int kActOffset = (kHidden / 64) * 256;  // act slice and down row sums after the gate/up fragments
static_assert(kSliceTiles * kTileRows * kFfnSlices == kGateUpRows && kDownItemTiles * 512 <= kSlotBytes &&
                  kDownItems * kDownItemTiles * kTileRows == kHidden,
              "FFN slices cover gate/up and down, a down item fits a slot");
static_assert(kActOffset + (64 + kHidden) * 4 <= kFragBytes, "act slice and down row sums fit the fragment area");
static_assert((16 * kQStride + 2 * kHeadDim + kMegaConsumerWarps * 4 * kCmbStride) * 4 <= kFragBytes,
              "attention staging fits the fragment area");

// ---- small PTX wrappers (the mbarrier and bulk-copy ones are in async.cuh) ----
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kMegaConsumers) : "memory"); }

// Bounded wait on an mbarrier phase; false when the launch already failed or
// this wait gave up (then *error is set).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, int *error)
{
    unsigned spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (++spins > kSpinLimit) {
            atomicExch(error, 1);
            return false;
        }
        if ((spins & 255u) == 0 && *(volatile int *)error) return false;
    }
    return true;
}

// ---- the stream: which bytes each CTA needs, in consumption order -----------
enum { kPhQKV, kPhO, kPhGateUp, kPhDown, kPhHead };

// This CTA's share of one phase: `items` consecutive items of `item_bytes`
// starting at src. FP8 phases: whole 8-row tiles from tile `first`, each
// split into K-chunks; head: 2-row items of the BF16 embedding from row `first`;
// down (tma = layer + 1): item i is the box {0, first, 24 i, layer} of the
// down tensor map (act slice `first`, tiles 24 i .. 24 i + 23).
struct PhaseSpan {
    const uint8_t *src;
    int items;
    int item_bytes;
    int first;
    int tma;
};

__device__ __forceinline__ void cta_range(int units, int &u0, int &u1)
{
    u0 = (int)(((long long)units * blockIdx.x) / gridDim.x);
    u1 = (int)(((long long)units * (blockIdx.x + 1)) / gridDim.x);
}

// blocks per item: qkv, o, gate/up, down
__host__ __device__ constexpr int item_blocks(int ph) { return ph == kPhO ? 8 : 12; }

__device__ __forceinline__ PhaseSpan phase_span(const MegaParams &p, int layer, int ph)
{
    constexpr size_t lq = (size_t)kQKVRows * kHidden, lo = (size_t)kHidden * kQuery,
                     lg = (size_t)kGateUpRows * kHidden, ld = (size_t)kHidden * kInner;
    if (ph == kPhHead) {
        int g0, g1;
        cta_range(kVocab / 4, g0, g1);  // 4-row groups, two items each
        return {reinterpret_cast<const uint8_t *>(p.embedding) + (size_t)g0 * 4 * kHidden * 2, 2 * (g1 - g0),
                2 * kHidden * 2, 4 * g0};
    }
    const uint8_t *base = p.w8 + (size_t)layer * (lq + lo + lg + ld);
    if (ph == kPhGateUp || ph == kPhDown) {
        const int s = blockIdx.x;  // act slice of this CTA; CTAs past the last slice idle in the FFN
        if (s >= kFfnSlices) return {base, 0, kSlotBytes, 0, 0};
        if (ph == kPhDown) return {nullptr, kDownItems, kDownItemTiles * 512, s, layer + 1};
        constexpr int nb = kHidden / kBlockCols, cb = item_blocks(kPhGateUp);
        return {base + lq + lo + (size_t)s * kSliceTiles * nb * kBlockBytes, kSliceTiles * (nb / cb),
                cb * kBlockBytes, s * kSliceTiles, 0};
    }
    const uint8_t *m;
    int tiles, nb;
    switch (ph) {
    case kPhQKV: m = base; tiles = kQKVRows / kTileRows; nb = kHidden / kBlockCols; break;
    default: m = base + lq; tiles = kHidden / kTileRows; nb = kQuery / kBlockCols; break;
    }
    const int cb = item_blocks(ph);
    int t0, t1;
    cta_range(tiles, t0, t1);
    return {m + (size_t)t0 * nb * kBlockBytes, (t1 - t0) * (nb / cb), cb * kBlockBytes, t0};
}

// Phase k of the launch's stream (steps repeat the same weights).
__device__ __forceinline__ PhaseSpan stream_span(const MegaParams &p, int k)
{
    k %= kPhasesPerStep;
    if (k == kLayers * 4) return phase_span(p, 0, kPhHead);
    return phase_span(p, k >> 2, k & 3);
}

struct Ring {
    uint8_t *slots;
    uint64_t *full, *empty;
};

// Slot of the k-th item taken by consumer warp w.
__device__ __forceinline__ unsigned slot_of(int w, unsigned k) { return w * kSlotsPerWarp + k % kSlotsPerWarp; }

// First item of a phase that belongs to this consumer warp, given the number
// of items the CTA's stream held before the phase.
__device__ __forceinline__ int first_item(unsigned seq0)
{
    const int warp = threadIdx.x >> 5;
    return (warp + kMegaConsumerWarps - (int)(seq0 % kMegaConsumerWarps)) % kMegaConsumerWarps;
}

// Position of one consumer warp's next item in the launch's stream: phase k,
// item i of that phase, seq0 items in the stream before phase k.
struct WarpCursor {
    int k, i;
    unsigned seq0;
    PhaseSpan sp;
};

// Move c to warp w's first item at or after c.i (item i of the stream belongs to
// warp (seq0 + i) mod 7); false past the launch's last phase.
__device__ __forceinline__ bool cursor_settle(const MegaParams &p, WarpCursor &c, int w, int total)
{
    while (c.i >= c.sp.items) {
        c.seq0 += (unsigned)c.sp.items;
        if (++c.k >= total) return false;
        c.sp = stream_span(p, c.k);
        c.i = (w + kMegaConsumerWarps - (int)(c.seq0 % kMegaConsumerWarps)) % kMegaConsumerWarps;
    }
    return true;
}

// Producer lane w (one per consumer warp): every item of warp w in stream
// order, each as one bulk copy into the warp's next slot once the warp released
// it. The seven lanes share one warp, so none of them may block it: they run
// one convergent loop in which each lane probes its next slot without waiting
// (mbarrier test_wait) and issues when it is free, so a slow consumer warp
// holds back only its own stream. Each lane also keeps its next items
// (p.l2_ahead / 7 bytes) prefetched into L2 while the layers run; the head
// reads nothing ahead. Down items are tensor copies through down_map (24
// pieces of 512 bytes, one per tile, gathered into one slot). A lane that sees
// no free slot for kSpinLimit probes sets *error and stops.
__device__ __forceinline__ void produce(const MegaParams &p, const Ring &r, int w, const void *down_map)
{
    constexpr unsigned kLanes = (1u << kMegaConsumerWarps) - 1;
    const int total = p.steps * kPhasesPerStep;
    WarpCursor rc = {0, w, 0u, stream_span(p, 0)}, pc = rc;
    bool more = cursor_settle(p, rc, w, total), pf_more = cursor_settle(p, pc, w, total);
    const unsigned budget = p.l2_ahead / kMegaConsumerWarps;
    const unsigned budget_ffn = p.l2_ahead_ffn / kMegaConsumerWarps;
    const bool hint_ring = p.l2_hints & 1u, hint_ahead = p.l2_hints & 2u;
    const uint64_t first_out = l2_policy_evict_first(), keep = l2_policy_evict_last();
    unsigned long long ring_bytes = 0, pf_bytes = 0;
    unsigned u = 0, idle = 0;
    while (__any_sync(kLanes, more)) {
        bool issued = false;
        if (more) {
            // the lookahead while the ring feeds the FFN (the layer's longest
            // stretch of pure weight streaming) may differ from the one while it
            // feeds qkv and o, whose phases wait on other CTAs
            const int kk = rc.k % kPhasesPerStep;
            const unsigned ahead = kk == kLayers * 4 ? 0u : ((kk & 3) >= kPhGateUp ? budget_ffn : budget);
            while (pf_more && pf_bytes < ring_bytes + ahead) {
                const unsigned n = (unsigned)pc.sp.item_bytes;
                if (pf_bytes >= ring_bytes) {  // not yet in the ring
                    if (pc.sp.tma) {
                        if (hint_ahead)
                            tma_prefetch_4d_hint(down_map, 0, pc.sp.first, pc.i * kDownItemTiles, pc.sp.tma - 1, keep);
                        else
                            tma_prefetch_4d(down_map, 0, pc.sp.first, pc.i * kDownItemTiles, pc.sp.tma - 1);
                    } else if (hint_ahead) {
                        l2_prefetch_hint(pc.sp.src + (size_t)pc.i * n, n, keep);
                    } else {
                        l2_prefetch(pc.sp.src + (size_t)pc.i * n, n);
                    }
                }
                pf_bytes += n;
                pc.i += kMegaConsumerWarps;
                pf_more = cursor_settle(p, pc, w, total);
            }
            const unsigned slot = slot_of(w, u), use = u / kSlotsPerWarp;
            if (!use || mbar_test_wait(&r.empty[slot], (use - 1) & 1)) {
                const unsigned n = (unsigned)rc.sp.item_bytes;
                mbar_expect_tx(&r.full[slot], n);
                uint8_t *dst = r.slots + (size_t)slot * kSlotBytes;
                if (rc.sp.tma) {
                    if (hint_ring)
                        tma_load_4d_hint(dst, down_map, 0, rc.sp.first, rc.i * kDownItemTiles, rc.sp.tma - 1,
                                         &r.full[slot], first_out);
                    else
                        tma_load_4d(dst, down_map, 0, rc.sp.first, rc.i * kDownItemTiles, rc.sp.tma - 1,
                                    &r.full[slot]);
                } else if (hint_ring) {
                    bulk_g2s_hint(dst, rc.sp.src + (size_t)rc.i * n, n, &r.full[slot], first_out);
                } else {
                    bulk_g2s(dst, rc.sp.src + (size_t)rc.i * n, n, &r.full[slot]);
                }
                ring_bytes += n;
                rc.i += kMegaConsumerWarps;
                more = cursor_settle(p, rc, w, total);
                u++;
                idle = 0;
                issued = true;
            } else if (++idle > kSpinLimit) {
                atomicExch(p.error, 1);
                more = false;
            } else if ((idle & 255u) == 0 && *(volatile int *)p.error) {
                more = false;
            }
        }
        // no slot was free: back off briefly instead of taking the issue slots
        // of the consumer warp that shares this scheduler
        if (!__any_sync(kLanes, issued)) __nanosleep(64);
    }
}

// ---- synchronisation --------------------------------------------------------
__device__ __forceinline__ unsigned *sync_word(const MegaParams &p, int index)
{
    return p.sync + (size_t)index * kSyncStride;
}

// Bounded wait of one thread until *word >= target (acquire).
__device__ __forceinline__ void thread_wait(const unsigned *word, unsigned target, int *error)
{
    unsigned spins = 0;
    while (ld_acquire_u32(word) < target) {
        if (++spins > kSpinLimit) {
            atomicExch(error, 1);
            return;
        }
        if ((spins & 255u) == 0 && *(volatile int *)error) return;
    }
}

__device__ __forceinline__ void record_mark(const MegaParams &p, bool rec, int mark)
{
    if (rec) p.timeline[kMegaTimelineHead + (size_t)mark * gridDim.x + blockIdx.x] = globaltimer_ns();
}

// Publish the CTA's global writes and add n to *word. One thread, after the
// consumers synchronised (bar.sync): the release add orders every write that
// happened before it in the CTA, so a reader that acquires the new count sees them.
__device__ __forceinline__ void signal_word(unsigned *word, unsigned n)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(word), "r"(n) : "memory");
}

// Grid barrier `target` (1, 2, ...) of this launch among all CTAs' consumers;
// with rec, this CTA's arrival goes to `mark` and CTA 0's exit to entry target.
__device__ __forceinline__ void grid_sync(const MegaParams &p, unsigned target, bool rec, int mark)
{
    consumers_sync();
    if (threadIdx.x == 0) {
        record_mark(p, rec, mark);
        if (!*(volatile int *)p.error) {
            // barrier k is passed once the arrival count reaches k * gridDim.x;
            // release add and acquire polls order the CTAs' writes around it
            unsigned *word = sync_word(p, kSyncBarrier);
            signal_word(word, 1u);
            thread_wait(word, target * gridDim.x, p.error);
        }
        if (rec && blockIdx.x == 0) p.timeline[target] = globaltimer_ns();
    }
    consumers_sync();
}

// ---- consumer helpers -------------------------------------------------------
// ---- tagged words (store_tagged) --------------------------------------------
__device__ __forceinline__ ulonglong2 ld_cg_u64x2(const unsigned long long *p)
{
    ulonglong2 v;
    asm volatile("ld.global.cg.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}

// Four tagged words at src -> v; true when all carry `want`.
__device__ __forceinline__ bool load_tagged4(const unsigned long long *src, unsigned want, float4 &v)
{
    const ulonglong2 a = ld_cg_u64x2(src), b = ld_cg_u64x2(src + 2);
    v = make_float4(__uint_as_float((unsigned)a.x), __uint_as_float((unsigned)a.y), __uint_as_float((unsigned)b.x),
                    __uint_as_float((unsigned)b.y));
    return (unsigned)(a.x >> 32) == want && (unsigned)(a.y >> 32) == want && (unsigned)(b.x >> 32) == want &&
           (unsigned)(b.y >> 32) == want;
}

// Poll four tagged words until they carry `want` (bounded).
__device__ __forceinline__ float4 poll_tagged4(const unsigned long long *src, unsigned want, int *error)
{
    float4 v;
    for (unsigned spins = 0; !load_tagged4(src, want, v);)
        if (++spins > kSpinLimit || ((spins & 255u) == 0 && *(volatile int *)error)) {
            atomicExch(error, 1);
            break;
        }
    return v;
}

__device__ __forceinline__ float consumers_sum(float v, float *red)
{
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    consumers_sync();
    if (lane == 0) red[warp] = v;
    consumers_sync();
    float t = lane < kMegaConsumerWarps ? red[lane] : 0.0f;
    return warp_sum(t);
}

// 64-bit fixed point with 32 fraction bits: the last layer's output x is summed
// in it (integer additions, so the sum does not depend on their order).
__device__ __forceinline__ float fixed_to_float(long long v) { return (float)v * 0x1p-32f; }
__device__ __forceinline__ long long float_to_fixed(float v) { return __float2ll_rn(v * 0x1p32f); }

// Rows [row0, row0 + n) of the layer input x -> shared memory, for an
// epilogue; the loads overlap the fragment staging that follows. x is the
// embedding row (emb) or the fixed-point sum xfix that other CTAs wrote.
__device__ __forceinline__ void stage_x_rows(float *dst, const long long *xfix, const uint16_t *emb, int row0, int n)
{
    for (int i = threadIdx.x; i < n; i += kMegaConsumers)
        dst[i] = emb ? bf16_lo((uint32_t)emb[row0 + i]) : fixed_to_float(__ldcg(&xfix[row0 + i]));
}

// Activation row -> hi/lo FP16 B fragments (lanes 0-7 of every half block, the
// layout of gemv_stage with one token), optionally RMS-normalised, in one pass:
// every consumer thread holds its float4s in registers while the sum of squares
// and the magnitude bound are reduced. src is another CTA's output (read through
// L2; or src64, the same in 64-bit fixed point) or, with emb, the BF16
// embedding row. Returns 2^-e, the inverse scale.
template <int K>
__device__ __forceinline__ float stage_frag(uint32_t *frag, const float *src, const long long *src64,
                                            const uint16_t *emb, const float *gain, float *red)
{
    constexpr int kF4 = K / 4;
    constexpr int kPer = (kF4 + kMegaConsumers - 1) / kMegaConsumers;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float4 *gain4 = reinterpret_cast<const float4 *>(gain);
    // the row and the gain in one round of loads
    float4 v[kPer], g[kPer];
#pragma unroll
    for (int u = 0; u < kPer; u++) {
        const int idx = threadIdx.x + u * kMegaConsumers;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        g[u] = make_float4(1.f, 1.f, 1.f, 1.f);
        if (idx < kF4) {
            if (gain) g[u] = __ldg(gain4 + idx);
            if (emb) {
                const uint2 e = *reinterpret_cast<const uint2 *>(emb + 4 * idx);
                v[u] = make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
            } else if (src64) {
                const longlong2 a = __ldcg(reinterpret_cast<const longlong2 *>(src64) + 2 * idx);
                const longlong2 b = __ldcg(reinterpret_cast<const longlong2 *>(src64) + 2 * idx + 1);
                v[u] = make_float4(fixed_to_float(a.x), fixed_to_float(a.y), fixed_to_float(b.x), fixed_to_float(b.y));
            } else {
                v[u] = __ldcg(reinterpret_cast<const float4 *>(src) + idx);
            }
        }
    }
    float ss = 0.0f, mx = 0.0f;
#pragma unroll
    for (int u = 0; u < kPer; u++) {
        const int idx = threadIdx.x + u * kMegaConsumers;
        if (idx < kF4) {
            const float4 x = v[u];
            ss += x.x * x.x;
            ss += x.y * x.y;
            ss += x.z * x.z;
            ss += x.w * x.w;
            const float4 gg = g[u];
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(gg.x * x.x), fabsf(gg.y * x.y)), fmaxf(fabsf(gg.z * x.z), fabsf(gg.w * x.w))));
        }
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if (lane == 0) {
        red[warp * 2] = ss;
        red[warp * 2 + 1] = mx;
    }
    consumers_sync();
    float tss = 0.0f, tmx = 0.0f;
#pragma unroll
    for (int w = 0; w < kMegaConsumerWarps; w++) {
        tss += red[w * 2];
        tmx = fmaxf(tmx, red[w * 2 + 1]);
    }
    const float rs = gain ? rsqrtf(tss / (float)K + kNormEps) : 1.0f;
    const int e = frag_exponent(tmx * rs * 1.0001f);
    const float sc = exp2i(e);
#pragma unroll
    for (int u = 0; u < kPer; u++) {
        const int idx = threadIdx.x + u * kMegaConsumers;
        if (idx < kF4) {
            float4 x = v[u];
            if (gain) {
                const float4 gg = g[u];
                x.x = gg.x * (x.x * rs);
                x.y = gg.y * (x.y * rs);
                x.z = gg.z * (x.z * rs);
                x.w = gg.w * (x.w * rs);
            }
            uint32_t hi, lo;
            split_hilo(x.x * sc, x.y * sc, hi, lo);
            frag_store_pair(frag, 8, 4 * idx, 0, hi);
            frag_store_pair(frag, 8, 4 * idx, 1, lo);
            split_hilo(x.z * sc, x.w * sc, hi, lo);
            frag_store_pair(frag, 8, 4 * idx + 2, 0, hi);
            frag_store_pair(frag, 8, 4 * idx + 2, 1, lo);
        }
    }
    consumers_sync();
    return exp2i(-e);
}

// One FP8 phase's items on this warp: CB blocks per item, NB blocks per row.
// Leaves the item's 8 partial row sums (hi + lo columns of both block halves)
// in partial[item][8]. B column n of lane (n, t4) is half (n >> 1) & 1, hi/lo n & 1
// of the token: lanes 0-15 load fragments, the rest stay zero.
template <int CB, int NB>
__device__ __forceinline__ void consume_fp8(const Ring &r, const PhaseSpan &sp, unsigned seq0, unsigned &taken,
                                            const uint4 *frag, float *partial, int *error)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kChunks = NB / CB;
    for (int i = first_item(seq0); i < sp.items; i += kMegaConsumerWarps) {
        const unsigned k = taken++;
        const unsigned slot = slot_of(warp, k), use = k / kSlotsPerWarp;
        mbar_wait(&r.full[slot], use & 1, error);
        const uint8_t *s = r.slots + (size_t)slot * kSlotBytes;
        __builtin_assume(__isShared(s));
        const uint4 *xf = frag + (size_t)(i % kChunks) * CB * 32;  // two 64-column pieces per block
        __builtin_assume(__isShared(xf));
        float c[4][4] = {};  // per k16 step j of a block: four independent accumulation chains
#pragma unroll 4
        for (int b = 0; b < CB; b++) {
            const uint4 wa = *reinterpret_cast<const uint4 *>(s + b * kBlockBytes + lane * 16);
            const uint4 wb = *reinterpret_cast<const uint4 *>(s + b * kBlockBytes + 512 + lane * 16);
            uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
            if (lane < 16) {
                const int piece = 2 * b + (lane >> 3);
                x0 = xf[(piece * 2) * 8 + (lane & 7)];
                x1 = xf[(piece * 2 + 1) * 8 + (lane & 7)];
            }
            mma_block4(c, wa, wb, x0, x1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&r.empty[slot]);
        // lane (g, t4): t4 = 0 holds half 0 of row g (A rows g), t4 = 1 half 1 (A rows g + 8)
        float v = (lane & 1) ? (c[0][2] + c[0][3]) + (c[1][2] + c[1][3]) + ((c[2][2] + c[2][3]) + (c[3][2] + c[3][3]))
                             : (c[0][0] + c[0][1]) + (c[1][0] + c[1][1]) + ((c[2][0] + c[2][1]) + (c[3][0] + c[3][1]));
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        if ((lane & 3) == 0) partial[i * 8 + (lane >> 2)] = v;
    }
}

// Sum each tile's chunk partials in chunk order and run the phase epilogue on
// its four row groups (groups spread over the consumer warps).
template <int EPI>
__device__ __forceinline__ void fp8_epilogue(const GemvParams &gp, const PhaseSpan &sp, int chunks,
                                             const float *partial, float inv_scale)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = (sp.items / chunks) * 2;
    for (int gi = warp; gi < groups; gi += kMegaConsumerWarps) {
        const int tl = gi >> 1, gq = gi & 1;
        float acc[4][1];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float s = 0.0f;
            for (int c = 0; c < chunks; c++) s += partial[(tl * chunks + c) * 8 + gq * 4 + i];
            acc[i][0] = s * inv_scale;
        }
        gemv_epilogue<1, EPI>(gp, (sp.first + tl) * 2 + gq, lane, acc);
    }
}

// Down items of this CTA's act slice (64 features, act_s in shared memory):
// each item holds kDownItemTiles tile pieces (8 rows x the slice's 64 columns),
// taken in pairs as the two 8-row halves of one m16n8k16 A tile, so every MMA
// row is a weight row and the B operand's columns 0 and 1 are the slice's hi
// and lo parts (same fragments for every pair; lanes 8-31 zero). The item's
// row sums (rows 8 kDownItemTiles i ..), scaled by 2^-e and the tensor's scale,
// go to rows_s[3072]; down_reduce then adds them into xfix.
__device__ __forceinline__ void consume_down(const Ring &r, const PhaseSpan &sp, unsigned seq0, unsigned &taken,
                                             const float *act_s, float *rows_s, float scale, int *error)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (first_item(seq0) >= sp.items) return;
    const float a0 = act_s[lane], a1 = act_s[lane + 32];
    const int e = frag_exponent(warp_max(fmaxf(fabsf(a0), fabsf(a1))) * 1.0001f);
    const float sc = exp2i(e), out_scale = scale * exp2i(-e);
    const int n = lane >> 2, t4 = lane & 3;
    uint32_t b[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    if (n < 2) {
        // k-step j: b0 = columns 16j + 2 t4 (+1), b1 = columns 16j + 2 t4 + 8 (+9)
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const int c = 16 * (q >> 1) + 2 * t4 + 8 * (q & 1);
            uint32_t hi, lo;
            split_hilo(act_s[c] * sc, act_s[c + 1] * sc, hi, lo);
            b[q] = n == 0 ? hi : lo;
        }
    }
    const uint4 x0 = make_uint4(b[0], b[1], b[2], b[3]), x1 = make_uint4(b[4], b[5], b[6], b[7]);
    for (int i = first_item(seq0); i < sp.items; i += kMegaConsumerWarps) {
        float *rows = rows_s + (size_t)i * kDownItemTiles * kTileRows;
        const unsigned k = taken++;
        const unsigned slot = slot_of(warp, k), use = k / kSlotsPerWarp;
        mbar_wait(&r.full[slot], use & 1, error);
        const uint8_t *s = r.slots + (size_t)slot * kSlotBytes;
        __builtin_assume(__isShared(s));
        // four pairs (64 rows) at a time: row 16 q + j of a group ends in lane
        // (16 q + j) % 32, register q / 2, moved there by shuffles, and the group
        // is stored once (a shared-memory store after every pair would hold the
        // next pairs' loads behind it)
#pragma unroll 1
        for (int q0 = 0; q0 < kDownItemTiles / 2; q0 += 4) {
            float res[2];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint4 wa = *reinterpret_cast<const uint4 *>(s + (q0 + q) * 1024 + lane * 16);
                const uint4 wb = *reinterpret_cast<const uint4 *>(s + (q0 + q) * 1024 + 512 + lane * 16);
                float c[4][4] = {};
                mma_block4(c, wa, wb, x0, x1);
                // lane (g, 0): row g of the pair's first tile (c0 hi + c1 lo) and of its second (c2 + c3)
                const float r0 =
                    (c[0][0] + c[0][1]) + (c[1][0] + c[1][1]) + ((c[2][0] + c[2][1]) + (c[3][0] + c[3][1]));
                const float r1 =
                    (c[0][2] + c[0][3]) + (c[1][2] + c[1][3]) + ((c[2][2] + c[2][3]) + (c[3][2] + c[3][3]));
                const int src = 4 * (lane & 7);
                const float v0 = __shfl_sync(0xffffffffu, r0, src), v1 = __shfl_sync(0xffffffffu, r1, src);
                if ((lane >> 4) == (q & 1)) res[q >> 1] = (lane & 8) ? v1 : v0;
            }
            rows[q0 * 16 + lane] = res[0] * out_scale;
            rows[q0 * 16 + 32 + lane] = res[1] * out_scale;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&r.empty[slot]);
    }
}

// The CTA's 3072 down row sums (rows_s) added into xfix, the layer output x
// in fixed point, with 64-bit integer reductions. A row sum the fixed point
// cannot hold (non-finite, or too large for 145 terms to stay in range) sets
// kFlagFixedRange, and the host reruns the step on the FP32 path.
__device__ __forceinline__ void down_reduce(const float *rows_s, long long *xfix, int *flag)
{
    bool out_of_range = false;
    for (int v = threadIdx.x; v < kHidden; v += kMegaConsumers) {
        const float r = rows_s[v];
        out_of_range |= !(fabsf(r) < kFixedTermLimit);
        asm volatile("red.global.add.u64 [%0], %1;" ::"l"(xfix + v), "l"(float_to_fixed(r)) : "memory");
    }
    if (__any_sync(0xffffffffu, out_of_range) && (threadIdx.x & 31) == 0) atomicOr(flag, kFlagFixedRange);
}

__device__ __forceinline__ void arg_better(float &v, int &i, float v2, int i2)
{
    if (v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

// Head phase: final-normed row staged with 8-column chunks; items of 2 BF16
// rows; logits, non-finite flag and per-warp best.
__device__ __forceinline__ void consume_head(const Ring &r, const PhaseSpan &sp, unsigned seq0, unsigned &taken,
                                             const MegaParams &p, const float4 *xs, float &best, int &best_i,
                                             int *error)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NQ = kHidden >> 3;  // 8-column chunks of a row
    int bad = 0;
    for (int i = first_item(seq0); i < sp.items; i += kMegaConsumerWarps) {
        const unsigned k = taken++;
        const unsigned slot = slot_of(warp, k), use = k / kSlotsPerWarp;
        mbar_wait(&r.full[slot], use & 1, error);
        const uint8_t *s = r.slots + (size_t)slot * kSlotBytes;
        float acc[2] = {0.f, 0.f};
#pragma unroll 4
        for (int qq = lane; qq < NQ; qq += 32) {
            const float4 x0 = xs[qq], x1 = xs[NQ + qq];
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const uint4 w = *reinterpret_cast<const uint4 *>(s + rr * kHidden * 2 + qq * 16);
                float a = acc[rr];
                a = fmaf(bf16_lo(w.x), x0.x, a);
                a = fmaf(bf16_hi(w.x), x0.y, a);
                a = fmaf(bf16_lo(w.y), x0.z, a);
                a = fmaf(bf16_hi(w.y), x0.w, a);
                a = fmaf(bf16_lo(w.z), x1.x, a);
                a = fmaf(bf16_hi(w.z), x1.y, a);
                a = fmaf(bf16_lo(w.w), x1.z, a);
                a = fmaf(bf16_hi(w.w), x1.w, a);
                acc[rr] = a;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&r.empty[slot]);
        const int row = sp.first + 2 * i;
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const float v = warp_sum(acc[rr]);
            if (lane == rr) {
                p.logits[row + rr] = v;
                bad |= !isfinite(v);
            }
            arg_better(best, best_i, v, row + rr);
        }
    }
    if (bad) atomicOr(p.nonfinite, kFlagNonfinite);
}

// Position ranges per KV head for `total` positions: at most 256 positions
// per range, at most one range per CTA.
__device__ __forceinline__ int attention_ranges(int total)
{
    int r = (total + 255) / 256;
    const int cap = min(kAttnMaxRanges, (int)gridDim.x / kKVHeads);
    return r < 1 ? 1 : (r > cap ? cap : r);
}

// The attention unit (KV head, range) of this CTA, or -1: unit u runs on CTA
// floor(u * gridDim / units), so units land on distinct CTAs spread over the grid.
__device__ __forceinline__ int attention_unit(int units)
{
    const long long G = gridDim.x, b = blockIdx.x;
    const int u = (int)((b * units + G - 1) / G);
    return (u < units && (int)((long long)u * G / units) == (int)b) ? u : -1;
}

// L2 prefetch of the K (kind 0) or V (kind 1) rows [begin, min(end, length))
// of an attention unit: per page one contiguous run of this KV head's slots.
__device__ __forceinline__ void attention_prefetch(const MegaParams &p, int layer, int length, int kvh, int range,
                                                   int ranges, int kind)
{
    int per = (length + 1 + ranges - 1) / ranges;
    per = (per + 7) & ~7;
    const int begin = range * per, end = min(begin + per, length);
    for (int p0 = begin; p0 < end;) {
        const int slot = p0 % kPage, n = min(kPage - slot, end - p0);
        const int page = p.page_table[p0 / kPage];
        l2_prefetch(p.kv + kv_offset(layer, p.num_pages, page, kind, kvh, slot), (unsigned)n * kHeadDim * 4);
        p0 += n;
    }
}

// K (lanes = position x dim quarter) and V (lanes = dims) of one 8-position
// sub-tile into registers; positions past `end` read as zero.
__device__ __forceinline__ float4 ld_cg_f4(const float4 *p)
{
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ void attention_load(const MegaParams &p, int layer, int kvh, int p0, int end, float4 (&kk)[8],
                                               float4 (&vv)[8])
{
    const int lane = threadIdx.x & 31, pp = lane >> 2, qd = lane & 3;
    const int n = min(8, end - p0);
    const int page = p.page_table[p0 / kPage];
    const float *kb = p.kv + kv_offset(layer, p.num_pages, page, 0, kvh, p0 % kPage);
    const float *vb = p.kv + kv_offset(layer, p.num_pages, page, 1, kvh, p0 % kPage);
    const float4 *krow = reinterpret_cast<const float4 *>(kb + pp * kHeadDim + qd * 32);
#pragma unroll
    for (int c = 0; c < 8; c++) kk[c] = pp < n ? ld_cg_f4(krow + c) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int t = 0; t < 8; t++)
        vv[t] = t < n ? ld_cg_f4(reinterpret_cast<const float4 *>(vb + t * kHeadDim) + lane)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
}

// K and V of one 8-position sub-tile with lanes = dims (lane l holds dims
// 4 l .. 4 l + 3 of each position): every load instruction reads one whole
// 512-byte row; positions past `end` read as zero.
__device__ __forceinline__ void attention_load_rows(const MegaParams &p, int layer, int kvh, int p0, int end,
                                                    float4 (&kk)[8], float4 (&vv)[8])
{
    const int lane = threadIdx.x & 31;
    const int n = min(8, end - p0);
    const int page = p.page_table[p0 / kPage];
    const float *kb = p.kv + kv_offset(layer, p.num_pages, page, 0, kvh, p0 % kPage);
    const float *vb = p.kv + kv_offset(layer, p.num_pages, page, 1, kvh, p0 % kPage);
#pragma unroll
    for (int t = 0; t < 8; t++) {
        kk[t] = t < n ? ld_cg_f4(reinterpret_cast<const float4 *>(kb + t * kHeadDim) + lane)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
        vv[t] = t < n ? ld_cg_f4(reinterpret_cast<const float4 *>(vb + t * kHeadDim) + lane)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

__device__ __forceinline__ void attention_patch_rows(int p0, int cur, const float *kcur, const float *vcur,
                                                     float4 (&kk)[8], float4 (&vv)[8])
{
    if (cur < p0 || cur >= p0 + 8) return;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < 8; t++)
        if (p0 + t == cur) {
            kk[t] = reinterpret_cast<const float4 *>(kcur)[lane];
            vv[t] = reinterpret_cast<const float4 *>(vcur)[lane];
        }
}

__device__ __forceinline__ float pick4(const float (&v)[4], int i)
{
    return i == 0 ? v[0] : i == 1 ? v[1] : i == 2 ? v[2] : v[3];
}

// The step's own position `cur` inside the sub-tile at p0: its k/v rows come
// from shared memory (staged from the tagged words), not from the pool.
__device__ __forceinline__ void attention_patch(int p0, int cur, const float *kcur, const float *vcur, float4 (&kk)[8],
                                                float4 (&vv)[8])
{
    if (cur < p0 || cur >= p0 + 8) return;
    const int lane = threadIdx.x & 31, pp = lane >> 2, qd = lane & 3;
    if (p0 + pp == cur)
#pragma unroll
        for (int c = 0; c < 8; c++) kk[c] = reinterpret_cast<const float4 *>(kcur + qd * 32)[c];
#pragma unroll
    for (int t = 0; t < 8; t++)
        if (p0 + t == cur) vv[t] = reinterpret_cast<const float4 *>(vcur)[lane];
}

// Merge the ranges of KV head kvh in range order (warps 0-3, one query head each).
__device__ __forceinline__ void merge_ranges(const MegaParams &p, int kvh, int ranges)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp >= 4) return;
    // last range of this KV head: merge all ranges in order
    const int hq = warp;
    float ms = -INFINITY, ls = 0.0f;
    if (lane < ranges) {
        const size_t at = ((size_t)(kvh * ranges + lane) * 4 + hq) * 2;
        ms = __ldcg(&p.part_ml[at]);
        ls = __ldcg(&p.part_ml[at + 1]);
    }
    const float M = warp_max(ls > 0.0f ? ms : -INFINITY);
    const float w = ls > 0.0f ? expf(ms - M) : 0.0f;
    const float L = warp_sum(w * ls);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s2 = 0; s2 < ranges; s2++) {
        const float ws = __shfl_sync(0xffffffffu, w, s2);
        const float4 v = __ldcg(
            reinterpret_cast<const float4 *>(p.part_acc + ((size_t)(kvh * ranges + s2) * 4 + hq) * kHeadDim) + lane);
        acc.x = fmaf(ws, v.x, acc.x);
        acc.y = fmaf(ws, v.y, acc.y);
        acc.z = fmaf(ws, v.z, acc.z);
        acc.w = fmaf(ws, v.w, acc.w);
    }
    const float inv = 1.0f / L;
    reinterpret_cast<float4 *>(p.attn + (size_t)(kvh * 4 + hq) * kHeadDim)[lane] =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

// One attention unit on the whole CTA: the four query heads of KV head kvh
// over one position range. Each warp takes sub-tiles of 8 positions (its first
// sub-tile's K/V loads are issued before the query rows are staged, so one
// memory round trip precedes the arithmetic), scores them with lanes =
// position x dim quarter, accumulates P.V with lanes = dims and keeps an online
// softmax per query head; the warps' (m, l, o) are merged in warp order in
// shared memory. With one range the result goes straight to attn; with several,
// each range leaves (m, l, unnormalised o) in global memory and the CTA that
// finishes a KV head's last range (ticket counter, `tickets` before this layer)
// merges them in range order. Replaces scores + attend
// (src/metal_kernels.metal:81-132).
template <int HQ>
__device__ __forceinline__ void cta_attention(const MegaParams &p, int layer, int length, int kvh, int h0, int range,
                                              int ranges, unsigned epoch, unsigned tag, unsigned tickets, float *qs,
                                              float *cmb, int *flag, bool rec)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, pp = lane >> 2, qd = lane & 3;
    const int total = length + 1;
    int per = (total + ranges - 1) / ranges;
    per = (per + 7) & ~7;
    const int begin = range * per, end = min(begin + per, total);
    float *kcur = qs + 16 * kQStride, *vcur = kcur + kHeadDim;
    // K/V of earlier steps' positions are in memory already: loaded first
    int p0 = begin + 8 * warp;
    float4 kk[8], vv[8];
    const bool rows = HQ == 4 && p.attn_rows;
    if (p0 < end) {
        if (rows) attention_load_rows(p, layer, kvh, p0, end, kk, vv);
        else attention_load(p, layer, kvh, p0, end, kk, vv);
    }
    // this layer's q rows of the four query heads and the position's k, v rows,
    // polled from the tagged words the qkv epilogues write (224 threads, 4 words each)
    {
        const unsigned long long *src;
        float *dst;
        if (threadIdx.x < 32 * HQ) {
            const int hq = threadIdx.x >> 5, d4 = threadIdx.x & 31;
            src = p.qkvt + (size_t)(kvh * 4 + h0 + hq) * kHeadDim + 4 * d4;
            dst = qs + (hq * 4 + (d4 >> 3)) * kQStride + (d4 & 7) * 4;
        } else if (threadIdx.x >= 128 && threadIdx.x < 160) {
            src = p.qkvt + kQuery + kvh * kHeadDim + 4 * (threadIdx.x - 128);
            dst = kcur + 4 * (threadIdx.x - 128);
        } else if (threadIdx.x >= 160 && threadIdx.x < 192) {
            src = p.qkvt + kQuery + kKV + kvh * kHeadDim + 4 * (threadIdx.x - 160);
            dst = vcur + 4 * (threadIdx.x - 160);
        } else {
            src = nullptr;
            dst = nullptr;
        }
        if (src) *reinterpret_cast<float4 *>(dst) = poll_tagged4(src, tag, p.error);
    }
    consumers_sync();
    if (rows) attention_patch_rows(p0, length, kcur, vcur, kk, vv);
    else attention_patch(p0, length, kcur, vcur, kk, vv);
    float m_run[HQ], l_run[HQ];
    float4 o[HQ];
#pragma unroll
    for (int hq = 0; hq < HQ; hq++) {
        m_run[hq] = -INFINITY;
        l_run[hq] = 0.0f;
        o[hq] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (rows) {
        // lanes = dims: this lane's 4 dims of the four query heads
        float4 qv[4];
#pragma unroll
        for (int hq = 0; hq < 4; hq++)
            qv[hq] = *reinterpret_cast<const float4 *>(qs + (hq * 4 + (lane >> 3)) * kQStride + (lane & 7) * 4);
        const int my_h = lane & 3, my_t = lane >> 2;
        for (; p0 < end; p0 += 8 * kMegaConsumerWarps) {
            if (p0 != begin + 8 * warp) {
                attention_load_rows(p, layer, kvh, p0, end, kk, vv);
                attention_patch_rows(p0, length, kcur, vcur, kk, vv);
            }
            // partial dots over this lane's 4 dims, index i = 4 t + hq
            float part[32];
#pragma unroll
            for (int t = 0; t < 8; t++)
#pragma unroll
                for (int hq = 0; hq < 4; hq++) {
                    float d = qv[hq].x * kk[t].x;
                    d = fmaf(qv[hq].y, kk[t].y, d);
                    d = fmaf(qv[hq].z, kk[t].z, d);
                    d = fmaf(qv[hq].w, kk[t].w, d);
                    part[4 * t + hq] = d;
                }
            // reduce-scatter over the warp: lane l ends with the full dot of index l
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) {
                const bool upper = (lane & off) != 0;
#pragma unroll
                for (int k = 0; k < off; k++) {
                    const float send = upper ? part[k] : part[k + off];
                    const float keep = upper ? part[k + off] : part[k];
                    part[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            const bool valid = my_t < min(8, end - p0);
            const float sc = valid ? part[0] * kScoreScale : -INFINITY;
            float tmax = sc;
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
            float m_new[4], corr[4];
#pragma unroll
            for (int hq = 0; hq < 4; hq++) {
                m_new[hq] = fmaxf(m_run[hq], __shfl_sync(0xffffffffu, tmax, hq));
                corr[hq] = m_run[hq] == -INFINITY ? 0.0f : expf(m_run[hq] - m_new[hq]);
            }
            const float pr = valid ? expf(sc - pick4(m_new, my_h)) : 0.0f;
            float ps = pr;
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            ps += __shfl_xor_sync(0xffffffffu, ps, 8);
            ps += __shfl_xor_sync(0xffffffffu, ps, 16);
#pragma unroll
            for (int hq = 0; hq < 4; hq++) {
                l_run[hq] = l_run[hq] * corr[hq] + __shfl_sync(0xffffffffu, ps, hq);
                m_run[hq] = m_new[hq];
                o[hq].x *= corr[hq];
                o[hq].y *= corr[hq];
                o[hq].z *= corr[hq];
                o[hq].w *= corr[hq];
            }
#pragma unroll
            for (int t = 0; t < 8; t++)
#pragma unroll
                for (int hq = 0; hq < 4; hq++) {
                    const float pt = __shfl_sync(0xffffffffu, pr, 4 * t + hq);
                    o[hq].x = fmaf(pt, vv[t].x, o[hq].x);
                    o[hq].y = fmaf(pt, vv[t].y, o[hq].y);
                    o[hq].z = fmaf(pt, vv[t].z, o[hq].z);
                    o[hq].w = fmaf(pt, vv[t].w, o[hq].w);
                }
        }
    } else
    for (; p0 < end; p0 += 8 * kMegaConsumerWarps) {
        if (p0 != begin + 8 * warp) {
            attention_load(p, layer, kvh, p0, end, kk, vv);
            attention_patch(p0, length, kcur, vcur, kk, vv);
        }
        const bool valid = pp < min(8, end - p0);
        float pr[HQ];
#pragma unroll
        for (int hq = 0; hq < HQ; hq++) {
            const float4 *qv = reinterpret_cast<const float4 *>(qs + (hq * 4 + qd) * kQStride);
            float d = 0.0f;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const float4 q4 = qv[c];
                d = fmaf(q4.x, kk[c].x, d);
                d = fmaf(q4.y, kk[c].y, d);
                d = fmaf(q4.z, kk[c].z, d);
                d = fmaf(q4.w, kk[c].w, d);
            }
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            const float s = valid ? d * kScoreScale : -INFINITY;
            float tmax = s;
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
            const float m_new = fmaxf(m_run[hq], tmax);
            const float corr = m_run[hq] == -INFINITY ? 0.0f : expf(m_run[hq] - m_new);
            pr[hq] = valid ? expf(s - m_new) : 0.0f;
            float ps = pr[hq];
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            ps += __shfl_xor_sync(0xffffffffu, ps, 8);
            ps += __shfl_xor_sync(0xffffffffu, ps, 16);
            l_run[hq] = l_run[hq] * corr + ps;
            m_run[hq] = m_new;
            o[hq].x *= corr;
            o[hq].y *= corr;
            o[hq].z *= corr;
            o[hq].w *= corr;
        }
#pragma unroll
        for (int t = 0; t < 8; t++) {
#pragma unroll
            for (int hq = 0; hq < HQ; hq++) {
                const float pt = __shfl_sync(0xffffffffu, pr[hq], t * 4);
                o[hq].x = fmaf(pt, vv[t].x, o[hq].x);
                o[hq].y = fmaf(pt, vv[t].y, o[hq].y);
                o[hq].z = fmaf(pt, vv[t].z, o[hq].z);
                o[hq].w = fmaf(pt, vv[t].w, o[hq].w);
            }
        }
    }
    // the warps' partials -> shared memory: [warp][head] o[128], m, l
#pragma unroll
    for (int hq = 0; hq < HQ; hq++) {
        float *slot = cmb + (warp * 4 + hq) * kCmbStride;
        reinterpret_cast<float4 *>(slot)[lane] = o[hq];
        if (lane == 0) {
            slot[128] = m_run[hq];
            slot[129] = l_run[hq];
        }
    }
    consumers_sync();
    if (warp < HQ) {
        const int hq = warp;
        float M = -INFINITY;
        for (int w = 0; w < kMegaConsumerWarps; w++) {
            const float *slot = cmb + (w * 4 + hq) * kCmbStride;
            if (slot[129] > 0.0f) M = fmaxf(M, slot[128]);
        }
        float L = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < kMegaConsumerWarps; w++) {
            const float *slot = cmb + (w * 4 + hq) * kCmbStride;
            if (!(slot[129] > 0.0f)) continue;
            const float wt = expf(slot[128] - M);
            const float4 v = reinterpret_cast<const float4 *>(slot)[lane];
            L = fmaf(wt, slot[129], L);
            acc.x = fmaf(wt, v.x, acc.x);
            acc.y = fmaf(wt, v.y, acc.y);
            acc.z = fmaf(wt, v.z, acc.z);
            acc.w = fmaf(wt, v.w, acc.w);
        }
        if (ranges == 1) {
            const float inv = 1.0f / L;
            reinterpret_cast<float4 *>(p.attn + (size_t)(kvh * 4 + h0 + hq) * kHeadDim)[lane] =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        } else {
            const size_t at = (size_t)(kvh * ranges + range) * 4 + hq;
            reinterpret_cast<float4 *>(p.part_acc + at * kHeadDim)[lane] = acc;
            if (lane == 0) {
                p.part_ml[at * 2] = M;
                p.part_ml[at * 2 + 1] = L;
            }
        }
    }
    consumers_sync();
    if (ranges == 1) {
        if (threadIdx.x == 0) {
            signal_word(sync_word(p, kSyncAttn), 1);
            record_mark(p, rec, layer * kMarksPerLayer + 3);
        }
        return;
    }
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned old = atomicAdd(sync_word(p, kSyncTicket + kvh), 1u);
        *flag = old == tickets + (unsigned)ranges - 1;
        __threadfence();
    }
    consumers_sync();
    if (!*flag) return;
    merge_ranges(p, kvh, ranges);
    consumers_sync();
    if (threadIdx.x == 0) {
        signal_word(sync_word(p, kSyncAttn), 1);
        record_mark(p, rec, layer * kMarksPerLayer + 3);
    }
}

__global__ void __launch_bounds__(kMegaThreads, 1)
    decode_mega_kernel(MegaParams p, const __grid_constant__ CUtensorMap down_map)
{
    extern __shared__ __align__(128) uint8_t mega_smem[];
    __shared__ float red[32];
    __shared__ float best_v[kMegaConsumerWarps];
    __shared__ int best_i[kMegaConsumerWarps];
    __shared__ int last_cta, flag;
    __shared__ float rope_s[2 * kHeadDim];       // cos | sin of the step's position
    __shared__ float res_s[kMegaMaxTiles * 16];  // residual rows of this CTA's tiles
    Ring ring;
    ring.slots = mega_smem;
    uint32_t *frag = reinterpret_cast<uint32_t *>(mega_smem + (size_t)kRingSlots * kSlotBytes);
    float *partial = reinterpret_cast<float *>(mega_smem + (size_t)kRingSlots * kSlotBytes + kFragBytes);
    ring.full = reinterpret_cast<uint64_t *>(partial + kMegaMaxItems * 16);
    ring.empty = ring.full + kRingSlots;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRingSlots; s++) {
            mbar_init(&ring.full[s], 1);
            mbar_init(&ring.empty[s], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (p.timeline && blockIdx.x == 0) p.timeline[0] = globaltimer_ns();
    }
    __syncthreads();

    if (threadIdx.x >= kMegaConsumers) {
        const int lane = threadIdx.x & 31;
        if (lane < kMegaConsumerWarps) produce(p, ring, lane, &down_map);
        return;
    }

    const uint4 *frag4 = reinterpret_cast<const uint4 *>(frag);
    float *xs_head = reinterpret_cast<float *>(frag);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned barrier = 0, taken = 0, seq = 0, tickets = 0, attn_target = 0;
    for (int s = 0; s < p.steps; s++) {
        const bool rec = p.timeline && s == 0;
        const int length = __ldcg(&p.step->length);
        const int id = __ldcg(&p.step->ids[0]);
        const uint16_t *emb_row = p.embedding + (size_t)id * kHidden;
        for (int i = threadIdx.x; i < 2 * kHeadDim; i += kMegaConsumers)
            rope_s[i] = i < kHeadDim ? p.rope_cos[(size_t)length * kHeadDim + i]
                                     : p.rope_sin[(size_t)length * kHeadDim + i - kHeadDim];
        // attention units: short contexts give each query head its own CTA
        // (32 units); longer ones split each KV head's positions into ranges
        const bool head_mode = length + 1 <= kHeadModeMax && (int)gridDim.x >= kQueryHeads;
        const int ranges = head_mode ? 1 : attention_ranges(length + 1);
        const int unit = attention_unit(head_mode ? kQueryHeads : kKVHeads * ranges);
        const int akvh = unit < 0 ? 0 : (head_mode ? unit / 4 : unit / ranges);
        const int ah0 = head_mode ? unit % 4 : 0, arange = head_mode ? 0 : unit - akvh * ranges;
        const unsigned attn_signals = head_mode ? kQueryHeads : kKVHeads;
        for (int layer = 0; layer < kLayers; layer++) {
            const unsigned epoch = (unsigned)(s * kLayers + layer) + 1;  // layers run by the launch, this one included
            const float *sc = p.scales + layer * 7;
            GemvParams gp;
            memset(&gp, 0, sizeof gp);
            gp.kv = p.kv;
            gp.page_table = p.page_table;
            gp.num_pages = p.num_pages;
            gp.layer = layer;
            gp.rope_row = rope_s;
            gp.length = length;
            // qkv: input norm, RoPE, KV store
            PhaseSpan sp = phase_span(p, layer, kPhQKV);
            gp.rows = kQKVRows;
            gp.cols = kHidden;
            gp.scale[0] = sc[0];
            gp.scale[1] = sc[1];
            gp.scale[2] = sc[2];
            gp.bound[0] = kQuery;
            gp.bound[1] = kQuery + kKV;
            gp.qkv_tagged = p.qkvt;
            gp.ytag = p.tag_base + epoch - 1;
            const int mk = layer * kMarksPerLayer;
            // the layer input x: the embedding row, else the last layer's xfix
            // (its h, stored by its o epilogue, plus every act slice's down rows)
            const int cur = (layer & 1) * kHidden, prev = kHidden - cur;  // hbuf / xfix halves
            // the attention unit's K/V rows of earlier steps do not depend on
            // this layer's qkv: start them towards L2 now
            if (unit >= 0 && threadIdx.x < 2) attention_prefetch(p, layer, length, akvh, arange, ranges, threadIdx.x);
            float inv = stage_frag<kHidden>(frag, nullptr, p.xfix + prev, layer == 0 ? emb_row : nullptr,
                                            p.norms + (size_t)(2 * layer) * kHidden, red);
            if (threadIdx.x == 0) record_mark(p, rec, mk);
            consume_fp8<item_blocks(kPhQKV), kHidden / kBlockCols>(ring, sp, seq, taken, frag4, partial, p.error);
            seq += sp.items;
            consumers_sync();
            if (threadIdx.x == 0) record_mark(p, rec, mk + 1);
            fp8_epilogue<kEpiQKV>(gp, sp, kHidden / kBlockCols / item_blocks(kPhQKV), partial, inv);
            gp.qkv_tagged = nullptr;
            if (rec) {
                consumers_sync();
                if (threadIdx.x == 0) record_mark(p, rec, mk + 2);
            }
            if (unit >= 0) {
                float *qs = reinterpret_cast<float *>(frag);
                if (head_mode)
                    cta_attention<1>(p, layer, length, akvh, ah0, 0, 1, epoch, gp.ytag, tickets, qs,
                                     qs + 16 * kQStride + 2 * kHeadDim, &flag, rec);
                else
                    cta_attention<4>(p, layer, length, akvh, 0, arange, ranges, epoch, gp.ytag, tickets, qs,
                                     qs + 16 * kQStride + 2 * kHeadDim, &flag, rec);
                consumers_sync();
            }
            if (ranges > 1) tickets += (unsigned)ranges;
            attn_target += attn_signals;
            // o + residual (x)
            sp = phase_span(p, layer, kPhO);
            gp.rows = kHidden;
            gp.cols = kQuery;
            gp.scale[0] = gp.scale[1] = gp.scale[2] = sc[3];
            gp.bound[0] = gp.bound[1] = 1 << 30;
            gp.res_shared = res_s;
            gp.res_base = sp.first * kTileRows;
            // h = x + o, as a float for the FFN's norm and as the starting
            // value of this layer's xfix (read only after the FFN barrier)
            gp.y = p.hbuf + cur;
            gp.y_fixed = p.xfix + cur;
            gp.range_flag = p.nonfinite;
            gp.y_stride = kHidden;
            stage_x_rows(res_s, p.xfix + prev, layer == 0 ? emb_row : nullptr, gp.res_base,
                         sp.items / (kQuery / kBlockCols / item_blocks(kPhO)) * kTileRows);
            // every KV head's attention output stored
            if (threadIdx.x == 0) thread_wait(sync_word(p, kSyncAttn), attn_target, p.error);
            consumers_sync();
            inv = stage_frag<kQuery>(frag, p.attn, nullptr, nullptr, nullptr, red);
            if (threadIdx.x == 0) record_mark(p, rec, mk + 4);
            consume_fp8<item_blocks(kPhO), kQuery / kBlockCols>(ring, sp, seq, taken, frag4, partial, p.error);
            seq += sp.items;
            consumers_sync();
            if (threadIdx.x == 0) record_mark(p, rec, mk + 5);
            fp8_epilogue<kEpiResidual>(gp, sp, kQuery / kBlockCols / item_blocks(kPhO), partial, inv);
            grid_sync(p, ++barrier, rec, mk + 6);
            // long contexts: the next layer's K/V rows of this CTA's attention
            // unit start towards L2 while the FFN streams its weights, so that
            // the next attention reads L2 instead of waiting on HBM
            if (p.kv_early && !head_mode && unit >= 0 && threadIdx.x < 2 && layer + 1 < kLayers)
                attention_prefetch(p, layer + 1, length, akvh, arange, ranges, threadIdx.x);
            // FFN of act slice s = blockIdx.x: post norm, the slice's 16 gate/up
            // tiles and SwiGLU into shared memory (act never leaves the CTA), then
            // the slice's 64 columns of down for every row, added into xfix;
            // the next layer reads x from xfix after one barrier
            sp = phase_span(p, layer, kPhGateUp);
            gp.rows = kGateUpRows;
            gp.cols = kHidden;
            gp.scale[0] = sc[4];
            gp.scale[1] = sc[5];
            gp.res_shared = nullptr;
            gp.y_fixed = nullptr;
            // features 64 s .. 64 s + 63 land in act_s[0 .. 63]
            float *act_s = reinterpret_cast<float *>(mega_smem + (size_t)kRingSlots * kSlotBytes + kActOffset);
            gp.y = act_s;
            gp.y_base = blockIdx.x * 64;
            gp.y_stride = kInner;
            inv = stage_frag<kHidden>(frag, p.hbuf + cur, nullptr, nullptr, p.norms + (size_t)(2 * layer + 1) * kHidden,
                                      red);
            if (threadIdx.x == 0) record_mark(p, rec, mk + 7);
            consume_fp8<item_blocks(kPhGateUp), kHidden / kBlockCols>(ring, sp, seq, taken, frag4, partial, p.error);
            seq += sp.items;
            consumers_sync();
            if (threadIdx.x == 0) record_mark(p, rec, mk + 8);
            fp8_epilogue<kEpiSwiGLU>(gp, sp, kHidden / kBlockCols / item_blocks(kPhGateUp), partial, inv);
            consumers_sync();
            if (threadIdx.x == 0) record_mark(p, rec, mk + 9);
            sp = phase_span(p, layer, kPhDown);
            consume_down(ring, sp, seq, taken, act_s, act_s + 64, sc[6], p.error);
            seq += sp.items;
            consumers_sync();
            if (sp.items) down_reduce(act_s + 64, p.xfix + cur, p.nonfinite);
            if (threadIdx.x == 0) record_mark(p, rec, mk + 11);
            grid_sync(p, ++barrier, rec, mk + 12);
        }
        // final norm + tied head, 8-column staging; the last layer's x from xfix
        // (CTA 0 also stores it, the step's final residual stream)
        {
            const long long *xl = p.xfix + (size_t)((kLayers - 1) & 1) * kHidden;
            float ss = 0.0f;
            for (int c = threadIdx.x; c < kHidden; c += kMegaConsumers) {
                const float v = fixed_to_float(__ldcg(&xl[c]));
                ss += v * v;
            }
            ss = consumers_sum(ss, red);
            const float rs = rsqrtf(ss / (float)kHidden + kNormEps);
            const int NQ = kHidden >> 3;
            for (int c = threadIdx.x; c < kHidden; c += kMegaConsumers) {
                const float v = fixed_to_float(__ldcg(&xl[c]));
                if (blockIdx.x == 0) p.x[c] = v;
                xs_head[((size_t)((c >> 2) & 1) * NQ + (c >> 3)) * 4 + (c & 3)] = p.final_norm[c] * (v * rs);
            }
            consumers_sync();
        }
        float best = -INFINITY;
        int bi = 0x7fffffff;
        const PhaseSpan hs = phase_span(p, 0, kPhHead);
        consume_head(ring, hs, seq, taken, p, reinterpret_cast<const float4 *>(xs_head), best, bi, p.error);
        seq += hs.items;
        if (lane == 0) {
            best_v[warp] = best;
            best_i[warp] = bi;
        }
        consumers_sync();
        if (threadIdx.x == 0) {
            float v = best_v[0];
            int i = best_i[0];
            for (int w = 1; w < kMegaConsumerWarps; w++) arg_better(v, i, best_v[w], best_i[w]);
            p.arg_val[blockIdx.x] = v;
            p.arg_idx[blockIdx.x] = i;
            __threadfence();
            last_cta = atomicAdd(sync_word(p, kSyncPick), 1u) == gridDim.x * (unsigned)(s + 1) - 1;
        }
        consumers_sync();
        if (last_cta && warp == 0) {
            // the last CTA to finish the head picks the token (strict '>', lowest id)
            __threadfence();
            float v = -INFINITY;
            int i = 0x7fffffff;
            for (int b = lane; b < (int)gridDim.x; b += 32)
                arg_better(v, i, __ldcg(&p.arg_val[b]), __ldcg(&p.arg_idx[b]));
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                float v2 = __shfl_xor_sync(0xffffffffu, v, o);
                int i2 = __shfl_xor_sync(0xffffffffu, i, o);
                arg_better(v, i, v2, i2);
            }
            if (lane == 0) {
                const int next = (i < 0 || i >= kVocab) ? 0 : i;
                const int generated = __ldcg(&p.step->generated);
                p.tokens[generated] = next;
                p.step->generated = generated + 1;
                p.step->ids[0] = next;
                p.step->length = length + 1;
            }
        }
        grid_sync(p, ++barrier, rec, kLayers * kMarksPerLayer);
    }
}

}  // namespace lun
