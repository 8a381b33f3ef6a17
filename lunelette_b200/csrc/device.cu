// CUDA layer of the B200 backend: device allocations, weight upload and the
// per-call launch sequence that replaces the reference's command-buffer encoder
// (src/metal_encode.m:124-215) and execute() commit/wait (src/metal_runtime.m:349-432).
#include "device.h"
#include "kernels.h"
#include "mega_params.cuh"

#include <new>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

using namespace lun;

namespace {

constexpr size_t kLayerQKV = (size_t)kQKVRows * kHidden;            // 18,874,368
constexpr size_t kLayerO = (size_t)kHidden * kQuery;                // 12,582,912
constexpr size_t kLayerGateUp = (size_t)kGateUpRows * kHidden;      // 56,623,104
constexpr size_t kLayerDown = (size_t)kHidden * kInner;             // 28,311,552
constexpr size_t kLayerBytes = kLayerQKV + kLayerO + kLayerGateUp + kLayerDown;
constexpr size_t kStagingBytes = (size_t)32 << 20;
constexpr size_t kPartSlots = 8192;  // (token, head, split) partial slots

size_t pages_for(size_t context) { return (context + kPage - 1) / kPage; }

}  // namespace

struct lun_device {
    int ordinal = -1;
    int sm_count = 0;
    size_t context = 0, block = 0;
    int num_pages = 0;
    cudaStream_t stream = nullptr;
    uint8_t *w8 = nullptr;
    float scales[kLayers][LUN_SLOT_COUNT] = {};
    uint16_t *embedding = nullptr;
    float *norms = nullptr, *final_norm = nullptr;
    float *kv = nullptr;
    int *page_table = nullptr;          // the table the kernels read (a session's row in batch mode)
    int *own_table = nullptr;           // the identity table allocated with the device
    float *rope_cos = nullptr, *rope_sin = nullptr;
    StepParams *d_step = nullptr, *h_step = nullptr;
    float *x = nullptr, *h = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
    float *logits = nullptr, *part_acc = nullptr, *part_ml = nullptr;
    int *d_flag = nullptr, *h_flag = nullptr;
    float *h_logits = nullptr;
    void *staging[2] = {nullptr, nullptr};
    cudaEvent_t staging_done[2] = {nullptr, nullptr};
    uint8_t *upload_raw = nullptr;  // row-major tensor on its way to the tiled layout (upload only)
    int trace = 0;
    float *trace_buf = nullptr;
    size_t trace_count = 0;
    // device greedy decode loop (benchmarks): one captured step, replayed
    int *d_tokens = nullptr, *d_partials = nullptr;
    cudaGraphExec_t decode_graph = nullptr;
    int launches_per_step = 0;
    // persistent decode kernel state
    bool use_mega = true;
    float *d_scales = nullptr;          // [26][7]
    unsigned *mega_sync = nullptr;      // kSyncWords lines, zeroed before every launch
    unsigned long long *mega_qkvt = nullptr;  // tagged q/k/v words the persistent kernel exchanges
    float *mega_ffn = nullptr;                // [2][3072] h, then [2][3072] 64-bit xfix (MegaParams::hbuf, xfix)
    alignas(64) unsigned char down_map[128];  // tensor map of the down projections (lun_down_slice_map)
    bool down_map_ready = false;
    unsigned mega_tag = 1;                    // tag of the next launch's first layer (never 0)
    unsigned l2_ahead = 0;              // persistent kernel's L2 lookahead (bytes per CTA)
    unsigned l2_ahead_ffn = 0;          // the same while the ring is filled with FFN items
    unsigned l2_hints = 0;              // persistent kernel's L2 eviction hints (MegaParams::l2_hints)
    bool kv_early = true;               // persistent kernel: next layer's K/V into L2 during the FFN
    bool head_tc = true;                // batched head on tcgen05 (head_tc.cuh) instead of mma.sync
    int *mega_error = nullptr, *h_error = nullptr;
    float *arg_val = nullptr;
    int *arg_idx = nullptr;
    bool prefetch = true;                        // next-matrix L2 prefetch
    // blocks of more than kGemvMaxTokens tokens: tcgen05 GEMM projections
    PrefillWorkspace pf = {};
    bool use_gemm = true;
    int *h_pf_error = nullptr;
    unsigned long long *timeline = nullptr;      // per-barrier timestamps (optional)
    bool record_timeline = false;
    lun_device_bytes owned = {};
    size_t part_slots = kPartSlots;
    // batched decode over sessions (lun_device_create_batch)
    int max_sessions = 0, session_pages = 0;
    int *session_tables = nullptr;      // [max_sessions][session_pages] page ids
    int *d_meta = nullptr, *h_meta = nullptr;  // [block] positions, then [block] session of each token
    float *batch_logits = nullptr;      // [block][vocab]
    uint16_t *head_stage = nullptr;     // B operand staging of the batched head (lun_launch_head_mma)
    int *d_next = nullptr, *h_next = nullptr;
};

static int fail(char *error, size_t capacity, const char *what, cudaError_t e)
{
    if (error && capacity) snprintf(error, capacity, "%s: %s", what, cudaGetErrorString(e));
    return -1;
}

extern "C" void lun_device_plan(size_t context, size_t block, lun_device_bytes *bytes)
{
    bytes->weight_bytes = (uint64_t)kLayerBytes * kLayers + (uint64_t)kVocab * kHidden * 2 +
                          (uint64_t)(2 * kLayers + 1) * kHidden * 4;
    bytes->kv_bytes = (uint64_t)kLayers * pages_for(context) * 2 * kPageKind * sizeof(float);
    uint64_t scratch = 0;
    scratch += sizeof(StepParams);
    scratch += (uint64_t)block * (2 * kHidden + 2 * kQuery + kInner) * 4;  // x h q attn act
    scratch += (uint64_t)kVocab * 4;                                       // logits
    scratch += (uint64_t)kPartSlots * (kHeadDim + 2) * 4;                  // attention partials (decode)
    scratch += (uint64_t)context * kHeadDim * 2 * 4;                       // rope tables
    scratch += (uint64_t)pages_for(context) * 4 + 4;                        // page table + flag
    if (block > kGemvMaxTokens) {  // prefill GEMM workspace (sized for a 148-SM B200)
        size_t xs, inv, ws;
        lun_prefill_workspace_bytes((int)block, 148, &xs, &inv, &ws);
        scratch += xs + inv + ws + 4;
    }
    bytes->scratch_bytes = scratch;
}

template <class T>
static cudaError_t dalloc(T **p, size_t bytes, uint64_t *counter)
{
    cudaError_t e = cudaMalloc((void **)p, bytes);
    if (e == cudaSuccess && counter) *counter += bytes;
    return e;
}

// context: positions of one sequence (RoPE table, bounds); kv_pages: pages of
// the KV pool; part_slots: attention partial slots.
static lun_device *create_device(size_t context, size_t kv_pages, size_t block, size_t part_slots, char *error,
                                 size_t capacity)
{
    lun_device_bytes plan;
    lun_device_plan(context, block, &plan);
    plan.kv_bytes = (uint64_t)kLayers * kv_pages * 2 * kPageKind * sizeof(float);
    plan.scratch_bytes += (uint64_t)(part_slots > kPartSlots ? part_slots - kPartSlots : 0) * (kHeadDim + 2) * 4;
    int ordinal = 0;
    cudaError_t e = cudaGetDevice(&ordinal);
    if (e != cudaSuccess) {
        fail(error, capacity, "CUDA device unavailable", e);
        return nullptr;
    }
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, ordinal);
    if (e != cudaSuccess) {
        fail(error, capacity, "CUDA device query failed", e);
        return nullptr;
    }
    if (prop.major != 10) {
        if (error && capacity)
            snprintf(error, capacity, "requires an sm_100 (B200) device, found sm_%d%d", prop.major,
                     prop.minor);
        return nullptr;
    }
    size_t free_bytes = 0, total_bytes = 0;
    e = cudaMemGetInfo(&free_bytes, &total_bytes);
    uint64_t need = plan.weight_bytes + plan.kv_bytes + plan.scratch_bytes + ((uint64_t)1 << 30);
    if (e != cudaSuccess || free_bytes < need) {
        if (error && capacity)
            snprintf(error, capacity, "insufficient device memory: need %llu bytes, %zu free",
                     (unsigned long long)need, free_bytes);
        return nullptr;
    }
    lun_device *d = new (std::nothrow) lun_device();
    if (!d) {
        if (error && capacity) snprintf(error, capacity, "device context allocation failed");
        return nullptr;
    }
    d->ordinal = ordinal;
    d->sm_count = prop.multiProcessorCount;
    d->context = context;
    d->block = block;
    d->num_pages = (int)kv_pages;
    d->part_slots = part_slots;
    uint64_t *wc = &d->owned.weight_bytes, *kc = &d->owned.kv_bytes, *sc = &d->owned.scratch_bytes;
    const char *what = "stream";
    if ((e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking)) != cudaSuccess) goto bad;
    what = "weights";
    if ((e = dalloc(&d->w8, kLayerBytes * kLayers, wc)) != cudaSuccess ||
        (e = dalloc(&d->embedding, (size_t)kVocab * kHidden * 2, wc)) != cudaSuccess ||
        (e = dalloc(&d->norms, (size_t)(2 * kLayers + 1) * kHidden * 4, wc)) != cudaSuccess)
        goto bad;
    d->final_norm = d->norms + (size_t)2 * kLayers * kHidden;
    what = "KV cache";
    if ((e = dalloc(&d->kv, (size_t)kLayers * d->num_pages * 2 * kPageKind * sizeof(float), kc)) !=
        cudaSuccess)
        goto bad;
    what = "scratch";
    if ((e = dalloc(&d->d_step, sizeof(StepParams), sc)) != cudaSuccess ||
        (e = dalloc(&d->x, block * kHidden * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->h, block * kHidden * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->q, block * kQuery * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->attn, block * kQuery * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->act, block * kInner * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->logits, (size_t)kVocab * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->part_acc, part_slots * kHeadDim * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->part_ml, part_slots * 2 * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->rope_cos, context * kHeadDim * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->rope_sin, context * kHeadDim * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->own_table, (size_t)d->num_pages * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->d_flag, 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->d_scales, (size_t)kLayers * LUN_SLOT_COUNT * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->mega_sync, kSyncWords * kSyncStride * sizeof(unsigned), sc)) != cudaSuccess ||
        (e = dalloc(&d->mega_qkvt, (size_t)kQKVRows * sizeof(unsigned long long), sc)) != cudaSuccess ||
        (e = dalloc(&d->mega_ffn, (size_t)6 * kHidden * sizeof(float), sc)) != cudaSuccess ||
        (e = dalloc(&d->mega_error, sizeof(int), sc)) != cudaSuccess ||
        (e = dalloc(&d->arg_val, (size_t)d->sm_count * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->arg_idx, (size_t)d->sm_count * 4, sc)) != cudaSuccess ||
        (e = dalloc(&d->d_tokens, context * sizeof(int), sc)) != cudaSuccess)
        goto bad;
    if (block > kGemvMaxTokens) {
        lun_prefill_workspace_bytes((int)block, d->sm_count, &d->pf.xs_bytes, &d->pf.inv_bytes, &d->pf.ws_bytes);
        if ((e = dalloc(&d->pf.xs, d->pf.xs_bytes, sc)) != cudaSuccess ||
            (e = dalloc(&d->pf.inv_scale, d->pf.inv_bytes, sc)) != cudaSuccess ||
            (e = dalloc(&d->pf.ws, d->pf.ws_bytes, sc)) != cudaSuccess ||
            (e = dalloc(&d->pf.error, sizeof(int), sc)) != cudaSuccess ||
            (e = cudaMemset(d->pf.error, 0, sizeof(int))) != cudaSuccess)
            goto bad;
    }
    if ((e = cudaMemset(d->mega_error, 0, sizeof(int))) != cudaSuccess ||
        (e = cudaMemset(d->mega_qkvt, 0, (size_t)kQKVRows * sizeof(unsigned long long))) != cudaSuccess)
        goto bad;
    {
        const char *mega = getenv("LUNELETTE_MEGA");
        d->use_mega = !(mega && mega[0] == '0') && lun_mega_supported(d->sm_count);
        const char *gemm = getenv("LUNELETTE_PREFILL_GEMM");
        d->use_gemm = !(gemm && gemm[0] == '0') && d->pf.ws;
        const char *prefetch = getenv("LUNELETTE_PREFETCH");
        d->prefetch = !(prefetch && prefetch[0] == '0');
        // L2 lookahead of the persistent kernel's weight stream, per CTA; longer
        // lookaheads measured slower, with or without eviction hints (256 KB:
        // -2 %, 512 KB: -7 %, 1 MB: -27 %): the extra requests in flight
        // lengthen the latency of the phases' cross-CTA exchanges
        const char *ahead = getenv("LUNELETTE_L2_AHEAD_KB");
        d->l2_ahead = (ahead ? (unsigned)strtoul(ahead, nullptr, 10) : 128u) << 10;
        const char *ahead_ffn = getenv("LUNELETTE_L2_AHEAD_FFN_KB");
        d->l2_ahead_ffn = ahead_ffn ? (unsigned)strtoul(ahead_ffn, nullptr, 10) << 10 : d->l2_ahead;
        // L2 eviction hints of the persistent kernel's weight stream
        // (MegaParams::l2_hints): ring copies evict_first measured +1.8 % on C0
        // (1002 against 984 tok/s); evict_last on the prefetches gained nothing
        const char *early = getenv("LUNELETTE_KV_EARLY");
        d->kv_early = !(early && early[0] == '0');
        const char *hints = getenv("LUNELETTE_L2_HINTS");
        d->l2_hints = hints ? (unsigned)strtoul(hints, nullptr, 10) : 1u;
        // the batched head's kernel: tcgen05 (its bounded waits report through
        // the GEMM's error word) unless LUNELETTE_HEAD_TC=0 selects the mma.sync
        // kernel for comparison (64-session step at short contexts: 3.00 against
        // 3.28 ms)
        const char *head = getenv("LUNELETTE_HEAD_TC");
        d->head_tc = !(head && head[0] == '0') && d->pf.error;
    }
    what = "pinned host buffers";
    if ((e = cudaMallocHost((void **)&d->h_step, sizeof(StepParams))) != cudaSuccess ||
        (e = cudaMallocHost((void **)&d->h_logits, (size_t)kVocab * 4)) != cudaSuccess ||
        (e = cudaMallocHost((void **)&d->h_flag, 4)) != cudaSuccess ||
        (e = cudaMallocHost((void **)&d->h_error, 4)) != cudaSuccess ||
        (e = cudaMallocHost((void **)&d->h_pf_error, 4)) != cudaSuccess ||
        (e = cudaMallocHost(&d->staging[0], kStagingBytes)) != cudaSuccess ||
        (e = cudaMallocHost(&d->staging[1], kStagingBytes)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&d->staging_done[0], cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&d->staging_done[1], cudaEventDisableTiming)) != cudaSuccess)
        goto bad;
    {
        // single-sequence context: identity page table
        int *table = (int *)malloc((size_t)d->num_pages * sizeof(int));
        if (!table) {
            e = cudaErrorMemoryAllocation;
            goto bad;
        }
        for (int i = 0; i < d->num_pages; i++) table[i] = i;
        d->page_table = d->own_table;
        e = cudaMemcpy(d->page_table, table, (size_t)d->num_pages * 4, cudaMemcpyHostToDevice);
        free(table);
        if (e != cudaSuccess) goto bad;
    }
    what = "kernel setup";
    if ((e = lun_kernels_ensure()) != cudaSuccess) goto bad;
    return d;
bad:
    fail(error, capacity, what, e);
    lun_device_destroy(d);
    return nullptr;
}

// Attention partial slots: the decode splits, and for blocks of tokens up to 17
// key splits per (token, query head).
static size_t part_slots_for(size_t block)
{
    const size_t prefill = block * kQueryHeads * 17;
    return prefill > kPartSlots ? prefill : kPartSlots;
}

extern "C" lun_device *lun_device_create(size_t context, size_t block, char *error, size_t capacity)
{
    return create_device(context, pages_for(context), block, part_slots_for(block), error, capacity);
}

extern "C" lun_device *lun_device_create_batch(size_t pool_pages, size_t session_context, size_t block,
                                               size_t max_sessions, char *error, size_t capacity)
{
    if (!pool_pages || !session_context || block <= (size_t)kGemvMaxTokens || block > 256 || !max_sessions ||
        max_sessions > 65536) {
        if (error && capacity) snprintf(error, capacity, "batch: invalid pool, context, block or sessions");
        return nullptr;
    }
    // partial slots for block tokens x 32 heads x up to 16 position splits
    lun_device *d = create_device(session_context, pool_pages, block, part_slots_for(block), error, capacity);
    if (!d) return nullptr;
    d->max_sessions = (int)max_sessions;
    d->session_pages = (int)pages_for(session_context);
    uint64_t *sc = &d->owned.scratch_bytes;
    cudaError_t e;
    const char *what = "batch tables";
    if ((e = dalloc(&d->session_tables, (size_t)max_sessions * d->session_pages * sizeof(int), sc)) != cudaSuccess ||
        (e = cudaMemset(d->session_tables, 0, (size_t)max_sessions * d->session_pages * sizeof(int))) !=
            cudaSuccess ||
        (e = dalloc(&d->d_meta, 2 * block * sizeof(int), sc)) != cudaSuccess || !d->pf.ws ||
        (e = dalloc(&d->batch_logits, block * (size_t)kVocab * sizeof(float), sc)) != cudaSuccess ||
        (e = dalloc(&d->head_stage, lun_head_mma_stage_bytes(), sc)) != cudaSuccess ||
        (e = dalloc(&d->d_next, block * sizeof(int), sc)) != cudaSuccess ||
        (e = cudaMallocHost((void **)&d->h_meta, 2 * block * sizeof(int))) != cudaSuccess ||
        (e = cudaMallocHost((void **)&d->h_next, block * sizeof(int))) != cudaSuccess) {
        fail(error, capacity, what, e);
        lun_device_destroy(d);
        return nullptr;
    }
    return d;
}

extern "C" int lun_device_session_table(lun_device *d, int session, const int *pages, size_t n)
{
    if (!d->session_tables || session < 0 || session >= d->max_sessions || n > (size_t)d->session_pages) return -1;
    for (size_t i = 0; i < n; i++)
        if (pages[i] < 0 || pages[i] >= d->num_pages) return -1;
    if (cudaSetDevice(d->ordinal) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(d->stream) != cudaSuccess) return -1;
    return cudaMemcpy(d->session_tables + (size_t)session * d->session_pages, pages, n * sizeof(int),
                      cudaMemcpyHostToDevice) == cudaSuccess
               ? 0
               : -1;
}

extern "C" int lun_device_use_session(lun_device *d, int session)
{
    if (!d->session_tables || session < 0 || session >= d->max_sessions) return -1;
    d->page_table = d->session_tables + (size_t)session * d->session_pages;
    return 0;
}

extern "C" int lun_device_copy_page(lun_device *d, int src_page, int dst_page, int slots)
{
    if (!d->d_meta || src_page < 0 || src_page >= d->num_pages || dst_page < 0 || dst_page >= d->num_pages ||
        src_page == dst_page || slots < 1 || slots > kPage)
        return -1;
    if (cudaSetDevice(d->ordinal) != cudaSuccess || cudaStreamSynchronize(d->stream) != cudaSuccess) return -1;
    // the pair goes through the batch metadata words (free between calls)
    const int pair[2] = {src_page, dst_page};
    if (cudaMemcpy(d->d_meta, pair, sizeof pair, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    KvCopyParams p;
    p.kv = d->kv;
    p.num_pages = d->num_pages;
    p.src_pages = d->d_meta;
    p.dst_pages = d->d_meta + 1;
    p.pairs = 1;
    p.last_slots = slots;
    if (lun_launch_kv_copy(p, kLayers, d->stream) != cudaSuccess) return -1;
    return cudaStreamSynchronize(d->stream) == cudaSuccess ? 0 : -1;
}

extern "C" void lun_device_destroy(lun_device *d)
{
    if (!d) return;
    if (d->stream) cudaStreamSynchronize(d->stream);
    cudaFree(d->w8);
    cudaFree(d->embedding);
    cudaFree(d->norms);
    cudaFree(d->kv);
    cudaFree(d->d_step);
    cudaFree(d->x);
    cudaFree(d->h);
    cudaFree(d->q);
    cudaFree(d->attn);
    cudaFree(d->act);
    cudaFree(d->logits);
    cudaFree(d->part_acc);
    cudaFree(d->part_ml);
    cudaFree(d->rope_cos);
    cudaFree(d->rope_sin);
    cudaFree(d->own_table);
    cudaFree(d->d_flag);
    cudaFree(d->trace_buf);
    cudaFree(d->d_tokens);
    cudaFree(d->d_partials);
    cudaFree(d->d_scales);
    cudaFree(d->mega_sync);
    cudaFree(d->session_tables);
    cudaFree(d->d_meta);
    cudaFree(d->batch_logits);
    cudaFree(d->head_stage);
    cudaFree(d->d_next);
    cudaFreeHost(d->h_meta);
    cudaFreeHost(d->h_next);
    cudaFree(d->mega_qkvt);
    cudaFree(d->mega_ffn);
    cudaFree(d->mega_error);
    cudaFree(d->arg_val);
    cudaFree(d->arg_idx);
    cudaFree(d->timeline);
    cudaFree(d->upload_raw);
    cudaFree(d->pf.xs);
    cudaFree(d->pf.inv_scale);
    cudaFree(d->pf.ws);
    cudaFree(d->pf.error);
    cudaFreeHost(d->h_pf_error);
    cudaFreeHost(d->h_error);
    if (d->decode_graph) cudaGraphExecDestroy(d->decode_graph);
    cudaFreeHost(d->h_step);
    cudaFreeHost(d->h_logits);
    cudaFreeHost(d->h_flag);
    cudaFreeHost(d->staging[0]);
    cudaFreeHost(d->staging[1]);
    for (int i = 0; i < 2; i++)
        if (d->staging_done[i]) cudaEventDestroy(d->staging_done[i]);
    if (d->stream) cudaStreamDestroy(d->stream);
    delete d;
}

extern "C" int lun_device_ordinal(const lun_device *d) { return d->ordinal; }

extern "C" void lun_device_bytes_owned(const lun_device *d, lun_device_bytes *bytes)
{
    *bytes = d->owned;
}

extern "C" size_t lun_device_staging_bytes(void) { return kStagingBytes; }

extern "C" void *lun_device_staging(lun_device *d, int index) { return d->staging[index & 1]; }

extern "C" int lun_device_staging_wait(lun_device *d, int index)
{
    return cudaEventSynchronize(d->staging_done[index & 1]) == cudaSuccess ? 0 : -1;
}

static uint8_t *layer_base(lun_device *d, int layer) { return d->w8 + (size_t)layer * kLayerBytes; }

// FP8 linears are stored tiled (gemv.cuh): the row-major tensor is copied to a
// device buffer and a tile kernel writes it into its matrix, placing q/k/v rows
// so that RoPE pairs are adjacent and interleaving gate/up rows (gate f -> 2f,
// up f -> 2f + 1), which the fused epilogues rely on.
extern "C" int lun_device_upload_linear(lun_device *d, int index, int layer, int slot, size_t rows,
                                        size_t cols, float scale)
{
    if (rows * cols > kStagingBytes || (cols % 128) || (rows % 8)) return -1;
    uint8_t *base = layer_base(d, layer);
    d->scales[layer][slot] = scale;
    uint8_t *matrix;
    int order = kOrderRows, row0 = 0;
    switch (slot) {
    case LUN_SLOT_Q:
    case LUN_SLOT_K:
    case LUN_SLOT_V:
        matrix = base;
        order = kOrderRopePairs;
        row0 = slot == LUN_SLOT_Q ? 0 : (slot == LUN_SLOT_K ? kQuery : kQuery + kKV);
        break;
    case LUN_SLOT_O: matrix = base + kLayerQKV; break;
    case LUN_SLOT_GATE:
    case LUN_SLOT_UP:
        matrix = base + kLayerQKV + kLayerO;
        order = kOrderInterleave;
        row0 = slot == LUN_SLOT_UP ? 1 : 0;
        break;
    case LUN_SLOT_DOWN: matrix = base + kLayerQKV + kLayerO + kLayerGateUp; break;
    default: return -1;
    }
    if (!d->upload_raw && cudaMalloc((void **)&d->upload_raw, kStagingBytes) != cudaSuccess) return -1;
    if (cudaMemcpyAsync(d->upload_raw, d->staging[index & 1], rows * cols, cudaMemcpyHostToDevice, d->stream) !=
            cudaSuccess ||
        cudaEventRecord(d->staging_done[index & 1], d->stream) != cudaSuccess)
        return -1;
    return lun_launch_tile_fp8(d->upload_raw, (int)rows, (int)cols, matrix, (int)(cols / 128), order, row0,
                               d->stream) == cudaSuccess
               ? 0
               : -1;
}

extern "C" int lun_device_upload_embedding(lun_device *d, int index, size_t offset, size_t bytes)
{
    if (cudaMemcpyAsync((uint8_t *)d->embedding + offset, d->staging[index & 1], bytes,
                        cudaMemcpyHostToDevice, d->stream) != cudaSuccess)
        return -1;
    return cudaEventRecord(d->staging_done[index & 1], d->stream) == cudaSuccess ? 0 : -1;
}

extern "C" int lun_device_upload_norms(lun_device *d, const float *norms, const float *final_norm)
{
    if (cudaMemcpy(d->norms, norms, (size_t)2 * kLayers * kHidden * 4, cudaMemcpyHostToDevice) !=
        cudaSuccess)
        return -1;
    return cudaMemcpy(d->final_norm, final_norm, (size_t)kHidden * 4, cudaMemcpyHostToDevice) ==
                   cudaSuccess
               ? 0
               : -1;
}

extern "C" int lun_device_upload_rope(lun_device *d, const float *cosine, const float *sine,
                                      size_t positions)
{
    if (positions > d->context) return -1;
    if (cudaMemcpy(d->rope_cos, cosine, positions * kHeadDim * 4, cudaMemcpyHostToDevice) !=
        cudaSuccess)
        return -1;
    return cudaMemcpy(d->rope_sin, sine, positions * kHeadDim * 4, cudaMemcpyHostToDevice) ==
                   cudaSuccess
               ? 0
               : -1;
}

extern "C" int lun_device_upload_finish(lun_device *d, char *error, size_t capacity)
{
    cudaError_t e = cudaStreamSynchronize(d->stream);
    cudaFree(d->upload_raw);
    d->upload_raw = nullptr;
    if (e != cudaSuccess) return fail(error, capacity, "weight upload failed", e);
    e = cudaMemcpy(d->d_scales, d->scales, sizeof d->scales, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail(error, capacity, "scale upload failed", e);
    return 0;
}

extern "C" float *lun_device_host_logits(lun_device *d) { return d->h_logits; }

// ---------------------------------------------------------------------------

static GemvParams layer_gemv(lun_device *d, int layer, int which)
{
    GemvParams p;
    memset(&p, 0, sizeof p);
    uint8_t *base = layer_base(d, layer);
    const float *s = d->scales[layer];
    p.step = d->d_step;
    p.kv = d->kv;
    p.page_table = d->page_table;
    p.num_pages = d->num_pages;
    p.layer = layer;
    p.rope_cos = d->rope_cos;
    p.rope_sin = d->rope_sin;
    p.bound[0] = p.bound[1] = 1 << 30;
    p.scale[0] = p.scale[1] = p.scale[2] = 1.0f;
    switch (which) {
    case 0:  // qkv with input norm
        p.W = base;
        p.rows = kQKVRows;
        p.cols = kHidden;
        p.gain = d->norms + (size_t)(2 * layer) * kHidden;
        p.scale[0] = s[LUN_SLOT_Q];
        p.scale[1] = s[LUN_SLOT_K];
        p.scale[2] = s[LUN_SLOT_V];
        p.bound[0] = kQuery;
        p.bound[1] = kQuery + kKV;
        break;
    case 1:  // o + residual
        p.W = base + kLayerQKV;
        p.rows = kHidden;
        p.cols = kQuery;
        p.scale[0] = s[LUN_SLOT_O];
        break;
    case 2:  // gate/up with post-attention norm, SwiGLU
        p.W = base + kLayerQKV + kLayerO;
        p.rows = kGateUpRows;
        p.cols = kHidden;
        p.gain = d->norms + (size_t)(2 * layer + 1) * kHidden;
        p.scale[0] = s[LUN_SLOT_GATE];
        p.scale[1] = s[LUN_SLOT_UP];
        break;
    default:  // down + residual
        p.W = base + kLayerQKV + kLayerO + kLayerGateUp;
        p.rows = kHidden;
        p.cols = kInner;
        p.scale[0] = s[LUN_SLOT_DOWN];
        break;
    }
    // The step reads the FP8 weights front to back (qkv, o, gate/up, down, next
    // layer's qkv): each projection prefetches the next matrix into L2.
    static const size_t next_bytes[4] = {kLayerO, kLayerGateUp, kLayerDown, kLayerQKV};
    if (which < 3 || layer + 1 < kLayers) {
        p.prefetch = p.W + (which == 0 ? kLayerQKV : which == 1 ? kLayerO
                            : which == 2 ? kLayerGateUp : kLayerDown);
        p.prefetch_bytes = next_bytes[which];
    }
    return p;
}

// Launch `which` projection of `layer` over all `count` tokens in groups of <= 4.
// Projection `which` of `layer` for the tokens from t0: weights, scales,
// epilogue operands (x/y/res rows of the block's scratch).
static cudaError_t run_attention(lun_device *d, int layer, int count, size_t length, bool fixed_plan = false);

static GemvParams projection_params(lun_device *d, int layer, int which, int t0)
{
    GemvParams p = layer_gemv(d, layer, which);
    p.token_offset = t0;
    switch (which) {
    case 0:
        p.x = d->x + (size_t)t0 * kHidden;
        p.x_stride = kHidden;
        p.y = d->q + (size_t)t0 * kQuery;
        p.y_stride = kQuery;
        break;
    case 1:
        p.x = d->attn + (size_t)t0 * kQuery;
        p.x_stride = kQuery;
        p.res = d->x + (size_t)t0 * kHidden;
        p.res_stride = kHidden;
        p.y = d->h + (size_t)t0 * kHidden;
        p.y_stride = kHidden;
        break;
    case 2:
        p.x = d->h + (size_t)t0 * kHidden;
        p.x_stride = kHidden;
        p.y = d->act + (size_t)t0 * kInner;
        p.y_stride = kInner;
        break;
    default:
        p.x = d->act + (size_t)t0 * kInner;
        p.x_stride = kInner;
        p.res = d->h + (size_t)t0 * kHidden;
        p.res_stride = kHidden;
        p.y = d->x + (size_t)t0 * kHidden;
        p.y_stride = kHidden;
        break;
    }
    p.prefetch = nullptr;
    return p;
}

// batched: tokens of independent sessions (batched decode): always the
// tcgen05 path, whose QKV epilogue takes per-token positions and page tables.
static cudaError_t run_projection(lun_device *d, int layer, int which, int count, bool batched = false)
{
    static const int epi[4] = {kEpiQKV, kEpiResidual, kEpiSwiGLU, kEpiResidual};
    const bool gemm = batched || (count > kGemvMaxTokens && d->use_gemm);
    for (int t0 = 0; t0 < count; t0 += gemm ? count : kGemvMaxTokens) {
        int m = count - t0 < kGemvMaxTokens ? count - t0 : kGemvMaxTokens;
        GemvParams p = projection_params(d, layer, which, t0);
        if (gemm) {
            if (batched) {
                p.positions = d->d_meta;
                p.token_table = d->d_meta + d->block;
                p.table_stride = d->session_pages;
                p.page_table = d->session_tables;
            }
            return lun_launch_prefill(p, count, epi[which], d->pf, d->sm_count, d->stream);
        }
        if (!gemm) p.prefetch = layer_gemv(d, layer, which).prefetch;  // next-matrix L2 prefetch (GEMV)
        cudaError_t e = lun_launch_gemv(p, m, epi[which], d->sm_count, d->stream);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Blocks of more than kGemvMaxTokens tokens of one sequence on the tcgen05
// path, each finish fused with the next projection's split: per layer split
// (attn), 4 GEMMs, the QKV finish, attention and three finish+split kernels.
static cudaError_t run_prefill_layers(lun_device *d, int count, size_t length)
{
    cudaError_t e;
    const int sms = d->sm_count;
    if ((e = lun_launch_prefill_split(projection_params(d, 0, 0, 0), count, d->pf, sms, d->stream)) != cudaSuccess)
        return e;
    for (int layer = 0; layer < kLayers; layer++) {
        const GemvParams qkv = projection_params(d, layer, 0, 0), o = projection_params(d, layer, 1, 0),
                         gu = projection_params(d, layer, 2, 0), down = projection_params(d, layer, 3, 0);
        if ((e = lun_launch_prefill_gemm(qkv, count, d->pf, sms, d->stream)) != cudaSuccess ||
            (e = lun_launch_prefill_finish(qkv, count, kEpiQKV, d->pf, sms, d->stream)) != cudaSuccess ||
            (e = run_attention(d, layer, count, length)) != cudaSuccess ||
            (e = lun_launch_prefill_split(o, count, d->pf, sms, d->stream)) != cudaSuccess ||
            (e = lun_launch_prefill_gemm(o, count, d->pf, sms, d->stream)) != cudaSuccess ||
            (e = lun_launch_prefill_finish_split(o, count, kEpiResidual, d->pf, sms, gu.gain, gu.rows, true,
                                                 d->stream)) != cudaSuccess ||
            (e = lun_launch_prefill_gemm(gu, count, d->pf, sms, d->stream)) != cudaSuccess)
            return e;
        GemvParams gux = gu;
        gux.y = nullptr;  // act feeds only the down projection's operand tiles
        const bool last = layer + 1 == kLayers;
        const float *next_gain = last ? nullptr : d->norms + (size_t)(2 * (layer + 1)) * kHidden;
        if ((e = lun_launch_prefill_finish_split(gux, count, kEpiSwiGLU, d->pf, sms, nullptr, down.rows, true,
                                                 d->stream)) != cudaSuccess ||
            (e = lun_launch_prefill_gemm(down, count, d->pf, sms, d->stream)) != cudaSuccess ||
            (e = lun_launch_prefill_finish_split(down, count, kEpiResidual, d->pf, sms, next_gain, kQKVRows, !last,
                                                 d->stream)) != cudaSuccess)
            return e;
        if (d->trace && (e = cudaMemcpyAsync(d->trace_buf + (size_t)layer * count * kHidden, d->x,
                                             (size_t)count * kHidden * 4, cudaMemcpyDeviceToDevice, d->stream)) !=
                            cudaSuccess)
            return e;
    }
    return cudaSuccess;
}

static cudaError_t run_attention(lun_device *d, int layer, int count, size_t length, bool fixed_plan)
{
    AttnParams a;
    memset(&a, 0, sizeof a);
    a.q = d->q;
    a.kv = d->kv;
    a.page_table = d->page_table;
    a.num_pages = d->num_pages;
    a.layer = layer;
    a.step = d->d_step;
    a.out = d->attn;
    a.part_acc = d->part_acc;
    a.part_ml = d->part_ml;
    a.error = d->pf.error;  // the tcgen05 kernel's bounded waits report here, as the GEMM's do
    // A captured graph serves every length, so it plans for the full context;
    // splits past the current length find no positions and contribute nothing.
    int total = fixed_plan ? (int)d->context : (int)(length + count);
    lun_attention_plan(&a, total, count, d->sm_count, (int)d->part_slots);
    return lun_launch_attention(a, count, d->stream);
}

// The persistent decode kernel for `steps` batch-1 steps starting from d_step
// (length and ids[0]); it advances d_step and logs the greedy ids in d_tokens.
static cudaError_t launch_mega(lun_device *d, int steps)
{
    MegaParams p;
    memset(&p, 0, sizeof p);
    p.w8 = d->w8;
    p.scales = d->d_scales;
    p.embedding = d->embedding;
    p.norms = d->norms;
    p.final_norm = d->final_norm;
    p.kv = d->kv;
    p.page_table = d->page_table;
    p.num_pages = d->num_pages;
    p.rope_cos = d->rope_cos;
    p.rope_sin = d->rope_sin;
    p.step = d->d_step;
    p.x = d->x;
    p.hbuf = d->mega_ffn;
    p.xfix = reinterpret_cast<long long *>(d->mega_ffn + 2 * kHidden);
    // tags of this launch's layers: mega_tag .. mega_tag + 26 * steps - 1; a
    // wrap restarts from 1 over freshly zeroed words, so no old word matches
    const unsigned long long span = (unsigned long long)steps * kLayers;
    if ((unsigned long long)d->mega_tag + span >= 0xffffffffull) {
        cudaError_t z = cudaMemsetAsync(d->mega_qkvt, 0, (size_t)kQKVRows * sizeof(unsigned long long), d->stream);
        if (z != cudaSuccess) return z;
        d->mega_tag = 1;
    }
    p.qkvt = d->mega_qkvt;
    p.tag_base = d->mega_tag;
    d->mega_tag += (unsigned)span;
    p.attn = d->attn;
    p.part_acc = d->part_acc;
    p.part_ml = d->part_ml;
    p.logits = d->logits;
    p.nonfinite = d->d_flag;
    p.arg_val = d->arg_val;
    p.arg_idx = d->arg_idx;
    p.tokens = d->d_tokens;
    p.sync = d->mega_sync;
    p.error = d->mega_error;
    p.steps = steps;
    p.timeline = d->record_timeline ? d->timeline : nullptr;
    p.l2_ahead = d->l2_ahead;
    p.l2_ahead_ffn = d->l2_ahead_ffn;
    p.l2_hints = d->l2_hints;
    p.kv_early = d->kv_early ? 1u : 0u;
    {
        const char *rows = getenv("LUNELETTE_ATTN_ROWS");
        p.attn_rows = !(rows && rows[0] == '0');
    }
    cudaError_t e;
    if (!d->down_map_ready) {
        if ((e = lun_down_slice_map(d->down_map, layer_base(d, 0) + kLayerQKV + kLayerO + kLayerGateUp,
                                    kLayerBytes)) != cudaSuccess)
            return e;
        d->down_map_ready = true;
    }
    e = cudaMemsetAsync(d->mega_sync, 0, kSyncWords * kSyncStride * sizeof(unsigned), d->stream);
    if (e != cudaSuccess) return e;
    return lun_launch_decode_mega(p, d->down_map, d->sm_count, d->stream);
}

// One decode step reading length/ids from d_step, ending with device greedy
// selection that advances d_step; capturable.
static cudaError_t enqueue_decode_step(lun_device *d, int *launches)
{
    int n = 0;
    cudaError_t e = lun_launch_embed(d->embedding, d->d_step, d->x, 1, d->stream);
    n++;
    for (int layer = 0; e == cudaSuccess && layer < kLayers; layer++) {
        if ((e = run_projection(d, layer, 0, 1)) != cudaSuccess ||
            (e = run_attention(d, layer, 1, 0, true)) != cudaSuccess ||
            (e = run_projection(d, layer, 1, 1)) != cudaSuccess ||
            (e = run_projection(d, layer, 2, 1)) != cudaSuccess ||
            (e = run_projection(d, layer, 3, 1)) != cudaSuccess)
            break;
        AttnParams a;
        lun_attention_plan(&a, (int)d->context, 1, d->sm_count, (int)d->part_slots);
        n += 5 + (a.splits > 1 ? 1 : 0);
    }
    if (e != cudaSuccess) return e;
    HeadParams hp;
    hp.W = d->embedding;
    hp.rows = kVocab;
    hp.cols = kHidden;
    hp.x = d->x;
    hp.gain = d->final_norm;
    hp.logits = d->logits;
    hp.nonfinite = d->d_flag;
    if ((e = lun_launch_head(hp, d->sm_count, d->stream)) != cudaSuccess) return e;
    if ((e = lun_launch_greedy(d->logits, kVocab, d->d_partials, d->d_step, d->d_tokens,
                               d->stream)) != cudaSuccess)
        return e;
    *launches = n + 3;
    return cudaSuccess;
}

extern "C" int lun_device_decode_loop(lun_device *d, int64_t first_token, size_t length,
                                      size_t steps, int64_t *tokens, float *milliseconds,
                                      int *launches, char *error, size_t capacity)
{
    cudaError_t e = cudaSetDevice(d->ordinal);
    if (e != cudaSuccess) return fail(error, capacity, "cudaSetDevice", e);
    if (!steps || length == 0 || length + steps > d->context || first_token < 0 ||
        first_token >= kVocab) {
        if (error && capacity) snprintf(error, capacity, "decode loop: bad length/steps/token");
        return -1;
    }
    const char *what = "decode loop setup";
    cudaEvent_t start = nullptr, stop = nullptr;
    int *host_tokens = nullptr;
    if (!d->d_partials &&
        (e = cudaMalloc((void **)&d->d_partials, 2 * kArgmaxBlocks * sizeof(int))) != cudaSuccess)
        goto bad;
    if (d->use_mega) {
        what = "decode loop (persistent kernel)";
        d->h_step->length = (int)length;
        d->h_step->count = 1;
        d->h_step->generated = 0;
        d->h_step->ids[0] = (int)first_token;
        if ((e = cudaEventCreate(&start)) != cudaSuccess || (e = cudaEventCreate(&stop)) != cudaSuccess ||
            (e = cudaMemcpyAsync(d->d_step, d->h_step, sizeof(StepParams), cudaMemcpyHostToDevice,
                                 d->stream)) != cudaSuccess ||
            (e = cudaMemsetAsync(d->d_flag, 0, 4, d->stream)) != cudaSuccess ||
            (e = cudaEventRecord(start, d->stream)) != cudaSuccess ||
            (e = launch_mega(d, (int)steps)) != cudaSuccess ||
            (e = cudaEventRecord(stop, d->stream)) != cudaSuccess ||
            (e = cudaMemcpyAsync(d->h_error, d->mega_error, 4, cudaMemcpyDeviceToHost, d->stream)) !=
                cudaSuccess ||
            (e = cudaMemcpyAsync(d->h_flag, d->d_flag, 4, cudaMemcpyDeviceToHost, d->stream)) != cudaSuccess ||
            (e = cudaStreamSynchronize(d->stream)) != cudaSuccess)
            goto bad;
        if (*d->h_error) {
            cudaMemset(d->mega_error, 0, sizeof(int));
            e = cudaErrorLaunchTimeout;
            what = "decode loop: grid barrier wait gave up";
            goto bad;
        }
        // the loop picks tokens on the device, so it cannot rerun a step on the
        // FP32 path: a flagged step fails the call (lunelette_metal_decode
        // handles such values)
        if (*d->h_flag) {
            if (error && capacity)
                snprintf(error, capacity, "decode loop: %s",
                         (*d->h_flag & kFlagNonfinite) ? "non-finite logit"
                                                        : "hidden value outside the fixed-point range");
            free(host_tokens);
            cudaEventDestroy(start);
            cudaEventDestroy(stop);
            return -1;
        }
        if (milliseconds && (e = cudaEventElapsedTime(milliseconds, start, stop)) != cudaSuccess) goto bad;
        d->launches_per_step = 1;
    } else if (!d->decode_graph) {
        what = "decode graph capture";
        cudaGraph_t graph = nullptr;
        if ((e = cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeRelaxed)) != cudaSuccess)
            goto bad;
        cudaError_t ce = enqueue_decode_step(d, &d->launches_per_step);
        e = cudaStreamEndCapture(d->stream, &graph);
        if (ce != cudaSuccess) e = ce;
        if (e == cudaSuccess) e = cudaGraphInstantiate(&d->decode_graph, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (e != cudaSuccess) {
            d->decode_graph = nullptr;
            goto bad;
        }
    }
    if (!d->use_mega) {
        what = "decode loop";
        d->h_step->length = (int)length;
        d->h_step->count = 1;
        d->h_step->generated = 0;
        d->h_step->ids[0] = (int)first_token;
        if ((e = cudaEventCreate(&start)) != cudaSuccess || (e = cudaEventCreate(&stop)) != cudaSuccess ||
            (e = cudaMemcpyAsync(d->d_step, d->h_step, sizeof(StepParams), cudaMemcpyHostToDevice,
                                 d->stream)) != cudaSuccess ||
            (e = cudaEventRecord(start, d->stream)) != cudaSuccess)
            goto bad;
        for (size_t s = 0; s < steps; s++)
            if ((e = cudaGraphLaunch(d->decode_graph, d->stream)) != cudaSuccess) goto bad;
        if ((e = cudaEventRecord(stop, d->stream)) != cudaSuccess ||
            (e = cudaStreamSynchronize(d->stream)) != cudaSuccess)
            goto bad;
        if (milliseconds && (e = cudaEventElapsedTime(milliseconds, start, stop)) != cudaSuccess)
            goto bad;
    }
    host_tokens = (int *)malloc(steps * sizeof(int));
    if (!host_tokens) {
        e = cudaErrorMemoryAllocation;
        goto bad;
    }
    if ((e = cudaMemcpy(host_tokens, d->d_tokens, steps * sizeof(int), cudaMemcpyDeviceToHost)) !=
        cudaSuccess)
        goto bad;
    for (size_t s = 0; s < steps; s++) tokens[s] = host_tokens[s];
    free(host_tokens);
    if (launches) *launches = d->use_mega ? 1 : d->launches_per_step * (int)steps;
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    return 0;
bad:
    free(host_tokens);
    if (start) cudaEventDestroy(start);
    if (stop) cudaEventDestroy(stop);
    return fail(error, capacity, what, e);
}

// Embedding, the 26 layers on the per-projection kernels (GEMV for up to
// kGemvMaxTokens tokens, tcgen05 GEMMs beyond), the optional trace copies and
// the head over the last row, for the n tokens described by d_step.
static cudaError_t enqueue_block(lun_device *d, int n, size_t length)
{
    cudaError_t e = lun_launch_embed(d->embedding, d->d_step, d->x, n, d->stream);
    if (e != cudaSuccess) return e;
    if (n > kGemvMaxTokens && d->use_gemm) {
        if ((e = run_prefill_layers(d, n, length)) != cudaSuccess) return e;
    } else {
        for (int layer = 0; layer < kLayers; layer++) {
            if ((e = run_projection(d, layer, 0, n)) != cudaSuccess ||
                (e = run_attention(d, layer, n, length)) != cudaSuccess ||
                (e = run_projection(d, layer, 1, n)) != cudaSuccess ||
                (e = run_projection(d, layer, 2, n)) != cudaSuccess ||
                (e = run_projection(d, layer, 3, n)) != cudaSuccess)
                return e;
            if (d->trace && (e = cudaMemcpyAsync(d->trace_buf + (size_t)layer * n * kHidden, d->x,
                                                 (size_t)n * kHidden * 4, cudaMemcpyDeviceToDevice,
                                                 d->stream)) != cudaSuccess)
                return e;
        }
    }
    if (d->trace) {
        if ((e = lun_launch_rmsnorm(d->final_norm, d->x, d->trace_buf + (size_t)kLayers * n * kHidden, kHidden, n,
                                    d->stream)) != cudaSuccess)
            return e;
        d->trace_count = (size_t)n;
    }
    HeadParams hp;
    hp.W = d->embedding;
    hp.rows = kVocab;
    hp.cols = kHidden;
    hp.x = d->x + (size_t)(n - 1) * kHidden;
    hp.gain = d->final_norm;
    hp.logits = d->logits;
    hp.nonfinite = d->d_flag;
    return lun_launch_head(hp, d->sm_count, d->stream);
}

extern "C" int lun_device_run(lun_device *d, const int64_t *ids, size_t count, size_t length,
                              const float **logits, int *nonfinite, char *error, size_t capacity)
{
    cudaError_t e = cudaSetDevice(d->ordinal);
    if (e != cudaSuccess) return fail(error, capacity, "cudaSetDevice", e);
    if (!count || count > d->block || length + count > d->context) {
        if (error && capacity) snprintf(error, capacity, "device run: block/context exceeded");
        return -1;
    }
    const int n = (int)count;
    // single-token calls run the persistent decode kernel (one launch); blocks of
    // several tokens and traced calls run the per-projection kernels. A
    // persistent step whose fixed-point residual sums left their range (a
    // non-finite or huge hidden value) is run again on the FP32 kernels, which
    // write the same KV rows and give the reference's answer for such values.
    bool mega = count == 1 && !d->trace && d->use_mega;
    const char *what = "step upload";
    for (;;) {
        d->h_step->length = (int)length;
        d->h_step->count = n;
        for (size_t i = 0; i < count; i++) d->h_step->ids[i] = (int)ids[i];
        d->h_step->generated = 0;
        what = "step upload";
        if ((e = cudaMemcpyAsync(d->d_step, d->h_step, sizeof(StepParams), cudaMemcpyHostToDevice,
                                 d->stream)) != cudaSuccess ||
            (e = cudaMemsetAsync(d->d_flag, 0, 4, d->stream)) != cudaSuccess)
            goto bad;
        what = "kernel launch";
        if (mega) {
            if ((e = launch_mega(d, 1)) != cudaSuccess ||
                (e = cudaMemcpyAsync(d->h_error, d->mega_error, 4, cudaMemcpyDeviceToHost, d->stream)) !=
                    cudaSuccess)
                goto bad;
        } else if ((e = enqueue_block(d, n, length)) != cudaSuccess) {
            goto bad;
        }
        what = "logits download";
        if ((e = cudaMemcpyAsync(d->h_logits, d->logits, (size_t)kVocab * 4, cudaMemcpyDeviceToHost,
                                 d->stream)) != cudaSuccess ||
            (e = cudaMemcpyAsync(d->h_flag, d->d_flag, 4, cudaMemcpyDeviceToHost, d->stream)) != cudaSuccess)
            goto bad;
        if (d->pf.error &&
            (e = cudaMemcpyAsync(d->h_pf_error, d->pf.error, 4, cudaMemcpyDeviceToHost, d->stream)) != cudaSuccess)
            goto bad;
        what = "execution";
        if ((e = cudaStreamSynchronize(d->stream)) != cudaSuccess) goto bad;
        if (d->pf.error && *d->h_pf_error) {
            cudaMemset(d->pf.error, 0, sizeof(int));
            if (error && capacity) snprintf(error, capacity, "prefill: tensor-core pipeline wait gave up (GEMM or block attention)");
            return -1;
        }
        if (mega && *d->h_error) {
            cudaMemset(d->mega_error, 0, sizeof(int));
            if (error && capacity) snprintf(error, capacity, "decode: grid barrier wait gave up");
            return -1;
        }
        if (mega && (*d->h_flag & kFlagFixedRange)) {
            mega = false;
            continue;
        }
        break;
    }
    *logits = d->h_logits;
    *nonfinite = (*d->h_flag & kFlagNonfinite) != 0;
    return 0;
bad:
    return fail(error, capacity, what, e);
}

// One decode step for n tokens of n sessions: token i (id ids[i]) at position
// positions[i] of session sessions[i]. The projections run on the tcgen05 path
// for all n tokens at once (weights read once per step), attention per token
// over its own session's pages, then the tied head over the rows and a greedy
// id per row. Writes next[i] (host) and, when logits is not NULL, the n x 131072
// logits (host).
extern "C" int lun_device_batch_decode(lun_device *d, const int *sessions, const int64_t *ids, const int *positions,
                                       size_t n, float *logits, int64_t *next, int *nonfinite, char *error,
                                       size_t capacity)
{
    cudaError_t e = cudaSetDevice(d->ordinal);
    if (e != cudaSuccess) return fail(error, capacity, "cudaSetDevice", e);
    if (!d->session_tables || !n || n > d->block || !sessions || !ids || !positions) {
        if (error && capacity) snprintf(error, capacity, "batch decode: invalid arguments");
        return -1;
    }
    int longest = 0;
    for (size_t i = 0; i < n; i++) {
        if (sessions[i] < 0 || sessions[i] >= d->max_sessions || positions[i] < 0 ||
            (size_t)positions[i] >= d->context || ids[i] < 0 || ids[i] >= kVocab) {
            if (error && capacity) snprintf(error, capacity, "batch decode: token %zu out of range", i);
            return -1;
        }
        d->h_step->ids[i] = (int)ids[i];
        d->h_meta[i] = positions[i];
        d->h_meta[d->block + i] = sessions[i];
        longest = positions[i] + 1 > longest ? positions[i] + 1 : longest;
    }
    d->h_step->length = 0;
    d->h_step->count = (int)n;
    d->h_step->generated = 0;
    const int count = (int)n;
    const char *what = "batch upload";
    if ((e = cudaMemcpyAsync(d->d_step, d->h_step, sizeof(StepParams), cudaMemcpyHostToDevice, d->stream)) !=
            cudaSuccess ||
        (e = cudaMemcpyAsync(d->d_meta, d->h_meta, 2 * d->block * sizeof(int), cudaMemcpyHostToDevice,
                             d->stream)) != cudaSuccess ||
        (e = cudaMemsetAsync(d->d_flag, 0, 4, d->stream)) != cudaSuccess)
        return fail(error, capacity, what, e);
    what = "batch kernels";
    if ((e = lun_launch_embed(d->embedding, d->d_step, d->x, count, d->stream)) != cudaSuccess)
        return fail(error, capacity, what, e);
    for (int layer = 0; layer < kLayers; layer++) {
        AttnParams a;
        memset(&a, 0, sizeof a);
        a.q = d->q;
        a.kv = d->kv;
        a.page_table = d->session_tables;
        a.num_pages = d->num_pages;
        a.layer = layer;
        a.out = d->attn;
        a.part_acc = d->part_acc;
        a.part_ml = d->part_ml;
        a.positions = d->d_meta;
        a.token_table = d->d_meta + d->block;
        a.table_stride = d->session_pages;
        lun_attention_plan(&a, longest, count, d->sm_count, (int)d->part_slots);
        if ((e = run_projection(d, layer, 0, count, true)) != cudaSuccess ||
            (e = lun_launch_attention(a, count, d->stream)) != cudaSuccess ||
            (e = run_projection(d, layer, 1, count, true)) != cudaSuccess ||
            (e = run_projection(d, layer, 2, count, true)) != cudaSuccess ||
            (e = run_projection(d, layer, 3, count, true)) != cudaSuccess)
            return fail(error, capacity, what, e);
    }
    for (int t0 = 0; t0 < count; t0 += lun_head_mma_tokens()) {
        HeadMmaParams hp;
        hp.W = d->embedding;
        hp.rows = kVocab;
        hp.x = d->x + (size_t)t0 * kHidden;
        hp.x_stride = kHidden;
        hp.count = count - t0 < lun_head_mma_tokens() ? count - t0 : lun_head_mma_tokens();
        hp.gain = d->final_norm;
        hp.xb = d->head_stage;
        hp.logits = d->batch_logits + (size_t)t0 * kVocab;
        hp.logits_stride = kVocab;
        hp.nonfinite = d->d_flag;
        hp.error = d->pf.error;
        if ((e = d->head_tc ? lun_launch_head_tc(hp, d->stream) : lun_launch_head_mma(hp, d->stream)) != cudaSuccess)
            return fail(error, capacity, what, e);
    }
    if ((e = lun_launch_argmax_rows(d->batch_logits, kVocab, kVocab, count, d->d_next, d->stream)) != cudaSuccess)
        return fail(error, capacity, what, e);
    what = "batch download";
    if ((e = cudaMemcpyAsync(d->h_next, d->d_next, n * sizeof(int), cudaMemcpyDeviceToHost, d->stream)) !=
            cudaSuccess ||
        (e = cudaMemcpyAsync(d->h_flag, d->d_flag, 4, cudaMemcpyDeviceToHost, d->stream)) != cudaSuccess ||
        (logits && (e = cudaMemcpyAsync(logits, d->batch_logits, n * (size_t)kVocab * sizeof(float),
                                        cudaMemcpyDeviceToHost, d->stream)) != cudaSuccess))
        return fail(error, capacity, what, e);
    what = "batch execution";
    if ((e = cudaStreamSynchronize(d->stream)) != cudaSuccess) return fail(error, capacity, what, e);
    if (d->pf.error && (e = cudaMemcpy(d->h_pf_error, d->pf.error, 4, cudaMemcpyDeviceToHost)) == cudaSuccess &&
        *d->h_pf_error) {
        cudaMemset(d->pf.error, 0, sizeof(int));
        if (error && capacity) snprintf(error, capacity, "batch decode: tensor-core pipeline wait gave up (GEMM or head)");
        return -1;
    }
    if (next)
        for (size_t i = 0; i < n; i++) next[i] = d->h_next[i];
    if (nonfinite) *nonfinite = *d->h_flag != 0;
    return 0;
}

// CTA 0's barrier exits, then every CTA's marks (mega_params.cuh)
static size_t timeline_entries(const lun_device *d)
{
    return (size_t)kMegaTimelineHead + (size_t)kMegaMarksPerStep * d->sm_count;
}

extern "C" int lun_device_timeline(lun_device *d, int enable)
{
    if (enable && !d->timeline &&
        cudaMalloc((void **)&d->timeline, timeline_entries(d) * sizeof(unsigned long long)) != cudaSuccess)
        return -1;
    d->record_timeline = enable != 0;
    return 0;
}

extern "C" int lun_device_timeline_copy(lun_device *d, unsigned long long *out, size_t entries)
{
    if (!d->timeline || entries > timeline_entries(d)) return -1;
    return cudaMemcpy(out, d->timeline, entries * sizeof(unsigned long long), cudaMemcpyDeviceToHost) ==
                   cudaSuccess
               ? 0
               : -1;
}

extern "C" int lun_device_trace(lun_device *d, int enable)
{
    if (enable && !d->trace_buf) {
        if (cudaMalloc((void **)&d->trace_buf, (size_t)(kLayers + 1) * d->block * kHidden * 4) !=
            cudaSuccess)
            return -1;
    }
    d->trace = enable != 0;
    return 0;
}

extern "C" size_t lun_device_trace_rows(const lun_device *d)
{
    return d->trace && d->trace_buf ? d->trace_count : 0;
}

extern "C" int lun_device_trace_copy(lun_device *d, int which, float *out, size_t floats)
{
    if (!d->trace_buf || which < 0 || which > kLayers || floats != d->trace_count * kHidden)
        return -1;
    return cudaMemcpy(out, d->trace_buf + (size_t)which * d->trace_count * kHidden, floats * 4,
                      cudaMemcpyDeviceToHost) == cudaSuccess
               ? 0
               : -1;
}
