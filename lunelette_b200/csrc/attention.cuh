// Causal GQA attention over the paged FP32 KV pool, split over positions.
//
// Replaces scores + attend (src/metal_kernels.metal:81-132), which materialise a
// [count,32,C] probability matrix; here each block streams K/V tiles of 32
// positions through shared memory once for the four query heads of one KV head
// (GQA group h -> h/4) and keeps an online softmax, so nothing of size C is
// written. Scores are (q . k) * 0.08838834764831845f as in the reference.
//
// Grid: (splits, 8 KV heads, count). Split s covers positions
// [s*split_len, min((s+1)*split_len, length+t+1)) for query token t. With one
// split the block writes the final output; otherwise it writes (max, sum, acc)
// partials that attention_combine_kernel merges in split order, so results do
// not depend on block scheduling.
#pragma once
#include "common.cuh"

namespace lun {

struct AttnParams {
    const float *q;          // [count][4096], RoPE'd and query-scaled
    const float *kv;         // FP32 pool
    const int *page_table;
    int num_pages, layer;
    const StepParams *step;  // length before this call (device), or nullptr to
    int length;              //   use this value instead
    int token_offset;        // first query token of this launch within the call
    int split_len;           // positions per split (multiple of 32)
    int splits;
    float *out;              // [count][4096] when splits == 1
    float *part_acc;         // [count][32][splits][128]
    float *part_ml;          // [count][32][splits][2]
    // Batched decode over independent sessions: token t sits at position
    // positions[t] of the session whose page table is page_table +
    // token_table[t] * table_stride (nullptr: one sequence, positions
    // length + token_offset + t over page_table).
    const int *positions, *token_table;
    int table_stride;
};

constexpr int kTile = 32;
constexpr int kKPad = 132;  // padded K row (floats): conflict-free 16-byte reads across lanes
constexpr int kStageFloats = kTile * kKPad + kTile * kHeadDim;
// dynamic shared memory: q for 4 heads + two K/V tile stages
constexpr int kAttnSmemBytes = (4 * kHeadDim + 2 * kStageFloats) * 4;

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool full)
{
    unsigned dst = (unsigned)__cvta_generic_to_shared(smem);
    int bytes = full ? 16 : 0;  // 0: no global read, zero-fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Issue the copies of one 32-position K/V tile (2 x 16 KB) into a stage. A tile
// starts on a multiple of 32 and so lies in one page: the page lookup and the
// row addresses are computed once per tile, not per 16-byte chunk.
__device__ __forceinline__ void attention_issue_tile(const AttnParams &p, const int *table, float *stage, int kvh,
                                                     int p0, int end)
{
    float *ks = stage, *vs = stage + kTile * kKPad;
    const int page = table[p0 / kPage], slot0 = p0 % kPage;
    const float *kb = p.kv + kv_offset(p.layer, p.num_pages, page, 0, kvh, slot0);
    const float *vb = p.kv + kv_offset(p.layer, p.num_pages, page, 1, kvh, slot0);
    const int rows = end - p0;
#pragma unroll 4
    for (int c = threadIdx.x; c < kTile * 32; c += blockDim.x) {
        const int row = c >> 5, chunk = c & 31;
        const bool in = row < rows;
        cp_async16(ks + row * kKPad + chunk * 4, in ? kb + row * kHeadDim + chunk * 4 : kb, in);
        cp_async16(vs + row * kHeadDim + chunk * 4, in ? vb + row * kHeadDim + chunk * 4 : vb, in);
    }
    cp_async_commit();
}

// Kernels defined in headers have internal linkage: each translation unit that
// launches one compiles its own copy.
static __global__ void __launch_bounds__(128) attention_split_kernel(AttnParams p)
{
    extern __shared__ float4 attn_smem4[];
    float *sm = reinterpret_cast<float *>(attn_smem4);
    float *qs = sm;  // [4][128]
    float *stages = sm + 4 * kHeadDim;
    const int split = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = kvh * 4 + warp;
    pdl_wait();  // q and the newest K/V rows come from the previous kernel
    pdl_launch_dependents();
    const int total = p.positions ? p.positions[t] + 1
                                  : (p.step ? p.step->length : p.length) + p.token_offset + t + 1;
    const int *table = p.positions ? p.page_table + (size_t)p.token_table[t] * p.table_stride : p.page_table;
    const int begin = split * p.split_len;
    const int end = min(begin + p.split_len, total);
    const int tiles = end > begin ? (end - begin + kTile - 1) / kTile : 0;
    if (tiles > 0) attention_issue_tile(p, table, stages, kvh, begin, end);

    for (int i = threadIdx.x; i < 4 * kHeadDim; i += blockDim.x)
        qs[i] = p.q[(size_t)t * kQuery + kvh * 4 * kHeadDim + i];

    float m_run = -INFINITY, l_run = 0.0f;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int it = 0; it < tiles; it++) {
        const int p0 = begin + it * kTile;
        if (it + 1 < tiles)
            attention_issue_tile(p, table, stages + ((it + 1) & 1) * kStageFloats, kvh, p0 + kTile, end);
        else cp_async_commit();  // empty group keeps the wait count uniform
        cp_async_wait_one();
        __syncthreads();
        const float *ks = stages + (it & 1) * kStageFloats;
        const float *vs = ks + kTile * kKPad;
        // scores: lane -> position p0 + lane
        float s = -INFINITY;
        if (p0 + lane < end) {
            float dot = 0.0f;
#pragma unroll
            for (int c = 0; c < 32; c++) {
                float4 kk = *reinterpret_cast<const float4 *>(ks + lane * kKPad + c * 4);
                float4 qa = *reinterpret_cast<const float4 *>(qs + warp * kHeadDim + c * 4);
                dot = fmaf(qa.x, kk.x, dot);
                dot = fmaf(qa.y, kk.y, dot);
                dot = fmaf(qa.z, kk.z, dot);
                dot = fmaf(qa.w, kk.w, dot);
            }
            s = dot * kScoreScale;
        }
        float m_new = fmaxf(m_run, warp_max(s));
        float correction = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
        float prob = s == -INFINITY ? 0.0f : expf(s - m_new);
        l_run = l_run * correction + warp_sum(prob);
        m_run = m_new;
#pragma unroll
        for (int d = 0; d < 4; d++) o[d] *= correction;
        const int rows = min(kTile, end - p0);
        for (int j = 0; j < rows; j++) {
            float pj = __shfl_sync(0xffffffffu, prob, j);
            float4 vv = *reinterpret_cast<const float4 *>(vs + j * kHeadDim + lane * 4);
            o[0] = fmaf(pj, vv.x, o[0]);
            o[1] = fmaf(pj, vv.y, o[1]);
            o[2] = fmaf(pj, vv.z, o[2]);
            o[3] = fmaf(pj, vv.w, o[3]);
        }
        __syncthreads();  // this stage is refilled two iterations later
    }
    if (p.splits == 1) {
        float inv = 1.0f / l_run;
        float4 r = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
        *reinterpret_cast<float4 *>(&p.out[(size_t)t * kQuery + head * kHeadDim + lane * 4]) = r;
    } else {
        size_t slot = ((size_t)t * kQueryHeads + head) * p.splits + split;
        *reinterpret_cast<float4 *>(&p.part_acc[slot * kHeadDim + lane * 4]) =
            make_float4(o[0], o[1], o[2], o[3]);
        if (lane == 0) {
            p.part_ml[slot * 2] = m_run;
            p.part_ml[slot * 2 + 1] = l_run;
        }
    }
}

// grid (32 heads, count), block 128 (one thread per dim).
static __global__ void __launch_bounds__(128) attention_combine_kernel(AttnParams p)
{
    const int head = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    const size_t base = ((size_t)t * kQueryHeads + head) * p.splits;
    float m = -INFINITY;
    for (int s = 0; s < p.splits; s++) {
        if (p.part_ml[(base + s) * 2 + 1] > 0.0f) m = fmaxf(m, p.part_ml[(base + s) * 2]);
    }
    float l = 0.0f, acc = 0.0f;
    for (int s = 0; s < p.splits; s++) {
        float ls = p.part_ml[(base + s) * 2 + 1];
        if (ls > 0.0f) {
            float w = expf(p.part_ml[(base + s) * 2] - m);
            l += ls * w;
            acc += p.part_acc[(base + s) * kHeadDim + d] * w;
        }
    }
    p.out[(size_t)t * kQuery + head * kHeadDim + d] = acc / l;
}

// ---- blocks of query tokens (prefill, append) ------------------------------------
// One block per (8 query tokens, KV head): the 32 query rows (8 tokens x the
// 4 query heads of the GQA group, row 4 * token + head) stream the causal K/V
// range once, a 64-position page at a time, instead of once per token. K and V
// tiles arrive by cp.async (a page of one head is 32 KB contiguous per kind);
// the next tile's K loads during this tile's P V and the next V during the
// next S, so one buffer each suffices. S = Q K^T and O += P V run as 4 x 4 and
// 4 x 8 register tiles per thread: thread (rg, cg) owns rows 4rg..4rg+3, keys
// cg + 16j (conflict-free 16-byte reads of the padded K rows) and dims
// 8cg..8cg+7; the online softmax of a row lives in the 16 threads of a half
// warp, the same in both phases.
constexpr int kPfTokens = 8;                    // query tokens per block
constexpr int kPfRows = 4 * kPfTokens;          // 32 query rows
constexpr int kPfKeys = kPage;                  // positions per K/V tile (one page)
constexpr int kPfRowStride = kHeadDim + 4;      // padded Q and K rows (floats)
constexpr int kPfPStride = kPfRows + 4;         // P^T row
constexpr int kPfThreads = 128;
constexpr int kPfSmemFloats =
    kPfRows * kPfRowStride + kPfKeys * kPfRowStride + kPfKeys * kHeadDim + kPfKeys * kPfPStride;
constexpr int kPfSmemBytes = kPfSmemFloats * 4;

// Copy rows [0, keys) of a 64 x 128 tile (zero the rest) into rows of `stride` floats.
__device__ __forceinline__ void pf_issue_tile(float *dst, const float *src, int keys, int stride)
{
    for (int i = threadIdx.x; i < kPfKeys * (kHeadDim / 4); i += kPfThreads) {
        const int row = i >> 5, c = i & 31;
        const bool in = row < keys;
        cp_async16(dst + row * stride + 4 * c, in ? src + (size_t)row * kHeadDim + 4 * c : src, in);
    }
    cp_async_commit();
}

// Grid (ceil(count / 8), 8 KV heads, splits), 128 threads. Split s covers the
// keys [s * split_len, (s + 1) * split_len) of the causal range (split_len a
// multiple of 64); with one split the block writes the output, otherwise
// (m, l, unnormalised o) per row for attention_combine_kernel.
static __global__ void __launch_bounds__(kPfThreads) attention_prefill_kernel(AttnParams p, int count)
{
    extern __shared__ float4 pf_smem4[];
    float *qs = reinterpret_cast<float *>(pf_smem4);     // [32][kPfRowStride]
    float *ks = qs + kPfRows * kPfRowStride;             // [64][kPfRowStride]
    float *vs = ks + kPfKeys * kPfRowStride;             // [64][128]
    float *pt = vs + kPfKeys * kHeadDim;                 // [64][kPfPStride]: P^T of the tile
    const int kvh = blockIdx.y, t0 = blockIdx.x * kPfTokens, tid = threadIdx.x;
    const int rg = tid >> 4, cg = tid & 15;
    pdl_wait();
    pdl_launch_dependents();
    const int length = (p.step ? p.step->length : p.length) + p.token_offset;
    const int last = min(t0 + kPfTokens, count) - 1;      // last query token of the block
    const int split = blockIdx.z;
    const int k0 = split * p.split_len;                   // first key of this split
    const int total = min(length + last + 1, k0 + p.split_len);  // keys the block needs (end)
    const int tiles = total > k0 ? (total - k0 + kPfKeys - 1) / kPfKeys : 0;

    auto kv_tile = [&](int tile, int kind) {
        const int page = p.page_table[k0 / kPfKeys + tile];
        return p.kv + kv_offset(p.layer, p.num_pages, page, kind, kvh, 0);
    };
    if (tiles > 0) {
        pf_issue_tile(ks, kv_tile(0, 0), min(kPfKeys, total - k0), kPfRowStride);
        pf_issue_tile(vs, kv_tile(0, 1), min(kPfKeys, total - k0), kHeadDim);
    }
    for (int i = tid; i < kPfRows * kHeadDim / 4; i += kPfThreads) {
        const int r = i >> 5, c = i & 31, tk = r >> 2, hh = r & 3;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + tk < count)
            v = *reinterpret_cast<const float4 *>(p.q + (size_t)(t0 + tk) * kQuery + (kvh * 4 + hh) * kHeadDim + 4 * c);
        *reinterpret_cast<float4 *>(qs + r * kPfRowStride + 4 * c) = v;
    }
    // the causal limit of each of this thread's rows: key position <= length + token
    int limit[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int tk = t0 + ((4 * rg + i) >> 2);
        limit[i] = tk < count ? length + tk : -1;
    }
    float m_run[4], l_run[4], o[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m_run[i] = -INFINITY;
        l_run[i] = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; e++) o[i][e] = 0.0f;
    }
    for (int tile = 0; tile < tiles; tile++) {
        const int p0 = k0 + tile * kPfKeys, keys = min(kPfKeys, total - p0);
        cp_async_wait_one();  // K of this tile (its V may still be in flight)
        __syncthreads();
        // S = Q K^T for rows 4rg.., keys p0 + cg + 16j
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[i][j] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < kHeadDim; d += 4) {
            float4 a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = *reinterpret_cast<const float4 *>(qs + (4 * rg + i) * kPfRowStride + d);
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = *reinterpret_cast<const float4 *>(ks + (cg + 16 * j) * kPfRowStride + d);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    s[i][j] = fmaf(a[i].x, b[j].x, s[i][j]);
                    s[i][j] = fmaf(a[i].y, b[j].y, s[i][j]);
                    s[i][j] = fmaf(a[i].z, b[j].z, s[i][j]);
                    s[i][j] = fmaf(a[i].w, b[j].w, s[i][j]);
                }
        }
        __syncthreads();  // K consumed: the next tile's K may load
        if (tile + 1 < tiles)
            pf_issue_tile(ks, kv_tile(tile + 1, 0), min(kPfKeys, total - p0 - kPfKeys), kPfRowStride);
        else
            cp_async_commit();
        // online softmax per row over the 16 threads of the half warp
        float prob[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int pos = p0 + cg + 16 * j;
                s[i][j] = pos <= limit[i] ? s[i][j] * kScoreScale : -INFINITY;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_run[i], mx);
            const float corr = m_run[i] == -INFINITY ? 0.0f : expf(m_run[i] - m_new);
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                prob[i][j] = s[i][j] == -INFINITY ? 0.0f : expf(s[i][j] - m_new);
                sum += prob[i][j];
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l_run[i] = l_run[i] * corr + sum;
            m_run[i] = m_new;
#pragma unroll
            for (int e = 0; e < 8; e++) o[i][e] *= corr;
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            *reinterpret_cast<float4 *>(pt + (cg + 16 * j) * kPfPStride + 4 * rg) =
                make_float4(prob[0][j], prob[1][j], prob[2][j], prob[3][j]);
        cp_async_wait_one();  // V of this tile (the next K may still be in flight)
        __syncthreads();
        // O += P V for rows 4rg.., dims 8cg..8cg+7
#pragma unroll 4
        for (int j = 0; j < keys; j++) {
            const float4 pj = *reinterpret_cast<const float4 *>(pt + j * kPfPStride + 4 * rg);
            const float4 v0 = *reinterpret_cast<const float4 *>(vs + j * kHeadDim + 8 * cg);
            const float4 v1 = *reinterpret_cast<const float4 *>(vs + j * kHeadDim + 8 * cg + 4);
            const float pv[4] = {pj.x, pj.y, pj.z, pj.w};
            const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int e = 0; e < 8; e++) o[i][e] = fmaf(pv[i], vv[e], o[i][e]);
        }
        __syncthreads();  // V and P consumed: the next tile's V may load
        if (tile + 1 < tiles)
            pf_issue_tile(vs, kv_tile(tile + 1, 1), min(kPfKeys, total - p0 - kPfKeys), kHeadDim);
        else
            cp_async_commit();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = 4 * rg + i, tk = t0 + (r >> 2), head = kvh * 4 + (r & 3);
        if (tk >= count) continue;
        if (p.splits == 1) {
            const float inv = 1.0f / l_run[i];
            float *dst = p.out + (size_t)tk * kQuery + head * kHeadDim + 8 * cg;
            *reinterpret_cast<float4 *>(dst) =
                make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
            *reinterpret_cast<float4 *>(dst + 4) =
                make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
        } else {
            // a split past this token's causal range leaves l = 0 (the combine skips it)
            const size_t slot = ((size_t)tk * kQueryHeads + head) * p.splits + split;
            float *dst = p.part_acc + slot * kHeadDim + 8 * cg;
            *reinterpret_cast<float4 *>(dst) = make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
            *reinterpret_cast<float4 *>(dst + 4) = make_float4(o[i][4], o[i][5], o[i][6], o[i][7]);
            if (cg == 0) {
                p.part_ml[slot * 2] = m_run[i];
                p.part_ml[slot * 2 + 1] = l_run[i];
            }
        }
    }
}

// ---- KV prefix copy / remap ---------------------------------------------------------
// Copies KV pages of the pool: for pair i, every layer's K and V rows of page
// src_pages[i] go to page dst_pages[i] (slots [0, 64), or [0, last_slots) for
// the last pair). A sequence that forks from another shares its full pages
// through the page table and copies only the partial last page (copy on write),
// or copies its whole prefix to pages of its own. Grid (pairs, layers * 16):
// one block per (pair, layer, kind, KV head) segment of up to 32 KB.
struct KvCopyParams {
    float *kv;
    int num_pages;
    const int *src_pages, *dst_pages;
    int pairs, last_slots;
};

static __global__ void __launch_bounds__(256) kv_copy_kernel(KvCopyParams p)
{
    const int i = blockIdx.x, seg = blockIdx.y;
    const int layer = seg >> 4, kind = (seg >> 3) & 1, head = seg & 7;
    const int slots = i == p.pairs - 1 ? p.last_slots : kPage;
    const float4 *src =
        reinterpret_cast<const float4 *>(p.kv + kv_offset(layer, p.num_pages, p.src_pages[i], kind, head, 0));
    float4 *dst = reinterpret_cast<float4 *>(p.kv + kv_offset(layer, p.num_pages, p.dst_pages[i], kind, head, 0));
    const int n = slots * (kHeadDim / 4);
    for (int j = threadIdx.x; j < n; j += blockDim.x) dst[j] = __ldcg(src + j);
}

// x[t][c] = widen(E[ids[t]][c]) for the call's tokens (src/metal_runtime.m:391-395).
static __global__ void embed_kernel(const uint16_t *embedding, const StepParams *step, float *x,
                             int count)
{
    const int t = blockIdx.x;
    pdl_wait();  // ids come from the host copy or the previous step's greedy kernel
    pdl_launch_dependents();
    if (t >= count) return;
    const uint16_t *row = embedding + (size_t)step->ids[t] * kHidden;
    for (int c = threadIdx.x; c < kHidden / 2; c += blockDim.x) {
        uint32_t w = reinterpret_cast<const uint32_t *>(row)[c];
        x[(size_t)t * kHidden + 2 * c] = bf16_lo(w);
        x[(size_t)t * kHidden + 2 * c + 1] = bf16_hi(w);
    }
}

}  // namespace lun
