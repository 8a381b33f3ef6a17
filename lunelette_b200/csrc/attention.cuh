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
    int *error;  // set when the tensor-core kernel's bounded waits give up (nullptr: not reported)
};

constexpr int kTile = 32;
constexpr int kKPad = 132;  // padded K row (floats): conflict-free 16-byte reads across lanes
constexpr int kStageFloats = kTile * kKPad + kTile * kHeadDim;
// dynamic shared memory: the warps' merge area (4 x 4 x 128 o + 32 m/l) + two K/V tile stages
constexpr int kAttnSmemBytes = (4 * 4 * kHeadDim + 32 + 2 * kStageFloats) * 4;

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
    float *merge = sm;                     // [4 warps][4 heads][128] partial o, then [4][4][2] (m, l)
    float *stages = sm + 4 * kHeadDim * 4 + 32;
    const int split = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();  // q and the newest K/V rows come from the previous kernel
    pdl_launch_dependents();
    const int total = p.positions ? p.positions[t] + 1
                                  : (p.step ? p.step->length : p.length) + p.token_offset + t + 1;
    const int *table = p.positions ? p.page_table + (size_t)p.token_table[t] * p.table_stride : p.page_table;
    const int begin = split * p.split_len;
    const int end = min(begin + p.split_len, total);
    const int tiles = end > begin ? (end - begin + kTile - 1) / kTile : 0;
    if (tiles > 0) attention_issue_tile(p, table, stages, kvh, begin, end);

    // every warp holds the four query heads of the group, lane l owning dims 4l..4l+3;
    // warp w takes positions 8w..8w+7 of each tile, so K and V are read once per block
    float4 q[4];
#pragma unroll
    for (int h = 0; h < 4; h++)
        q[h] = *reinterpret_cast<const float4 *>(p.q + (size_t)t * kQuery + (kvh * 4 + h) * kHeadDim + 4 * lane);
    float m_run = -INFINITY, l_run = 0.0f;  // of head lane & 3, over this warp's positions
    float4 o[4];
#pragma unroll
    for (int h = 0; h < 4; h++) o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int it = 0; it < tiles; it++) {
        const int p0 = begin + it * kTile;
        if (it + 1 < tiles)
            attention_issue_tile(p, table, stages + ((it + 1) & 1) * kStageFloats, kvh, p0 + kTile, end);
        else cp_async_commit();  // empty group keeps the wait count uniform
        cp_async_wait_one();
        __syncthreads();
        const float *ks = stages + (it & 1) * kStageFloats;
        const float *vs = ks + kTile * kKPad;
        // partial dots of (position j, head h) over this lane's dims, index 4 j + h
        float d[32];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 k4 = *reinterpret_cast<const float4 *>(ks + (8 * warp + j) * kKPad + 4 * lane);
#pragma unroll
            for (int h = 0; h < 4; h++)
                d[4 * j + h] = fmaf(q[h].x, k4.x, fmaf(q[h].y, k4.y, fmaf(q[h].z, k4.z, q[h].w * k4.w)));
        }
        // reduce-scatter over the warp: lane l ends with the full dot of index l
#pragma unroll
        for (int width = 16; width >= 1; width >>= 1) {
            const bool upper = (lane & width) != 0;
#pragma unroll
            for (int i = 0; i < width; i++) {
                const float mine = upper ? d[i + width] : d[i];
                const float other = upper ? d[i] : d[i + width];
                d[i] = mine + __shfl_xor_sync(0xffffffffu, other, width);
            }
        }
        // lane l: position p0 + 8 warp + (l >> 2), head l & 3
        const int pos = p0 + 8 * warp + (lane >> 2);
        const float sc = pos < end ? d[0] * kScoreScale : -INFINITY;
        float tmax = sc;
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
        const float m_new = fmaxf(m_run, tmax);
        const float corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
        const float prob = sc == -INFINITY ? 0.0f : expf(sc - m_new);
        float psum = prob;
        psum += __shfl_xor_sync(0xffffffffu, psum, 4);
        psum += __shfl_xor_sync(0xffffffffu, psum, 8);
        psum += __shfl_xor_sync(0xffffffffu, psum, 16);
        l_run = l_run * corr + psum;
        m_run = m_new;
        // O += P V for this warp's positions; head h's factors sit in lanes h, h + 4, ...
#pragma unroll
        for (int h = 0; h < 4; h++) {
            const float c = __shfl_sync(0xffffffffu, corr, h);
            o[h].x *= c;
            o[h].y *= c;
            o[h].z *= c;
            o[h].w *= c;
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 v4 = *reinterpret_cast<const float4 *>(vs + (8 * warp + j) * kHeadDim + 4 * lane);
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const float pj = __shfl_sync(0xffffffffu, prob, 4 * j + h);
                o[h].x = fmaf(pj, v4.x, o[h].x);
                o[h].y = fmaf(pj, v4.y, o[h].y);
                o[h].z = fmaf(pj, v4.z, o[h].z);
                o[h].w = fmaf(pj, v4.w, o[h].w);
            }
        }
        __syncthreads();  // this stage is refilled two iterations later
    }
    // merge the four warps' (m, l, o) per head in warp order; warp h writes head h
    float *ml = merge + 4 * 4 * kHeadDim;
#pragma unroll
    for (int h = 0; h < 4; h++)
        *reinterpret_cast<float4 *>(merge + (warp * 4 + h) * kHeadDim + 4 * lane) = o[h];
    if (lane < 4) {
        ml[(warp * 4 + lane) * 2] = m_run;
        ml[(warp * 4 + lane) * 2 + 1] = l_run;
    }
    __syncthreads();
    const int h = warp, head = kvh * 4 + h;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; w++)
        if (ml[(w * 4 + h) * 2 + 1] > 0.0f) M = fmaxf(M, ml[(w * 4 + h) * 2]);
    float L = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 4; w++) {
        const float lw = ml[(w * 4 + h) * 2 + 1];
        if (!(lw > 0.0f)) continue;
        const float wt = expf(ml[(w * 4 + h) * 2] - M);
        const float4 v = *reinterpret_cast<const float4 *>(merge + (w * 4 + h) * kHeadDim + 4 * lane);
        L = fmaf(wt, lw, L);
        acc.x = fmaf(wt, v.x, acc.x);
        acc.y = fmaf(wt, v.y, acc.y);
        acc.z = fmaf(wt, v.z, acc.z);
        acc.w = fmaf(wt, v.w, acc.w);
    }
    if (p.splits == 1) {
        const float inv = 1.0f / L;
        *reinterpret_cast<float4 *>(&p.out[(size_t)t * kQuery + head * kHeadDim + lane * 4]) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    } else {
        // an empty split leaves l = 0 and m = -inf (the combine skips it)
        size_t slot = ((size_t)t * kQueryHeads + head) * p.splits + split;
        *reinterpret_cast<float4 *>(&p.part_acc[slot * kHeadDim + lane * 4]) = acc;
        if (lane == 0) {
            p.part_ml[slot * 2] = M;
            p.part_ml[slot * 2 + 1] = L;
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

// ---- blocks of query tokens (prefill, append) on the tensor cores ----------------------
// One block per (32 query tokens, KV head) and key range: the 128 query rows
// (32 tokens x the 4 query heads of the GQA group) stream the causal K/V range
// once, instead of once per token. Split s covers the keys [s * split_len,
// (s + 1) * split_len) of the causal range (split_len a multiple of 64); with
// one split the block writes the output, otherwise (m, l, unnormalised o) per
// row for attention_combine_kernel. S = Q K^T and O += P V run on
// mma.sync.m16n8k16 in FP16: every FP32 operand x is split into hi = fp16(x)
// and lo = fp16(x - hi) (22 significant bits together) and each product takes
// three MMAs (hi.hi + hi.lo + lo.hi, FP32 accumulation), so S and O keep
// near-FP32 accuracy. Block: 8 warps x 16 rows (4 query tokens x the 4 query
// heads of KV head blockIdx.y); keys stream in tiles of 32 (half a page): the
// FP32 K and V rows are copied (cp.async), converted once per tile into FP16
// hi/lo parts (K row-major, V transposed, both padded so the fragment loads are
// conflict-free) shared by the block's 8 warps, and the next tile's copy
// overlaps this tile's MMAs. The online softmax (running max, rescaled sum
// and output, exp of the scaled scores) runs on the S fragments: a row's 32
// keys sit in one lane quad.
constexpr int kPmWarps = 8;                                     // 16 rows (4 tokens x 4 heads) each
constexpr int kPmTokens = 4 * kPmWarps;                         // query tokens per block
constexpr int kPmThreads = 32 * kPmWarps;
constexpr int kPmKeys = 32;                                     // keys per tile
constexpr int kPmKStride = kHeadDim + 8;                        // halves per K row
constexpr int kPmVStride = kPmKeys + 8;                         // halves per V^T row
constexpr int kPmStageBytes = 2 * kPmKeys * kHeadDim * 4;       // FP32 K and V of a tile
constexpr int kPmKBytes = kPmKeys * kPmKStride * 2;             // one FP16 part of K
constexpr int kPmVBytes = kHeadDim * kPmVStride * 2;            // one FP16 part of V^T
constexpr int kPmSmemBytes = kPmStageBytes + 2 * kPmKBytes + 2 * kPmVBytes;

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// (a, b) -> FP16x2 hi = round(a, b) and lo = round(a - hi, b - hi): packed conversions
__device__ __forceinline__ void split_half2(float a, float b, uint32_t &hi, uint32_t &lo)
{
    const __half2 h = __floats2half2_rn(a, b);
    const float2 back = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - back.x, b - back.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Grid (ceil(count / 32), 8 KV heads, splits), 256 threads, kPmSmemBytes.
static __global__ void __launch_bounds__(kPmThreads) attention_prefill_mma_kernel(AttnParams p, int count)
{
    extern __shared__ __align__(16) uint8_t pm_smem[];
    float *stage_k = reinterpret_cast<float *>(pm_smem);  // [32][128] FP32
    float *stage_v = stage_k + kPmKeys * kHeadDim;        // [32][128] FP32
    __half *kh = reinterpret_cast<__half *>(pm_smem + kPmStageBytes);  // [32][kPmKStride]
    __half *kl = kh + kPmKeys * kPmKStride;
    __half *vth = kl + kPmKeys * kPmKStride;  // [128][kPmVStride]: V^T
    __half *vtl = vth + kHeadDim * kPmVStride;
    const int kvh = blockIdx.y, t0 = blockIdx.x * kPmTokens, split = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    pdl_wait();
    pdl_launch_dependents();
    const int length = (p.step ? p.step->length : p.length) + p.token_offset;
    const int last = min(t0 + kPmTokens, count) - 1;  // last query token of the block
    const int k0 = split * p.split_len;               // first key of this split
    const int total = min(length + last + 1, k0 + p.split_len);
    const int tiles = total > k0 ? (total - k0 + kPmKeys - 1) / kPmKeys : 0;

    // rows [0, keys) of the 32-key tile at p0 (one page holds it), the rest zero
    auto issue = [&](int p0) {
        const int page = p.page_table[p0 / kPage], slot0 = p0 % kPage;
        const float *kb = p.kv + kv_offset(p.layer, p.num_pages, page, 0, kvh, slot0);
        const float *vb = p.kv + kv_offset(p.layer, p.num_pages, page, 1, kvh, slot0);
        const int keys = min(kPmKeys, total - p0);
#pragma unroll 4
        for (int i = threadIdx.x; i < kPmKeys * (kHeadDim / 4); i += kPmThreads) {
            const int row = i >> 5, c = i & 31;
            const bool in = row < keys;
            cp_async16(stage_k + row * kHeadDim + 4 * c, in ? kb + row * kHeadDim + 4 * c : kb, in);
            cp_async16(stage_v + row * kHeadDim + 4 * c, in ? vb + row * kHeadDim + 4 * c : vb, in);
        }
        cp_async_commit();
    };
    if (tiles > 0) issue(k0);

    // this warp's rows: r = g (token ta) and g + 8 (token tb), head kvh * 4 + (g & 3)
    const int head = kvh * 4 + (g & 3);
    const int ta = t0 + 4 * warp + (g >> 2), tb = ta + 2;
    const int limit_a = ta < count ? length + ta : -1, limit_b = tb < count ? length + tb : -1;
    // Q as A fragments, hi and lo, per k16 step of the head dimension
    uint32_t qh[8][4], ql[8][4];
    {
        const float *qa = p.q + (size_t)(ta < count ? ta : 0) * kQuery + head * kHeadDim;
        const float *qb = p.q + (size_t)(tb < count ? tb : 0) * kQuery + head * kHeadDim;
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
            const int d = 16 * ks + 2 * t4;
            float2 v[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            if (ta < count) {
                v[0] = *reinterpret_cast<const float2 *>(qa + d);
                v[2] = *reinterpret_cast<const float2 *>(qa + d + 8);
            }
            if (tb < count) {
                v[1] = *reinterpret_cast<const float2 *>(qb + d);
                v[3] = *reinterpret_cast<const float2 *>(qb + d + 8);
            }
#pragma unroll
            for (int r = 0; r < 4; r++) split_half2(v[r].x, v[r].y, qh[ks][r], ql[ks][r]);
        }
    }
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
    float o[16][4];
#pragma unroll
    for (int nb = 0; nb < 16; nb++) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.0f;

    for (int tile = 0; tile < tiles; tile++) {
        const int p0 = k0 + tile * kPmKeys;
        cp_async_wait_all();
        __syncthreads();  // the tile is staged; every warp is done with the last tile's FP16 parts
        // K: [key][dim] hi/lo; V: transposed [dim][key] hi/lo, two keys per store
        for (int i = threadIdx.x; i < kPmKeys * (kHeadDim / 4); i += kPmThreads) {
            const int row = i >> 5, c = i & 31;
            const float4 k4 = *reinterpret_cast<const float4 *>(stage_k + row * kHeadDim + 4 * c);
            uint2 hi, lo;
            split_half2(k4.x, k4.y, hi.x, lo.x);
            split_half2(k4.z, k4.w, hi.y, lo.y);
            *reinterpret_cast<uint2 *>(kh + row * kPmKStride + 4 * c) = hi;
            *reinterpret_cast<uint2 *>(kl + row * kPmKStride + 4 * c) = lo;
        }
        for (int i = threadIdx.x; i < (kPmKeys / 2) * kHeadDim; i += kPmThreads) {
            const int d = i & (kHeadDim - 1), kp = i >> 7;
            uint32_t hi, lo;
            split_half2(stage_v[(2 * kp) * kHeadDim + d], stage_v[(2 * kp + 1) * kHeadDim + d], hi, lo);
            *reinterpret_cast<uint32_t *>(vth + d * kPmVStride + 2 * kp) = hi;
            *reinterpret_cast<uint32_t *>(vtl + d * kPmVStride + 2 * kp) = lo;
        }
        __syncthreads();  // parts ready, staging free
        if (tile + 1 < tiles) issue(p0 + kPmKeys);

        // S = Q K^T: 4 key blocks of 8 x 8 k16 steps, three MMAs each; the
        // blocks interleave so consecutive MMAs never feed one another
        float s[4][4];
#pragma unroll
        for (int nb = 0; nb < 4; nb++) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
            uint32_t bh[4][2], bl[4][2];
#pragma unroll
            for (int nb = 0; nb < 4; nb++) {
                const int off = (nb * 8 + g) * kPmKStride + 16 * ks + 2 * t4;
                bh[nb][0] = *reinterpret_cast<const uint32_t *>(kh + off);
                bh[nb][1] = *reinterpret_cast<const uint32_t *>(kh + off + 8);
                bl[nb][0] = *reinterpret_cast<const uint32_t *>(kl + off);
                bl[nb][1] = *reinterpret_cast<const uint32_t *>(kl + off + 8);
            }
#pragma unroll
            for (int nb = 0; nb < 4; nb++) mma_16816(s[nb], qh[ks], bh[nb][0], bh[nb][1]);
#pragma unroll
            for (int nb = 0; nb < 4; nb++) mma_16816(s[nb], qh[ks], bl[nb][0], bl[nb][1]);
#pragma unroll
            for (int nb = 0; nb < 4; nb++) mma_16816(s[nb], ql[ks], bh[nb][0], bh[nb][1]);
        }
        // mask, scale, online softmax; lane quad (g, t4 = 0..3) holds rows g / g + 8, keys 8 nb + 2 t4 (+1)
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int nb = 0; nb < 4; nb++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int pos = p0 + 8 * nb + 2 * t4 + e;
                s[nb][e] = pos <= limit_a ? s[nb][e] * kScoreScale : -INFINITY;
                s[nb][2 + e] = pos <= limit_b ? s[nb][2 + e] * kScoreScale : -INFINITY;
                mx_a = fmaxf(mx_a, s[nb][e]);
                mx_b = fmaxf(mx_b, s[nb][2 + e]);
            }
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float corr_a = m_a == -INFINITY ? 0.0f : expf(m_a - mn_a);
        const float corr_b = m_b == -INFINITY ? 0.0f : expf(m_b - mn_b);
        float sum_a = 0.0f, sum_b = 0.0f;
#pragma unroll
        for (int nb = 0; nb < 4; nb++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                s[nb][e] = s[nb][e] == -INFINITY ? 0.0f : expf(s[nb][e] - mn_a);
                s[nb][2 + e] = s[nb][2 + e] == -INFINITY ? 0.0f : expf(s[nb][2 + e] - mn_b);
                sum_a += s[nb][e];
                sum_b += s[nb][2 + e];
            }
        }
        sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 1);
        sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 2);
        sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 1);
        sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 2);
        l_a = l_a * corr_a + sum_a;
        l_b = l_b * corr_b + sum_b;
        m_a = mn_a;
        m_b = mn_b;
#pragma unroll
        for (int nb = 0; nb < 16; nb++) {
            o[nb][0] *= corr_a;
            o[nb][1] *= corr_a;
            o[nb][2] *= corr_b;
            o[nb][3] *= corr_b;
        }
        // O += P V: P's S fragments are the A fragments of two k16 steps of keys
#pragma unroll
        for (int j = 0; j < 2; j++) {
            uint32_t ph[4], pl[4];
            split_half2(s[2 * j][0], s[2 * j][1], ph[0], pl[0]);
            split_half2(s[2 * j][2], s[2 * j][3], ph[1], pl[1]);
            split_half2(s[2 * j + 1][0], s[2 * j + 1][1], ph[2], pl[2]);
            split_half2(s[2 * j + 1][2], s[2 * j + 1][3], ph[3], pl[3]);
#pragma unroll
            for (int n0 = 0; n0 < 16; n0 += 4) {
                uint32_t bh[4][2], bl[4][2];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int off = ((n0 + u) * 8 + g) * kPmVStride + 16 * j + 2 * t4;
                    bh[u][0] = *reinterpret_cast<const uint32_t *>(vth + off);
                    bh[u][1] = *reinterpret_cast<const uint32_t *>(vth + off + 8);
                    bl[u][0] = *reinterpret_cast<const uint32_t *>(vtl + off);
                    bl[u][1] = *reinterpret_cast<const uint32_t *>(vtl + off + 8);
                }
#pragma unroll
                for (int u = 0; u < 4; u++) mma_16816(o[n0 + u], ph, bh[u][0], bh[u][1]);
#pragma unroll
                for (int u = 0; u < 4; u++) mma_16816(o[n0 + u], ph, bl[u][0], bl[u][1]);
#pragma unroll
                for (int u = 0; u < 4; u++) mma_16816(o[n0 + u], pl, bh[u][0], bh[u][1]);
            }
        }
    }
    // rows g (token ta) and g + 8 (token tb); lane holds dims 8 nb + 2 t4 (+1)
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const int tk = half ? tb : ta;
        if (tk >= count) continue;
        const float l = half ? l_b : l_a, m = half ? m_b : m_a;
        if (p.splits == 1) {
            const float inv = 1.0f / l;
            float *dst = p.out + (size_t)tk * kQuery + head * kHeadDim + 2 * t4;
#pragma unroll
            for (int nb = 0; nb < 16; nb++)
                *reinterpret_cast<float2 *>(dst + 8 * nb) =
                    make_float2(o[nb][2 * half] * inv, o[nb][2 * half + 1] * inv);
        } else {
            // a split past this token's causal range leaves l = 0 (the combine skips it)
            const size_t slot = ((size_t)tk * kQueryHeads + head) * p.splits + split;
            float *dst = p.part_acc + slot * kHeadDim + 2 * t4;
#pragma unroll
            for (int nb = 0; nb < 16; nb++)
                *reinterpret_cast<float2 *>(dst + 8 * nb) = make_float2(o[nb][2 * half], o[nb][2 * half + 1]);
            if (t4 == 0) {
                p.part_ml[slot * 2] = m;
                p.part_ml[slot * 2 + 1] = l;
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
