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
};

constexpr int kTile = 32;
constexpr int kKPad = 132;  // padded K row (floats): conflict-free 16-byte reads across lanes

// Kernels defined in headers have internal linkage: each translation unit that
// launches one compiles its own copy.
static __global__ void __launch_bounds__(128) attention_split_kernel(AttnParams p)
{
    __shared__ __align__(16) float qs[4][kHeadDim];
    __shared__ __align__(16) float ks[kTile][kKPad];
    __shared__ __align__(16) float vs[kTile][kHeadDim];
    const int split = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = kvh * 4 + warp;
    const int total = (p.step ? p.step->length : p.length) + p.token_offset + t + 1;
    const int begin = split * p.split_len;
    const int end = min(begin + p.split_len, total);

    for (int i = threadIdx.x; i < 4 * kHeadDim; i += blockDim.x)
        qs[i / kHeadDim][i % kHeadDim] = p.q[(size_t)t * kQuery + kvh * 4 * kHeadDim + i];

    float m_run = -INFINITY, l_run = 0.0f;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int p0 = begin; p0 < end; p0 += kTile) {
        __syncthreads();
        // cooperative tile load: 32 rows x 512 B for K and for V = 2048 16-byte chunks
        for (int c = threadIdx.x; c < 2 * kTile * 32; c += blockDim.x) {
            int kind = c >> 10, row = (c >> 5) & 31, chunk = c & 31;
            int pos = p0 + row;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (pos < end) {
                int page = p.page_table[pos / kPage];
                const float *src = p.kv + kv_offset(p.layer, p.num_pages, page, kind, kvh,
                                                    pos % kPage);
                v = *reinterpret_cast<const float4 *>(src + chunk * 4);
            }
            if (kind == 0) *reinterpret_cast<float4 *>(&ks[row][chunk * 4]) = v;
            else *reinterpret_cast<float4 *>(&vs[row][chunk * 4]) = v;
        }
        __syncthreads();
        // scores: lane -> position p0 + lane
        float s = -INFINITY;
        if (p0 + lane < end) {
            float dot = 0.0f;
#pragma unroll
            for (int c = 0; c < 32; c++) {
                float4 kk = *reinterpret_cast<const float4 *>(&ks[lane][c * 4]);
                float4 qa = *reinterpret_cast<const float4 *>(&qs[warp][c * 4]);
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
            float4 vv = *reinterpret_cast<const float4 *>(&vs[j][lane * 4]);
            o[0] = fmaf(pj, vv.x, o[0]);
            o[1] = fmaf(pj, vv.y, o[1]);
            o[2] = fmaf(pj, vv.z, o[2]);
            o[3] = fmaf(pj, vv.w, o[3]);
        }
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

// x[t][c] = widen(E[ids[t]][c]) for the call's tokens (src/metal_runtime.m:391-395).
static __global__ void embed_kernel(const uint16_t *embedding, const StepParams *step, float *x,
                             int count)
{
    const int t = blockIdx.x;
    if (t >= count) return;
    const uint16_t *row = embedding + (size_t)step->ids[t] * kHidden;
    for (int c = threadIdx.x; c < kHidden / 2; c += blockDim.x) {
        uint32_t w = reinterpret_cast<const uint32_t *>(row)[c];
        x[(size_t)t * kHidden + 2 * c] = bf16_lo(w);
        x[(size_t)t * kHidden + 2 * c + 1] = bf16_hi(w);
    }
}

}  // namespace lun
