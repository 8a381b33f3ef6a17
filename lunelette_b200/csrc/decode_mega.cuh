// Persistent cooperative decode kernel: one CTA per SM runs whole batch-1
// decode steps (26 layers, final norm, tied head, greedy pick) with grid-wide
// barriers between the phases of the reference's layer graph
// (src/metal_encode.m:124-215). Per layer:
//   qkv   input norm + q/k/v GEMV + RoPE + KV store          (prefetches o)
//   attn  split-K attention; the last split of a KV head combines (fixed order)
//   o     o GEMV + residual                                  (prefetches gate/up)
//   ffn   post norm + gate/up GEMV + SwiGLU                  (prefetches down)
//   down  down GEMV + residual                               (prefetches next qkv)
// Each phase issues an L2 prefetch of the next matrix before computing, so HBM
// keeps streaming weights through the barriers; the weights themselves never
// depend on activations. Activations produced by other CTAs are read through L2
// (ld.cg / cp.async.cg), never from a possibly stale L1.
//
// Barrier waits are bounded: past kSpinLimit polls a CTA sets *error and stops
// waiting for the rest of the launch; the host then reports a failed call.
#pragma once
#include "attention.cuh"
#include "gemv.cuh"
#include "mega_params.cuh"

namespace lun {

constexpr int kMegaThreads = 512;
constexpr int kMegaWarps = kMegaThreads / 32;
constexpr int kMegaAttnWorkers = kMegaThreads / 128;  // 4-warp workers (one warp per query head)
constexpr int kMegaWorkerFloats = 4 * kHeadDim + kTile * kKPad + kTile * kHeadDim;
constexpr int kMegaSmemBytes = kMegaAttnWorkers * kMegaWorkerFloats * 4;  // >= 9216 floats for x
constexpr unsigned kSpinLimit = 1u << 22;
static_assert(kMegaSmemBytes >= kInner * 4, "x buffer must fit in the attention buffers");



__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_cg_int(const int *p) { return __ldcg(p); }

__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Grid-wide barrier number `target` (1, 2, ...) of this launch.
__device__ __forceinline__ void mega_sync(const MegaParams &p, unsigned target)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        unsigned arrived = atomicAdd(&p.barrier[0], 1u);
        if (arrived == gridDim.x - 1) {
            p.barrier[0] = 0;
            __threadfence();
            atomicExch(&p.barrier[1], target);
        } else {
            unsigned spins = 0;
            while ((int)(ld_acquire_u32(&p.barrier[1]) - target) < 0) {
                if (*(volatile int *)p.error) break;
                if (++spins > kSpinLimit) {
                    atomicExch(p.error, 1);
                    break;
                }
                __nanosleep(32);
            }
        }
        __threadfence();
        if (p.timeline && blockIdx.x == 0 && target <= (unsigned)kMegaBarriersPerStep)
            p.timeline[target] = globaltimer_ns();
    }
    __syncthreads();
}

__device__ __forceinline__ void named_sync(int id, int threads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// One activation row into the GEMV's permuted shared layout (16-column chunks),
// optionally RMS-normalised; src rows come from other CTAs (read through L2) or
// from the BF16 embedding.
__device__ __forceinline__ void mega_load_row(float4 *xs, const float *src, const uint16_t *emb,
                                              const float *gain, int cols, float *red)
{
    const int NQ = cols >> 4;
    float *xf = reinterpret_cast<float *>(xs);
    float rs = 1.0f;
    if (gain) {
        float ss = 0.0f;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            float v = emb ? bf16_lo((uint32_t)emb[c]) : __ldcg(&src[c]);
            ss += v * v;
        }
        ss = block_sum(ss, red);
        rs = rsqrtf(ss / (float)cols + kNormEps);
    }
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float v = emb ? bf16_lo((uint32_t)emb[c]) : __ldcg(&src[c]);
        if (gain) v = gain[c] * (v * rs);
        xf[((size_t)((c >> 2) & 3) * NQ + (c >> 4)) * 4 + (c & 3)] = v;
    }
    __syncthreads();
}

template <int EPI>
__device__ __forceinline__ void mega_gemv(const GemvParams &gp, const float4 *xs)
{
    const int lane = threadIdx.x & 31;
    const int groups = (gp.rows + 3) >> 2;
    const int warps = gridDim.x * kMegaWarps;
    for (int g = blockIdx.x * kMegaWarps + (threadIdx.x >> 5); g < groups; g += warps) {
        float acc[4][1];
        gemv_group<1, EPI>(gp, xs, g, lane, acc);
        gemv_epilogue<1, EPI>(gp, g, lane, acc);
    }
}

// Split-K attention of the step's single query row; worker = 4 warps.
__device__ __forceinline__ void mega_attention(const MegaParams &p, int layer, int length,
                                               float *smem)
{
    const int worker = threadIdx.x >> 7, wt = threadIdx.x & 127;
    const int warp = wt >> 5, lane = threadIdx.x & 31;
    float *qs = smem + worker * kMegaWorkerFloats;
    float *ks = qs + 4 * kHeadDim;
    float *vs = ks + kTile * kKPad;
    __shared__ int last_flag[kMegaAttnWorkers];
    const int total = length + 1;
    const int live = (total + p.split_len - 1) / p.split_len;  // splits holding positions
    const int items = kKVHeads * live;
    for (int item = blockIdx.x * kMegaAttnWorkers + worker; item < items;
         item += gridDim.x * kMegaAttnWorkers) {
        const int kvh = item % kKVHeads, split = item / kKVHeads;
        const int head = kvh * 4 + warp;
        const int begin = split * p.split_len, end = min(begin + p.split_len, total);
        for (int i = wt; i < 4 * kHeadDim; i += 128) qs[i] = __ldcg(&p.q[kvh * 4 * kHeadDim + i]);
        float m_run = -INFINITY, l_run = 0.0f;
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        for (int p0 = begin; p0 < end; p0 += kTile) {
            named_sync(1 + worker, 128);
            for (int c = wt; c < 2 * kTile * 32; c += 128) {
                int kind = c >> 10, row = (c >> 5) & 31, chunk = c & 31;
                int pos = p0 + row;
                bool in = pos < end;
                const float *src = p.kv;
                if (in)
                    src = p.kv + kv_offset(layer, p.num_pages, p.page_table[pos / kPage], kind, kvh,
                                           pos % kPage) + chunk * 4;
                float *dst = kind == 0 ? ks + row * kKPad + chunk * 4 : vs + row * kHeadDim + chunk * 4;
                cp_async16(dst, src, in);
            }
            cp_async_commit();
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            named_sync(1 + worker, 128);
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
        }
        size_t slot = (size_t)head * p.splits + split;
        *reinterpret_cast<float4 *>(&p.part_acc[slot * kHeadDim + lane * 4]) =
            make_float4(o[0], o[1], o[2], o[3]);
        if (lane == 0) {
            p.part_ml[slot * 2] = m_run;
            p.part_ml[slot * 2 + 1] = l_run;
        }
        __threadfence();
        named_sync(1 + worker, 128);
        if (wt == 0) last_flag[worker] = atomicAdd(&p.attn_count[kvh], 1u) == (unsigned)(live - 1);
        named_sync(1 + worker, 128);
        if (last_flag[worker]) {
            // every split of this KV head has written its partials: merge them in
            // split order for the four query heads (thread = head-dim column)
            __threadfence();
            for (int hq = 0; hq < 4; hq++) {
                const size_t base = (size_t)(kvh * 4 + hq) * p.splits;
                float m = -INFINITY;
                for (int s2 = 0; s2 < live; s2++)
                    if (__ldcg(&p.part_ml[(base + s2) * 2 + 1]) > 0.0f)
                        m = fmaxf(m, __ldcg(&p.part_ml[(base + s2) * 2]));
                float l = 0.0f, acc = 0.0f;
                for (int s2 = 0; s2 < live; s2++) {
                    float ls = __ldcg(&p.part_ml[(base + s2) * 2 + 1]);
                    if (ls > 0.0f) {
                        float w = expf(__ldcg(&p.part_ml[(base + s2) * 2]) - m);
                        l += ls * w;
                        acc += __ldcg(&p.part_acc[(base + s2) * kHeadDim + wt]) * w;
                    }
                }
                p.attn[(kvh * 4 + hq) * kHeadDim + wt] = acc / l;
            }
            if (wt == 0) p.attn_count[kvh] = 0;
        }
    }
}

__device__ __forceinline__ void arg_better(float &v, int &i, float v2, int i2)
{
    if (v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

// Final norm + tied BF16 head over this CTA's rows, then a per-CTA argmax.
__device__ __forceinline__ void mega_head(const MegaParams &p, float4 *xs, float *red)
{
    const int cols = kHidden, NQ = cols >> 3;
    {
        float ss = 0.0f;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            float v = __ldcg(&p.x[c]);
            ss += v * v;
        }
        ss = block_sum(ss, red);
        float rs = rsqrtf(ss / (float)cols + kNormEps);
        float *xf = reinterpret_cast<float *>(xs);
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            float v = p.final_norm[c] * (__ldcg(&p.x[c]) * rs);
            xf[((size_t)((c >> 2) & 1) * NQ + (c >> 3)) * 4 + (c & 3)] = v;
        }
        __syncthreads();
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int groups = kVocab / 4;
    const int warps = gridDim.x * kMegaWarps;
    float best = -INFINITY;
    int best_i = 0x7fffffff, bad = 0;
    for (int g = blockIdx.x * kMegaWarps + warp; g < groups; g += warps) {
        const uint16_t *wr[4];
#pragma unroll
        for (int i = 0; i < 4; i++) wr[i] = p.embedding + (size_t)(g * 4 + i) * cols;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int q0 = lane; q0 < NQ; q0 += 64) {
            uint4 w[2][4];
#pragma unroll
            for (int u = 0; u < 2; u++)
#pragma unroll
                for (int i = 0; i < 4; i++) w[u][i] = ld_stream(wr[i] + (size_t)(q0 + 32 * u) * 8);
#pragma unroll
            for (int u = 0; u < 2; u++) {
                int q = q0 + 32 * u;
                float4 x0 = xs[q], x1 = xs[NQ + q];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float a = acc[i];
                    a = fmaf(bf16_lo(w[u][i].x), x0.x, a);
                    a = fmaf(bf16_hi(w[u][i].x), x0.y, a);
                    a = fmaf(bf16_lo(w[u][i].y), x0.z, a);
                    a = fmaf(bf16_hi(w[u][i].y), x0.w, a);
                    a = fmaf(bf16_lo(w[u][i].z), x1.x, a);
                    a = fmaf(bf16_hi(w[u][i].z), x1.y, a);
                    a = fmaf(bf16_lo(w[u][i].w), x1.z, a);
                    a = fmaf(bf16_hi(w[u][i].w), x1.w, a);
                    acc[i] = a;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float v = warp_sum(acc[i]);
            if (lane == i) {
                p.logits[g * 4 + i] = v;
                bad |= !isfinite(v);
            }
            arg_better(best, best_i, v, g * 4 + i);
        }
    }
    if (bad) atomicOr(p.nonfinite, 1);
    // CTA argmax over its warps (value, then lowest id)
    __shared__ float bv[kMegaWarps];
    __shared__ int bi[kMegaWarps];
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = bv[0];
        int i = bi[0];
        for (int w = 1; w < kMegaWarps; w++) arg_better(v, i, bv[w], bi[w]);
        p.arg_val[blockIdx.x] = v;
        p.arg_idx[blockIdx.x] = i;
    }
}

__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega_kernel(MegaParams p)
{
    extern __shared__ float4 mega_smem[];
    float4 *xs = mega_smem;
    __shared__ float red[32];
    unsigned barrier = 0;
    if (p.timeline && blockIdx.x == 0 && threadIdx.x == 0) p.timeline[0] = globaltimer_ns();
    const size_t layer_bytes = (size_t)kQKVRows * kHidden + (size_t)kHidden * kQuery +
                               (size_t)kGateUpRows * kHidden + (size_t)kHidden * kInner;
    for (int s = 0; s < p.steps; s++) {
        const int length = ld_cg_int(&p.step->length);
        const int id = ld_cg_int(&p.step->ids[0]);
        const uint16_t *emb_row = p.embedding + (size_t)id * kHidden;
        for (int layer = 0; layer < kLayers; layer++) {
            const uint8_t *base = p.w8 + (size_t)layer * layer_bytes;
            const float *sc = p.scales + layer * 7;
            GemvParams gp;
            memset(&gp, 0, sizeof gp);
            gp.kv = p.kv;
            gp.page_table = p.page_table;
            gp.num_pages = p.num_pages;
            gp.layer = layer;
            gp.rope_cos = p.rope_cos;
            gp.rope_sin = p.rope_sin;
            gp.length = length;
            gp.bound[0] = gp.bound[1] = 1 << 30;
            // qkv
            gp.W = base;
            gp.rows = kQKVRows;
            gp.cols = kHidden;
            gp.scale[0] = sc[0];
            gp.scale[1] = sc[1];
            gp.scale[2] = sc[2];
            gp.bound[0] = kQuery;
            gp.bound[1] = kQuery + kKV;
            gp.y = p.q;
            if (p.prefetch) l2_prefetch_share(base + (size_t)kQKVRows * kHidden, (size_t)kHidden * kQuery);
            mega_load_row(xs, p.x, layer == 0 ? emb_row : nullptr, p.norms + (size_t)(2 * layer) * kHidden,
                          kHidden, red);
            if (layer == 0 && blockIdx.x == 0)
                for (int c = threadIdx.x; c < kHidden; c += blockDim.x) p.x[c] = bf16_lo((uint32_t)emb_row[c]);
            mega_gemv<kEpiQKV>(gp, xs);
            mega_sync(p, ++barrier);
            // attention
            mega_attention(p, layer, length, reinterpret_cast<float *>(mega_smem));
            mega_sync(p, ++barrier);
            // o + residual
            gp.W = base + (size_t)kQKVRows * kHidden;
            gp.rows = kHidden;
            gp.cols = kQuery;
            gp.scale[0] = gp.scale[1] = gp.scale[2] = sc[3];
            gp.bound[0] = gp.bound[1] = 1 << 30;
            gp.res = p.x;
            gp.y = p.h;
            if (p.prefetch) l2_prefetch_share(gp.W + (size_t)kHidden * kQuery, (size_t)kGateUpRows * kHidden);
            mega_load_row(xs, p.attn, nullptr, nullptr, kQuery, red);
            mega_gemv<kEpiResidual>(gp, xs);
            mega_sync(p, ++barrier);
            // post norm + gate/up + SwiGLU
            gp.W = base + (size_t)kQKVRows * kHidden + (size_t)kHidden * kQuery;
            gp.rows = kGateUpRows;
            gp.cols = kHidden;
            gp.scale[0] = sc[4];
            gp.scale[1] = sc[5];
            gp.y = p.act;
            if (p.prefetch) l2_prefetch_share(gp.W + (size_t)kGateUpRows * kHidden, (size_t)kHidden * kInner);
            mega_load_row(xs, p.h, nullptr, p.norms + (size_t)(2 * layer + 1) * kHidden, kHidden, red);
            mega_gemv<kEpiSwiGLU>(gp, xs);
            mega_sync(p, ++barrier);
            // down + residual
            gp.W = base + (size_t)kQKVRows * kHidden + (size_t)kHidden * kQuery +
                   (size_t)kGateUpRows * kHidden;
            gp.rows = kHidden;
            gp.cols = kInner;
            gp.scale[0] = gp.scale[1] = gp.scale[2] = sc[6];
            gp.res = p.h;
            gp.y = p.x;
            if (layer + 1 < kLayers) if (p.prefetch) l2_prefetch_share(base + layer_bytes, (size_t)kQKVRows * kHidden);
            mega_load_row(xs, p.act, nullptr, nullptr, kInner, red);
            mega_gemv<kEpiResidual>(gp, xs);
            mega_sync(p, ++barrier);
        }
        mega_head(p, xs, red);
        mega_sync(p, ++barrier);
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            float v = __ldcg(&p.arg_val[0]);
            int i = __ldcg(&p.arg_idx[0]);
            for (int b = 1; b < (int)gridDim.x; b++) arg_better(v, i, __ldcg(&p.arg_val[b]), __ldcg(&p.arg_idx[b]));
            int next = (i < 0 || i >= kVocab) ? 0 : i;
            int generated = ld_cg_int(&p.step->generated);
            p.tokens[generated] = next;
            p.step->generated = generated + 1;
            p.step->ids[0] = next;
            p.step->length = length + 1;
        }
        mega_sync(p, ++barrier);
    }
}

}  // namespace lun
