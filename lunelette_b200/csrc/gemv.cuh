// FP8-E4M3 weight GEMV family for decode (M = 1..4 token rows).
//
// Replaces project_fp8 / project_fp8_lookup (src/metal_kernels.metal:136-177,
// 249-272) and, by fusion, the norm, rope, element and KV-blit steps that the
// reference encodes around each projection (src/metal_encode.m:124-187).
// K and V rows are stored in FP32, the reference's KV precision.
//
// Layout: W is row-major [rows][cols] E4M3 bytes; one warp owns a group of four
// rows and streams them with 16-byte loads (16 codes per lane per load, two
// loads in flight per row), dequantises in registers (cvt e4m3x2 -> f16x2 ->
// f32, exact), and accumulates in FP32 against the activation rows held in
// shared memory. The per-tensor scale multiplies the reduced sum. The warp
// reduction is a fixed xor butterfly, so results are run-to-run deterministic.
//
// Shared-memory activation layout: row m, 16-column chunk q, 4-column piece p
// lives at float4 index m*4*NQ + p*NQ + q (NQ = cols/16). Consecutive lanes read
// consecutive float4s, so the loads are bank-conflict free.
#pragma once
#include "common.cuh"

namespace lun {

enum GemvEpilogue : int {
    kEpiStore = 0,     // y[m][r] = acc * scale(r)
    kEpiResidual = 1,  // y[m][r] = res[m][r] + acc * scale(r)
    kEpiQKV = 2,       // rows [q|k|v]: RoPE on q,k (+query scale); q -> y, k/v -> KV pool
    kEpiSwiGLU = 3,    // alternating gate/up rows: y[m][f] = silu(g) * u
};

struct GemvParams {
    const uint8_t *W;
    int rows, cols;
    const float *x;      // [M][x_stride] activations (pre-norm when gain != nullptr)
    int x_stride;
    const float *gain;   // RMSNorm gain (FP32) fused as prologue, or nullptr
    float scale[3];      // per-tensor scales by row range
    int bound[2];        // rows < bound[0] -> scale[0]; < bound[1] -> scale[1]; else scale[2]
    float *y;            // output rows [M][y_stride]
    int y_stride;
    const float *res;    // residual rows [M][res_stride] (kEpiResidual)
    int res_stride;
    // kEpiQKV
    const float *rope_cos, *rope_sin;  // [context][128]
    const StepParams *step;            // device: sequence length before this call, or
    int length;                        //   nullptr to use this value instead
    int token_offset;                  // first token of this launch within the call
    float *kv;                         // FP32 KV pool
    const int *page_table;
    int num_pages, layer;
    // Weights of the next projection in the step, fetched into L2 while this one
    // runs so that HBM keeps streaming across kernel boundaries (or nullptr).
    const uint8_t *prefetch;
    size_t prefetch_bytes;
};

template <int M>
__device__ __forceinline__ void gemv_load_x(const GemvParams &p, float4 *xs, float *red)
{
    const int cols = p.cols, NQ = cols >> 4;
    float *xf = reinterpret_cast<float *>(xs);
#pragma unroll
    for (int m = 0; m < M; m++) {
        const float *xr = p.x + (size_t)m * p.x_stride;
        float rs = 1.0f;
        if (p.gain) {
            float ss = 0.0f;
            for (int c = threadIdx.x; c < cols; c += blockDim.x) ss += xr[c] * xr[c];
            ss = block_sum(ss, red);
            rs = rsqrtf(ss / (float)cols + kNormEps);
        }
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            float v = xr[c];
            if (p.gain) v = p.gain[c] * (v * rs);
            int q = c >> 4, piece = (c >> 2) & 3, e = c & 3;
            xf[((size_t)m * 4 * NQ + (size_t)piece * NQ + q) * 4 + e] = v;
        }
    }
}

// Storage is group-major: group g occupies rows 4g..4g+3 of the matrix on the
// device. For q/k/v a group is two RoPE pairs of one 128-row head, stored as
// (j, j+64, j+1, j+65); for gate/up it is (gate f, up f, gate f+1, up f+1) with
// f = 2g. logical_row() maps element i of group g back to the row index of the
// checkpoint's tensor (q|k|v concatenated) for scales, RoPE and outputs.
template <int EPI>
__device__ __forceinline__ int logical_row(int g, int i)
{
    if (EPI == kEpiQKV) {
        int head = g >> 5, j = (g & 31) * 2;
        return head * 128 + j + (i & 1) * 64 + (i >> 1);
    } else {
        return g * 4 + i;
    }
}

// Per-tensor scale of element i of group g: gate/up alternate (odd = up);
// otherwise by logical row range (q, k, v).
template <int EPI>
__device__ __forceinline__ float elem_scale(const GemvParams &p, int g, int i)
{
    if (EPI == kEpiSwiGLU) return (i & 1) ? p.scale[1] : p.scale[0];
    int r = logical_row<EPI>(g, i);
    return r < p.bound[0] ? p.scale[0] : (r < p.bound[1] ? p.scale[1] : p.scale[2]);
}

template <int M, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams &p, int g, int lane,
                                              float (&acc)[4][M])
{
    // Every lane holds the reduced sums; lane k < 2*M handles pair (k/M, k%M).
    if constexpr (EPI == kEpiStore || EPI == kEpiResidual) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                if (lane == i * M + m) {
                    int r = logical_row<EPI>(g, i);
                    if (r < p.rows) {
                        float v = acc[i][m] * elem_scale<EPI>(p, g, i);
                        if (EPI == kEpiResidual) v = __ldcg(&p.res[(size_t)m * p.res_stride + r]) + v;
                        p.y[(size_t)m * p.y_stride + r] = v;
                    }
                }
            }
        }
    } else {
#pragma unroll
    for (int pair = 0; pair < 2; pair++) {
#pragma unroll
        for (int m = 0; m < M; m++) {
            if (lane != pair * M + m) continue;
            int ra = logical_row<EPI>(g, pair * 2), rb = logical_row<EPI>(g, pair * 2 + 1);
            float a = acc[pair * 2][m] * elem_scale<EPI>(p, g, pair * 2);
            float b = acc[pair * 2 + 1][m] * elem_scale<EPI>(p, g, pair * 2 + 1);
            if (EPI == kEpiSwiGLU) {
                // a = gate, b = up of feature 2g + pair
                int f = 2 * g + pair;
                float silu = a / (1.0f + expf(-a));
                p.y[(size_t)m * p.y_stride + f] = silu * b;
            } else {
                // QKV: ra = head*128 + j (j < 64), rb = ra + 64
                int pos = (p.step ? p.step->length : p.length) + p.token_offset + m;
                int j = ra & 127;
                if (ra < kQuery + kKV) {
                    const float *cs = p.rope_cos + (size_t)pos * 128;
                    const float *sn = p.rope_sin + (size_t)pos * 128;
                    float lo = a * cs[j] + (-b) * sn[j];
                    float hi = b * cs[j + 64] + a * sn[j + 64];
                    a = lo;
                    b = hi;
                }
                if (ra < kQuery) {
                    float qs = query_scale(pos);
                    p.y[(size_t)m * p.y_stride + ra] = a * qs;
                    p.y[(size_t)m * p.y_stride + rb] = b * qs;
                } else {
                    int kind = ra < kQuery + kKV ? 0 : 1;
                    int head = (ra - kQuery - kind * kKV) >> 7;
                    int page = p.page_table[pos / kPage], slot = pos % kPage;
                    float *dst = p.kv + kv_offset(p.layer, p.num_pages, page, kind, head, slot);
                    dst[j] = a;
                    dst[j + 64] = b;
                }
            }
        }
    }
    }
}

// Dot products of the four rows of group g against the M activation rows in
// shared memory; every lane ends with the full (butterfly-reduced) sums.
template <int M, int EPI>
__device__ __forceinline__ void gemv_group(const GemvParams &p, const float4 *xs, int g, int lane,
                                           float (&acc)[4][M])
{
    const int NQ = p.cols >> 4;
    const uint8_t *wr[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int r = 4 * g + i;  // storage row
        wr[i] = p.W + (size_t)(r < p.rows ? r : p.rows - 1) * p.cols;
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int m = 0; m < M; m++) acc[i][m] = 0.0f;

    for (int q0 = lane; q0 < NQ; q0 += 64) {
        uint4 w[2][4];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            int q = q0 + 32 * u;
#pragma unroll
            for (int i = 0; i < 4; i++)
                w[u][i] = q < NQ ? ld_stream(wr[i] + (size_t)q * 16) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 2; u++) {
            int q = q0 + 32 * u;
            if (q >= NQ) break;
#pragma unroll
            for (int piece = 0; piece < 4; piece++) {
                float4 xv[M];
#pragma unroll
                for (int m = 0; m < M; m++) xv[m] = xs[(size_t)m * 4 * NQ + (size_t)piece * NQ + q];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    uint32_t word = piece == 0 ? w[u][i].x : piece == 1 ? w[u][i].y
                                  : piece == 2 ? w[u][i].z : w[u][i].w;
                    float2 lo = e4m3x2_to_float2(word);
                    float2 hi = e4m3x2_to_float2(word >> 16);
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        float a = acc[i][m];
                        a = fmaf(lo.x, xv[m].x, a);
                        a = fmaf(lo.y, xv[m].y, a);
                        a = fmaf(hi.x, xv[m].z, a);
                        a = fmaf(hi.y, xv[m].w, a);
                        acc[i][m] = a;
                    }
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int m = 0; m < M; m++) acc[i][m] = warp_sum(acc[i][m]);
}

// One launch: blockDim 256 (8 warps); grid-stride over row groups of 4.
template <int M, int EPI>
__global__ void __launch_bounds__(256) gemv_fp8_kernel(GemvParams p)
{
    extern __shared__ float4 xs[];
    __shared__ float red[32];
    l2_prefetch_share(p.prefetch, p.prefetch_bytes);
    pdl_wait();
    pdl_launch_dependents();
    gemv_load_x<M>(p, xs, red);
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int groups = (p.rows + 3) >> 2;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups; g += warps) {
        float acc[4][M];
        gemv_group<M, EPI>(p, xs, g, lane, acc);
        gemv_epilogue<M, EPI>(p, g, lane, acc);
    }
}

// ---------------------------------------------------------------------------
// Tied LM head: BF16 weights [vocab][cols], final RMSNorm fused as prologue,
// one token row. Widening BF16 -> FP32 is exact (bit shift). Also flags any
// non-finite logit for the host's finiteness contract.
struct HeadParams {
    const uint16_t *W;
    int rows, cols;
    const float *x;     // the last token's hidden row
    const float *gain;  // final norm gain
    float *logits;
    int *nonfinite;     // set to 1 when any logit is NaN/Inf
};

static __global__ void __launch_bounds__(256) head_bf16_kernel(HeadParams p)
{
    extern __shared__ float4 xs[];
    __shared__ float red[32];
    const int cols = p.cols, NQ = cols >> 3;  // 8-column chunks (16 bytes of BF16)
    pdl_wait();
    pdl_launch_dependents();
    {
        float ss = 0.0f;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) ss += p.x[c] * p.x[c];
        ss = block_sum(ss, red);
        float rs = rsqrtf(ss / (float)cols + kNormEps);
        float *xf = reinterpret_cast<float *>(xs);
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            float v = p.gain[c] * (p.x[c] * rs);
            int q = c >> 3, piece = (c >> 2) & 1, e = c & 3;
            xf[((size_t)piece * NQ + q) * 4 + e] = v;
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int groups = (p.rows + 3) >> 2;
    const int warps = gridDim.x * (blockDim.x >> 5);
    int bad = 0;
    for (int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups; g += warps) {
        const uint16_t *wr[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int r = g * 4 + i;
            wr[i] = p.W + (size_t)(r < p.rows ? r : p.rows - 1) * cols;
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int q0 = lane; q0 < NQ; q0 += 64) {
            uint4 w[2][4];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                int q = q0 + 32 * u;
#pragma unroll
                for (int i = 0; i < 4; i++)
                    w[u][i] = q < NQ ? ld_stream(wr[i] + (size_t)q * 8) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                int q = q0 + 32 * u;
                if (q >= NQ) break;
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
            int r = g * 4 + i;
            if (lane == i && r < p.rows) {
                p.logits[r] = v;
                bad |= !isfinite(v);
            }
        }
    }
    if (bad) atomicOr(p.nonfinite, 1);
}

}  // namespace lun
