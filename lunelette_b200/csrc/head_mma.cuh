// Tied head of a batched decode step on the tensor cores: logits[t][v] =
// sum_c E[v][c] * norm(x_t)[c] for up to 64 tokens per pass, E the BF16
// embedding (131072 x 3072). Replaces the head projection of the reference's
// step (src/metal_encode.m:206-215) for many sessions at once.
//
// head_mma_split_kernel: per token, the final RMSNorm times the gain (the
// reference's rule, as in head_bf16_kernel) split into BF16 hi = bf16(v) and
// lo = bf16(v - hi); both become columns of the MMA's B operand (column
// n = 2 token + part), staged in chunks of 64 K values: xb[chunk][n][64].
//
// head_mma_kernel: a block of 8 warps takes 128 vocabulary rows, a warp 16 of
// them, over 48 chunks of 64 columns. Lane (g, t4) loads 16 consecutive BF16 of
// rows g and g + 8 from global memory (columns 16 t4 .. 16 t4 + 15 of the
// chunk) and uses them as the A fragments of four m16n8k16 steps: k step s
// takes the columns 16 t4 + 4 s + {0, 1} and {2, 3} as its k = 2 t4 (+1) and
// 2 t4 + 8 (+9) pairs; the staged B rows are read with the same column order,
// so the products pair the same columns. Every product of two BF16 values is
// exact in FP32; hi and lo columns are added in the epilogue (16 significant
// bits of the normed activation).
#pragma once
#include "attention.cuh"
#include "gemv.cuh"

namespace lun {

constexpr int kHmTokens = 64;                     // tokens per pass: N = 128 (hi and lo)
constexpr int kHmN = 2 * kHmTokens;
constexpr int kHmChunk = 64;                      // K columns per chunk
constexpr int kHmChunks = kHidden / kHmChunk;     // 48
constexpr int kHmRowStride = kHmChunk + 8;        // BF16 per staged B row (144 bytes)
constexpr int kHmWarps = 8;
constexpr int kHmRows = 16 * kHmWarps;            // vocabulary rows per block
constexpr int kHmThreads = 32 * kHmWarps;
constexpr int kHmSmemBytes = 2 * kHmN * kHmRowStride * 2;  // two B stages
constexpr size_t kHmStageElems = (size_t)kHmChunks * kHmN * kHmChunk;  // xb: BF16 elements

__device__ __forceinline__ uint16_t bf16_bits(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

// grid kHmTokens, 256 threads
static __global__ void __launch_bounds__(256) head_mma_split_kernel(HeadMmaParams p)
{
    __shared__ float red[32];
    const int tok = blockIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    uint16_t *hi_row = p.xb + (size_t)(2 * tok) * kHmChunk;
    uint16_t *lo_row = hi_row + kHmChunk;
    if (tok >= p.count) {
        for (int c = threadIdx.x; c < kHidden; c += blockDim.x) {
            const size_t at = (size_t)(c / kHmChunk) * kHmN * kHmChunk + c % kHmChunk;
            hi_row[at] = 0;
            lo_row[at] = 0;
        }
        return;
    }
    const float *x = p.x + (size_t)tok * p.x_stride;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) ss += x[c] * x[c];
    ss = block_sum(ss, red);
    const float rs = rsqrtf(ss / (float)kHidden + kNormEps);
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) {
        const float v = p.gain[c] * (x[c] * rs);
        const uint16_t h = bf16_bits(v);
        const float back = __bfloat162float(__ushort_as_bfloat16(h));
        const size_t at = (size_t)(c / kHmChunk) * kHmN * kHmChunk + c % kHmChunk;
        hi_row[at] = h;
        lo_row[at] = bf16_bits(v - back);
    }
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// grid rows / 128, kHmThreads, kHmSmemBytes
static __global__ void __launch_bounds__(kHmThreads) head_mma_kernel(HeadMmaParams p)
{
    extern __shared__ __align__(16) uint16_t hm_smem[];  // [2][kHmN][kHmRowStride]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const int row0 = blockIdx.x * kHmRows + warp * 16;
    const uint16_t *wa = p.W + (size_t)min(row0 + g, p.rows - 1) * kHidden + 16 * t4;
    const uint16_t *wb = p.W + (size_t)min(row0 + g + 8, p.rows - 1) * kHidden + 16 * t4;
    auto stage = [&](int c, int s) {
        uint16_t *dst = hm_smem + (size_t)s * kHmN * kHmRowStride;
        const uint16_t *src = p.xb + (size_t)c * kHmN * kHmChunk;
        for (int i = threadIdx.x; i < kHmN * (kHmChunk / 8); i += kHmThreads) {
            const int n = i >> 3, q = i & 7;
            cp_async16(dst + n * kHmRowStride + 8 * q, src + n * kHmChunk + 8 * q, true);
        }
        cp_async_commit();
    };
    // weights do not depend on earlier kernels: start the first chunks before the wait
    uint4 a_cur[4], a_next[4];
    a_cur[0] = __ldg(reinterpret_cast<const uint4 *>(wa));
    a_cur[1] = __ldg(reinterpret_cast<const uint4 *>(wa + 8));
    a_cur[2] = __ldg(reinterpret_cast<const uint4 *>(wb));
    a_cur[3] = __ldg(reinterpret_cast<const uint4 *>(wb + 8));
#pragma unroll
    for (int c = 1; c <= 4; c++) {
        prefetch_l2(wa + c * kHmChunk);
        prefetch_l2(wb + c * kHmChunk);
    }
    pdl_wait();  // xb comes from head_mma_split_kernel
    pdl_launch_dependents();
    stage(0, 0);
    float acc[16][4];
#pragma unroll
    for (int nb = 0; nb < 16; nb++) acc[nb][0] = acc[nb][1] = acc[nb][2] = acc[nb][3] = 0.0f;
    for (int c = 0; c < kHmChunks; c++) {
        if (c + 1 < kHmChunks) {
            stage(c + 1, (c + 1) & 1);
            const int off = (c + 1) * kHmChunk;
            a_next[0] = __ldg(reinterpret_cast<const uint4 *>(wa + off));
            a_next[1] = __ldg(reinterpret_cast<const uint4 *>(wa + off + 8));
            a_next[2] = __ldg(reinterpret_cast<const uint4 *>(wb + off));
            a_next[3] = __ldg(reinterpret_cast<const uint4 *>(wb + off + 8));
            if (c + 5 < kHmChunks) {
                prefetch_l2(wa + (c + 5) * kHmChunk);
                prefetch_l2(wb + (c + 5) * kHmChunk);
            }
        } else {
            cp_async_commit();  // empty group keeps the wait count uniform
        }
        cp_async_wait_one();
        __syncthreads();
        const uint16_t *bs = hm_smem + (size_t)(c & 1) * kHmN * kHmRowStride;
        const uint32_t ar[8] = {a_cur[0].x, a_cur[0].y, a_cur[0].z, a_cur[0].w,
                                a_cur[1].x, a_cur[1].y, a_cur[1].z, a_cur[1].w};
        const uint32_t br[8] = {a_cur[2].x, a_cur[2].y, a_cur[2].z, a_cur[2].w,
                                a_cur[3].x, a_cur[3].y, a_cur[3].z, a_cur[3].w};
#pragma unroll
        for (int nb = 0; nb < 16; nb++) {
            const uint16_t *brow = bs + (8 * nb + g) * kHmRowStride + 16 * t4;
            const uint4 b0 = *reinterpret_cast<const uint4 *>(brow);
            const uint4 b1 = *reinterpret_cast<const uint4 *>(brow + 8);
            mma_bf16_16816(acc[nb], ar[0], br[0], ar[1], br[1], b0.x, b0.y);
            mma_bf16_16816(acc[nb], ar[2], br[2], ar[3], br[3], b0.z, b0.w);
            mma_bf16_16816(acc[nb], ar[4], br[4], ar[5], br[5], b1.x, b1.y);
            mma_bf16_16816(acc[nb], ar[6], br[6], ar[7], br[7], b1.z, b1.w);
        }
        __syncthreads();  // this stage is refilled by the next iteration's copy
#pragma unroll
        for (int i = 0; i < 4; i++) a_cur[i] = a_next[i];
    }
    // column n = 8 nb + 2 t4 (+1) is token 4 nb + t4, part hi (lo)
    int bad = 0;
#pragma unroll
    for (int nb = 0; nb < 16; nb++) {
        const int tok = 4 * nb + t4;
        if (tok >= p.count) continue;
        float *out = p.logits + (size_t)tok * p.logits_stride;
        if (row0 + g < p.rows) {
            const float v = acc[nb][0] + acc[nb][1];
            out[row0 + g] = v;
            bad |= !isfinite(v);
        }
        if (row0 + g + 8 < p.rows) {
            const float v = acc[nb][2] + acc[nb][3];
            out[row0 + g + 8] = v;
            bad |= !isfinite(v);
        }
    }
    if (bad) atomicOr(p.nonfinite, 1);
}

}  // namespace lun
