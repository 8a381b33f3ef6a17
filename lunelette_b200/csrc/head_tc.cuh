// Tied head of a batched decode step on tcgen05 (5th-generation tensor cores):
// logits[t][v] = sum_c E[v][c] * norm(x_t)[c] for up to 64 tokens per pass, E
// the BF16 embedding (131072 x 3072). The same arithmetic as head_mma_kernel
// (BF16 hi and lo parts of the normed activation, every product exact in
// FP32, the two parts added in the epilogue), with the products on the
// tcgen05 pipe and the accumulator in tensor memory. Replaces the head
// projection of the reference's step (src/metal_encode.m:206-215) for many
// sessions at once.
//
// head_tc_split_kernel: per token, the final RMSNorm times the gain (the rule
// of head_mma_split_kernel, value for value) split into BF16 hi = bf16(v) and
// lo = bf16(v - hi), written as rows 2 t (hi) and 2 t + 1 (lo) of the MMA's B
// operand: K-major, one 16 KB tile of 128 rows x 64 columns per chunk of 64
// K values, already in the 128-byte-swizzled order the tensor core reads, so
// one bulk copy moves a chunk into shared memory as it is.
//
// head_tc_kernel: a CTA takes 128 vocabulary rows (MMA M = 128, TMEM lanes)
// against all 128 B rows (N = 128), K in 48 chunks of 64 through a ring of
// kHtStages stages. Warp 0 loads: the chunk's 128 x 64 embedding tile by a 2-D
// tensor copy with the 128-byte swizzle (the rows do not depend on earlier
// kernels, so the first stages are in flight before the wait for the split
// kernel) and the chunk's B tile by a bulk copy. Warp 1 allocates the 128
// accumulator columns and issues four K = 16 MMAs per chunk; warps 2-5 (one
// per TMEM lane quarter) read the accumulator once every MMA completed: lane
// = vocabulary row, column 2 t + part, and store hi + lo for each token, so a
// warp writes 32 consecutive logits of a token. Two CTAs fit on an SM (shared
// memory and tensor memory), so one CTA's epilogue and prologue overlap the
// other's stream. Every wait is bounded: one that gives up sets p.error and
// the CTA stores nothing.
#pragma once
#include "head_mma.cuh"
#include "tcgen05.cuh"

namespace lun {

constexpr int kHtRows = 128;                        // vocabulary rows per CTA (MMA M, TMEM lanes)
constexpr int kHtN = kHmN;                          // B rows: token 2 t + part (MMA N)
constexpr int kHtChunk = 64;                        // K columns per stage: one 128-byte swizzle row
constexpr int kHtChunks = kHidden / kHtChunk;       // 48
constexpr int kHtStages = 3;
constexpr int kHtABytes = kHtRows * kHtChunk * 2;   // 16384: embedding tile of a stage
constexpr int kHtBBytes = kHtN * kHtChunk * 2;      // 16384: B tile of a stage (and of a chunk in xb)
constexpr int kHtStageBytes = kHtABytes + kHtBBytes;
constexpr int kHtBarOffset = kHtStages * kHtStageBytes;
constexpr int kHtSmemBytes = 1024 + kHtBarOffset + 128;  // alignment slack, ring, barriers
constexpr int kHtThreads = 192;                     // load warp, MMA warp, four epilogue warps
constexpr int kHtTmemCols = 128;                    // one FP32 accumulator of N columns
static_assert(kHtStages <= kHtChunks, "the first stages are issued unconditionally");
static_assert((size_t)kHtChunks * kHtBBytes == kHmStageElems * sizeof(uint16_t),
              "the swizzled B operand fills the batched head's staging buffer");

// Instruction descriptor of kind::f16 with BF16 A and B (formats in bits 7-9
// and 10-12), FP32 D, K-major operands.
__host__ __device__ constexpr uint32_t bf16_idesc(int m, int n) { return f16_idesc(m, n) | (1u << 7) | (1u << 10); }

// Byte offset of B element (row n, column c) in the staging buffer.
__host__ __device__ __forceinline__ size_t head_tc_b_offset(int n, int c)
{
    return (size_t)(c / kHtChunk) * kHtBBytes + sw128_offset(n, c % kHtChunk);
}

// grid kHmTokens, 256 threads
static __global__ void __launch_bounds__(256) head_tc_split_kernel(HeadMmaParams p)
{
    __shared__ float red[32];
    const int tok = blockIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    uint8_t *xb = reinterpret_cast<uint8_t *>(p.xb);
    if (tok >= p.count) {
        for (int c = threadIdx.x; c < kHidden; c += blockDim.x) {
            *reinterpret_cast<uint16_t *>(xb + head_tc_b_offset(2 * tok, c)) = 0;
            *reinterpret_cast<uint16_t *>(xb + head_tc_b_offset(2 * tok + 1, c)) = 0;
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
        *reinterpret_cast<uint16_t *>(xb + head_tc_b_offset(2 * tok, c)) = h;
        *reinterpret_cast<uint16_t *>(xb + head_tc_b_offset(2 * tok + 1, c)) = bf16_bits(v - back);
    }
}

// Grid rows / 128, kHtThreads threads, kHtSmemBytes. emap: the embedding as a
// 2-D BF16 tensor {3072, rows} with box {64, 128} and the 128-byte swizzle.
static __global__ void __launch_bounds__(kHtThreads, 2)
    head_tc_kernel(HeadMmaParams p, const __grid_constant__ CUtensorMap emap)
{
    extern __shared__ __align__(1024) uint8_t ht_raw[];
    const uint32_t raw = smem_u32(ht_raw);
    uint8_t *base = ht_raw + (((raw + 1023u) & ~1023u) - raw);  // swizzled tiles start on 1024 bytes
    uint64_t *full = reinterpret_cast<uint64_t *>(base + kHtBarOffset);
    uint64_t *empty = full + kHtStages;
    uint64_t *accf = empty + kHtStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);
    volatile int *abort_word = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kHtRows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kHtStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        *abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, kHtTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // the embedding rows depend on no earlier kernel: the first stages' tiles
    // are in flight before the wait for the split kernel (programmatic launch)
    if (warp == 0 && lane == 0)
        for (int c = 0; c < kHtStages; c++) {
            mbar_expect_tx(&full[c], kHtStageBytes);
            tma_load_2d(base + c * kHtStageBytes, &emap, c * kHtChunk, row0, &full[c]);
        }
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        // ---- loads: stage s of chunk c holds the embedding tile (16 KB) then
        // the B tile (16 KB); chunk c refills stage c % kHtStages once the MMAs
        // of chunk c - kHtStages released it
        int issued = kHtStages;
        if (lane == 0) {
            const uint8_t *xb = reinterpret_cast<const uint8_t *>(p.xb);
            for (int c = 0; c < kHtStages; c++)
                bulk_g2s(base + c * kHtStageBytes + kHtABytes, xb + (size_t)c * kHtBBytes, kHtBBytes, &full[c]);
            for (int c = kHtStages; c < kHtChunks; c++) {
                const int s = c % kHtStages, u = c / kHtStages;
                if (!mbar_wait_bounded(&empty[s], (u - 1) & 1, abort_word, p.error, kWaitSpinLimit)) break;
                uint8_t *st = base + s * kHtStageBytes;
                mbar_expect_tx(&full[s], kHtStageBytes);
                tma_load_2d(st, &emap, c * kHtChunk, row0, &full[s]);
                bulk_g2s(st + kHtABytes, xb + (size_t)c * kHtBBytes, kHtBBytes, &full[s]);
                issued = c + 1;
            }
        }
        issued = __shfl_sync(0xffffffffu, issued, 0);
        // every copy issued has landed before the CTA ends (the latest phase of
        // each stage's barrier is the last copy into it)
        if (lane == 0)
            for (int c = issued - kHtStages; c < issued; c++)
                mbar_wait_bounded(&full[c % kHtStages], (c / kHtStages) & 1, abort_word, p.error, kWaitSpinLimit);
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = bf16_idesc(kHtRows, kHtN);
            for (int c = 0; c < kHtChunks; c++) {
                const int s = c % kHtStages;
                if (!mbar_wait_bounded(&full[s], (c / kHtStages) & 1, abort_word, p.error, kWaitSpinLimit)) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(base + s * kHtStageBytes), b0 = a0 + kHtABytes;
#pragma unroll
                for (int k = 0; k < kHtChunk / 16; k++)
                    tc_mma_f16(tmem, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), idesc, (c | k) != 0);
                tc_commit(&empty[s]);  // the stage may refill once these MMAs read it
            }
            // completes once every MMA issued completed (also after a wait gave
            // up, so that no MMA is in flight when the columns are freed)
            tc_commit(accf);
            mbar_wait_bounded(accf, 0, abort_word, p.error, kWaitSpinLimit);
        }
        __syncwarp();
    } else {
        // ---- epilogue: warp w reads TMEM lane quarter w % 4 (rows 32 q .. 32 q + 31
        // of the CTA's 128); the tensor-memory loads are warp-collective, so the
        // test is warp-uniform
        const int q = warp & 3;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const int row = row0 + 32 * q + lane;
        if (__all_sync(0xffffffffu, warp_wait(accf, 0, abort_word, p.error) && !*abort_word)) {
            tc_fence_after();
            int bad = 0;
            for (int cb = 0; cb < kHtN / 32; cb++) {
                if (16 * cb >= p.count) break;  // 16 tokens per 32 columns; the same for the whole warp
                uint32_t d[32];
                tmem_ld32(tmem + lane_base + (uint32_t)(32 * cb), d);
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int tok = 16 * cb + j;
                    if (tok < p.count && row < p.rows) {
                        const float v = __uint_as_float(d[2 * j]) + __uint_as_float(d[2 * j + 1]);
                        p.logits[(size_t)tok * p.logits_stride + row] = v;
                        bad |= !isfinite(v);
                    }
                }
            }
            if (bad) atomicOr(p.nonfinite, 1);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kHtTmemCols);
    }
}

}  // namespace lun
