// Projections of small token blocks (decode batches over many sessions, short
// prompts) on the tcgen05 tensor cores with the weights as the MMA's A operand
// in tensor memory.
//
// For a block of up to kTmMaxTokens tokens the work of a projection is the
// weight stream itself: 116 MB of FP8 per layer, which the pair GEMM
// (prefill_gemm.cuh) converts to FP16 through shared memory, tiles 256 tokens
// per MMA whatever the block holds and so runs about as long at 64 tokens as
// at 256. Here one CTA owns 128 weight rows and a K range for all the block's
// tokens (MMA M = 128 rows, N = 2 x the tokens rounded up to 16: the hi and
// the lo activation tiles side by side, one MMA per k-step for both):
//   warp 0      tensor copies of the FP8 weight stages (128 rows x 64 columns:
//               one 512-byte piece of each of 16 tiles, a 3-D map of 8-byte
//               elements) and bulk copies of the split activations' hi and lo
//               operand tiles, each into its own ring;
//   warp 1      allocates tensor memory; one lane issues the MMAs
//               (tcgen05.mma.cta_group::1.kind::f16 with A in tensor memory,
//               B = activations in shared memory), alternating between two
//               accumulators, and commits;
//   warps 2-9   convert, in two groups of four (one warp per TMEM lane
//               quarter) that take alternating stages: thread = weight row,
//               its 64 FP8 bytes of the stage to 32 FP16 pairs in registers
//               and one tcgen05.st into that stage's A buffer; the 16-byte
//               reads start at a chunk rotated by lane so a warp's reads
//               spread over the shared-memory banks; then the epilogue (group g
//               takes tokens 32 g .. 32 g + 31): the accumulators' hi and lo
//               columns added, times the token's 2^-e, into the FP32 partials
//               of its K range, which the finish kernels add in order as for
//               the pair GEMM.
// The FP16 weights never touch shared memory, and the MMA does no work for
// token tiles the block does not have.
//
// The CTA takes all 512 tensor-memory columns of its SM; its 198 KB of shared
// memory keep any other tcgen05 kernel of this library off that SM meanwhile,
// so the allocation never waits.
//
// Tensor-memory A operand (kind::f16, M = 128, cta_group::1): row r in lane r,
// K element k of a 16-element step in 32-bit column k / 2 (low half even k),
// consecutive steps in consecutive 8-column groups.
#pragma once
#include "prefill_gemm.cuh"

namespace lun {

constexpr int kTmMaxTokens = 64;                      // tokens of a block this GEMM takes
constexpr int kTmConverters = 8;                      // converter warps (two per TMEM lane quarter)
constexpr int kTmThreads = 32 * (2 + kTmConverters);  // load warp, MMA warp, converters
constexpr int kTmRows = 128;                          // weight rows per CTA (MMA M, TMEM lanes)
constexpr int kTmWStages = 8;                         // FP8 weight stages in shared memory
constexpr int kTmAStages = 8;                         // activation stages in shared memory
constexpr int kTmTStages = 8;                         // A stages in tensor memory
constexpr int kTmW8 = kTmRows * kPgK;                 // 8192: one stage of FP8 weights
constexpr int kTmABytes = (kTmMaxTokens / 8) * 1024;  // 8192: one part (hi or lo) of a stage's activations
constexpr int kTmStageCols = kPgK / 2;                // 32 TMEM columns: one stage's A (64 FP16 per row)
// A stage's activations are one B operand of N = 2 n rows: the hi tile's n
// token rows followed by the lo tile's (n = tokens rounded up to 16), so one
// MMA per k-step covers both parts (MMA issue, not tensor work, is what a
// stage of this small GEMM spends); D column t is W.hi_t and column n + t is
// W.lo_t. The k-steps alternate between two accumulators, added in the epilogue.
constexpr int kTmAccCols = 2 * kTmMaxTokens;          // columns of one accumulator (2 n)
constexpr int kTmAccs = 2;
constexpr int kTmTmemCols = 512;                      // accumulator + A stages, a power of two
constexpr int kTmWOffset = 0;
constexpr int kTmAOffset = kTmWOffset + kTmWStages * kTmW8;
constexpr int kTmBarOffset = kTmAOffset + kTmAStages * 2 * kTmABytes;
constexpr int kTmSmemBytes = 1024 + kTmBarOffset + 512;
static_assert(kTmAccs * kTmAccCols + kTmTStages * kTmStageCols <= kTmTmemCols && kTmAccCols >= kTmMaxTokens,
              "accumulator and A stages fit the allocation");
static_assert(kTmSmemBytes <= 232448, "small GEMM shared memory");

struct TmGemmParams {
    int rows, kchunks, count, splits;
    const uint8_t *xs;        // split activations: [kchunks][hi, lo][kPgATile] of token tile 0
    const float *inv_scale;   // [128]: 2^-e per token
    float *ws;                // [splits][t_stride][ws_rows] FP32 partials
    int t_stride, ws_rows;
    int *error;
};

// Grid (ceil(rows / 128), 1, splits), kTmThreads threads. wmap: the weight
// matrix as 8-byte elements {64, 2 nb, tiles} (a box {64, 1, 16} is one
// 64-column piece of 16 tiles = 128 rows, in 16 rows of 512 bytes).
static __global__ void __launch_bounds__(kTmThreads, 1)
    prefill_gemm_tmem_kernel(TmGemmParams p, const __grid_constant__ CUtensorMap wmap)
{
    extern __shared__ __align__(1024) uint8_t tm_raw[];
    const uint32_t raw = smem_u32(tm_raw);
    uint8_t *base = tm_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *wring = base + kTmWOffset, *aring = base + kTmAOffset;
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + kTmBarOffset);
    uint64_t *wfull = bars, *wempty = wfull + kTmWStages;
    uint64_t *afull = wempty + kTmWStages, *aempty = afull + kTmAStages;
    uint64_t *tfull = aempty + kTmAStages, *tempty = tfull + kTmTStages;
    uint64_t *accf = tempty + kTmTStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);
    volatile int *abort_word = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.z;
    const int k0 = (int)((long long)split * p.kchunks / p.splits);
    const int nk = (int)((long long)(split + 1) * p.kchunks / p.splits) - k0;
    const int tile0 = blockIdx.x * (kTmRows / kTileRows);
    const int count = min(p.count, kTmMaxTokens);
    const int n = (count + 15) & ~15;                            // MMA N
    const uint32_t nbytes = (uint32_t)(n / 8) * 1024;             // 8-token atoms of a part (n rows)

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTmWStages; s++) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], 4);  // the converter group of the stage (one warp per quarter)
        }
        for (int s = 0; s < kTmAStages; s++) {
            mbar_init(&afull[s], 1);
            mbar_init(&aempty[s], 1);
        }
        for (int s = 0; s < kTmTStages; s++) {
            mbar_init(&tfull[s], 4);   // after that group's tensor-memory stores
            mbar_init(&tempty[s], 1);
        }
        mbar_init(accf, 1);
        *abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // the weights depend on no earlier kernel: the first stages are in flight
    // before the wait for the previous kernel (programmatic launch)
    const int pre = min(nk, kTmWStages);
    if (warp == 0 && lane == 0)
        for (int iw = 0; iw < pre; iw++) {
            mbar_expect_tx(&wfull[iw], kTmW8);
            tma_load_3d(wring + iw * kTmW8, &wmap, 0, k0 + iw, tile0, &wfull[iw]);
        }
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        // ---- loads: weights into their ring, activations into theirs, each as
        // far ahead as its ring allows (non-blocking probes)
        int iw = pre, ia = 0;
        if (lane == 0) {
            unsigned idle = 0;
            while ((iw < nk || ia < nk) && !*abort_word) {
                bool progressed = false;
                if (iw < nk) {
                    const int s = iw % kTmWStages, u = iw / kTmWStages;
                    if (u == 0 || mbar_test_wait(&wempty[s], (u - 1) & 1)) {
                        mbar_expect_tx(&wfull[s], kTmW8);
                        tma_load_3d(wring + s * kTmW8, &wmap, 0, k0 + iw, tile0, &wfull[s]);
                        iw++;
                        progressed = true;
                    }
                }
                if (ia < nk) {
                    const int s = ia % kTmAStages, u = ia / kTmAStages;
                    if (u == 0 || mbar_test_wait(&aempty[s], (u - 1) & 1)) {
                        uint8_t *st = aring + s * 2 * kTmABytes;
                        const uint8_t *a = p.xs + ((size_t)(k0 + ia) * 2) * kPgATile;
                        mbar_expect_tx(&afull[s], 2 * nbytes);
                        bulk_g2s(st, a, nbytes, &afull[s]);                   // hi: B rows 0 .. n - 1
                        bulk_g2s(st + nbytes, a + kPgATile, nbytes, &afull[s]);  // lo: B rows n .. 2 n - 1
                        ia++;
                        progressed = true;
                    }
                }
                if (progressed) {
                    idle = 0;
                } else if (++idle > 64u * kPgSpinLimit) {
                    *abort_word = 1;
                    atomicExch(p.error, 1);
                    break;
                }
            }
        }
        iw = __shfl_sync(0xffffffffu, iw, 0);
        ia = __shfl_sync(0xffffffffu, ia, 0);
        // every copy issued has landed before the CTA ends
        for (int i = max(0, iw - kTmWStages); i < iw; i++)
            mbar_wait_bounded(&wfull[i % kTmWStages], (i / kTmWStages) & 1, abort_word, p.error, kPgSpinLimit);
        for (int i = max(0, ia - kTmAStages); i < ia; i++)
            mbar_wait_bounded(&afull[i % kTmAStages], (i / kTmAStages) & 1, abort_word, p.error, kPgSpinLimit);
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = f16_idesc(kTmRows, 2 * n);
            bool ok = true;
            for (int i = 0; i < nk && ok; i++) {
                const int s = i % kTmAStages, t = i % kTmTStages;
                ok = mbar_wait_bounded(&tfull[t], (i / kTmTStages) & 1, abort_word, p.error, kPgSpinLimit) &&
                     mbar_wait_bounded(&afull[s], (i / kTmAStages) & 1, abort_word, p.error, kPgSpinLimit);
                if (!ok) break;
                tc_fence_after();
                const uint32_t b0 = smem_u32(aring + s * 2 * kTmABytes);
                const uint32_t a_cols = tmem + (uint32_t)(kTmAccs * kTmAccCols + t * kTmStageCols);
#pragma unroll
                for (int k = 0; k < kPgK / 16; k++) {
                    const int acc = k % kTmAccs;
                    tc_mma_f16_tmem_a(tmem + (uint32_t)(acc * kTmAccCols), a_cols + (uint32_t)(k * 8),
                                      sw128_desc(b0 + k * 32), idesc, i > 0 || k >= kTmAccs);
                }
                tc_commit(&aempty[s]);
                tc_commit(&tempty[t]);
            }
            tc_commit(accf);
            mbar_wait_bounded(accf, 0, abort_word, p.error, kPgSpinLimit);
        }
        __syncwarp();
    } else {
        // ---- converters: thread = weight row 32 q + lane of the CTA's 128, in
        // TMEM lane quarter q = warp % 4 (the quarter this warp may access);
        // two groups of four warps take alternating stages, so that one
        // group's tensor-memory stores are in flight while the other converts
        const int q = warp & 3, grp = (warp - 2) >> 2, r = 32 * q + lane;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const int rot = (lane >> 1) & 3;  // first chunk this lane reads
        for (int i = grp; i < nk; i += 2) {
            const int s = i % kTmWStages, t = i % kTmTStages, ut = i / kTmTStages;
            if (!warp_wait(&wfull[s], (i / kTmWStages) & 1, abort_word, p.error)) break;
            if (ut > 0 && !warp_wait(&tempty[t], (ut - 1) & 1, abort_word, p.error)) break;
            // tile r >> 3 of the stage holds the 64 columns of its 8 rows in 512
            // bytes; row g's four 16-byte chunks (lanes 4 g .. 4 g + 3 of the
            // fragment layout) are contiguous: chunk c, word j carries columns
            // 16 j + 2 c + {0, 1} (low half) and 16 j + 2 c + {8, 9} (high half);
            // lanes start at chunk rot so a warp's reads spread over the banks
            const uint8_t *src = wring + s * kTmW8 + (r >> 3) * 512 + (r & 7) * 64;
            uint4 w[4];
#pragma unroll
            for (int k = 0; k < 4; k++) w[k] = *reinterpret_cast<const uint4 *>(src + 16 * ((k + rot) & 3));
            __syncwarp();
            if (lane == 0) mbar_arrive(&wempty[s]);  // the FP8 slot may refill
            uint32_t a[32];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int d = (c - rot) & 3;  // chunk c was read in step d
                const uint4 v = d == 0 ? w[0] : d == 1 ? w[1] : d == 2 ? w[2] : w[3];
                const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    a[8 * j + c] = e4m3x2_to_f16x2(words[j]);
                    a[8 * j + c + 4] = e4m3x2_to_f16x2(words[j] >> 16);
                }
            }
            tmem_st32(tmem + lane_base + (uint32_t)(kTmAccs * kTmAccCols + t * kTmStageCols), a);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tfull[t]);
        }
        const int hf = grp;  // the epilogue: group g takes tokens 32 g .. 32 g + 31
        // accf completes once every MMA of the CTA did (the A stages in tensor
        // memory are free then too). The tensor-memory load below is
        // warp-collective: a warp-uniform test
        if (__all_sync(0xffffffffu, warp_wait(accf, 0, abort_word, p.error) && !*abort_word) && 32 * hf < n) {
            tc_fence_after();
            // accumulator: lane = weight row, column = token; half hf takes
            // tokens 32 hf .. 32 hf + 31
            const int row = blockIdx.x * kTmRows + r, cb = 32 * hf;
            // (acc 0 + acc 1) of the hi column plus the same of the lo column
            float sum[32];
#pragma unroll 1
            for (int part = 0; part < 2; part++) {
                float ps[32];
#pragma unroll 1
                for (int acc = 0; acc < kTmAccs; acc++) {
                    uint32_t d[32];
                    tmem_ld32(tmem + lane_base + (uint32_t)(acc * kTmAccCols + part * n + cb), d);
#pragma unroll
                    for (int j = 0; j < 32; j++) ps[j] = acc ? ps[j] + __uint_as_float(d[j]) : __uint_as_float(d[j]);
                }
#pragma unroll
                for (int j = 0; j < 32; j++) sum[j] = part ? sum[j] + ps[j] : ps[j];
            }
            if (row < p.rows)
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const int tok = cb + j;
                    if (tok < count)
                        __stcg(p.ws + ((size_t)split * p.t_stride + tok) * p.ws_rows + row, sum[j] * p.inv_scale[tok]);
                }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmTmemCols);
    }
}

}  // namespace lun
