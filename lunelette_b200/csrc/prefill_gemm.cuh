// Prefill projections on the 5th-generation tensor cores (tcgen05, TMEM).
//
// Replaces the reference's MPS matrix multiplications of multi-token blocks
// (src/metal_mps.m:26-111, encoded by src/metal_encode.m:124-187 for prefill
// and append) and, by fusion, the norm, rope, element and KV-blit steps around
// them. Y[t][r] = scale * sum_k X[t][k] * W[r][k] for a block of T tokens:
//
//   prefill_split_kernel   X (optionally RMS-normed) -> per token an exact power
//                          of two 2^e and FP16 hi + lo parts (the GEMV's
//                          split, gemv.cuh), written as ready-swizzled operand
//                          tiles;
//   prefill_gemm_pair_kernel  one CTA pair per (512 weight rows, 256 tokens,
//                          K range): bulk copies of the activation tiles and of
//                          the FP8 weight tiles, FP8 -> FP16 conversion into
//                          shared memory, tcgen05.mma.cta_group::2 (kind::f16,
//                          M = 256 tokens, N = 256 rows, K = 16) with the hi and
//                          the lo part accumulating into the same FP32 TMEM
//                          accumulator; the epilogue reads TMEM, applies 2^-e
//                          and writes FP32 partial rows of its K range;
//   prefill_finish_kernel  adds the K ranges in a fixed order, applies the
//                          per-tensor scale and the fused epilogue of the
//                          projection (store, residual, RoPE + query scale +
//                          KV store, SwiGLU).
//
// Operand layout (K-major, 128-byte swizzle, the tcgen05 canonical form): a
// tile of R rows x 64 FP16 columns is R/8 atoms of 1024 bytes; element (r, k)
// sits at byte (r >> 3) * 1024 + (r & 7) * 128 + (((k >> 3) ^ (r & 7)) << 4) +
// (k & 7) * 2 of the tile, which must start on a 1024-byte boundary. The split
// kernel writes activations in this form, so one 16 KB bulk copy lands a
// 128-token operand; the converters write the weights in it.
//
// Precision: E4M3 -> FP16 is exact; hi + lo carry 22 significant bits of each
// scaled activation; FP16 x FP16 products are exact in FP32. Only the order of
// the FP32 additions differs from the reference's dot products.
#pragma once
#include <cuda.h>

#include "async.cuh"
#include "gemv.cuh"
#include "tcgen05.cuh"

namespace lun {

constexpr int kPgM = 128;                           // tokens per CTA (TMEM lanes; a pair's MMA has M = 256)
constexpr int kPgN = 256;                           // N of one MMA (TMEM columns of one accumulator)
constexpr int kPgK = 64;                            // K columns per stage
constexpr int kPgThreads = 192;                     // warp 0 loads, warp 1 MMA, warps 2-5 convert + epilogue
constexpr int kPgATile = kPgM * kPgK * 2;           // 16384: one activation part of a stage
constexpr unsigned kPgSpinLimit = 1u << 20;  // polls of a bounded wait; the loaders idle up to 64x this

// ---- activation split --------------------------------------------------------------
struct PrefillSplitParams {
    const float *x;      // [count][x_stride]
    int x_stride;
    const float *gain;   // RMSNorm gain, or nullptr
    int cols, kchunks, count;
    uint8_t *xs;         // [count tiles][kchunks][hi, lo][kPgATile]
    float *inv_scale;    // [count tiles * 128]: 2^-e (0 for padding tokens)
};

// One block per token of the padded block (padding tokens write zeros). The
// row is read once into registers (kSplitVec float4 per thread), so every load
// of the block is in flight at once.
constexpr int kSplitThreads = 256;
constexpr int kSplitVec = 16;                                   // float4 per thread
constexpr int kSplitMaxCols = kSplitThreads * 4 * kSplitVec;    // 16384
// The split of one token row held in registers (v: the row, float4 slot
// threadIdx.x + kSplitThreads * i; g: the gain, 1 without norm): the
// statistics of gemv_stage (sum of squares of x, max of |gain * x|), the
// exponent, and the hi/lo parts into the swizzled operand tiles.
template <int THREADS, int VEC>
__device__ __forceinline__ void split_emit(const PrefillSplitParams &p, int t, bool live, const float4 (&v)[VEC],
                                           const float4 (&g)[VEC])
{
    __shared__ float red[2][THREADS / 32];
    const int tt = t >> 7, m = t & 127;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int vecs = (p.kchunks * kPgK) / 4;  // float4 slots of the padded row
    float ss = 0.0f, mx = 0.0f;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(g[i].x * v[i].x), fabsf(g[i].y * v[i].y)),
                             fmaxf(fabsf(g[i].z * v[i].z), fabsf(g[i].w * v[i].w))));
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if (lane == 0) {
        red[0][warp] = ss;
        red[1][warp] = mx;
    }
    __syncthreads();
    float s = 0.0f, x = 0.0f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; w++) {
        s += red[0][w];
        x = fmaxf(x, red[1][w]);
    }
    const float rs = p.gain ? rsqrtf(s / (float)p.cols + kNormEps) : 1.0f;
    const int e = live ? frag_exponent(x * rs * 1.0001f) : 0;
    const float sc = exp2i(e);
    if (threadIdx.x == 0) p.inv_scale[t] = live ? exp2i(-e) : 0.0f;
    uint8_t *tile = p.xs + (size_t)tt * p.kchunks * 2 * kPgATile;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
        const int slot = threadIdx.x + THREADS * i;
        if (slot >= vecs) break;
        const int c = 4 * slot;
        float a0 = v[i].x, a1 = v[i].y, a2 = v[i].z, a3 = v[i].w;
        if (p.gain) {
            a0 = g[i].x * (a0 * rs);
            a1 = g[i].y * (a1 * rs);
            a2 = g[i].z * (a2 * rs);
            a3 = g[i].w * (a3 * rs);
        }
        uint32_t h0 = 0, l0 = 0, h1 = 0, l1 = 0;
        if (live) {
            split_hilo(a0 * sc, a1 * sc, h0, l0);
            split_hilo(a2 * sc, a3 * sc, h1, l1);
        }
        // columns c..c+3 share one 16-byte chunk of the swizzled row
        uint8_t *dst = tile + (size_t)(c >> 6) * 2 * kPgATile + sw128_offset(m, c & 63);
        *reinterpret_cast<uint2 *>(dst) = make_uint2(h0, h1);
        *reinterpret_cast<uint2 *>(dst + kPgATile) = make_uint2(l0, l1);
    }
}

static __global__ void __launch_bounds__(kSplitThreads) prefill_split_kernel(PrefillSplitParams p)
{
    pdl_wait();  // the rows come from the previous kernel, and the last GEMM read the operand tiles
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const bool live = t < p.count;
    const float *xr = p.x + (size_t)(live ? t : 0) * p.x_stride;
    float4 v[kSplitVec], g[kSplitVec];
#pragma unroll
    for (int i = 0; i < kSplitVec; i++) {
        const int c = 4 * (threadIdx.x + kSplitThreads * i);
        v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        g[i] = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        if (live && c < p.cols) {
            v[i] = *reinterpret_cast<const float4 *>(xr + c);
            if (p.gain) g[i] = *reinterpret_cast<const float4 *>(p.gain + c);
        }
    }
    split_emit<kSplitThreads, kSplitVec>(p, t, live, v, g);
}

// ---- the GEMM ---------------------------------------------------------------------
struct PrefillGemmParams {
    const uint8_t *W;         // tiled FP8 matrix (gemv.cuh), nb blocks per tile
    int rows, nb, kchunks;    // rows % 8 == 0; kchunks = ceil(cols / 64)
    const uint8_t *xs;        // split activations (prefill_split_kernel)
    int token_tiles, count;
    int splits;               // K ranges (gridDim.z)
    const float *inv_scale;
    float *ws;                // [splits][token_tiles * 128][ws_rows] FP32 partials
    int ws_rows;              // gridDim.x * 256
    int *error;
};

// ---- the GEMM on a CTA pair (tcgen05 cta_group::2) ------------------------------------
// A cluster of two CTAs computes 256 tokens x 512 weight rows. CTA r loads the
// activation tiles of its 128 tokens (the MMA's A rows 128r..128r+127; only the
// 8-row atoms that hold tokens) and converts weight rows h*256 + 128r + [0, 128)
// for h = 0, 1 (the B halves it holds); CTA 0 issues tcgen05.mma.cta_group::2
// (M = 256, N = 256) twice per K step and part, once per 256-row half h, into
// TMEM accumulator h (columns 256h..256h+255) of each CTA. Each activation tile
// loaded thus serves 512 weight rows: the activations (4 bytes per token and
// column: FP16 hi and lo) are the operand every CTA streams, and L2 -> SM
// traffic, not the tensor core, bounds this GEMM at 256 rows per tile.
constexpr int kP2Acc = 2;                                // accumulators (256-row halves) per CTA
constexpr int kP2N = kPgN * kP2Acc;                      // 512 weight rows per pair
constexpr int kP2Rows = kPgN / 2;                        // 128 rows of each half per CTA
// Three rings: activations (freed when the MMA of the stage completed), FP8
// weights (freed as soon as they are converted, so the weight stream from HBM
// runs further ahead) and converted FP16 weights (freed when the MMA completed).
constexpr int kP2AStages = 3;
constexpr int kP2WStages = 4;
constexpr int kP2BStages = 2;
constexpr int kP2ABytes = 2 * kPgATile;                  // 32768: hi and lo of 128 tokens
constexpr int kP2W8 = kP2Acc * kP2Rows * kPgK;           // 16384
constexpr int kP2BHalf = kP2Rows * kPgK * 2;             // 16384: one half's FP16 rows
constexpr int kP2BBytes = kP2Acc * kP2BHalf;             // 32768
constexpr int kP2WOffset = kP2AStages * kP2ABytes;
constexpr int kP2BOffset = kP2WOffset + kP2WStages * kP2W8;
constexpr int kP2BarOffset = kP2BOffset + kP2BStages * kP2BBytes;
constexpr int kP2SmemBytes = 1024 + kP2BarOffset + 256;
constexpr int kP2TmemCols = kPgN * kP2Acc;               // 512
static_assert(kP2SmemBytes <= 232448, "pair GEMM shared memory");

__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive (release at cluster scope) on the mbarrier at the same offset in CTA `rank`.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t *bar, uint32_t rank)
{
    asm volatile(
        "{\n\t.reg .b32 ra;\n\t"
        "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
        "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
        "r"(rank)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, unsigned parity)
{
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot, uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                bool accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// Arrive on the mbarrier at this offset in both CTAs of the pair once every
// MMA issued so far completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t *bar)
{
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}

// Grid (2 * ceil(rows / 512), ceil(token tiles / 2), splits), clusters of 2 along x.
// wmap: the tiled weight matrix as a 4-D uint8 tensor {256, 2, 2 * nb, rows / 8}
// (bytes of a 512-byte half block, its two 256-byte pieces, the half blocks of
// a tile, the tiles) with box {256, 2, 1, 16}: one copy brings one 64-column
// half block of 16 consecutive tiles (8 KB); tiles past the matrix read zeros.
static __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPgThreads, 1)
    prefill_gemm_pair_kernel(PrefillGemmParams p, const __grid_constant__ CUtensorMap wmap)
{
    extern __shared__ __align__(1024) uint8_t pg2_raw[];
    const uint32_t raw = smem_u32(pg2_raw);
    uint8_t *base = pg2_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *aring = base, *wring = base + kP2WOffset, *bring = base + kP2BOffset;
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + kP2BarOffset);
    uint64_t *afull = bars, *aempty = afull + kP2AStages;
    uint64_t *wfull = aempty + kP2AStages, *wempty = wfull + kP2WStages;
    uint64_t *bfull = wempty + kP2WStages, *bempty = bfull + kP2BStages;
    uint64_t *accf = bempty + kP2BStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);
    volatile int *abort_word = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int rt = blockIdx.x >> 1, split = blockIdx.z;
    const int tt = 2 * blockIdx.y + (int)rank;  // this CTA's token tile
    const int tokens = max(0, min(kPgM, p.count - tt * kPgM));
    const uint32_t abytes = (uint32_t)((tokens + 7) / 8) * 1024;  // 8-token atoms of a part
    const int k0 = (int)((long long)split * p.kchunks / p.splits);
    const int nk = (int)((long long)(split + 1) * p.kchunks / p.splits) - k0;
    // this CTA's weight tiles: 16 per half, half h from tile0 + 32 h
    const int tile0 = rt * (kP2N / kTileRows) + (int)rank * (kP2Rows / kTileRows);
    static_assert(kP2Acc == 2, "two 256-row halves");

    if (threadIdx.x == 0) {
        for (int s = 0; s < kP2AStages; s++) {
            mbar_init(&afull[s], 1);
            mbar_init(&aempty[s], 1);
        }
        for (int s = 0; s < kP2WStages; s++) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], 4);  // this CTA's converter warps
        }
        for (int b = 0; b < kP2BStages; b++) {
            mbar_init(&bfull[b], 2 * 4);  // the converter warps of both CTAs
            mbar_init(&bempty[b], 1);
        }
        mbar_init(accf, 1);
        *abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, kP2TmemCols);
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // the weights do not depend on earlier kernels: their first stages are in
    // flight before the wait for the previous kernel (programmatic launch); the
    // activations, the partials this grid writes and the rest come after it
    const int pre = min(nk, kP2WStages);
    if (warp == 0 && lane == 0)
        for (int iw = 0; iw < pre; iw++) {
            uint8_t *dst = wring + iw * kP2W8;
            mbar_expect_tx(&wfull[iw], kP2W8);
            tma_load_4d(dst, &wmap, 0, 0, k0 + iw, tile0, &wfull[iw]);
            tma_load_4d(dst + kP2W8 / 2, &wmap, 0, 0, k0 + iw, tile0 + kPgN / kTileRows, &wfull[iw]);
        }
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        // ---- loads. Weights: per stage two tensor copies (the 16 tiles of each
        // 256-row half) into the weight ring; activations: the hi and lo atoms of
        // this CTA's tokens into the activation ring. Each stream goes as far
        // ahead as its ring allows; the warp issues whichever next copy has a
        // free slot (non-blocking probes, so one full ring never stalls the other).
        int iw = pre, ia = 0;
        if (lane == 0) {
            unsigned idle = 0;
            while ((iw < nk || ia < nk) && !*abort_word) {
                bool progressed = false;
                if (iw < nk) {
                    const int s = iw % kP2WStages, u = iw / kP2WStages;
                    if (u == 0 || mbar_test_wait(&wempty[s], (u - 1) & 1)) {
                        const int kc = k0 + iw;
                        uint8_t *dst = wring + s * kP2W8;
                        mbar_expect_tx(&wfull[s], kP2W8);
                        tma_load_4d(dst, &wmap, 0, 0, kc, tile0, &wfull[s]);
                        tma_load_4d(dst + kP2W8 / 2, &wmap, 0, 0, kc, tile0 + kPgN / kTileRows, &wfull[s]);
                        iw++;
                        progressed = true;
                    }
                }
                if (ia < nk && ia < iw) {
                    const int s = ia % kP2AStages, u = ia / kP2AStages;
                    if (u == 0 || mbar_test_wait(&aempty[s], (u - 1) & 1)) {
                        const int kc = k0 + ia;
                        uint8_t *st = aring + s * kP2ABytes;
                        mbar_expect_tx(&afull[s], 2 * abytes);
                        if (abytes) {
                            const uint8_t *a = p.xs + ((size_t)(tt * p.kchunks + kc) * 2) * kPgATile;
                            bulk_g2s(st, a, abytes, &afull[s]);
                            bulk_g2s(st + kPgATile, a + kPgATile, abytes, &afull[s]);
                        }
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
        // before the CTA ends: every copy issued has landed, and the leader's
        // releases of the last activation stages (multicast arrivals on this
        // CTA's barriers) too
        for (int i = max(0, iw - kP2WStages); i < iw; i++)
            mbar_wait_bounded(&wfull[i % kP2WStages], (i / kP2WStages) & 1, abort_word, p.error, kPgSpinLimit);
        for (int i = max(0, ia - kP2AStages); i < ia; i++)
            mbar_wait_bounded(&aempty[i % kP2AStages], (i / kP2AStages) & 1, abort_word, p.error, kPgSpinLimit);
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = f16_idesc(2 * kPgM, kPgN);
            bool ok = true;
            for (int i = 0; i < nk && ok; i++) {
                const int s = i % kP2AStages, b = i % kP2BStages, v = i / kP2BStages;
                // both CTAs' converters arrive once their activations and FP16 weights are in place
                unsigned spins = 0;
                while (!mbar_try_wait_cluster(&bfull[b], v & 1)) {
                    if (++spins > kPgSpinLimit || (((spins & 63u) == 0) && *abort_word)) {
                        *abort_word = 1;
                        atomicExch(p.error, 1);
                        ok = false;
                        break;
                    }
                }
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(aring + s * kP2ABytes), b0 = smem_u32(bring + b * kP2BBytes);
#pragma unroll
                for (int k = 0; k < kPgK / 16; k++) {
#pragma unroll
                    for (int part = 0; part < 2; part++) {
                        const uint64_t adesc = sw128_desc(a0 + part * kPgATile + k * 32);
#pragma unroll
                        for (int hh = 0; hh < kP2Acc; hh++)
                            tc_mma_f16_pair(tmem + (uint32_t)(hh * kPgN), adesc,
                                            sw128_desc(b0 + hh * kP2BHalf + k * 32), idesc, (i | k | part) != 0);
                    }
                }
                tc_commit_pair(&aempty[s]);
                tc_commit_pair(&bempty[b]);
            }
            tc_commit_pair(accf);
            mbar_wait_bounded(accf, 0, abort_word, p.error, kPgSpinLimit);
        }
        __syncwarp();
    } else {
        // ---- converters: this CTA's 256 weight rows to FP16, then the epilogue
        const int c = threadIdx.x - 64;
        int done = 0;
        for (int i = 0; i < nk; i++) {
            const int s = i % kP2WStages, u = i / kP2WStages, b = i % kP2BStages, v = i / kP2BStages;
            if (!warp_wait(&wfull[s], u & 1, abort_word, p.error)) break;
            if (v > 0 && !warp_wait(&bempty[b], (v - 1) & 1, abort_word, p.error)) break;
            const uint8_t *w8 = wring + s * kP2W8;
            uint8_t *bb = bring + b * kP2BBytes;
#pragma unroll
            for (int q = 0; q < kP2W8 / 16 / 128; q++) {
                // 32 half blocks (half tl >> 4, tile tl & 15), stored in that order
                // in the weight ring and, 16 KB per half, in the FP16 buffer
                const int chunk = q * 128 + c, tl = chunk >> 5, L = chunk & 31;
                const uint4 w = *reinterpret_cast<const uint4 *>(w8 + chunk * 16);  // zero past the matrix
                // lane L of a half block holds tile row L >> 2, columns
                // 16j + 2(L & 3) + {0, 1} (bytes 4j, 4j+1) and + {8, 9} (bytes 4j+2, 4j+3)
                const int r = L >> 2;
                uint8_t *row = bb + tl * 1024 + r * 128 + 4 * (L & 3);
                const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    *reinterpret_cast<uint32_t *>(row + (((2 * j) ^ r) << 4)) = e4m3x2_to_f16x2(words[j]);
                    *reinterpret_cast<uint32_t *>(row + (((2 * j + 1) ^ r) << 4)) =
                        e4m3x2_to_f16x2(words[j] >> 16);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&wempty[s]);  // the FP8 slot may refill
            fence_proxy_async_smem();
            // the stage's activations must have landed in this CTA too
            if (!warp_wait(&afull[i % kP2AStages], (i / kP2AStages) & 1, abort_word, p.error)) break;
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(&bfull[b], 0);
            done = i + 1;
        }
        // the leader's releases of the last FP16 buffers land before the CTA ends
        for (int i = max(0, done - kP2BStages); i < done; i++)
            warp_wait(&bempty[i % kP2BStages], (i / kP2BStages) & 1, abort_word, p.error);
        // (the tensor-memory loads below are warp-collective: a warp-uniform test)
        if (__all_sync(0xffffffffu, warp_wait(accf, 0, abort_word, p.error) && !*abort_word) && tokens > 0) {
            tc_fence_after();
            // each 32 x 32 block (this warp's 32 tokens x 32 accumulator columns)
            // goes through shared memory (the activation ring is idle now), so
            // every store writes four whole 128-byte rows of the partials
            const int quarter = warp & 3, m = 32 * quarter + lane;
            const float inv = p.inv_scale[tt * kPgM + m];
            float *tile = reinterpret_cast<float *>(aring) + (warp - 2) * 32 * 33;
            const int row_lane = lane & 7, token_lane = lane >> 3;
            for (int cb = 0; cb < kP2TmemCols / 32; cb++) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(cb * 32), r);
#pragma unroll
                for (int i = 0; i < 32; i++) tile[lane * 33 + i] = __uint_as_float(r[i]) * inv;
                __syncwarp();
#pragma unroll
                for (int g = 0; g < 8; g++) {
                    const int tk = 4 * g + token_lane, t = tt * kPgM + 32 * quarter + tk;
                    if (t < p.count) {
                        const float *src = tile + tk * 33 + 4 * row_lane;
                        // accumulator h column j is pair row 256 h + j
                        *reinterpret_cast<float4 *>(p.ws + ((size_t)split * p.token_tiles * kPgM + t) * p.ws_rows +
                                                    (size_t)rt * kP2N + cb * 32 + 4 * row_lane) =
                            make_float4(src[0], src[1], src[2], src[3]);
                    }
                }
                __syncwarp();
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kP2TmemCols);
    }
}

// ---- finish: K ranges in order, per-tensor scale, fused epilogue -------------------------
struct PrefillFinishParams {
    const float *ws;
    int splits, t_stride, ws_rows;  // t_stride = token_tiles * 128
    int rows, count;
    float scale[3];
    int bound[2];                   // logical rows < bound[0] -> scale[0]; < bound[1] -> scale[1]; else scale[2]
    float *y;
    int y_stride;
    const float *res;
    int res_stride;
    // kEpiQKV (gemv.cuh semantics)
    const float *rope_cos, *rope_sin;
    const StepParams *step;
    int length;
    float *kv;
    const int *page_table;
    int num_pages, layer;
    const int *positions, *token_table;  // batched decode (GemvParams)
    int table_stride;
};

__device__ __forceinline__ float finish_scale(const PrefillFinishParams &p, int r)
{
    return r < p.bound[0] ? p.scale[0] : (r < p.bound[1] ? p.scale[1] : p.scale[2]);
}

// Grid (ceil(rows / 2 / 256), count): one thread per token and storage row pair.
template <int EPI>
static __global__ void __launch_bounds__(256) prefill_finish_kernel(PrefillFinishParams p)
{
    pdl_wait();  // the partials come from the GEMM
    pdl_launch_dependents();
    const int t = blockIdx.y;
    const int pr = blockIdx.x * blockDim.x + threadIdx.x;
    if (2 * pr >= p.rows) return;
    float a = 0.0f, b = 0.0f;
    for (int s = 0; s < p.splits; s++) {
        const float2 v = __ldcg(reinterpret_cast<const float2 *>(p.ws + ((size_t)s * p.t_stride + t) * p.ws_rows) + pr);
        a += v.x;
        b += v.y;
    }
    if constexpr (EPI == kEpiStore || EPI == kEpiResidual) {
        const int r = 2 * pr;
        a *= finish_scale(p, r);
        b *= finish_scale(p, r + 1);
        if (EPI == kEpiResidual) {
            a = p.res[(size_t)t * p.res_stride + r] + a;
            b = p.res[(size_t)t * p.res_stride + r + 1] + b;
        }
        p.y[(size_t)t * p.y_stride + r] = a;
        p.y[(size_t)t * p.y_stride + r + 1] = b;
    } else if constexpr (EPI == kEpiSwiGLU) {
        // storage row 2f is gate f, 2f + 1 is up f
        const float g = a * p.scale[0], u = b * p.scale[1];
        const float silu = g / (1.0f + expf(-g));
        p.y[(size_t)t * p.y_stride + pr] = silu * u;
    } else {
        // storage rows (2j, 2j + 1) of a 128-row head hold logical rows (j, j + 64)
        const int head = pr >> 6, j = pr & 63;
        const int ra = head * kHeadDim + j, rb = ra + 64;
        a *= finish_scale(p, ra);
        b *= finish_scale(p, rb);
        const int pos = p.positions ? p.positions[t] : (p.step ? p.step->length : p.length) + t;
        if (ra < kQuery + kKV) {
            const float *cs = p.rope_cos + (size_t)pos * 128, *sn = p.rope_sin + (size_t)pos * 128;
            const float lo = a * cs[j] + (-b) * sn[j];
            const float hi = b * cs[j + 64] + a * sn[j + 64];
            a = lo;
            b = hi;
        }
        if (ra < kQuery) {
            const float qs = query_scale(pos);
            p.y[(size_t)t * p.y_stride + ra] = a * qs;
            p.y[(size_t)t * p.y_stride + rb] = b * qs;
        } else {
            const int kind = ra < kQuery + kKV ? 0 : 1;
            const int kvh = (ra - kQuery - kind * kKV) >> 7;
            const int *table = p.positions ? p.page_table + (size_t)p.token_table[t] * p.table_stride : p.page_table;
            const int page = table[pos / kPage], slot = pos % kPage;
            float *dst = p.kv + kv_offset(p.layer, p.num_pages, page, kind, kvh, slot);
            dst[j] = a;
            dst[j + 64] = b;
        }
    }
}

// ---- finish + the next projection's split, per token ----------------------------------
// The residual (o, down) or SwiGLU (gate/up) epilogue of one token's row from
// the K-range partials, in the same order as prefill_finish_kernel, kept in
// registers; written to f.y when the row is needed later (h, x); then split
// (RMS-normed with sp.gain) into the next projection's operand tiles. act,
// which only the down projection reads, never goes to memory.
constexpr int kFsThreads = 512;
constexpr int kFsVec = kSplitMaxCols / (4 * kFsThreads);  // float4 per thread
template <int EPI>
static __global__ void __launch_bounds__(kFsThreads) prefill_finish_split_kernel(PrefillFinishParams f,
                                                                                  PrefillSplitParams sp)
{
    pdl_wait();  // the partials come from the GEMM, which also read the operand tiles this kernel rewrites
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const bool live = t < f.count;
    const int width = EPI == kEpiSwiGLU ? f.rows / 2 : f.rows;
    const float *ws = f.ws + (size_t)(live ? t : 0) * f.ws_rows;
    const size_t split_stride = (size_t)f.t_stride * f.ws_rows;
    float4 v[kFsVec], g[kFsVec];
#pragma unroll
    for (int i = 0; i < kFsVec; i++) {
        const int c = 4 * (threadIdx.x + kFsThreads * i);
        v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        g[i] = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        if (live && c < width) {
            if (sp.gain) g[i] = *reinterpret_cast<const float4 *>(sp.gain + c);
            if constexpr (EPI == kEpiSwiGLU) {
                // features c..c+3: gate at storage rows 2f, up at 2f + 1
                float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
                for (int s = 0; s < f.splits; s++) {
                    const float4 a = __ldcg(reinterpret_cast<const float4 *>(ws + s * split_stride + 2 * c));
                    const float4 b = __ldcg(reinterpret_cast<const float4 *>(ws + s * split_stride + 2 * c + 4));
                    lo.x += a.x; lo.y += a.y; lo.z += a.z; lo.w += a.w;
                    hi.x += b.x; hi.y += b.y; hi.z += b.z; hi.w += b.w;
                }
                const float gv[4] = {lo.x * f.scale[0], lo.z * f.scale[0], hi.x * f.scale[0], hi.z * f.scale[0]};
                const float uv[4] = {lo.y * f.scale[1], lo.w * f.scale[1], hi.y * f.scale[1], hi.w * f.scale[1]};
                float o[4];
#pragma unroll
                for (int k = 0; k < 4; k++) o[k] = (gv[k] / (1.0f + expf(-gv[k]))) * uv[k];
                v[i] = make_float4(o[0], o[1], o[2], o[3]);
            } else {
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int s = 0; s < f.splits; s++) {
                    const float4 b = __ldcg(reinterpret_cast<const float4 *>(ws + s * split_stride + c));
                    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
                }
                const float4 r = *reinterpret_cast<const float4 *>(f.res + (size_t)t * f.res_stride + c);
                v[i] = make_float4(r.x + a.x * finish_scale(f, c), r.y + a.y * finish_scale(f, c + 1),
                                   r.z + a.z * finish_scale(f, c + 2), r.w + a.w * finish_scale(f, c + 3));
            }
            if (f.y) *reinterpret_cast<float4 *>(f.y + (size_t)t * f.y_stride + c) = v[i];
        }
    }
    if (!sp.xs) return;
    split_emit<kFsThreads, kFsVec>(sp, t, live, v, g);
}

}  // namespace lun
