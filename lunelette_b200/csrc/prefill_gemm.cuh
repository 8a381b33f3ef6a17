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
//   prefill_gemm_kernel    one CTA per (256 weight rows, 128 tokens, K range):
//                          bulk copies of the activation tiles and of the FP8
//                          weight tiles, FP8 -> FP16 conversion into shared
//                          memory, tcgen05.mma (kind::f16, M = 128 tokens,
//                          N = 256 rows, K = 16) with the hi and the lo part
//                          accumulating into the same FP32 TMEM accumulator;
//                          the epilogue reads TMEM, applies 2^-e and writes
//                          FP32 partial rows of its K range;
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
#include "async.cuh"
#include "gemv.cuh"

namespace lun {

constexpr int kPgM = 128;                           // tokens per tile (MMA M, TMEM lanes)
constexpr int kPgN = 256;                           // weight rows per CTA (MMA N, TMEM columns)
constexpr int kPgK = 64;                            // K columns per stage
constexpr int kPgStages = 3;                        // load ring: activation hi, lo, FP8 weights
constexpr int kPgBStages = 2;                       // ring of converted FP16 weights
constexpr int kPgThreads = 192;                     // warp 0 loads, warp 1 MMA, warps 2-5 convert + epilogue
constexpr int kPgATile = kPgM * kPgK * 2;           // 16384: one activation part of a stage
constexpr int kPgW8 = kPgN * kPgK;                  // 16384: FP8 weights of a stage
constexpr int kPgStageBytes = 2 * kPgATile + kPgW8;  // 49152
constexpr int kPgBBytes = kPgN * kPgK * 2;          // 32768: FP16 weights of a stage
constexpr int kPgBarOffset = kPgStages * kPgStageBytes + kPgBStages * kPgBBytes;
constexpr int kPgSmemBytes = 1024 + kPgBarOffset + 256;  // + alignment slack + barriers
constexpr unsigned kPgSpinLimit = 1u << 20;
static_assert(kPgSmemBytes <= 232448, "prefill GEMM shared memory");

// Byte offset of element (r, k) (k < 64) inside a swizzled K-major tile.
__host__ __device__ __forceinline__ uint32_t sw128_offset(int r, int k)
{
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 3) ^ (r & 7)) & 7) << 4) + (k & 7) * 2);
}

// ---- tcgen05 wrappers ------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole warp: allocate `cols` TMEM columns, address written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (stride byte offset), leading byte offset 16 (unused by the
// swizzled K-major form), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: FP16 A and B (K-major), FP32 D, M x N.
__host__ __device__ constexpr uint32_t f16_idesc(int m, int n)
{
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// One thread: D[tmem] (+)= A[smem] * B[smem]^T.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           bool accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// One thread: arrive on *bar once every tcgen05.mma it issued so far completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Whole warp: 32 consecutive FP32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- activation split --------------------------------------------------------------
struct PrefillSplitParams {
    const float *x;      // [count][x_stride]
    int x_stride;
    const float *gain;   // RMSNorm gain, or nullptr
    int cols, kchunks, count;
    uint8_t *xs;         // [count tiles][kchunks][hi, lo][kPgATile]
    float *inv_scale;    // [count tiles * 128]: 2^-e (0 for padding tokens)
};

// One block per token of the padded block (padding tokens write zeros).
static __global__ void __launch_bounds__(256) prefill_split_kernel(PrefillSplitParams p)
{
    __shared__ float red[2][8];
    const int t = blockIdx.x, tt = t >> 7, m = t & 127;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool live = t < p.count;
    const float *xr = p.x + (size_t)(live ? t : 0) * p.x_stride;
    float rs = 1.0f, sc = 1.0f;
    int e = 0;
    if (live) {
        // the same statistics and order as gemv_stage
        float ss = 0.0f, mx = 0.0f;
        for (int c = threadIdx.x; c < p.cols; c += blockDim.x) {
            const float v = xr[c];
            ss += v * v;
            mx = fmaxf(mx, fabsf(p.gain ? p.gain[c] * v : v));
        }
        ss = warp_sum(ss);
        mx = warp_max(mx);
        if (lane == 0) {
            red[0][warp] = ss;
            red[1][warp] = mx;
        }
        __syncthreads();
        float s = 0.0f, x = 0.0f;
        for (int w = 0; w < 8; w++) {
            s += red[0][w];
            x = fmaxf(x, red[1][w]);
        }
        rs = p.gain ? rsqrtf(s / (float)p.cols + kNormEps) : 1.0f;
        e = frag_exponent(x * rs * 1.0001f);
        sc = exp2i(e);
    }
    if (threadIdx.x == 0) p.inv_scale[t] = live ? exp2i(-e) : 0.0f;
    uint8_t *tile = p.xs + (size_t)tt * p.kchunks * 2 * kPgATile;
    for (int c = 2 * threadIdx.x; c < kPgK * p.kchunks; c += 2 * blockDim.x) {
        uint32_t hi = 0, lo = 0;
        if (live && c < p.cols) {
            float a = xr[c], b = xr[c + 1];
            if (p.gain) {
                a = p.gain[c] * (a * rs);
                b = p.gain[c + 1] * (b * rs);
            }
            split_hilo(a * sc, b * sc, hi, lo);
        }
        uint8_t *dst = tile + (size_t)(c >> 6) * 2 * kPgATile + sw128_offset(m, c & 63);
        *reinterpret_cast<uint32_t *>(dst) = hi;
        *reinterpret_cast<uint32_t *>(dst + kPgATile) = lo;
    }
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

// Warp-uniform bounded wait: every lane polls; the warp goes on only if all saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, unsigned parity, volatile int *abort_word, int *error)
{
    const bool ok = mbar_wait_bounded(bar, parity, abort_word, error, kPgSpinLimit);
    return __all_sync(0xffffffffu, ok);
}

static __global__ void __launch_bounds__(kPgThreads, 1) prefill_gemm_kernel(PrefillGemmParams p)
{
    extern __shared__ __align__(1024) uint8_t pg_raw[];
    const uint32_t raw = smem_u32(pg_raw);
    uint8_t *base = pg_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *ring = base;
    uint8_t *bring = base + kPgStages * kPgStageBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + kPgBarOffset);
    uint64_t *full = bars, *empty = bars + kPgStages, *bfull = bars + 2 * kPgStages,
             *bempty = bars + 2 * kPgStages + kPgBStages, *accf = bars + 2 * kPgStages + 2 * kPgBStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);
    volatile int *abort_word = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt = blockIdx.x, tt = blockIdx.y, split = blockIdx.z;
    const int k0 = (int)((long long)split * p.kchunks / p.splits);
    const int nk = (int)((long long)(split + 1) * p.kchunks / p.splits) - k0;
    const int tile0 = rt * (kPgN / kTileRows);
    const int ntiles = min(kPgN / kTileRows, p.rows / kTileRows - tile0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPgStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < kPgBStages; b++) {
            mbar_init(&bfull[b], 4);
            mbar_init(&bempty[b], 1);
        }
        mbar_init(accf, 1);
        *abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, kPgN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- loads: activation hi and lo (one 16 KB copy each) and the FP8
        // weights (a 512-byte half block of each of the 32 tiles)
        const uint32_t tx = 2 * kPgATile + (uint32_t)ntiles * 512;
        int issued = 0;
        for (int i = 0; i < nk; i++) {
            const int s = i % kPgStages, u = i / kPgStages;
            if (u > 0 && !warp_wait(&empty[s], (u - 1) & 1, abort_word, p.error)) break;
            uint8_t *st = ring + s * kPgStageBytes;
            const int kc = k0 + i;
            if (lane == 0) mbar_expect_tx(&full[s], tx);
            __syncwarp();
            const uint8_t *a = p.xs + ((size_t)(tt * p.kchunks + kc) * 2) * kPgATile;
            if (lane == 0) bulk_g2s(st, a, kPgATile, &full[s]);
            if (lane == 1) bulk_g2s(st + kPgATile, a + kPgATile, kPgATile, &full[s]);
            if (lane < ntiles)
                bulk_g2s(st + 2 * kPgATile + lane * 512,
                         p.W + (size_t)(tile0 + lane) * p.nb * kBlockBytes + (size_t)(kc >> 1) * kBlockBytes +
                             (kc & 1) * 512,
                         512, &full[s]);
            issued = i + 1;
        }
        // no copy may still be in flight when the CTA ends: wait for the
        // stages whose slots were not reused
        for (int i = max(0, issued - kPgStages); i < issued; i++) {
            for (unsigned spins = 0; !mbar_try_wait(&full[i % kPgStages], (i / kPgStages) & 1); spins++) {
                if (spins > kPgSpinLimit) {
                    *abort_word = 1;
                    atomicExch(p.error, 1);
                    break;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = f16_idesc(kPgM, kPgN);
            for (int i = 0; i < nk; i++) {
                const int s = i % kPgStages, u = i / kPgStages, b = i % kPgBStages, v = i / kPgBStages;
                if (!mbar_wait_bounded(&full[s], u & 1, abort_word, p.error, kPgSpinLimit) ||
                    !mbar_wait_bounded(&bfull[b], v & 1, abort_word, p.error, kPgSpinLimit))
                    break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(ring + s * kPgStageBytes), b0 = smem_u32(bring + b * kPgBBytes);
#pragma unroll
                for (int k = 0; k < kPgK / 16; k++) {
#pragma unroll
                    for (int part = 0; part < 2; part++)
                        tc_mma_f16(tmem, sw128_desc(a0 + part * kPgATile + k * 32), sw128_desc(b0 + k * 32), idesc,
                                   (i | k | part) != 0);
                }
                tc_commit(&empty[s]);
                tc_commit(&bempty[b]);
            }
            tc_commit(accf);
            // the accumulator (and every MMA) is done before the CTA tears down
            mbar_wait_bounded(accf, 0, abort_word, p.error, kPgSpinLimit);
        }
        __syncwarp();
    } else {
        // ---- converters: FP8 half blocks (fragment order, gemv.cuh) -> FP16
        // K-major swizzled rows; then the epilogue
        const int c = threadIdx.x - 64;
        for (int i = 0; i < nk; i++) {
            const int s = i % kPgStages, u = i / kPgStages, b = i % kPgBStages, v = i / kPgBStages;
            if (!warp_wait(&full[s], u & 1, abort_word, p.error)) break;
            if (v > 0 && !warp_wait(&bempty[b], (v - 1) & 1, abort_word, p.error)) break;
            const uint8_t *w8 = ring + s * kPgStageBytes + 2 * kPgATile;
            uint8_t *bb = bring + b * kPgBBytes;
#pragma unroll 4
            for (int q = 0; q < kPgW8 / 16 / 128; q++) {
                const int chunk = q * 128 + c, tl = chunk >> 5, L = chunk & 31;
                uint4 w = make_uint4(0, 0, 0, 0);
                if (tl < ntiles) w = *reinterpret_cast<const uint4 *>(w8 + chunk * 16);
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
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bfull[b]);
        }
        // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = tokens of the tile
        if (warp_wait(accf, 0, abort_word, p.error) && !*abort_word) {
            tc_fence_after();
            const int quarter = warp & 3, m = 32 * quarter + lane, t = tt * kPgM + m;
            const float inv = p.inv_scale[t];
            float *dst = p.ws + ((size_t)split * p.token_tiles * kPgM + t) * p.ws_rows + (size_t)rt * kPgN;
            for (int cb = 0; cb < kPgN / 32; cb++) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(cb * 32), r);
                if (t < p.count) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(dst + cb * 32 + i) =
                            make_float4(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv,
                                        __uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kPgN);
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
};

__device__ __forceinline__ float finish_scale(const PrefillFinishParams &p, int r)
{
    return r < p.bound[0] ? p.scale[0] : (r < p.bound[1] ? p.scale[1] : p.scale[2]);
}

// Grid (ceil(rows / 2 / 256), count): one thread per token and storage row pair.
template <int EPI>
static __global__ void __launch_bounds__(256) prefill_finish_kernel(PrefillFinishParams p)
{
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
        const int pos = (p.step ? p.step->length : p.length) + t;
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
            const int page = p.page_table[pos / kPage], slot = pos % kPage;
            float *dst = p.kv + kv_offset(p.layer, p.num_pages, page, kind, kvh, slot);
            dst[j] = a;
            dst[j + 64] = b;
        }
    }
}

}  // namespace lun
