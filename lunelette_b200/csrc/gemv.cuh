// FP8-E4M3 weight GEMV family for decode and short chunks (M = 1..4 token rows).
//
// Replaces project_fp8 / project_fp8_lookup (src/metal_kernels.metal:136-177,
// 249-272) and, by fusion, the norm, rope, element and KV-blit steps that the
// reference encodes around each projection (src/metal_encode.m:124-187).
// K and V rows are stored in FP32, the reference's KV precision.
//
// Tiled weight layout. Every FP8 matrix [rows][K] lives on the device as
// 8-row tiles; a tile is ceil(K/128) blocks of 1 KB (8 rows x 128 columns),
// stored in the order the m16n8k16 tensor-core MMA consumes them: byte
// h*512 + lane*16 + j*4 + i of a block holds tile row lane >> 2 and block column
// 64h + 16j + 2(lane & 3) + (i & 1) + 8(i >> 1). The MMA's 16 A rows are the
// tile's 8 rows twice, over the block's two 64-column halves (A row g: half 0,
// A row g + 8: half 1), so one coalesced 16-byte load per lane per half yields
// the A fragments of the block's four k16 MMAs. Rows past the matrix and
// columns past K are zero. Eight-row tiles split a 3072-row matrix over 148
// SMs as 2-3 tiles each instead of 1-2 sixteen-row tiles.
//
// Arithmetic. E4M3 codes become FP16 exactly (cvt.rn.f16x2.e4m3x2). The FP32
// activation row is scaled by an exact power of two 2^e (so its largest value
// sits in [2^14, 2^15)) and split into FP16 hi + lo halves (hi = rn(x),
// lo = rn(x - hi): 22 significant bits). The MMA's B operand carries hi and lo
// of each token and half as four columns (n = 4 * (token & 1) + 2 * half + lo);
// FP16 x FP16 products are exact and accumulate in FP32 on the tensor core, and
// a row's sum is its hi and lo columns of both halves times 2^-e, times the
// per-tensor scale in the epilogue. This keeps the projections within
// FP32 summation noise of the reference's FP32 dot products while replacing ten
// CUDA-core instructions per four weights with two conversions and a quarter MMA.
#pragma once
#include "common.cuh"
#include "async.cuh"

namespace lun {

enum GemvEpilogue : int {
    kEpiStore = 0,     // y[m][r] = acc * scale(r)
    kEpiResidual = 1,  // y[m][r] = res[m][r] + acc * scale(r)
    kEpiQKV = 2,       // rows [q|k|v]: RoPE on q,k (+query scale); q -> y, k/v -> KV pool
    kEpiSwiGLU = 3,    // alternating gate/up rows: y[m][f] = silu(g) * u
};

constexpr int kTileRows = 8;
constexpr int kBlockCols = 128;
constexpr int kBlockBytes = 1024;

// Bytes of a matrix in the tiled layout (rows padded to 8, columns to 128).
__host__ __device__ constexpr size_t tiled_bytes(size_t rows, size_t cols)
{
    return ((rows + 7) / 8) * 8 * ((cols + 127) / 128) * 128;
}

// Row orders the upload applies before tiling (storage row of source row r):
//   kOrderRows       row0 + r
//   kOrderRopePairs  inside every 128-row head, row j < 64 -> 2j, j + 64 -> 2j + 1
//                    (RoPE pairs adjacent), offset by row0
//   kOrderInterleave 2r + row0 (gate rows even, up rows odd)
enum TileOrder : int { kOrderRows = 0, kOrderRopePairs = 1, kOrderInterleave = 2 };

__host__ __device__ __forceinline__ int tile_storage_row(int order, int row0, int r)
{
    if (order == kOrderRopePairs) {
        const int j = r & 127;
        return row0 + (r & ~127) + (j < 64 ? 2 * j : 2 * (j - 64) + 1);
    }
    if (order == kOrderInterleave) return 2 * r + row0;
    return row0 + r;
}

// Row-major [rows][cols] codes (cols % 16 == 0) -> tiled matrix of dst_nb blocks
// per tile; one thread per 16-column chunk. Padding is the caller's (zeroed) memory.
static __global__ void tile_fp8_kernel(const uint8_t *src, int rows, int cols, uint8_t *dst, int dst_nb,
                                       int order, int row0)
{
    const int chunks_per_row = cols >> 4;
    const size_t chunks = (size_t)rows * chunks_per_row;
    for (size_t u = (size_t)blockIdx.x * blockDim.x + threadIdx.x; u < chunks; u += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(u / chunks_per_row), q = (int)(u % chunks_per_row);
        const uint4 v = *reinterpret_cast<const uint4 *>(src + (size_t)r * cols + (size_t)q * 16);
        const int s = tile_storage_row(order, row0, r);
        const int tile = s >> 3, g = s & 7, kb = q >> 3, h = (q >> 2) & 1, j = q & 3;
        uint8_t *blk = dst + ((size_t)tile * dst_nb + kb) * kBlockBytes + h * 512 + j * 4;
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int t4 = 0; t4 < 4; t4++) {
            const int sh = 16 * (t4 & 1);
            const uint32_t lo = (w[t4 >> 1] >> sh) & 0xffffu, hi = (w[2 + (t4 >> 1)] >> sh) & 0xffffu;
            *reinterpret_cast<uint32_t *>(blk + (g * 4 + t4) * 16) = lo | (hi << 16);
        }
    }
}

// ---- MMA helpers -------------------------------------------------------------
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_codes)
{
    uint32_t h;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)(two_codes & 0xffffu)));
    return h;
}

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The four k16 MMAs of one block: wa/wb are this lane's 16 bytes of tile row g
// in the block's two halves, x0/x1 its B fragments (zero on unused lanes).
__device__ __forceinline__ void mma_block(float (&c)[4], const uint4 &wa, const uint4 &wb, const uint4 &x0,
                                          const uint4 &x1)
{
    mma_f16_16816(c, e4m3x2_to_f16x2(wa.x), e4m3x2_to_f16x2(wb.x), e4m3x2_to_f16x2(wa.x >> 16),
                  e4m3x2_to_f16x2(wb.x >> 16), x0.x, x0.y);
    mma_f16_16816(c, e4m3x2_to_f16x2(wa.y), e4m3x2_to_f16x2(wb.y), e4m3x2_to_f16x2(wa.y >> 16),
                  e4m3x2_to_f16x2(wb.y >> 16), x0.z, x0.w);
    mma_f16_16816(c, e4m3x2_to_f16x2(wa.z), e4m3x2_to_f16x2(wb.z), e4m3x2_to_f16x2(wa.z >> 16),
                  e4m3x2_to_f16x2(wb.z >> 16), x1.x, x1.y);
    mma_f16_16816(c, e4m3x2_to_f16x2(wa.w), e4m3x2_to_f16x2(wb.w), e4m3x2_to_f16x2(wa.w >> 16),
                  e4m3x2_to_f16x2(wb.w >> 16), x1.z, x1.w);
}

// The same four MMAs with k16 step j accumulating into c[j]: independent
// accumulators let consecutive MMAs issue back to back instead of each waiting
// for the previous one's result.
__device__ __forceinline__ void mma_block4(float (&c)[4][4], const uint4 &wa, const uint4 &wb, const uint4 &x0,
                                           const uint4 &x1)
{
    mma_f16_16816(c[0], e4m3x2_to_f16x2(wa.x), e4m3x2_to_f16x2(wb.x), e4m3x2_to_f16x2(wa.x >> 16),
                  e4m3x2_to_f16x2(wb.x >> 16), x0.x, x0.y);
    mma_f16_16816(c[1], e4m3x2_to_f16x2(wa.y), e4m3x2_to_f16x2(wb.y), e4m3x2_to_f16x2(wa.y >> 16),
                  e4m3x2_to_f16x2(wb.y >> 16), x0.z, x0.w);
    mma_f16_16816(c[2], e4m3x2_to_f16x2(wa.z), e4m3x2_to_f16x2(wb.z), e4m3x2_to_f16x2(wa.z >> 16),
                  e4m3x2_to_f16x2(wb.z >> 16), x1.x, x1.y);
    mma_f16_16816(c[3], e4m3x2_to_f16x2(wa.w), e4m3x2_to_f16x2(wb.w), e4m3x2_to_f16x2(wa.w >> 16),
                  e4m3x2_to_f16x2(wb.w >> 16), x1.z, x1.w);
}

// ---- activation fragments ------------------------------------------------------
// Staged per 64-column piece c64 of the activation rows: `lanes` = 8 * tokens
// lanes per half piece, as uint4 index (c64 * 2 + half) * lanes + 4u + t4 for
// u = 2 * token + (0 hi, 1 lo). Word (j & 1) * 2 + b of that uint4 holds MMA j
// (j >> 1 == half) register b: columns 16j + 2t4 + 8b and the next one. An MMA
// lane with B column n reads piece 2 * block + ((n >> 1) & 1), u = 2 * token + (n & 1).
__device__ __forceinline__ void frag_store_pair(uint32_t *frag, int lanes, int c, int n, uint32_t pair)
{
    const int kb = c >> 6, w = c & 63, j = w >> 4, ww = w & 15;
    const int t4 = (ww & 7) >> 1, b = ww >> 3;
    frag[((size_t)(kb * 2 + (j >> 1)) * lanes + n * 4 + t4) * 4 + (j & 1) * 2 + b] = pair;
}

__device__ __forceinline__ uint32_t half2_bits(__half a, __half b)
{
    __half2 h = __halves2half2(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// hi/lo FP16 split of two (already scaled) values.
__device__ __forceinline__ void split_hilo(float a, float b, uint32_t &hi, uint32_t &lo)
{
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    hi = half2_bits(ha, hb);
    lo = half2_bits(__float2half_rn(a - __half2float(ha)), __float2half_rn(b - __half2float(hb)));
}

// Exponent e with bound * 2^e < 2^15 for an upper bound of the row's magnitudes
// (0 for an all-zero or non-finite row, whose NaN/Inf then propagate).
__device__ __forceinline__ int frag_exponent(float bound)
{
    if (!(bound > 0.0f) || !isfinite(bound)) return 0;
    const int e = 14 - ((int)((__float_as_uint(bound) >> 23) & 0xffu) - 127);
    return e < -100 ? -100 : (e > 100 ? 100 : e);
}

__device__ __forceinline__ float exp2i(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

// ---- multi-token GEMV ------------------------------------------------------------
struct GemvParams {
    const uint8_t *W;    // tiled matrix
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
    // One-token callers may stage epilogue operands in shared memory: the RoPE
    // row of the position (cos[128] then sin[128]) and residual rows
    // [res_base, ...) of token 0; nullptr reads the global arrays above.
    const float *rope_row;
    const float *res_shared;
    int res_base;
    // kEpiResidual, one token: the output rows also as 64-bit fixed point
    // (value * 2^32, rounded), or nullptr; a value the fixed point cannot hold
    // sets kFlagFixedRange in *range_flag
    long long *y_fixed;
    int *range_flag;
    // kEpiSwiGLU, one token: feature f goes to y[f - y_base] (a slice of the
    // features staged in shared memory); 0 otherwise
    int y_base;
    // One-token QKV epilogue for readers on other CTAs: q rows and the
    // position's k and v rows also go out as tagged words (store_tagged) to
    // qkv_tagged[0..4096) (q), [4096..5120) (k), [5120..6144) (v), tag ytag;
    // q then skips y.
    unsigned long long *qkv_tagged;
    unsigned ytag;
    // Batched decode over independent sessions (the tcgen05 path's QKV
    // epilogue): token t at position positions[t] of page table page_table +
    // token_table[t] * table_stride; nullptr for one sequence.
    const int *positions, *token_table;
    int table_stride;
};

// A value and the tag of the phase that produced it in one 64-bit word: a
// reader that sees the expected tag sees the value written with it (a single
// aligned 8-byte store), so no separate flag, fence or counter is needed.
__device__ __forceinline__ void store_tagged(unsigned long long *dst, float v, unsigned tag)
{
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.global.u64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
}

// Stage M activation rows (normed when p.gain) as hi/lo B fragments for the
// whole block; inv_scale[m] = 2^-e of row m. red: 16 * M floats of scratch.
template <int M>
__device__ __forceinline__ void gemv_stage(const GemvParams &p, uint32_t *frag, float *inv_scale, float *red)
{
    const int cols = p.cols, NB = 2 * ((cols + 127) >> 7), lanes = 8 * M;  // 64-column pieces
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    float ss[M], mx[M];
#pragma unroll
    for (int m = 0; m < M; m++) {
        ss[m] = 0.0f;
        mx[m] = 0.0f;
        const float *xr = p.x + (size_t)m * p.x_stride;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            const float v = xr[c];
            ss[m] += v * v;
            mx[m] = fmaxf(mx[m], fabsf(p.gain ? p.gain[c] * v : v));
        }
        ss[m] = warp_sum(ss[m]);
        mx[m] = warp_max(mx[m]);
        if (lane == 0) {
            red[(warp * M + m) * 2] = ss[m];
            red[(warp * M + m) * 2 + 1] = mx[m];
        }
    }
    __syncthreads();
    float rs[M], sc[M];
#pragma unroll
    for (int m = 0; m < M; m++) {
        float s = 0.0f, x = 0.0f;
        for (int w = 0; w < warps; w++) {
            s += red[(w * M + m) * 2];
            x = fmaxf(x, red[(w * M + m) * 2 + 1]);
        }
        rs[m] = p.gain ? rsqrtf(s / (float)cols + kNormEps) : 1.0f;
        const int e = frag_exponent(x * rs[m] * 1.0001f);
        sc[m] = exp2i(e);
        if (threadIdx.x == 0) inv_scale[m] = exp2i(-e);
    }
    // column pairs (c, c+1); columns in [cols, 64 * NB) are zero
    for (int c = 2 * threadIdx.x; c < 64 * NB; c += 2 * blockDim.x) {
        float g0 = 1.0f, g1 = 1.0f;
        if (p.gain && c < cols) {
            g0 = p.gain[c];
            g1 = p.gain[c + 1];
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            uint32_t hi = 0, lo = 0;
            if (c < cols) {
                const float *xr = p.x + (size_t)m * p.x_stride;
                float a = xr[c], b = xr[c + 1];
                if (p.gain) {
                    a = g0 * (a * rs[m]);
                    b = g1 * (b * rs[m]);
                }
                split_hilo(a * sc[m], b * sc[m], hi, lo);
            }
            frag_store_pair(frag, lanes, c, 2 * m, hi);
            frag_store_pair(frag, lanes, c, 2 * m + 1, lo);
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
                        if (EPI == kEpiResidual)
                            v = (p.res_shared ? p.res_shared[r - p.res_base]
                                              : __ldcg(&p.res[(size_t)m * p.res_stride + r])) +
                                v;
                        p.y[(size_t)m * p.y_stride + r] = v;
                        if (EPI == kEpiResidual && p.y_fixed) {
                            p.y_fixed[r] = __float2ll_rn(v * 0x1p32f);
                            if (!(fabsf(v) < kFixedTermLimit)) atomicOr(p.range_flag, kFlagFixedRange);
                        }
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
                p.y[(size_t)m * p.y_stride + f - p.y_base] = silu * b;
            } else {
                // QKV: ra = head*128 + j (j < 64), rb = ra + 64
                int pos = (p.step ? p.step->length : p.length) + p.token_offset + m;
                int j = ra & 127;
                if (ra < kQuery + kKV) {
                    const float *cs = p.rope_row ? p.rope_row : p.rope_cos + (size_t)pos * 128;
                    const float *sn = p.rope_row ? p.rope_row + 128 : p.rope_sin + (size_t)pos * 128;
                    float lo = a * cs[j] + (-b) * sn[j];
                    float hi = b * cs[j + 64] + a * sn[j + 64];
                    a = lo;
                    b = hi;
                }
                if (ra < kQuery) {
                    float qs = query_scale(pos);
                    if (p.qkv_tagged) {
                        store_tagged(p.qkv_tagged + ra, a * qs, p.ytag);
                        store_tagged(p.qkv_tagged + rb, b * qs, p.ytag);
                    } else {
                        p.y[(size_t)m * p.y_stride + ra] = a * qs;
                        p.y[(size_t)m * p.y_stride + rb] = b * qs;
                    }
                } else {
                    int kind = ra < kQuery + kKV ? 0 : 1;
                    int head = (ra - kQuery - kind * kKV) >> 7;
                    int page = p.page_table[pos / kPage], slot = pos % kPage;
                    float *dst = p.kv + kv_offset(p.layer, p.num_pages, page, kind, head, slot);
                    dst[j] = a;
                    dst[j + 64] = b;
                    if (p.qkv_tagged) {
                        store_tagged(p.qkv_tagged + ra, a, p.ytag);
                        store_tagged(p.qkv_tagged + rb, b, p.ytag);
                    }
                }
            }
        }
    }
    }
}

// One launch: 8 warps per block, grid-stride over 8-row tiles. The warps split
// a tile's blocks (warp w takes blocks w, w+8, ...), one MMA per token pair and
// k16 step; their partial row sums are added in warp order (deterministic) and
// warps 0-1 run the epilogue of the tile's two row groups.
template <int M, int EPI>
__global__ void __launch_bounds__(256) gemv_tiled_kernel(GemvParams p)
{
    constexpr int kPairs = (M + 1) / 2;
    extern __shared__ uint4 frag4[];
    __shared__ float part[8][8][M];
    __shared__ float inv_scale[M];
    __shared__ float red[16 * M];
    // this block's first tiles (contiguous NB KB each) start towards L2 before
    // the activation row is staged: the weights depend on no earlier kernel
    {
        const int NB = (p.cols + 127) >> 7, tiles = (p.rows + 7) >> 3;
        const int tile = blockIdx.x + (int)threadIdx.x * (int)gridDim.x;
        if (threadIdx.x < 4 && tile < tiles)
            l2_prefetch(p.W + (size_t)tile * NB * kBlockBytes, (unsigned)(NB * kBlockBytes));
    }
    l2_prefetch_share(p.prefetch, p.prefetch_bytes);
    pdl_wait();
    pdl_launch_dependents();
    gemv_stage<M>(p, reinterpret_cast<uint32_t *>(frag4), inv_scale, red);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const int NB = (p.cols + 127) >> 7, tiles = (p.rows + 7) >> 3, lanes = 8 * M;
    // this lane's B column g: token 2 * pair + (g >> 2), half (g >> 1) & 1, hi/lo g & 1
    const int slot = (2 * (g >> 2) + (g & 1)) * 4 + t4;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const uint8_t *tw = p.W + (size_t)tile * NB * kBlockBytes;
        float c[kPairs][4];
#pragma unroll
        for (int tp = 0; tp < kPairs; tp++) c[tp][0] = c[tp][1] = c[tp][2] = c[tp][3] = 0.0f;
#pragma unroll 2
        for (int kb = warp; kb < NB; kb += 8) {
            const uint4 wa = ld_stream(tw + (size_t)kb * kBlockBytes + lane * 16);
            const uint4 wb = ld_stream(tw + (size_t)kb * kBlockBytes + 512 + lane * 16);
            const int piece = 2 * kb + ((g >> 1) & 1);
#pragma unroll
            for (int tp = 0; tp < kPairs; tp++) {
                uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
                if (2 * tp + (g >> 2) < M) {
                    const int l = slot + 16 * tp;
                    x0 = frag4[(piece * 2) * lanes + l];
                    x1 = frag4[(piece * 2 + 1) * lanes + l];
                }
                mma_block(c[tp], wa, wb, x0, x1);
            }
        }
        // lane (g, t4) holds token 2 * pair + (t4 >> 1), half t4 & 1 of row g
#pragma unroll
        for (int tp = 0; tp < kPairs; tp++) {
            float v = (t4 & 1) ? c[tp][2] + c[tp][3] : c[tp][0] + c[tp][1];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            const int m = 2 * tp + (t4 >> 1);
            if (!(t4 & 1) && m < M) part[warp][g][m] = v;
        }
        __syncthreads();
        if (warp < 2) {
            float acc[4][M];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int m = 0; m < M; m++) {
                    float s = 0.0f;
#pragma unroll
                    for (int w = 0; w < 8; w++) s += part[w][warp * 4 + i][m];
                    acc[i][m] = s * inv_scale[m];
                }
            gemv_epilogue<M, EPI>(p, tile * 2 + warp, lane, acc);
        }
        __syncthreads();
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

// ---- tied head over several token rows (batched decode) -----------------------------
// Parameters of the tensor-core head of head_mma.cuh: logits[r][v] =
// E[v] . rmsnorm(x[r]) for r < count (at most 64 rows per launch pair).
struct HeadMmaParams {
    const uint16_t *W;     // BF16 [rows][3072]
    int rows;
    const float *x;        // [count][x_stride] hidden rows
    int x_stride, count;   // count <= kHmTokens
    const float *gain;
    uint16_t *xb;          // kHmStageElems staged B operand
    float *logits;         // [count][logits_stride]
    int logits_stride;
    int *nonfinite;
    int *error;            // set when a bounded wait of the tcgen05 head gives up
};

}  // namespace lun
