#include "kernels.h"

#include <atomic>
#include <mutex>

#include <cudaTypedefs.h>

#include "attention_tc.cuh"
#include "head_mma.cuh"
#include "head_tc.cuh"
#include "launch.h"

#include <stdlib.h>

using namespace lun;

namespace {

constexpr int kMaxGemvSmem = (kInner / 64) * 256 * 4;  // B fragments of 4 rows x 9216 columns

template <int M, int EPI>
cudaError_t setup_one()
{
    return cudaFuncSetAttribute(gemv_tiled_kernel<M, EPI>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxGemvSmem);
}

template <int EPI>
cudaError_t setup_epi()
{
    cudaError_t e;
    if ((e = setup_one<1, EPI>()) != cudaSuccess) return e;
    if ((e = setup_one<2, EPI>()) != cudaSuccess) return e;
    if ((e = setup_one<3, EPI>()) != cudaSuccess) return e;
    return setup_one<4, EPI>();
}

// B fragments: 256 bytes per token per 64-column piece (columns padded to 128).
template <int M, int EPI>
cudaError_t launch_one(const GemvParams &p, int sm_count, cudaStream_t stream)
{
    const size_t smem = (size_t)((p.cols + 127) / 128) * 2 * 256 * M;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_tiled_kernel<M, EPI>,
                                                                  256, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    int blocks = (p.rows + 7) / 8;
    int limit = sm_count * per_sm;
    if (blocks > limit) blocks = limit;
    return launch(gemv_tiled_kernel<M, EPI>, dim3(blocks), dim3(256), smem, stream, p);
}

template <int EPI>
cudaError_t launch_epi(const GemvParams &p, int m, int sm_count, cudaStream_t stream)
{
    switch (m) {
    case 1: return launch_one<1, EPI>(p, sm_count, stream);
    case 2: return launch_one<2, EPI>(p, sm_count, stream);
    case 3: return launch_one<3, EPI>(p, sm_count, stream);
    case 4: return launch_one<4, EPI>(p, sm_count, stream);
    default: return cudaErrorInvalidValue;
    }
}

__global__ void rmsnorm_kernel(const float *gain, const float *x, float *out, int width)
{
    __shared__ float red[32];
    pdl_wait();
    pdl_launch_dependents();
    const float *xr = x + (size_t)blockIdx.x * width;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < width; c += blockDim.x) ss += xr[c] * xr[c];
    ss = block_sum(ss, red);
    float rs = rsqrtf(ss / (float)width + kNormEps);
    for (int c = threadIdx.x; c < width; c += blockDim.x)
        out[(size_t)blockIdx.x * width + c] = gain[c] * (xr[c] * rs);
}

__global__ void fp8_decode_kernel(const uint8_t *codes, size_t n, float scale, float *out)
{
    size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 2;
    if (i >= n) return;
    uint32_t two = codes[i] | (i + 1 < n ? (uint32_t)codes[i + 1] << 8 : 0u);
    float2 v = e4m3x2_to_float2(two);
    out[i] = v.x * scale;
    if (i + 1 < n) out[i + 1] = v.y * scale;
}

// Better of two (value, index) candidates: larger value, then lower index.
__device__ __forceinline__ void better(float &v, int &i, float v2, int i2)
{
    if (v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

__device__ __forceinline__ void block_best(float &v, int &i)
{
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        int i2 = __shfl_xor_sync(0xffffffffu, i, o);
        better(v, i, v2, i2);
    }
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = i;
    }
    __syncthreads();
    if (warp == 0) {
        int warps = blockDim.x >> 5;
        v = lane < warps ? sv[lane] : -INFINITY;
        i = lane < warps ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            int i2 = __shfl_xor_sync(0xffffffffu, i, o);
            better(v, i, v2, i2);
        }
    }
}

__global__ void __launch_bounds__(256) argmax_partial_kernel(const float *logits, int n, int *partials)
{
    pdl_wait();
    pdl_launch_dependents();
    int per = (n + gridDim.x - 1) / gridDim.x;
    int begin = blockIdx.x * per, end = min(begin + per, n);
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int k = begin + threadIdx.x; k < end; k += blockDim.x) better(v, i, logits[k], k);
    block_best(v, i);
    if (threadIdx.x == 0) {
        partials[2 * blockIdx.x] = __float_as_int(v);
        partials[2 * blockIdx.x + 1] = i;
    }
}

__global__ void __launch_bounds__(256) argmax_final_kernel(const int *partials, int blocks,
                                                           StepParams *step, int *tokens)
{
    pdl_wait();
    pdl_launch_dependents();
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int k = threadIdx.x; k < blocks; k += blockDim.x)
        better(v, i, __int_as_float(partials[2 * k]), partials[2 * k + 1]);
    block_best(v, i);
    if (threadIdx.x == 0) {
        int id = i == 0x7fffffff ? 0 : i;
        step->ids[0] = id;
        tokens[step->generated] = id;
        step->generated += 1;
        step->length += 1;
    }
}

}  // namespace

cudaError_t lun_launch_greedy(const float *logits, int n, int *partials, StepParams *step,
                              int *tokens, cudaStream_t stream)
{
    cudaError_t e = launch(argmax_partial_kernel, dim3(kArgmaxBlocks), dim3(256), 0, stream, logits, n,
                           partials);
    if (e != cudaSuccess) return e;
    return launch(argmax_final_kernel, dim3(1), dim3(256), 0, stream, (const int *)partials,
                  (int)kArgmaxBlocks, step, tokens);
}

cudaError_t lun_launch_embed(const uint16_t *embedding, const StepParams *step, float *x, int count,
                             cudaStream_t stream)
{
    return launch(embed_kernel, dim3(count), dim3(256), 0, stream, embedding, step, x, count);
}

// Function attributes apply to the current device; calling again is cheap.
cudaError_t lun_kernels_init()
{
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(attention_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kAttnSmemBytes)) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(attention_prefill_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kPmSmemBytes)) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(attention_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kTaSmemBytes)) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(head_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kHtSmemBytes)) !=
        cudaSuccess)
        return e;
    if ((e = setup_epi<kEpiStore>()) != cudaSuccess) return e;
    if ((e = setup_epi<kEpiResidual>()) != cudaSuccess) return e;
    if ((e = setup_epi<kEpiQKV>()) != cudaSuccess) return e;
    return setup_epi<kEpiSwiGLU>();
}

// Dynamic shared memory above 48 KB needs a per-device opt-in; do it on first
// use. Callers on several threads may arrive together: the flags are atomic and
// the set-up itself runs under a lock, once per device.
cudaError_t lun_kernels_ensure()
{
    static std::atomic<bool> done[128];
    static std::mutex setup;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return lun_kernels_init();
    if (done[dev].load(std::memory_order_acquire)) return cudaSuccess;
    std::lock_guard<std::mutex> lock(setup);
    if (done[dev].load(std::memory_order_relaxed)) return cudaSuccess;
    e = lun_kernels_init();
    if (e == cudaSuccess) done[dev].store(true, std::memory_order_release);
    return e;
}

cudaError_t lun_launch_gemv(const GemvParams &p, int m, int epilogue, int sm_count,
                            cudaStream_t stream)
{
    if (p.cols <= 0 || (p.cols & 15) || p.rows <= 0 || (size_t)m * p.cols * 4 > (size_t)kMaxGemvSmem)
        return cudaErrorInvalidValue;
    cudaError_t ie = lun_kernels_ensure();
    if (ie != cudaSuccess) return ie;
    switch (epilogue) {
    case kEpiStore: return launch_epi<kEpiStore>(p, m, sm_count, stream);
    case kEpiResidual: return launch_epi<kEpiResidual>(p, m, sm_count, stream);
    case kEpiQKV: return launch_epi<kEpiQKV>(p, m, sm_count, stream);
    case kEpiSwiGLU: return launch_epi<kEpiSwiGLU>(p, m, sm_count, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t lun_launch_head(const HeadParams &p, int sm_count, cudaStream_t stream)
{
    if (p.cols <= 0 || (p.cols & 7)) return cudaErrorInvalidValue;
    const size_t smem = (size_t)p.cols * 4;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, head_bf16_kernel, 256, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    int groups = (p.rows + 3) / 4;
    int blocks = (groups + 7) / 8;
    if (blocks > sm_count * per_sm) blocks = sm_count * per_sm;
    return launch(head_bf16_kernel, dim3(blocks), dim3(256), smem, stream, p);
}

constexpr int kAttnMaxSplit = 512;

// Blocks of more than kGemvMaxTokens tokens of one sequence run the tcgen05
// attention (attention_tc.cuh) unless LUNELETTE_TC_ATTENTION=0 selects the
// mma.sync kernel (attention.cuh).
static bool tc_attention_enabled()
{
    static const bool on = [] {
        const char *v = getenv("LUNELETTE_TC_ATTENTION");
        return !(v && v[0] == '0');
    }();
    return on;
}

void lun_attention_plan(AttnParams *a, int total, int count, int sm_count, int slots)
{
    if (count > kGemvMaxTokens && !a->positions) {
        // blocks of one sequence's tokens (attention_prefill_mma_kernel): key
        // ranges of whole pages split so that about two waves of blocks run
        // (the tcgen05 kernel holds a whole SM: at most one wave of its blocks)
        const int qtiles = (count + kPmTokens - 1) / kPmTokens;
        const int pages = (total + kPage - 1) / kPage;
        int splits = tc_attention_enabled() ? sm_count / (qtiles * kKVHeads)
                                            : (4 * sm_count + qtiles * kKVHeads - 1) / (qtiles * kKVHeads);
        const int cap = slots / (count * kQueryHeads);
        splits = splits > cap ? cap : splits;
        splits = splits < 1 ? 1 : (splits > pages ? pages : splits);
        const int per = (pages + splits - 1) / splits;
        a->split_len = per * kPage;
        a->splits = (pages + per - 1) / per;
        return;
    }
    int wanted = (2 * sm_count + 8 * count - 1) / (8 * count);  // splits per (token, kv head)
    // and no split longer than kAttnMaxSplit positions: a long sequence among
    // many short ones (batched decode) must not stream its prefix serially
    const int by_length = (total + kAttnMaxSplit - 1) / kAttnMaxSplit;
    if (wanted < by_length) wanted = by_length;
    if (wanted < 1) wanted = 1;
    int split_len = (total + wanted - 1) / wanted;
    split_len = (split_len + kTile - 1) / kTile * kTile;
    if (split_len < kTile) split_len = kTile;
    int splits = (total + split_len - 1) / split_len;
    int cap = slots / (count * kQueryHeads);
    if (cap < 1) cap = 1;
    if (splits > cap) {
        splits = cap;
        split_len = (total + splits - 1) / splits;
        split_len = (split_len + kTile - 1) / kTile * kTile;
        splits = (total + split_len - 1) / split_len;
    }
    a->split_len = split_len;
    a->splits = splits;
}

cudaError_t lun_launch_attention(const AttnParams &a, int count, cudaStream_t stream)
{
    cudaError_t e = lun_kernels_ensure();
    if (e != cudaSuccess) return e;
    if (count > kGemvMaxTokens && !a.positions) {  // blocks of one sequence's tokens: key pages per 8 query tokens
        if (a.splits < 1 || a.split_len < kPage || (a.split_len % kPage)) return cudaErrorInvalidValue;
        const dim3 grid((count + kPmTokens - 1) / kPmTokens, kKVHeads, a.splits);
        if (tc_attention_enabled())
            e = launch(attention_prefill_tc_kernel, grid, dim3(kTaThreads), kTaSmemBytes, stream, a, count);
        else
            e = launch(attention_prefill_mma_kernel, grid, dim3(kPmThreads), kPmSmemBytes, stream, a, count);
        if (e != cudaSuccess || a.splits == 1) return e;
        return launch(attention_combine_kernel, dim3(kQueryHeads, count), dim3(128), 0, stream, a);
    }
    if (a.splits < 1 || a.split_len < kTile || (a.split_len % kTile)) return cudaErrorInvalidValue;
    dim3 grid(a.splits, kKVHeads, count);
    e = launch(attention_split_kernel, grid, dim3(128), kAttnSmemBytes, stream, a);
    if (e != cudaSuccess || a.splits == 1) return e;
    return launch(attention_combine_kernel, dim3(kQueryHeads, count), dim3(128), 0, stream, a);
}

cudaError_t lun_launch_rmsnorm(const float *gain, const float *x, float *out, int width, int count,
                               cudaStream_t stream)
{
    if (width <= 0 || count <= 0) return cudaErrorInvalidValue;
    return launch(rmsnorm_kernel, dim3(count), dim3(256), 0, stream, gain, x, out, width);
}

cudaError_t lun_launch_tile_fp8(const uint8_t *src, int rows, int cols, uint8_t *dst, int dst_nb, int order,
                                int row0, cudaStream_t stream)
{
    if (rows <= 0 || cols <= 0 || (cols & 15) || dst_nb < (cols + 127) / 128) return cudaErrorInvalidValue;
    const size_t chunks = (size_t)rows * (cols / 16);
    size_t blocks = (chunks + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    tile_fp8_kernel<<<(unsigned)blocks, 256, 0, stream>>>(src, rows, cols, dst, dst_nb, order, row0);
    return cudaGetLastError();
}

cudaError_t lun_launch_fp8_decode(const uint8_t *codes, size_t n, float scale, float *out,
                                  cudaStream_t stream)
{
    if (!n) return cudaSuccess;
    size_t pairs = (n + 1) / 2;
    fp8_decode_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, stream>>>(codes, n, scale, out);
    return cudaGetLastError();
}

cudaError_t lun_launch_kv_copy(const KvCopyParams &p, int layers, cudaStream_t stream)
{
    if (p.pairs <= 0 || layers <= 0 || p.last_slots <= 0 || p.last_slots > kPage) return cudaErrorInvalidValue;
    kv_copy_kernel<<<dim3(p.pairs, layers * 2 * kKVHeads), 256, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t lun_launch_head_mma(const HeadMmaParams &p, cudaStream_t stream)
{
    if (p.count < 1 || p.count > kHmTokens || p.rows < kHmRows || (p.rows % kHmRows) || !p.xb)
        return cudaErrorInvalidValue;
    cudaError_t e = launch(head_mma_split_kernel, dim3(kHmTokens), dim3(256), 0, stream, p);
    if (e != cudaSuccess) return e;
    return launch(head_mma_kernel, dim3(p.rows / kHmRows), dim3(kHmThreads), kHmSmemBytes, stream, p);
}

PFN_cuTensorMapEncodeTiled_v12000 lun_tensor_map_encoder();

// The embedding as a 2-D BF16 tensor {3072, rows}: a box {64, 128} is one
// chunk of a CTA's 128 rows, landed in the 128-byte-swizzled K-major order the
// tensor core reads (head_tc_kernel).
static cudaError_t embedding_tensor_map(CUtensorMap *map, const uint16_t *E, int rows)
{
    PFN_cuTensorMapEncodeTiled_v12000 encode = lun_tensor_map_encoder();
    if (!encode || ((uintptr_t)E & 15)) return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {(cuuint64_t)kHidden, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kHidden * 2};
    const cuuint32_t box[2] = {kHtChunk, kHtRows};
    const cuuint32_t elem[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)E, dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t lun_launch_head_tc(const HeadMmaParams &p, cudaStream_t stream)
{
    if (p.count < 1 || p.count > kHmTokens || p.rows < kHtRows || (p.rows % kHtRows) || !p.xb || !p.error ||
        ((uintptr_t)p.xb & 15))
        return cudaErrorInvalidValue;
    cudaError_t e = lun_kernels_ensure();
    if (e != cudaSuccess) return e;
    CUtensorMap emap;
    if ((e = embedding_tensor_map(&emap, p.W, p.rows)) != cudaSuccess) return e;
    if ((e = launch(head_tc_split_kernel, dim3(kHmTokens), dim3(256), 0, stream, p)) != cudaSuccess) return e;
    return launch(head_tc_kernel, dim3(p.rows / kHtRows), dim3(kHtThreads), kHtSmemBytes, stream, p, emap);
}

size_t lun_head_mma_stage_bytes() { return kHmStageElems * sizeof(uint16_t); }
int lun_head_mma_tokens() { return kHmTokens; }

// out[t] = argmax of logits row t (strict '>', lowest id on ties:
// src/generation.c:8-34); one block of 1024 threads per row.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float *logits, int n, int stride, int *out)
{
    __shared__ float bv[32];
    __shared__ int bi[32];
    const float *row = logits + (size_t)blockIdx.x * stride;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = row[i];
        if (x > v || (x == v && i < idx)) {
            v = x;
            idx = i;
        }
    }
    for (int o = 16; o; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (v2 > v || (v2 == v && i2 < idx)) {
            v = v2;
            idx = i2;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        bv[threadIdx.x >> 5] = v;
        bi[threadIdx.x >> 5] = idx;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        v = bv[threadIdx.x];
        idx = bi[threadIdx.x];
        for (int o = 16; o; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
            if (v2 > v || (v2 == v && i2 < idx)) {
                v = v2;
                idx = i2;
            }
        }
        if (threadIdx.x == 0) out[blockIdx.x] = idx < n ? idx : 0;
    }
}

cudaError_t lun_launch_argmax_rows(const float *logits, int n, int stride, int rows, int *out, cudaStream_t stream)
{
    if (rows <= 0 || n <= 0) return cudaErrorInvalidValue;
    argmax_rows_kernel<<<rows, 1024, 0, stream>>>(logits, n, stride, out);
    return cudaGetLastError();
}
