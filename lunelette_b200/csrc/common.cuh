// Shared device helpers for the sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lun {

constexpr int kHidden = 3072;
constexpr int kQuery = 4096;
constexpr int kKV = 1024;
constexpr int kInner = 9216;
constexpr int kLayers = 26;
constexpr int kVocab = 131072;
constexpr int kHeadDim = 128;
constexpr int kQueryHeads = 32;
constexpr int kKVHeads = 8;
constexpr int kPage = 64;                        // KV positions per page
constexpr int kPageKind = kKVHeads * kPage * kHeadDim;  // elements of K (or V) per page per layer
constexpr float kNormEps = 1e-5f;
constexpr float kScoreScale = 0.08838834764831845f;  // 1/sqrt(128) as the reference rounds it
constexpr int kQKVRows = kQuery + 2 * kKV;       // 6144
constexpr int kGateUpRows = 2 * kInner;          // 18432: gate and up rows alternate (2f, 2f+1)
// Bits of a step's flag word (the host reads it after the step):
//   kFlagNonfinite    the head produced a NaN or infinite logit
//   kFlagFixedRange   a term added into a 64-bit fixed-point sum (32 fraction
//                     bits, range +-2^31) was non-finite or not below
//                     kFixedTermLimit, so the sum cannot be trusted; the host
//                     reruns the step on the FP32 path
constexpr int kFlagNonfinite = 1;
constexpr int kFlagFixedRange = 2;
// At most 145 terms reach one fixed-point element per layer (h from the o
// epilogue plus 144 act slices of down); 145 * 2^23 < 2^31.
constexpr float kFixedTermLimit = 0x1p23f;

// Per-call parameters that kernels read from device memory, so that one
// captured graph serves every step: the sequence length before the call.
struct StepParams {
    int length;
    int count;
    int generated;  // device greedy loop: tokens appended so far
    int pad;
    int ids[256];
};

// Programmatic dependent launch: the next kernel in the stream may start before
// this one finishes; pdl_wait() blocks until the previous kernel completed and
// its writes are visible (a no-op when launched without the attribute).
// Everything before pdl_wait() may only read immutable data (weights).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Ask L2 to fetch this block's share of [base, base+bytes) (bytes and base
// 16-byte aligned), in 16 KB bulk prefetches spread over the block's threads.
// Fire-and-forget: nothing waits for it; a later read finds the lines in L2.
__device__ __forceinline__ void l2_prefetch_share(const void *base, size_t bytes)
{
    if (!base || !bytes) return;
    size_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
    size_t begin = (size_t)blockIdx.x * per;
    size_t end = begin + per < bytes ? begin + per : bytes;
    const char *p = static_cast<const char *>(base);
    for (size_t off = begin + (size_t)threadIdx.x * 16384; off < end; off += (size_t)blockDim.x * 16384) {
        uint32_t n = (uint32_t)(end - off < 16384 ? end - off : 16384);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(n) : "memory");
    }
}

// 16-byte streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Two E4M3FN codes (low byte first) -> two exact FP32 values. Every finite
// E4M3 value is exactly representable in FP16, so the hardware conversion to
// f16x2 followed by widening is exact.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two_codes)
{
    uint32_t h;
    uint16_t packed = (uint16_t)(two_codes & 0xffffu);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(packed));
    __half2 hv = *reinterpret_cast<__half2 *>(&h);
    return __half22float2(hv);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024); all threads get it.
__device__ __forceinline__ float block_sum(float v, float *scratch32)
{
    v = warp_sum(v);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch32[warp] = v;
    __syncthreads();
    int warps = blockDim.x >> 5;
    float t = lane < warps ? scratch32[lane] : 0.0f;
    return warp_sum(t);
}

// Query scale of the checkpoint's YaRN rule: 1 + 0.1 * ln(1 + floor(pos / 16384)).
__device__ __forceinline__ float query_scale(int position)
{
    return 1.0f + 0.1f * logf(1.0f + (float)(position / 16384));
}

// KV pool address (in elements): pool is layer-major [layer][page][kind][kv_head][slot][dim]
// FP32 — the reference's KV precision; narrower formats measurably break the
// per-layer parity gate on hidden states (BF16 KV: 0.38 max-abs at layer 25).
__device__ __forceinline__ size_t kv_offset(int layer, int num_pages, int page, int kind,
                                            int head, int slot)
{
    return ((((size_t)layer * num_pages + page) * 2 + kind) * kKVHeads + head) *
               (size_t)(kPage * kHeadDim) +
           (size_t)slot * kHeadDim;
}

}  // namespace lun
