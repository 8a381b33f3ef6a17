// Shared-memory mbarriers and bulk asynchronous copies (the TMA engine's
// cp.async.bulk), used by the persistent decode kernel and the prefill GEMM.
#pragma once
#include <cstdint>

namespace lun {

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity)
{
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Non-blocking probe of an mbarrier phase (mbarrier.try_wait may suspend the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, unsigned parity)
{
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Tiled 4-D tensor load (no multicast) of the box at {c0, c1, c2, c3}, completing on *bar.
__device__ __forceinline__ void tma_load_4d(void *dst, const void *tmap, int c0, int c1, int c2, int c3,
                                            uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}
// Tiled 3-D tensor load (no multicast) of the box at {c0, c1, c2}, completing on *bar.
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int c0, int c1, int c2, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
// Tiled 2-D tensor load (no multicast) of the box at {c0, c1}, completing on *bar.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int c0, int c1, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
// L2 prefetch of the box at {c0, c1, c2, c3} of a 4-D tensor map.
__device__ __forceinline__ void tma_prefetch_4d(const void *tmap, int c0, int c1, int c2, int c3)
{
    asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(tmap), "r"(c0),
                 "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
__device__ __forceinline__ void l2_prefetch(const void *src, unsigned bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// L2 eviction policies (createpolicy): evict_first for bytes read once (after
// the copy into shared memory the line is the first candidate for
// replacement), evict_last for bytes fetched ahead of their use.
__device__ __forceinline__ uint64_t l2_policy_evict_first()
{
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last()
{
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
// bulk_g2s with an L2 cache policy
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, unsigned bytes, uint64_t *bar,
                                              uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// tma_load_4d with an L2 cache policy (no multicast)
__device__ __forceinline__ void tma_load_4d_hint(void *dst, const void *tmap, int c0, int c1, int c2, int c3,
                                                 uint64_t *bar, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void l2_prefetch_hint(const void *src, unsigned bytes, uint64_t policy)
{
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src), "r"(bytes), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void tma_prefetch_4d_hint(const void *tmap, int c0, int c1, int c2, int c3, uint64_t policy)
{
    asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile.L2::cache_hint [%0, {%1, %2, %3, %4}], %5;" ::"l"(
                     tmap),
                 "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
                 : "memory");
}

// Bounded wait on an mbarrier phase for one thread: polls until the phase with
// `parity` completed, the CTA's abort word is set, or `limit` polls passed (then
// it sets the abort word and *error). False when the wait did not see the phase.
__device__ __forceinline__ unsigned long long wait_clock_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // one second

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, unsigned parity, volatile int *abort_word,
                                                  int *error, unsigned limit)
{
    // mbarrier.try_wait may suspend the thread for a system-defined time per
    // poll, so the poll count alone does not bound the wait: a clock does too
    unsigned spins = 0;
    unsigned long long start = 0;
    while (!mbar_try_wait(bar, parity)) {
        ++spins;
        if ((spins & 255u) == 1) {
            const unsigned long long now = wait_clock_ns();
            if (spins == 1) start = now;
            else if (now - start > kWaitLimitNs) spins = limit + 1;
        }
        if (spins > limit) {
            *abort_word = 1;
            atomicExch(error, 1);
            return false;
        }
        if ((spins & 63u) == 0 && *abort_word) return false;
    }
    return true;
}

// Polls of one bounded mbarrier wait in the tensor-core kernels.
constexpr unsigned kWaitSpinLimit = 1u << 20;

// Warp-uniform bounded wait: every lane polls; the warp goes on only if all saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, unsigned parity, volatile int *abort_word, int *error)
{
    const bool ok = mbar_wait_bounded(bar, parity, abort_word, error, kWaitSpinLimit);
    return __all_sync(0xffffffffu, ok);
}

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (bulk copies, tensor-core operand reads).
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace lun
