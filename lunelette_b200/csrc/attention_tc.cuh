// Causal GQA attention of a block of query tokens on the 5th-generation tensor
// cores (tcgen05, tensor memory): the prefill/append path that replaces
// scores + attend (src/metal_kernels.metal:81-132) for blocks of more than four
// tokens of one sequence.
//
// One CTA owns 128 query rows (32 tokens x the 4 query heads of one KV head)
// and a page-aligned key range (split) of the paged FP32 pool; it streams the
// range in tiles of 64 keys (one page):
//   warp 0     bulk copies of a tile's FP32 K rows and V rows (32 KB each, one
//              page of one KV head) into two separate two-stage rings, each
//              copy issued as soon as its slot is free (non-blocking probes);
//   warp 1     allocates tensor memory; one lane issues the MMAs
//              (tcgen05.mma.cta_group::1.kind::f16, A in tensor memory) and
//              commits: S = Q K^T into one of two S buffers, O += P V;
//   warps 2-3  convert a staged K tile into FP16 hi + lo parts in shared
//              memory ([64 keys x 128 dims], K-major, 128-byte swizzle);
//   warps 4-5  convert a staged V tile, transposed ([128 dims x 64 keys]), into
//              one of two buffers; V rows past the valid keys become zeros;
//              with two V buffers and separate rings the next tiles' loads and
//              conversions never wait for the current P V;
//   warps 6-9  one thread per query row (TMEM lane quarter = query head): Q's
//              hi + lo parts into tensor memory once; per tile the row's 64
//              scores from tensor memory, causal mask, online softmax with the
//              running maximum kept unless a tile raises it by more than 2^8
//              (then O's row is rescaled in tensor memory), P's hi + lo parts
//              written over the scores as the A operand of P V; at the end O / l
//              (or the unnormalised partial, m and l of the split).
// Each product is taken as hi.hi + hi.lo + lo.hi (FP16 parts of 11 significant
// bits each, 22 together; the lo.lo term, ~2^-22 relative, is dropped) with
// FP32 accumulation, as the mma.sync kernel in attention.cuh does; the softmax
// runs in base 2 (scores scaled by log2 e).
//
// The CTA takes all 512 tensor-memory columns of its SM: its 225 KB of shared
// memory leave no room for a second CTA of this or any other tcgen05 kernel of
// this library (each needs more than 128 KB), so the allocation never waits.
// Tensor memory (512 columns): Q hi [0, 64), Q lo [64, 128) (FP16 pairs),
// S/P buffers [128, 192) and [192, 256) (64 FP32 scores, then P hi in the first
// 32 columns and P lo in the next 32), O [256, 384) (128 FP32 dims). The MMAs of
// one thread run in issue order (S(0), S(1), PV(0), S(2), PV(1), ...), so S(j)
// completing implies PV(j - 2) completed, whose P the softmax of tile j then
// overwrites in the same buffer.
#pragma once
#include "async.cuh"
#include "attention.cuh"
#include "tcgen05.cuh"

namespace lun {

constexpr int kTaKeys = 64;                                   // keys per tile (one page)
constexpr int kTaThreads = 320;                               // 10 warps
constexpr int kTaKPart = kTaKeys * kHeadDim * 2;              // one FP16 part of K: 16384 (two 8 KB chunks)
constexpr int kTaVPart = kHeadDim * kTaKeys * 2;              // one FP16 part of V^T: 16384
constexpr int kTaRowBytes = kTaKeys * kHeadDim * 4;          // one FP32 K (or V) page of a head: 32768
constexpr int kTaKStageOffset = 0;                             // K ring: 2 x 32 KB
constexpr int kTaVStageOffset = kTaKStageOffset + 2 * kTaRowBytes;  // V ring: 2 x 32 KB
constexpr int kTaKOffset = kTaVStageOffset + 2 * kTaRowBytes;  // K hi | lo
constexpr int kTaVOffset = kTaKOffset + 2 * kTaKPart;          // two V buffers, each hi | lo
constexpr int kTaBarOffset = kTaVOffset + 4 * kTaVPart;
constexpr int kTaSmemBytes = 1024 + kTaBarOffset + 256;
static_assert(kTaSmemBytes <= 232448, "tensor-core attention shared memory");
constexpr uint32_t kTaQCol = 0, kTaSCol = 128, kTaOCol = 256, kTaTmemCols = 512;
constexpr float kTaLog2e = 1.4426950408889634f;
constexpr float kTaLn2 = 0.6931471805599453f;
constexpr float kTaScale2 = kScoreScale * kTaLog2e;           // scores in base-2 units
constexpr float kTaRescale = 8.0f;                            // keep the maximum unless raised by more (log2)

// Where the waits report giving up when the caller passed no error word.
static __device__ int tc_attention_error_sink;

// Grid (ceil(count / 32), 8 KV heads, splits), kTaThreads threads, kTaSmemBytes.
static __global__ void __launch_bounds__(kTaThreads, 1) attention_prefill_tc_kernel(AttnParams p, int count)
{
    extern __shared__ __align__(1024) uint8_t ta_raw[];
    const uint32_t raw = smem_u32(ta_raw);
    uint8_t *base = ta_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *kstage = base + kTaKStageOffset, *vstage = base + kTaVStageOffset;
    uint8_t *kc = base + kTaKOffset, *vc = base + kTaVOffset;  // K [hi | lo]; V buffer b at b * 2 parts
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + kTaBarOffset);
    uint64_t *kst_full = bars, *kst_empty = bars + 2, *vst_full = bars + 4, *vst_empty = bars + 6;
    uint64_t *k_ready = bars + 8, *k_free = bars + 9, *v_ready = bars + 10, *v_free = bars + 12;
    uint64_t *s_full = bars + 14, *p_ready = bars + 16, *o_done = bars + 18, *q_ready = bars + 19;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 20);
    volatile int *abort_word = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *error = p.error ? p.error : &tc_attention_error_sink;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = blockIdx.y, t0 = blockIdx.x * kPmTokens, split = blockIdx.z;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&kst_full[i], 1);
            mbar_init(&kst_empty[i], 2);  // K converter warps
            mbar_init(&vst_full[i], 1);
            mbar_init(&vst_empty[i], 2);  // V converter warps
            mbar_init(&v_ready[i], 2);
            mbar_init(&v_free[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_ready[i], 4);    // softmax warps
        }
        mbar_init(k_ready, 2);
        mbar_init(k_free, 1);
        mbar_init(o_done, 1);
        mbar_init(q_ready, 4);
        *abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTaTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // q and the KV rows of this block come from the qkv projection
    pdl_launch_dependents();

    const int length = (p.step ? p.step->length : p.length) + p.token_offset;
    const int last = min(t0 + kPmTokens, count) - 1;  // last query token of the block
    const int k0 = split * p.split_len;               // first key of this split (page-aligned)
    const int total = min(length + last + 1, k0 + p.split_len);
    const int tiles = total > k0 ? (total - k0 + kTaKeys - 1) / kTaKeys : 0;

    if (warp == 0) {
        // ---- loads: tile j's K page into K slot j % 2 and its V page into V
        // slot j % 2, each as soon as the converters released the slot
        if (lane == 0) {
            int ik = 0, iv = 0;
            unsigned idle = 0;
            const unsigned long long start = wait_clock_ns();
            while ((ik < tiles || iv < tiles) && !*abort_word) {
                bool progressed = false;
                if (ik < tiles && (ik < 2 || mbar_test_wait(&kst_empty[ik & 1], ((ik >> 1) - 1) & 1))) {
                    const int page = p.page_table[(k0 + ik * kTaKeys) / kPage];
                    mbar_expect_tx(&kst_full[ik & 1], kTaRowBytes);
                    bulk_g2s(kstage + (ik & 1) * kTaRowBytes, p.kv + kv_offset(p.layer, p.num_pages, page, 0, kvh, 0),
                             kTaRowBytes, &kst_full[ik & 1]);
                    ik++;
                    progressed = true;
                }
                if (iv < tiles && (iv < 2 || mbar_test_wait(&vst_empty[iv & 1], ((iv >> 1) - 1) & 1))) {
                    const int page = p.page_table[(k0 + iv * kTaKeys) / kPage];
                    mbar_expect_tx(&vst_full[iv & 1], kTaRowBytes);
                    bulk_g2s(vstage + (iv & 1) * kTaRowBytes, p.kv + kv_offset(p.layer, p.num_pages, page, 1, kvh, 0),
                             kTaRowBytes, &vst_full[iv & 1]);
                    iv++;
                    progressed = true;
                }
                if (progressed) {
                    idle = 0;
                } else if ((++idle & 1023u) == 0 && wait_clock_ns() - start > kWaitLimitNs) {
                    *abort_word = 1;
                    atomicExch(error, 1);
                    break;
                }
            }
            // every copy issued has landed before the CTA ends
            for (int j = max(0, ik - 2); j < ik; j++)
                mbar_wait_bounded(&kst_full[j & 1], (j >> 1) & 1, abort_word, error, kWaitSpinLimit);
            for (int j = max(0, iv - 2); j < iv; j++)
                mbar_wait_bounded(&vst_full[j & 1], (j >> 1) & 1, abort_word, error, kWaitSpinLimit);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issue: S(j) as soon as K(j) is converted, then PV(j - 1)
        if (lane == 0 && tiles > 0) {
            const uint32_t idesc_s = f16_idesc(128, kTaKeys), idesc_o = f16_idesc(128, kHeadDim);
            const uint32_t kc0 = smem_u32(kc), vc0 = smem_u32(vc);
            bool ok = mbar_wait_bounded(q_ready, 0, abort_word, error, kWaitSpinLimit);
            for (int j = 0; ok && j <= tiles; j++) {
                if (j < tiles) {
                    if (!(ok = mbar_wait_bounded(k_ready, j & 1, abort_word, error, kWaitSpinLimit))) break;
                    tc_fence_after();
                    const uint32_t sd = tmem + kTaSCol + 64u * (uint32_t)(j & 1);
#pragma unroll
                    for (int ks = 0; ks < kHeadDim / 16; ks++)
#pragma unroll
                        for (int term = 0; term < 3; term++) {
                            // hi.hi, hi.lo, lo.hi
                            const uint32_t a = tmem + kTaQCol + (term == 2 ? 64u : 0u) + 8u * (uint32_t)ks;
                            const uint32_t b = kc0 + (term == 1 ? kTaKPart : 0) + (ks >> 2) * 8192 + (ks & 3) * 32;
                            tc_mma_f16_tmem_a(sd, a, sw128_desc(b), idesc_s, (ks | term) != 0);
                        }
                    tc_commit(k_free);
                    tc_commit(&s_full[j & 1]);
                }
                if (j >= 1) {
                    const int jj = j - 1, vb = jj & 1;
                    if (!(ok = mbar_wait_bounded(&p_ready[vb], (jj >> 1) & 1, abort_word, error, kWaitSpinLimit) &&
                               mbar_wait_bounded(&v_ready[vb], (jj >> 1) & 1, abort_word, error, kWaitSpinLimit)))
                        break;
                    tc_fence_after();
                    const uint32_t pa = tmem + kTaSCol + 64u * (uint32_t)vb;
                    const uint32_t v0 = vc0 + (uint32_t)vb * 2 * kTaVPart;
#pragma unroll
                    for (int ks = 0; ks < kTaKeys / 16; ks++)
#pragma unroll
                        for (int term = 0; term < 3; term++) {
                            const uint32_t a = pa + (term == 2 ? 32u : 0u) + 8u * (uint32_t)ks;
                            const uint32_t b = v0 + (term == 1 ? kTaVPart : 0) + ks * 32;
                            tc_mma_f16_tmem_a(tmem + kTaOCol, a, sw128_desc(b), idesc_o, (jj | ks | term) != 0);
                        }
                    tc_commit(&v_free[vb]);
                    tc_commit(o_done);
                }
            }
        }
        __syncwarp();
    } else if (warp < 4) {
        // ---- K converters: staged FP32 K -> FP16 hi + lo operand tile
        const int ct = threadIdx.x - 64;  // 0..63
        for (int j = 0; j < tiles; j++) {
            const float *sk = reinterpret_cast<const float *>(kstage + (j & 1) * kTaRowBytes);
            if (!warp_wait(&kst_full[j & 1], (j >> 1) & 1, abort_word, error)) break;
            if (j >= 1 && !warp_wait(k_free, (j - 1) & 1, abort_word, error)) break;
            // unit g = (key, 8 dims); a warp reads two whole 512-byte rows
#pragma unroll 4
            for (int it = 0; it < 16; it++) {
                const int g = ct + 64 * it, key = g >> 4, grp = g & 15;
                const float4 a = *reinterpret_cast<const float4 *>(sk + key * kHeadDim + 8 * grp);
                const float4 b = *reinterpret_cast<const float4 *>(sk + key * kHeadDim + 8 * grp + 4);
                uint4 hi, lo;
                split_half2(a.x, a.y, hi.x, lo.x);
                split_half2(a.z, a.w, hi.y, lo.y);
                split_half2(b.x, b.y, hi.z, lo.z);
                split_half2(b.z, b.w, hi.w, lo.w);
                const uint32_t off = (grp >> 3) * 8192 + sw128_offset(key, (grp & 7) * 8);
                *reinterpret_cast<uint4 *>(kc + off) = hi;
                *reinterpret_cast<uint4 *>(kc + kTaKPart + off) = lo;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(k_ready);
                mbar_arrive(&kst_empty[j & 1]);
            }
        }
    } else if (warp < 6) {
        // ---- V converters: staged FP32 V -> transposed FP16 hi + lo tile in
        // buffer j % 2; keys past the valid ones are zeros (their stale pool
        // rows must not reach P V)
        const int ct = threadIdx.x - 128;  // 0..63
        for (int j = 0; j < tiles; j++) {
            const int vb = j & 1;
            const float *sv = reinterpret_cast<const float *>(vstage + vb * kTaRowBytes);
            uint8_t *vdst = vc + vb * 2 * kTaVPart;
            const int valid = min(kTaKeys, total - (k0 + j * kTaKeys));
            if (!warp_wait(&vst_full[vb], (j >> 1) & 1, abort_word, error)) break;
            if (j >= 2 && !warp_wait(&v_free[vb], ((j >> 1) - 1) & 1, abort_word, error)) break;
            // unit (dim d, keys 8 kg .. 8 kg + 7): d = ct + 64 (it & 1), kg = it >> 1
#pragma unroll 2
            for (int it = 0; it < 16; it++) {
                const int d = ct + 64 * (it & 1), kg = it >> 1;
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int key = 8 * kg + e;
                    v[e] = key < valid ? sv[key * kHeadDim + d] : 0.0f;
                }
                uint4 hi, lo;
                split_half2(v[0], v[1], hi.x, lo.x);
                split_half2(v[2], v[3], hi.y, lo.y);
                split_half2(v[4], v[5], hi.z, lo.z);
                split_half2(v[6], v[7], hi.w, lo.w);
                const uint32_t off = sw128_offset(d, 8 * kg);
                *reinterpret_cast<uint4 *>(vdst + off) = hi;
                *reinterpret_cast<uint4 *>(vdst + kTaVPart + off) = lo;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&v_ready[vb]);
                mbar_arrive(&vst_empty[vb]);
            }
        }
    } else {
        // ---- softmax: thread = query row (head hq = TMEM quarter, token lane)
        const int hq = warp & 3, tok = lane, t = t0 + tok;
        const bool live = t < count;
        const int limit = live ? length + t : -1;  // last key position this row sees
        const uint32_t lane_base = tmem + ((uint32_t)(32 * hq) << 16);
        const int head = kvh * 4 + hq;
        {
            // Q row -> hi and lo FP16 pairs in tensor memory (dim d in column d / 2)
            const float4 *qrow = reinterpret_cast<const float4 *>(p.q + (size_t)(live ? t : 0) * kQuery +
                                                                  (size_t)head * kHeadDim);
#pragma unroll
            for (int half = 0; half < 2; half++) {
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const float4 v = live ? qrow[16 * half + i] : make_float4(0.f, 0.f, 0.f, 0.f);
                    split_half2(v.x, v.y, hi[2 * i], lo[2 * i]);
                    split_half2(v.z, v.w, hi[2 * i + 1], lo[2 * i + 1]);
                }
                tmem_st32(lane_base + kTaQCol + 32u * (uint32_t)half, hi);
                tmem_st32(lane_base + kTaQCol + 64u + 32u * (uint32_t)half, lo);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_ready);
        }
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        for (int j = 0; j < tiles; j++) {
            if (!(ok = warp_wait(&s_full[j & 1], (j >> 1) & 1, abort_word, error))) break;
            tc_fence_after();
            const uint32_t sb = kTaSCol + 64u * (uint32_t)(j & 1);
            uint32_t raw_s[64];
            {
                uint32_t (&a)[32] = *reinterpret_cast<uint32_t (*)[32]>(&raw_s[0]);
                uint32_t (&b)[32] = *reinterpret_cast<uint32_t (*)[32]>(&raw_s[32]);
                tmem_ld32(lane_base + sb, a);
                tmem_ld32(lane_base + sb + 32u, b);
            }
            const int p0 = k0 + j * kTaKeys;
            float s[64];
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 64; c++) {
                s[c] = p0 + c <= limit ? __uint_as_float(raw_s[c]) * kTaScale2 : -INFINITY;
                mx = fmaxf(mx, s[c]);
            }
            // the running maximum changes only when this tile raises it by more
            // than 2^8 (P stays below 2^8 otherwise); a row without any key yet
            // (m_run = -inf) has O = 0 and l = 0 and just takes the tile's
            const bool raise = m_run != -INFINITY && mx > m_run + kTaRescale;
            const float corr = raise ? exp2f(m_run - mx) : 1.0f;
            const float m_use = (m_run == -INFINITY || raise) ? mx : m_run;
            if (__any_sync(0xffffffffu, raise)) {
                // O's row *= corr once P V of the previous tile has landed
                if (!(ok = warp_wait(o_done, (j - 1) & 1, abort_word, error))) break;
                tc_fence_after();
#pragma unroll 1
                for (int cb = 0; cb < 4; cb++) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + kTaOCol + 32u * (uint32_t)cb, o);
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
                    tmem_st32(lane_base + kTaOCol + 32u * (uint32_t)cb, o);
                }
            }
            l_run *= corr;
            m_run = m_use;
            float sum = 0.0f;
            uint32_t ph[32], pl[32];
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float a = s[2 * i] == -INFINITY ? 0.0f : exp2f(s[2 * i] - m_use);
                const float b = s[2 * i + 1] == -INFINITY ? 0.0f : exp2f(s[2 * i + 1] - m_use);
                sum += a + b;
                split_half2(a, b, ph[i], pl[i]);
            }
            l_run += sum;
            tmem_st32(lane_base + sb, ph);
            tmem_st32(lane_base + sb + 32u, pl);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_ready[j & 1]);
        }
        // ---- epilogue: O / l, or the split's unnormalised O with m and l. The
        // tensor-memory loads are warp-collective (.sync.aligned): every lane
        // runs them, and only the stores depend on this lane's token
        if (ok && tiles > 0) ok = warp_wait(o_done, (tiles - 1) & 1, abort_word, error);
        if (__all_sync(0xffffffffu, ok && !*abort_word)) {
            tc_fence_after();
            const bool whole = p.splits == 1;
            const float inv = whole && l_run > 0.0f ? 1.0f / l_run : 1.0f;
            const size_t tr = live ? (size_t)t : 0;  // rows past the block are never stored
            float *dst = whole ? p.out + tr * kQuery + (size_t)head * kHeadDim
                               : p.part_acc + ((tr * kQueryHeads + head) * p.splits + split) * kHeadDim;
#pragma unroll 1
            for (int cb = 0; cb < 4; cb++) {
                uint32_t o[32];
                if (tiles > 0) {
                    tmem_ld32(lane_base + kTaOCol + 32u * (uint32_t)cb, o);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = 0u;
                }
                if (live)
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        reinterpret_cast<float4 *>(dst + 32 * cb)[i] =
                            make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                        __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
            }
            if (!whole && live) {
                const size_t slot = ((size_t)t * kQueryHeads + head) * p.splits + split;
                // a split past this token's causal range leaves l = 0 (the combine skips it)
                p.part_ml[slot * 2] = m_run * kTaLn2;
                p.part_ml[slot * 2 + 1] = l_run;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTaTmemCols);
    }
}

}  // namespace lun
