// Kernel-level C-ABI: the product kernels on caller-provided device pointers,
// so tests can check each one against the CPU oracle on awkward shapes.
// Return 0 on success, -1 on invalid arguments or a CUDA launch error.
#include "kernels.h"
#include "prefill_gemm.cuh"

#include <stdlib.h>
#include <string.h>

#define LUN_API extern "C" __attribute__((visibility("default")))

using namespace lun;

static int sm_count_of_current()
{
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
    return sms;
}

static int ok(cudaError_t e) { return e == cudaSuccess ? 0 : -1; }

LUN_API int lunelette_cuda_kernels_init(void) { return ok(lun_kernels_init()); }

LUN_API int lunelette_cuda_fp8_decode(const uint8_t *codes, size_t n, float scale, float *out,
                                      void *stream)
{
    if ((!codes || !out) && n) return -1;
    return ok(lun_launch_fp8_decode(codes, n, scale, out, (cudaStream_t)stream));
}

static GemvParams plain(const uint8_t *W, size_t rows, size_t cols, float scale)
{
    GemvParams p;
    memset(&p, 0, sizeof p);
    p.W = W;
    p.rows = (int)rows;
    p.cols = (int)cols;
    p.scale[0] = p.scale[1] = p.scale[2] = scale;
    p.bound[0] = p.bound[1] = 1 << 30;
    p.length = 0;
    return p;
}

// Row-major FP8 codes -> the tiled layout that every GEMV entry point reads.
// order 0 keeps the rows; 1 takes q|k|v rows (rows % 128 == 0) and places the
// RoPE pairs (j, j + 64) of every 128-row head in adjacent rows; 2 takes gate
// rows followed by up rows (rows even) and interleaves them (gate f -> 2f,
// up f -> 2f + 1). Padding rows/columns of dst are zeroed.
LUN_API int lunelette_cuda_tile_fp8(const uint8_t *src, size_t rows, size_t cols, int order, uint8_t *dst,
                                    void *stream)
{
    if (!src || !dst || !rows || !cols || (cols % 16) || rows > (1u << 24) || cols > (1u << 16) || order < 0 ||
        order > 2 || (order == 1 && rows % 128) || (order == 2 && rows % 2))
        return -1;
    cudaStream_t st = (cudaStream_t)stream;
    const int nb = (int)((cols + 127) / 128);
    if (tiled_bytes(rows, cols) != rows * cols && cudaMemsetAsync(dst, 0, tiled_bytes(rows, cols), st) != cudaSuccess)
        return -1;
    if (order == 2) {
        const int half = (int)(rows / 2);
        if (lun_launch_tile_fp8(src, half, (int)cols, dst, nb, kOrderInterleave, 0, st) != cudaSuccess) return -1;
        return ok(lun_launch_tile_fp8(src + (size_t)half * cols, half, (int)cols, dst, nb, kOrderInterleave, 1, st));
    }
    return ok(lun_launch_tile_fp8(src, (int)rows, (int)cols, dst, nb, order == 1 ? kOrderRopePairs : kOrderRows, 0,
                                  st));
}

// y[t][r] = scale * sum_c decode(W[r][c]) * x[t][c] (+ res[t][r]), any count
// (processed in groups of 4 rows of x). W is tiled (lunelette_cuda_tile_fp8,
// order 0); cols must be a multiple of 16.
LUN_API int lunelette_cuda_gemv_fp8(const uint8_t *W, size_t rows, size_t cols, float scale,
                                    const float *x, const float *res, size_t count, float *y,
                                    void *stream)
{
    if (!W || !x || !y || !rows || !cols || (cols % 16) || !count || rows > (1u << 28) ||
        cols * 4 * 4 > 4 * 9216 * 4)
        return -1;
    int sms = sm_count_of_current();
    for (size_t t0 = 0; t0 < count; t0 += 4) {
        int m = (int)(count - t0 < 4 ? count - t0 : 4);
        GemvParams p = plain(W, rows, cols, scale);
        p.x = x + t0 * cols;
        p.x_stride = (int)cols;
        p.y = y + t0 * rows;
        p.y_stride = (int)rows;
        if (res) {
            p.res = res + t0 * rows;
            p.res_stride = (int)rows;
        }
        if (lun_launch_gemv(p, m, res ? kEpiResidual : kEpiStore, sms, (cudaStream_t)stream) !=
            cudaSuccess)
            return -1;
    }
    return 0;
}

// Fused input-norm + q/k/v projection + RoPE (+query scale) + KV store for
// tokens at positions length..length+count-1. W is the tiled [6144][3072] q|k|v
// matrix (lunelette_cuda_tile_fp8, order 1).
LUN_API int lunelette_cuda_qkv_rope(const uint8_t *W, const float *scales, const float *gain,
                                    const float *x, size_t count, size_t length,
                                    const float *rope_cos, const float *rope_sin, float *q_out,
                                    float *kv_pool, const int *page_table, size_t num_pages,
                                    size_t layer, void *stream)
{
    if (!W || !scales || !gain || !x || !count || !rope_cos || !rope_sin || !q_out || !kv_pool ||
        !page_table || !num_pages || length + count > num_pages * kPage)
        return -1;
    int sms = sm_count_of_current();
    for (size_t t0 = 0; t0 < count; t0 += 4) {
        int m = (int)(count - t0 < 4 ? count - t0 : 4);
        GemvParams p = plain(W, kQKVRows, kHidden, 1.0f);
        p.scale[0] = scales[0];
        p.scale[1] = scales[1];
        p.scale[2] = scales[2];
        p.bound[0] = kQuery;
        p.bound[1] = kQuery + kKV;
        p.gain = gain;
        p.x = x + t0 * kHidden;
        p.x_stride = kHidden;
        p.y = q_out + t0 * kQuery;
        p.y_stride = kQuery;
        p.length = (int)length;
        p.token_offset = (int)t0;
        p.rope_cos = rope_cos;
        p.rope_sin = rope_sin;
        p.kv = kv_pool;
        p.page_table = page_table;
        p.num_pages = (int)num_pages;
        p.layer = (int)layer;
        if (lun_launch_gemv(p, m, kEpiQKV, sms, (cudaStream_t)stream) != cudaSuccess) return -1;
    }
    return 0;
}

// Fused post-attention norm + gate/up projection + SwiGLU.
// W is the tiled [18432][3072] gate/up matrix (lunelette_cuda_tile_fp8, order 2:
// gate row f at 2f, up row f at 2f + 1).
LUN_API int lunelette_cuda_gateup_swiglu(const uint8_t *W, float scale_gate, float scale_up,
                                         const float *gain, const float *x, size_t count,
                                         float *act, void *stream)
{
    if (!W || !gain || !x || !act || !count) return -1;
    int sms = sm_count_of_current();
    for (size_t t0 = 0; t0 < count; t0 += 4) {
        int m = (int)(count - t0 < 4 ? count - t0 : 4);
        GemvParams p = plain(W, kGateUpRows, kHidden, 1.0f);
        p.scale[0] = scale_gate;
        p.scale[1] = scale_up;
        p.gain = gain;
        p.x = x + t0 * kHidden;
        p.x_stride = kHidden;
        p.y = act + t0 * kInner;
        p.y_stride = kInner;
        if (lun_launch_gemv(p, m, kEpiSwiGLU, sms, (cudaStream_t)stream) != cudaSuccess) return -1;
    }
    return 0;
}

// One projection through the tcgen05 prefill path with workspace allocated
// for this call (stream-ordered); -1 also when a bounded wait inside the GEMM
// gave up. Synchronises the stream.
static int run_prefill(const GemvParams &p, size_t count, int epilogue, cudaStream_t stream)
{
    if (!count || count > 65536) return -1;
    const int sms = sm_count_of_current();
    const PrefillPlan pl = lun_prefill_plan(p.rows, p.cols, (int)count, sms);
    PrefillWorkspace w;
    memset(&w, 0, sizeof w);
    w.xs_bytes = pl.xs_bytes;
    w.inv_bytes = pl.inv_bytes;
    w.ws_bytes = pl.ws_bytes;
    int rc = -1, error = 0;
    if (cudaMallocAsync((void **)&w.xs, w.xs_bytes, stream) == cudaSuccess &&
        cudaMallocAsync((void **)&w.inv_scale, w.inv_bytes, stream) == cudaSuccess &&
        cudaMallocAsync((void **)&w.ws, w.ws_bytes, stream) == cudaSuccess &&
        cudaMallocAsync((void **)&w.error, sizeof(int), stream) == cudaSuccess &&
        cudaMemsetAsync(w.error, 0, sizeof(int), stream) == cudaSuccess &&
        lun_launch_prefill(p, (int)count, epilogue, w, sms, stream) == cudaSuccess &&
        cudaMemcpyAsync(&error, w.error, sizeof(int), cudaMemcpyDeviceToHost, stream) == cudaSuccess &&
        cudaStreamSynchronize(stream) == cudaSuccess)
        rc = error ? -1 : 0;
    if (w.xs) cudaFreeAsync(w.xs, stream);
    if (w.inv_scale) cudaFreeAsync(w.inv_scale, stream);
    if (w.ws) cudaFreeAsync(w.ws, stream);
    if (w.error) cudaFreeAsync(w.error, stream);
    return rc;
}

// Mean device time of each prefill kernel (ms[0] split, ms[1] GEMM, ms[2]
// finish) over `reps` back-to-back runs of lunelette_cuda_gemm_fp8 (store
// epilogue), from CUDA events on the stream; run r reads weight copy r % copies
// of `copies` consecutive tiled matrices at W. A microbenchmark of the
// tensor-core path.
LUN_API int lunelette_cuda_gemm_fp8_timed(const uint8_t *W, size_t copies, size_t rows, size_t cols, float scale,
                                          const float *x, size_t count, float *y, int reps, float *ms,
                                          void *stream)
{
    if (!W || !copies || !x || !y || !ms || reps <= 0 || reps > 4096 || !rows || (rows % 8) || !cols ||
        (cols % 16) || !count || count > 65536 || rows > (1u << 24) || cols > kSplitMaxCols)
        return -1;
    cudaStream_t st = (cudaStream_t)stream;
    const int sms = sm_count_of_current();
    const size_t matrix = tiled_bytes(rows, cols);
    GemvParams p = plain(W, rows, cols, scale);
    p.x = x;
    p.x_stride = (int)cols;
    p.y = y;
    p.y_stride = (int)rows;
    const PrefillPlan pl = lun_prefill_plan(p.rows, p.cols, (int)count, sms);
    PrefillWorkspace w;
    memset(&w, 0, sizeof w);
    w.xs_bytes = pl.xs_bytes;
    w.inv_bytes = pl.inv_bytes;
    w.ws_bytes = pl.ws_bytes;
    cudaEvent_t *ev = (cudaEvent_t *)calloc((size_t)4 * reps, sizeof(cudaEvent_t));
    if (!ev) return -1;
    int rc = -1, error = 0;
    double sum[3] = {0, 0, 0};
    bool good = cudaMalloc((void **)&w.xs, w.xs_bytes) == cudaSuccess &&
                cudaMalloc((void **)&w.inv_scale, w.inv_bytes) == cudaSuccess &&
                cudaMalloc((void **)&w.ws, w.ws_bytes) == cudaSuccess &&
                cudaMalloc((void **)&w.error, sizeof(int)) == cudaSuccess &&
                cudaMemsetAsync(w.error, 0, sizeof(int), st) == cudaSuccess;
    for (int i = 0; i < 4 * reps && good; i++) good = cudaEventCreate(&ev[i]) == cudaSuccess;
    for (int r = 0; r < reps && good; r++) {
        p.W = W + (size_t)(r % copies) * matrix;
        good = lun_launch_prefill_marked(p, (int)count, kEpiStore, w, sms, st, ev + 4 * r) == cudaSuccess;
    }
    good = good && cudaStreamSynchronize(st) == cudaSuccess;
    for (int r = 0; r < reps && good; r++)
        for (int k = 0; k < 3 && good; k++) {
            float t = 0.0f;
            good = cudaEventElapsedTime(&t, ev[4 * r + k], ev[4 * r + k + 1]) == cudaSuccess;
            sum[k] += t;
        }
    if (good && cudaMemcpy(&error, w.error, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && !error) {
        for (int k = 0; k < 3; k++) ms[k] = (float)(sum[k] / reps);
        rc = 0;
    }
    for (int i = 0; i < 4 * reps; i++)
        if (ev[i]) cudaEventDestroy(ev[i]);
    free(ev);
    cudaFree(w.xs);
    cudaFree(w.inv_scale);
    cudaFree(w.ws);
    cudaFree(w.error);
    return rc;
}

// lunelette_cuda_gemv_fp8 through the tcgen05 prefill GEMM.
LUN_API int lunelette_cuda_gemm_fp8(const uint8_t *W, size_t rows, size_t cols, float scale, const float *x,
                                    const float *res, size_t count, float *y, void *stream)
{
    if (!W || !x || !y || !rows || (rows % 8) || !cols || (cols % 16) || rows > (1u << 24) || cols > kSplitMaxCols)
        return -1;
    GemvParams p = plain(W, rows, cols, scale);
    p.x = x;
    p.x_stride = (int)cols;
    p.y = y;
    p.y_stride = (int)rows;
    p.res = res;
    p.res_stride = (int)rows;
    return run_prefill(p, count, res ? kEpiResidual : kEpiStore, (cudaStream_t)stream);
}

// lunelette_cuda_qkv_rope through the tcgen05 prefill GEMM.
LUN_API int lunelette_cuda_gemm_qkv_rope(const uint8_t *W, const float *scales, const float *gain,
                                         const float *x, size_t count, size_t length, const float *rope_cos,
                                         const float *rope_sin, float *q_out, float *kv_pool,
                                         const int *page_table, size_t num_pages, size_t layer, void *stream)
{
    if (!W || !scales || !gain || !x || !count || !rope_cos || !rope_sin || !q_out || !kv_pool ||
        !page_table || !num_pages || length + count > num_pages * kPage)
        return -1;
    GemvParams p = plain(W, kQKVRows, kHidden, 1.0f);
    p.scale[0] = scales[0];
    p.scale[1] = scales[1];
    p.scale[2] = scales[2];
    p.bound[0] = kQuery;
    p.bound[1] = kQuery + kKV;
    p.gain = gain;
    p.x = x;
    p.x_stride = kHidden;
    p.y = q_out;
    p.y_stride = kQuery;
    p.length = (int)length;
    p.rope_cos = rope_cos;
    p.rope_sin = rope_sin;
    p.kv = kv_pool;
    p.page_table = page_table;
    p.num_pages = (int)num_pages;
    p.layer = (int)layer;
    return run_prefill(p, count, kEpiQKV, (cudaStream_t)stream);
}

// lunelette_cuda_gateup_swiglu through the tcgen05 prefill GEMM.
LUN_API int lunelette_cuda_gemm_gateup_swiglu(const uint8_t *W, float scale_gate, float scale_up,
                                              const float *gain, const float *x, size_t count, float *act,
                                              void *stream)
{
    if (!W || !gain || !x || !act || !count) return -1;
    GemvParams p = plain(W, kGateUpRows, kHidden, 1.0f);
    p.scale[0] = scale_gate;
    p.scale[1] = scale_up;
    p.gain = gain;
    p.x = x;
    p.x_stride = kHidden;
    p.y = act;
    p.y_stride = kInner;
    return run_prefill(p, count, kEpiSwiGLU, (cudaStream_t)stream);
}

LUN_API int lunelette_cuda_rmsnorm(const float *gain, const float *x, size_t width, size_t count,
                                   float *out, void *stream)
{
    if (!gain || !x || !out || !width || !count) return -1;
    return ok(lun_launch_rmsnorm(gain, x, out, (int)width, (int)count, (cudaStream_t)stream));
}

// Final norm + BF16 head over one hidden row; *nonfinite (device int) is OR-ed.
LUN_API int lunelette_cuda_head_bf16(const uint16_t *W, size_t rows, size_t cols, const float *x,
                                     const float *gain, float *logits, int *nonfinite, void *stream)
{
    if (!W || !x || !gain || !logits || !nonfinite || !rows || !cols || (cols % 8) ||
        cols > 9216)
        return -1;
    HeadParams p;
    p.W = W;
    p.rows = (int)rows;
    p.cols = (int)cols;
    p.x = x;
    p.gain = gain;
    p.logits = logits;
    p.nonfinite = nonfinite;
    return ok(lun_launch_head(p, sm_count_of_current(), (cudaStream_t)stream));
}

// Causal GQA attention of `count` query rows (positions length..length+count-1)
// over KV layer `layer` of a paged FP32 pool. part_acc/part_ml are caller scratch
// of (slots*128) and (slots*2) floats; slots >= count*32.
LUN_API int lunelette_cuda_attention(const float *q, const float *kv_pool, const int *page_table,
                                     size_t num_pages, size_t layer, size_t length, size_t count,
                                     float *out, float *part_acc, float *part_ml, size_t slots,
                                     void *stream)
{
    if (!q || !kv_pool || !page_table || !out || !count || !part_acc || !part_ml ||
        slots < count * kQueryHeads || length + count > num_pages * kPage)
        return -1;
    AttnParams a;
    memset(&a, 0, sizeof a);
    a.q = q;
    a.kv = kv_pool;
    a.page_table = page_table;
    a.num_pages = (int)num_pages;
    a.layer = (int)layer;
    a.length = (int)length;
    a.out = out;
    a.part_acc = part_acc;
    a.part_ml = part_ml;
    lun_attention_plan(&a, (int)(length + count), (int)count, sm_count_of_current(), (int)slots);
    return ok(lun_launch_attention(a, (int)count, (cudaStream_t)stream));
}

// KV prefix copy / remap: for i < pairs, all layers' K and V of page
// src_pages[i] -> page dst_pages[i] (device arrays), the last pair only its
// first last_slots positions.
LUN_API int lunelette_cuda_kv_copy(float *kv_pool, size_t num_pages, size_t layers, const int *src_pages,
                                   const int *dst_pages, size_t pairs, size_t last_slots, void *stream)
{
    if (!kv_pool || !src_pages || !dst_pages || !num_pages || !layers || layers > 1024 || !pairs ||
        pairs > num_pages || !last_slots || last_slots > (size_t)kPage)
        return -1;
    KvCopyParams p;
    p.kv = kv_pool;
    p.num_pages = (int)num_pages;
    p.src_pages = src_pages;
    p.dst_pages = dst_pages;
    p.pairs = (int)pairs;
    p.last_slots = (int)last_slots;
    return ok(lun_launch_kv_copy(p, (int)layers, (cudaStream_t)stream));
}
