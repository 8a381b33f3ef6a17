// Launch helpers shared by the runtime (device.cu) and the kernel-level C-ABI
// (kernel_api.cu). C++ only; nothing here crosses the public boundary.
#pragma once
#include "attention.cuh"
#include "gemv.cuh"

// One-time per-process kernel attribute setup (dynamic shared memory limits).
cudaError_t lun_kernels_init();
// lun_kernels_init() once per device (cached); call before any graph capture.
cudaError_t lun_kernels_ensure();

// Row-major FP8 [rows][cols] (cols % 16 == 0) -> the tiled layout of gemv.cuh
// with dst_nb blocks per tile, rows placed by lun::TileOrder from row0. Padding
// rows/columns of dst are left as they are (zero them first).
cudaError_t lun_launch_tile_fp8(const uint8_t *src, int rows, int cols, uint8_t *dst, int dst_nb, int order,
                                int row0, cudaStream_t stream);

// GEMV family over a tiled matrix: m token rows (1..kGemvMaxTokens), epilogue kind lun::GemvEpilogue.
constexpr int kGemvMaxTokens = 4;
cudaError_t lun_launch_gemv(const lun::GemvParams &p, int m, int epilogue, int sm_count,
                            cudaStream_t stream);
cudaError_t lun_launch_head(const lun::HeadParams &p, int sm_count, cudaStream_t stream);
// Batched tied head on the tensor cores (head_mma.cuh): up to lun_head_mma_tokens()
// tokens per launch pair; p.xb holds lun_head_mma_stage_bytes() of staging.
cudaError_t lun_launch_head_mma(const lun::HeadMmaParams &p, cudaStream_t stream);
// The same on tcgen05 (head_tc.cuh), same staging size, same logits; p.error
// receives a bounded wait that gave up.
cudaError_t lun_launch_head_tc(const lun::HeadMmaParams &p, cudaStream_t stream);
size_t lun_head_mma_stage_bytes();
int lun_head_mma_tokens();
// Greedy id of each of `rows` logits rows (stride floats apart).
cudaError_t lun_launch_argmax_rows(const float *logits, int n, int stride, int rows, int *out, cudaStream_t stream);

// Choose split_len/splits for `total` positions (max over the call's tokens),
// `count` query tokens and `slots` partial slots available.
void lun_attention_plan(lun::AttnParams *a, int total, int count, int sm_count, int slots);
cudaError_t lun_launch_attention(const lun::AttnParams &a, int count, cudaStream_t stream);

// KV page copies (attention.cuh kv_copy_kernel) over `layers` layers of the pool.
cudaError_t lun_launch_kv_copy(const lun::KvCopyParams &p, int layers, cudaStream_t stream);

// x[t] = widen(embedding[step->ids[t]]) for t < count.
cudaError_t lun_launch_embed(const uint16_t *embedding, const lun::StepParams *step, float *x, int count,
                             cudaStream_t stream);

// out[t][c] = gain[c] * (x[t][c] * rsqrt(mean(x[t]^2) + eps))
cudaError_t lun_launch_rmsnorm(const float *gain, const float *x, float *out, int width, int count,
                               cudaStream_t stream);

// Greedy selection on the device for the decode loop: argmax over logits with
// the reference's rule (strict '>', lowest id wins ties, src/generation.c:8-34);
// writes the id into step->ids[0], appends it to tokens[step->generated++] and
// advances step->length by one. partials: 2*kArgmaxBlocks ints.
constexpr int kArgmaxBlocks = 256;
cudaError_t lun_launch_greedy(const float *logits, int n, int *partials, lun::StepParams *step,
                              int *tokens, cudaStream_t stream);

// Persistent decode kernel (decode_mega.cuh): cooperative launch of one CTA per
// SM; the barrier words in p must be zero at launch.
namespace lun {
struct MegaParams;
}
cudaError_t lun_launch_decode_mega(const lun::MegaParams &p, const void *down_map, int sm_count,
                                   cudaStream_t stream);
// down_map (128 bytes, 64-byte aligned): the tensor map of every layer's down
// projection that the persistent kernel's FFN reads in act slices; down0 is
// layer 0's tiled down matrix, layer_stride the bytes between layers.
cudaError_t lun_down_slice_map(void *map, const uint8_t *down0, size_t layer_stride);
// Whether the persistent kernel's per-CTA work fits on a grid of sm_count CTAs.
bool lun_mega_supported(int sm_count);

// FP8 codes -> FP32 * scale through the same in-register conversion as the GEMV.
cudaError_t lun_launch_fp8_decode(const uint8_t *codes, size_t n, float scale, float *out,
                                  cudaStream_t stream);

// Prefill projections on the tcgen05 tensor cores (prefill_gemm.cuh): split
// activations, GEMM into per-K-range partials, ordered finish + fused epilogue.
struct PrefillPlan {
    int row_tiles, token_tiles, kchunks, splits;  // 512-row tiles, 128-token tiles, 64-column chunks, K ranges
    size_t xs_bytes, inv_bytes, ws_bytes;         // workspace this projection needs
    bool tmem_a;  // small blocks: the GEMM with the weights as tensor-memory A (128 rows per CTA)
};
PrefillPlan lun_prefill_plan(int rows, int cols, int count, int sm_count);
struct PrefillWorkspace {
    uint8_t *xs;        // split activation tiles
    float *inv_scale;   // per-token 2^-e
    float *ws;          // FP32 partials
    int *error;         // set when a bounded wait inside the GEMM gave up
    size_t xs_bytes, inv_bytes, ws_bytes;
};
// Workspace sizes covering the model's four projections for up to max_count tokens.
void lun_prefill_workspace_bytes(int max_count, int sm_count, size_t *xs_bytes, size_t *inv_bytes,
                                 size_t *ws_bytes);
// The projection of p (GemvParams fields: W tiled, rows % 8 == 0, cols % 16 == 0,
// x, gain, scales, y, res, RoPE/KV fields) for `count` tokens with a
// lun::GemvEpilogue, positions from p.step->length (or p.length + p.token_offset).
cudaError_t lun_launch_prefill(const lun::GemvParams &p, int count, int epilogue, const PrefillWorkspace &w,
                               int sm_count, cudaStream_t stream);
// The three steps separately, and the finish fused with the next projection's
// split (residual or SwiGLU epilogue written to p.y when p.y is set; the row
// then RMS-normed with next_gain (or not, nullptr) and split into the operand
// tiles of a projection of next_rows rows; split == false stops after the
// epilogue).
cudaError_t lun_launch_prefill_split(const lun::GemvParams &p, int count, const PrefillWorkspace &w, int sm_count,
                                     cudaStream_t stream);
cudaError_t lun_launch_prefill_gemm(const lun::GemvParams &p, int count, const PrefillWorkspace &w, int sm_count,
                                    cudaStream_t stream);
cudaError_t lun_launch_prefill_finish(const lun::GemvParams &p, int count, int epilogue, const PrefillWorkspace &w,
                                      int sm_count, cudaStream_t stream);
cudaError_t lun_launch_prefill_finish_split(const lun::GemvParams &p, int count, int epilogue,
                                            const PrefillWorkspace &w, int sm_count, const float *next_gain,
                                            int next_rows, bool split, cudaStream_t stream);
// The same with events recorded before the split, between the kernels and after
// the finish (marks[0..3]), for per-kernel timing.
cudaError_t lun_launch_prefill_marked(const lun::GemvParams &p, int count, int epilogue,
                                      const PrefillWorkspace &w, int sm_count, cudaStream_t stream,
                                      cudaEvent_t *marks);
