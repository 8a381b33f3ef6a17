// Launchers of the tcgen05 prefill projections (prefill_gemm.cuh).
#include <cudaTypedefs.h>
#include <string.h>
#include <atomic>

#include "kernels.h"
#include "launch.h"
#include "prefill_gemm.cuh"
#include "prefill_gemm_tmem.cuh"

#include <stdlib.h>


using namespace lun;

// Blocks of up to kTmMaxTokens tokens run the tensor-memory-A GEMM
// (prefill_gemm_tmem.cuh) unless LUNELETTE_TMEM_GEMM=0.
static bool tmem_gemm_enabled()
{
    static const int on = [] {
        const char *v = getenv("LUNELETTE_TMEM_GEMM");
        return v && v[0] == '0' ? 0 : 1;
    }();
    return on != 0;
}

PrefillPlan lun_prefill_plan(int rows, int cols, int count, int sm_count)
{
    PrefillPlan pl;
    pl.row_tiles = (rows + kP2N - 1) / kP2N;
    pl.token_tiles = (count + kPgM - 1) / kPgM;
    pl.kchunks = (cols + kPgK - 1) / kPgK;
    pl.tmem_a = count <= kTmMaxTokens && tmem_gemm_enabled();
    // K ranges fill the SMs when the output tiles alone do not (a CTA pair per
    // 512 rows x 256 tokens, or a CTA per 128 rows for small blocks); every
    // range keeps at least two stages
    const int ctas = pl.tmem_a ? (rows + kTmRows - 1) / kTmRows : 2 * pl.row_tiles * ((pl.token_tiles + 1) / 2);
    int splits = sm_count / (ctas > 0 ? ctas : 1);
    splits = splits < 1 ? 1 : splits;
    const int max_splits = pl.kchunks / 2 > 0 ? pl.kchunks / 2 : 1;
    pl.splits = splits > max_splits ? max_splits : splits;
    pl.xs_bytes = (size_t)pl.token_tiles * pl.kchunks * 2 * kPgATile;
    pl.inv_bytes = (size_t)pl.token_tiles * kPgM * sizeof(float);
    pl.ws_bytes = (size_t)pl.splits * pl.token_tiles * kPgM * pl.row_tiles * kP2N * sizeof(float);
    return pl;
}

void lun_prefill_workspace_bytes(int max_count, int sm_count, size_t *xs_bytes, size_t *inv_bytes,
                                 size_t *ws_bytes)
{
    static const int shapes[4][2] = {{kQKVRows, kHidden}, {kHidden, kQuery}, {kGateUpRows, kHidden}, {kHidden, kInner}};
    size_t xs = 0, ws = 0, inv = 0;
    for (const auto &s : shapes) {
        const PrefillPlan pl = lun_prefill_plan(s[0], s[1], max_count, sm_count);
        xs = pl.xs_bytes > xs ? pl.xs_bytes : xs;
        ws = pl.ws_bytes > ws ? pl.ws_bytes : ws;
        inv = pl.inv_bytes > inv ? pl.inv_bytes : inv;
    }
    *xs_bytes = xs;
    *inv_bytes = inv;
    *ws_bytes = ws;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 lun_tensor_map_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return (PFN_cuTensorMapEncodeTiled_v12000)f;
    }();
    return fn;
}

// The tiled FP8 matrix as the GEMM's 4-D weight tensor (prefill_gemm_pair_kernel).
static cudaError_t weight_tensor_map(CUtensorMap *map, const uint8_t *W, int rows, int nb)
{
    PFN_cuTensorMapEncodeTiled_v12000 encode = lun_tensor_map_encoder();
    if (!encode || ((uintptr_t)W & 15)) return cudaErrorInvalidValue;
    const cuuint64_t dims[4] = {256, 2, (cuuint64_t)(2 * nb), (cuuint64_t)(rows / kTileRows)};
    const cuuint64_t strides[3] = {256, 512, (cuuint64_t)nb * kBlockBytes};
    const cuuint32_t box[4] = {256, 2, 1, kP2Rows / kTileRows};
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, (void *)W, dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// The same matrix as 8-byte elements in three dimensions, {64 (one 512-byte
// piece: 8 rows x 64 columns), 2 * nb pieces per tile row, tiles}, for
// prefill_gemm_tmem_kernel: a box of {64, 1, 16} lands the same 8 KB (one
// piece of each of 16 tiles) as the 4-D map's box, in 16 box rows of 512 bytes
// instead of 32 of 256.
static cudaError_t weight_tensor_map_wide(CUtensorMap *map, const uint8_t *W, int rows, int nb)
{
    PFN_cuTensorMapEncodeTiled_v12000 encode = lun_tensor_map_encoder();
    if (!encode || ((uintptr_t)W & 15)) return cudaErrorInvalidValue;
    const cuuint64_t dims[3] = {64, (cuuint64_t)(2 * nb), (cuuint64_t)(rows / kTileRows)};
    const cuuint64_t strides[2] = {512, (cuuint64_t)nb * kBlockBytes};
    const cuuint32_t box[3] = {64, 1, kTmRows / kTileRows};
    const cuuint32_t elem[3] = {1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, (void *)W, dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// The GEMM's shared-memory opt-in, once per device (atomic flags: callers may
// be on several threads; setting the attribute twice is harmless).
static cudaError_t prefill_setup()
{
    static std::atomic<bool> done[128];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    if (done[dev].load(std::memory_order_acquire)) return cudaSuccess;
    e = cudaFuncSetAttribute(prefill_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kP2SmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_gemm_tmem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBytes);
    if (e == cudaSuccess) done[dev].store(true, std::memory_order_release);
    return e;
}

template <int EPI>
static cudaError_t launch_finish(const PrefillFinishParams &f, cudaStream_t stream)
{
    const dim3 grid((unsigned)((f.rows / 2 + 255) / 256), (unsigned)f.count);
    return launch(prefill_finish_kernel<EPI>, grid, dim3(256), 0, stream, f);
}

static cudaError_t check_prefill(const GemvParams &p, int count, const PrefillPlan &pl, const PrefillWorkspace &w)
{
    if (count <= 0 || p.rows <= 0 || (p.rows % kTileRows) || p.cols <= 0 || (p.cols & 15) || p.cols > kSplitMaxCols ||
        !w.xs || !w.inv_scale || !w.ws || !w.error)
        return cudaErrorInvalidValue;
    if (pl.xs_bytes > w.xs_bytes || pl.inv_bytes > w.inv_bytes || pl.ws_bytes > w.ws_bytes) return cudaErrorInvalidValue;
    return prefill_setup();
}

static PrefillSplitParams split_params(const PrefillPlan &pl, int cols, int count, const PrefillWorkspace &w)
{
    PrefillSplitParams sp;
    memset(&sp, 0, sizeof sp);
    sp.cols = cols;
    sp.kchunks = pl.kchunks;
    sp.count = count;
    sp.xs = w.xs;
    sp.inv_scale = w.inv_scale;
    return sp;
}

static PrefillFinishParams finish_params(const GemvParams &p, int count, const PrefillPlan &pl,
                                         const PrefillWorkspace &w)
{
    PrefillFinishParams f;
    memset(&f, 0, sizeof f);
    f.ws = w.ws;
    f.splits = pl.splits;
    f.t_stride = pl.token_tiles * kPgM;
    f.ws_rows = pl.row_tiles * kP2N;
    f.rows = p.rows;
    f.count = count;
    for (int i = 0; i < 3; i++) f.scale[i] = p.scale[i];
    f.bound[0] = p.bound[0];
    f.bound[1] = p.bound[1];
    f.y = p.y;
    f.y_stride = p.y_stride;
    f.res = p.res;
    f.res_stride = p.res_stride;
    f.rope_cos = p.rope_cos;
    f.rope_sin = p.rope_sin;
    f.step = p.step;
    f.length = p.length + p.token_offset;
    f.kv = p.kv;
    f.page_table = p.page_table;
    f.num_pages = p.num_pages;
    f.layer = p.layer;
    f.positions = p.positions;
    f.token_table = p.token_table;
    f.table_stride = p.table_stride;
    return f;
}

cudaError_t lun_launch_prefill_split(const GemvParams &p, int count, const PrefillWorkspace &w, int sm_count,
                                     cudaStream_t stream)
{
    const PrefillPlan pl = lun_prefill_plan(p.rows, p.cols, count, sm_count);
    cudaError_t e = check_prefill(p, count, pl, w);
    if (e != cudaSuccess) return e;
    if ((p.x_stride & 3) || ((uintptr_t)p.x & 15) || ((uintptr_t)p.gain & 15)) return cudaErrorInvalidValue;
    PrefillSplitParams sp = split_params(pl, p.cols, count, w);
    sp.x = p.x;
    sp.x_stride = p.x_stride;
    sp.gain = p.gain;
    return launch(prefill_split_kernel, dim3(pl.token_tiles * kPgM), dim3(kSplitThreads), 0, stream, sp);
}

cudaError_t lun_launch_prefill_gemm(const GemvParams &p, int count, const PrefillWorkspace &w, int sm_count,
                                    cudaStream_t stream)
{
    const PrefillPlan pl = lun_prefill_plan(p.rows, p.cols, count, sm_count);
    cudaError_t e = check_prefill(p, count, pl, w);
    if (e != cudaSuccess) return e;
    PrefillGemmParams g;
    g.W = p.W;
    g.rows = p.rows;
    g.nb = (p.cols + kBlockCols - 1) / kBlockCols;
    g.kchunks = pl.kchunks;
    g.xs = w.xs;
    g.token_tiles = pl.token_tiles;
    g.count = count;
    g.splits = pl.splits;
    g.inv_scale = w.inv_scale;
    g.ws = w.ws;
    g.ws_rows = pl.row_tiles * kP2N;
    g.error = w.error;
    if (pl.tmem_a) {
        TmGemmParams t;
        t.rows = p.rows;
        t.kchunks = pl.kchunks;
        t.count = count;
        t.splits = pl.splits;
        t.xs = w.xs;
        t.inv_scale = w.inv_scale;
        t.ws = w.ws;
        t.t_stride = pl.token_tiles * kPgM;
        t.ws_rows = pl.row_tiles * kP2N;
        t.error = w.error;
        CUtensorMap wide;
        if ((e = weight_tensor_map_wide(&wide, p.W, p.rows, g.nb)) != cudaSuccess) return e;
        return launch(prefill_gemm_tmem_kernel, dim3((p.rows + kTmRows - 1) / kTmRows, 1, pl.splits),
                      dim3(kTmThreads), kTmSmemBytes, stream, t, wide);
    }
    CUtensorMap wmap;
    if ((e = weight_tensor_map(&wmap, p.W, p.rows, g.nb)) != cudaSuccess) return e;
    return launch(prefill_gemm_pair_kernel, dim3(2 * pl.row_tiles, (pl.token_tiles + 1) / 2, pl.splits),
                  dim3(kPgThreads), kP2SmemBytes, stream, g, wmap);
}

cudaError_t lun_launch_prefill_finish(const GemvParams &p, int count, int epilogue, const PrefillWorkspace &w,
                                      int sm_count, cudaStream_t stream)
{
    const PrefillPlan pl = lun_prefill_plan(p.rows, p.cols, count, sm_count);
    cudaError_t e = check_prefill(p, count, pl, w);
    if (e != cudaSuccess) return e;
    if ((epilogue == kEpiQKV && (p.rows != kQKVRows || p.cols != kHidden)) || (epilogue == kEpiSwiGLU && (p.rows & 1)))
        return cudaErrorInvalidValue;
    const PrefillFinishParams f = finish_params(p, count, pl, w);
    switch (epilogue) {
    case kEpiStore: return launch_finish<kEpiStore>(f, stream);
    case kEpiResidual: return launch_finish<kEpiResidual>(f, stream);
    case kEpiQKV: return launch_finish<kEpiQKV>(f, stream);
    case kEpiSwiGLU: return launch_finish<kEpiSwiGLU>(f, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t lun_launch_prefill_finish_split(const GemvParams &p, int count, int epilogue, const PrefillWorkspace &w,
                                            int sm_count, const float *next_gain, int next_rows, bool split,
                                            cudaStream_t stream)
{
    const PrefillPlan pl = lun_prefill_plan(p.rows, p.cols, count, sm_count);
    cudaError_t e = check_prefill(p, count, pl, w);
    if (e != cudaSuccess) return e;
    const int width = epilogue == kEpiSwiGLU ? p.rows / 2 : p.rows;
    if ((epilogue != kEpiResidual && epilogue != kEpiSwiGLU) || width > kSplitMaxCols || (width & 15) ||
        (p.y && ((p.y_stride & 3) || ((uintptr_t)p.y & 15))) ||
        (epilogue == kEpiResidual && (!p.res || (p.res_stride & 3) || ((uintptr_t)p.res & 15))) ||
        ((uintptr_t)next_gain & 15))
        return cudaErrorInvalidValue;
    const PrefillFinishParams f = finish_params(p, count, pl, w);
    // the next projection reads `width` columns: its plan sizes the operand tiles
    const PrefillPlan next = lun_prefill_plan(next_rows > 0 ? next_rows : kTileRows, width, count, sm_count);
    if (next.xs_bytes > w.xs_bytes) return cudaErrorInvalidValue;
    PrefillSplitParams sp = split_params(next, width, count, w);
    sp.gain = next_gain;
    if (!split) sp.xs = nullptr;
    if (epilogue == kEpiSwiGLU)
        return launch(prefill_finish_split_kernel<kEpiSwiGLU>, dim3(pl.token_tiles * kPgM), dim3(kFsThreads), 0,
                      stream, f, sp);
    return launch(prefill_finish_split_kernel<kEpiResidual>, dim3(pl.token_tiles * kPgM), dim3(kFsThreads), 0, stream,
                  f, sp);
}

cudaError_t lun_launch_prefill(const GemvParams &p, int count, int epilogue, const PrefillWorkspace &w,
                               int sm_count, cudaStream_t stream)
{
    return lun_launch_prefill_marked(p, count, epilogue, w, sm_count, stream, nullptr);
}

cudaError_t lun_launch_prefill_marked(const GemvParams &p, int count, int epilogue, const PrefillWorkspace &w,
                                      int sm_count, cudaStream_t stream, cudaEvent_t *marks)
{
    cudaError_t e;
    if (marks && (e = cudaEventRecord(marks[0], stream)) != cudaSuccess) return e;
    if ((e = lun_launch_prefill_split(p, count, w, sm_count, stream)) != cudaSuccess) return e;
    if (marks && (e = cudaEventRecord(marks[1], stream)) != cudaSuccess) return e;
    if ((e = lun_launch_prefill_gemm(p, count, w, sm_count, stream)) != cudaSuccess) return e;
    if (marks && (e = cudaEventRecord(marks[2], stream)) != cudaSuccess) return e;
    if ((e = lun_launch_prefill_finish(p, count, epilogue, w, sm_count, stream)) != cudaSuccess) return e;
    if (marks && (e = cudaEventRecord(marks[3], stream)) != cudaSuccess) return e;
    return cudaSuccess;
}
