// Launchers of the tcgen05 prefill projections (prefill_gemm.cuh).
#include "kernels.h"
#include "prefill_gemm.cuh"

using namespace lun;

PrefillPlan lun_prefill_plan(int rows, int cols, int count, int sm_count)
{
    PrefillPlan pl;
    pl.row_tiles = (rows + kPgN - 1) / kPgN;
    pl.token_tiles = (count + kPgM - 1) / kPgM;
    pl.kchunks = (cols + kPgK - 1) / kPgK;
    // K ranges fill the SMs when the output tiles alone do not; every range
    // keeps at least two stages
    const int tiles = pl.row_tiles * pl.token_tiles;
    int splits = sm_count / (tiles > 0 ? tiles : 1);
    splits = splits < 1 ? 1 : splits;
    const int max_splits = pl.kchunks / 2 > 0 ? pl.kchunks / 2 : 1;
    pl.splits = splits > max_splits ? max_splits : splits;
    return pl;
}

void lun_prefill_workspace_bytes(int max_count, int sm_count, size_t *xs_bytes, size_t *inv_bytes,
                                 size_t *ws_bytes)
{
    static const int shapes[4][2] = {{kQKVRows, kHidden}, {kHidden, kQuery}, {kGateUpRows, kHidden}, {kHidden, kInner}};
    size_t xs = 0, ws = 0;
    for (const auto &s : shapes) {
        const PrefillPlan pl = lun_prefill_plan(s[0], s[1], max_count, sm_count);
        const size_t x = (size_t)pl.token_tiles * pl.kchunks * 2 * kPgATile;
        const size_t w = (size_t)pl.splits * pl.token_tiles * kPgM * pl.row_tiles * kPgN * sizeof(float);
        xs = x > xs ? x : xs;
        ws = w > ws ? w : ws;
    }
    *xs_bytes = xs;
    *inv_bytes = (size_t)((max_count + kPgM - 1) / kPgM) * kPgM * sizeof(float);
    *ws_bytes = ws;
}

static cudaError_t prefill_setup()
{
    static bool done[128] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    if (done[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(prefill_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPgSmemBytes);
    if (e == cudaSuccess) done[dev] = true;
    return e;
}

template <int EPI>
static cudaError_t launch_finish(const PrefillFinishParams &f, cudaStream_t stream)
{
    const dim3 grid((unsigned)((f.rows / 2 + 255) / 256), (unsigned)f.count);
    prefill_finish_kernel<EPI><<<grid, 256, 0, stream>>>(f);
    return cudaGetLastError();
}

cudaError_t lun_launch_prefill(const GemvParams &p, int count, int epilogue, const PrefillWorkspace &w,
                               int sm_count, cudaStream_t stream)
{
    if (count <= 0 || p.rows <= 0 || (p.rows % kTileRows) || p.cols <= 0 || (p.cols & 15) || !w.xs ||
        !w.inv_scale || !w.ws || !w.error)
        return cudaErrorInvalidValue;
    if ((epilogue == kEpiQKV && (p.rows != kQKVRows || p.cols != kHidden)) || (epilogue == kEpiSwiGLU && (p.rows & 1)))
        return cudaErrorInvalidValue;
    const PrefillPlan pl = lun_prefill_plan(p.rows, p.cols, count, sm_count);
    const size_t xs = (size_t)pl.token_tiles * pl.kchunks * 2 * kPgATile;
    const size_t inv = (size_t)pl.token_tiles * kPgM * sizeof(float);
    const size_t ws = (size_t)pl.splits * pl.token_tiles * kPgM * pl.row_tiles * kPgN * sizeof(float);
    if (xs > w.xs_bytes || inv > w.inv_bytes || ws > w.ws_bytes) return cudaErrorInvalidValue;
    cudaError_t e = prefill_setup();
    if (e != cudaSuccess) return e;

    PrefillSplitParams sp;
    sp.x = p.x;
    sp.x_stride = p.x_stride;
    sp.gain = p.gain;
    sp.cols = p.cols;
    sp.kchunks = pl.kchunks;
    sp.count = count;
    sp.xs = w.xs;
    sp.inv_scale = w.inv_scale;
    prefill_split_kernel<<<pl.token_tiles * kPgM, 256, 0, stream>>>(sp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

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
    g.ws_rows = pl.row_tiles * kPgN;
    g.error = w.error;
    prefill_gemm_kernel<<<dim3(pl.row_tiles, pl.token_tiles, pl.splits), kPgThreads, kPgSmemBytes, stream>>>(g);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    PrefillFinishParams f;
    f.ws = w.ws;
    f.splits = pl.splits;
    f.t_stride = pl.token_tiles * kPgM;
    f.ws_rows = g.ws_rows;
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
    switch (epilogue) {
    case kEpiStore: return launch_finish<kEpiStore>(f, stream);
    case kEpiResidual: return launch_finish<kEpiResidual>(f, stream);
    case kEpiQKV: return launch_finish<kEpiQKV>(f, stream);
    case kEpiSwiGLU: return launch_finish<kEpiSwiGLU>(f, stream);
    default: return cudaErrorInvalidValue;
    }
}
