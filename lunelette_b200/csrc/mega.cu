// Launcher of the persistent decode kernel (decode_mega.cuh).
#include <cudaTypedefs.h>
#include <string.h>

#include <atomic>

#include "decode_mega.cuh"
#include "kernels.h"

PFN_cuTensorMapEncodeTiled_v12000 lun_tensor_map_encoder();

using namespace lun;

// The partial sums of a phase's items and the residual rows of its tiles stay
// in shared memory: every CTA's share of every FP8 phase must fit kMegaMaxItems
// items and kMegaMaxTiles tiles.
bool lun_mega_supported(int sm_count)
{
    // one CTA per act slice in the FFN; a KV head per CTA in attention
    if (sm_count < kFfnSlices || sm_count < kQueryHeads) return false;
    // blocks of the largest CTA share: whole tiles of k / 64 blocks each
    auto tiles = [sm_count](int rows) { return (rows / kTileRows + sm_count - 1) / sm_count; };
    const int qkv = tiles(kQKVRows) * (kHidden / kBlockCols) / item_blocks(kPhQKV);
    const int o = tiles(kHidden) * (kQuery / kBlockCols) / item_blocks(kPhO);
    const int gateup = kSliceTiles * (kHidden / kBlockCols) / item_blocks(kPhGateUp);
    return qkv <= kMegaMaxItems && o <= kMegaMaxItems && gateup <= kMegaMaxItems && tiles(kHidden) <= kMegaMaxTiles;
}

// The down projections of all layers as one 4-D tensor of 16-bit elements:
// {256 (a 512-byte piece: 8 rows x 64 columns of one tile), 144 pieces per tile
// (act slice s = block s / 2, half s % 2), 384 tiles, 26 layers}; the box
// {256, 1, 24, 1} is one down item of the persistent kernel.
cudaError_t lun_down_slice_map(void *map, const uint8_t *down0, size_t layer_stride)
{
    PFN_cuTensorMapEncodeTiled_v12000 encode = lun_tensor_map_encoder();
    if (!encode || ((uintptr_t)down0 & 15) || (layer_stride & 15)) return cudaErrorInvalidValue;
    const cuuint64_t dims[4] = {256, (cuuint64_t)kFfnSlices, (cuuint64_t)(kHidden / kTileRows), (cuuint64_t)kLayers};
    const cuuint64_t strides[3] = {512, (cuuint64_t)(kInner / kBlockCols) * kBlockBytes, layer_stride};
    const cuuint32_t box[4] = {256, 1, kDownItemTiles, 1};
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    CUresult r = encode(reinterpret_cast<CUtensorMap *>(map), CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, (void *)down0, dims,
                        strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t lun_launch_decode_mega(const MegaParams &p, const void *down_map, int sm_count, cudaStream_t stream)
{
    if (!lun_mega_supported(sm_count)) return cudaErrorInvalidConfiguration;
    // the shared-memory opt-in, once per device (atomic flags: callers may be on
    // several threads; setting the attribute twice is harmless)
    static std::atomic<bool> attribute_set[128];
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    if (device < 0 || device >= 128) return cudaErrorInvalidDevice;
    if (!attribute_set[device].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(decode_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kMegaSmemBytes);
        if (e != cudaSuccess) return e;
        attribute_set[device].store(true, std::memory_order_release);
    }
    // every CTA must be resident at once (grid barriers): one per SM
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mega_kernel, kMegaThreads,
                                                      kMegaSmemBytes);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    MegaParams copy = p;
    CUtensorMap map;
    memcpy(&map, down_map, sizeof map);
    void *args[] = {&copy, &map};
    return cudaLaunchCooperativeKernel((const void *)decode_mega_kernel, dim3(sm_count),
                                       dim3(kMegaThreads), args, kMegaSmemBytes, stream);
}
