// Launcher of the persistent decode kernel (decode_mega.cuh).
#include "decode_mega.cuh"
#include "kernels.h"

using namespace lun;

// The partial sums of a phase's items and the residual rows of its tiles stay
// in shared memory: every CTA's share of every FP8 phase must fit kMegaMaxItems
// items and kMegaMaxTiles tiles.
bool lun_mega_supported(int sm_count)
{
    if (sm_count < kKVHeads) return false;
    // blocks of the largest CTA share: whole tiles of k / 64 blocks each
    auto tiles = [sm_count](int rows) { return (rows / kTileRows + sm_count - 1) / sm_count; };
    const int qkv = tiles(kQKVRows) * (kHidden / kBlockCols) / item_blocks(kPhQKV);
    const int o = tiles(kHidden) * (kQuery / kBlockCols) / item_blocks(kPhO);
    const int gateup = tiles(kGateUpRows) * (kHidden / kBlockCols) / item_blocks(kPhGateUp);
    const int down = tiles(kHidden) * (kInner / kBlockCols) / item_blocks(kPhDown);
    return qkv <= kMegaMaxItems && o <= kMegaMaxItems && gateup <= kMegaMaxItems && down <= kMegaMaxItems &&
           tiles(kHidden) <= kMegaMaxTiles;
}

cudaError_t lun_launch_decode_mega(const MegaParams &p, int sm_count, cudaStream_t stream)
{
    if (!lun_mega_supported(sm_count)) return cudaErrorInvalidConfiguration;
    static bool attribute_set[128] = {};
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    if (device < 0 || device >= 128) return cudaErrorInvalidDevice;
    if (!attribute_set[device]) {
        e = cudaFuncSetAttribute(decode_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kMegaSmemBytes);
        if (e != cudaSuccess) return e;
        attribute_set[device] = true;
    }
    // every CTA must be resident at once (grid barriers): one per SM
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mega_kernel, kMegaThreads,
                                                      kMegaSmemBytes);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    MegaParams copy = p;
    void *args[] = {&copy};
    return cudaLaunchCooperativeKernel((const void *)decode_mega_kernel, dim3(sm_count),
                                       dim3(kMegaThreads), args, kMegaSmemBytes, stream);
}
