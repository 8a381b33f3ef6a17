// Launcher of the persistent decode kernel (decode_mega.cuh).
#include "decode_mega.cuh"
#include "kernels.h"

using namespace lun;

cudaError_t lun_launch_decode_mega(const MegaParams &p, int sm_count, cudaStream_t stream)
{
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
