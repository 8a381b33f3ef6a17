/* The test hook the reference's real-weight comparator (tests/compare_metal.c)
 * declares and calls after each prefill/decode: borrowed host rows of the last
 * block's layer-25 output (normalized 0) or its final-norm rows (normalized 1).
 * The reference defines it over its Metal runtime's surviving scratch buffers
 * (tests/metal_snapshot.m:5-8); here it forwards to the library's traced
 * snapshot, so run the comparator with LUNELETTE_CUDA_TRACE=1. */
#include "lunelette_cuda.h"

const float *test_metal_snapshot(lunelette_metal *runtime, int normalized)
{
    return lunelette_cuda_snapshot(runtime, normalized);
}
