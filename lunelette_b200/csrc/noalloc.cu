// Allocation-free variant of the split-K attention entry point.
//
// Some callers cannot call cudaMalloc: an engine that has already reserved the
// whole device memory budget for its own pool, or a latency-critical serving loop
// in which cudaMalloc/cudaFree would synchronise the device and stall every other
// stream. lunelette_cuda_attention() asks those callers for two scratch buffers;
// this variant keeps its scratch in a fixed device array inside the library
// instead, so the caller passes only inputs and outputs and nothing is allocated.
#include "kernels.h"

#include <mutex>
#include <stdio.h>
#include <string.h>

#define LUN_API extern "C" __attribute__((visibility("default")))

using namespace lun;

namespace {

// Partial-result slots (one per query row, head and split): 4096 slots of 128
// accumulators plus (max, sum) = 2,129,920 bytes, held by every GPU that loads
// the library until the process exits.
constexpr int kScratchSlots = 4096;
constexpr size_t kScratchFloats = (size_t)kScratchSlots * (kHeadDim + 2);

__device__ __align__(256) float g_attention_scratch[kScratchFloats];

constexpr int kMaxDevices = 128;
float *g_scratch_address[kMaxDevices];  // device address of the array, per device
std::mutex g_setup;

// The array's name in host code only stands for the symbol; its device address
// on the current device comes from cudaGetSymbolAddress, looked up once per
// device and then reused.
int scratch_of_current_device(float **address, char *error, size_t capacity)
{
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess || device < 0 || device >= kMaxDevices) {
        if (error && capacity)
            snprintf(error, capacity, "attention_noalloc: no usable current device (%s)",
                     cudaGetErrorString(e));
        return -1;
    }
    std::lock_guard<std::mutex> lock(g_setup);
    if (!g_scratch_address[device]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (e != cudaSuccess || !p) {
            if (error && capacity)
                snprintf(error, capacity, "attention_noalloc: cudaGetSymbolAddress failed: %s",
                         cudaGetErrorString(e));
            return -1;
        }
        g_scratch_address[device] = static_cast<float *>(p);
    }
    *address = g_scratch_address[device];
    return 0;
}

int sm_count_of_current_device()
{
    int device = 0, sms = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 148;
    return sms;
}

}  // namespace

LUN_API int lunelette_cuda_attention_noalloc(const float *q, const float *kv_pool,
                                             const int *page_table, size_t num_pages, size_t layer,
                                             size_t length, size_t count, float *out, void *stream,
                                             char *error, size_t capacity)
{
    if (!q || !kv_pool || !page_table || !out || !count || !num_pages ||
        length + count > num_pages * kPage) {
        if (error && capacity) snprintf(error, capacity, "attention_noalloc: invalid arguments");
        return -1;
    }
    if (count * kQueryHeads > (size_t)kScratchSlots) {
        if (error && capacity)
            snprintf(error, capacity,
                     "attention_noalloc: count %zu exceeds the fixed scratch (at most %d query rows)",
                     count, kScratchSlots / kQueryHeads);
        return -1;
    }
    float *scratch = nullptr;
    if (scratch_of_current_device(&scratch, error, capacity)) return -1;
    AttnParams a;
    memset(&a, 0, sizeof a);
    a.q = q;
    a.kv = kv_pool;
    a.page_table = page_table;
    a.num_pages = (int)num_pages;
    a.layer = (int)layer;
    a.length = (int)length;
    a.out = out;
    // Every slot the combine step reads is written by the split step of the same
    // call, so nothing in the shared array has to be cleared between calls.
    a.part_acc = scratch;
    a.part_ml = scratch + (size_t)kScratchSlots * kHeadDim;
    lun_attention_plan(&a, (int)(length + count), (int)count, sm_count_of_current_device(),
                       kScratchSlots);
    cudaError_t e = lun_launch_attention(a, (int)count, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        if (error && capacity)
            snprintf(error, capacity, "attention_noalloc: launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
