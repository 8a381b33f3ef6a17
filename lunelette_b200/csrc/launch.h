// Kernel launches with programmatic dependent launch (PDL): a kernel may start
// while the previous kernel of the stream finishes; it runs griddepcontrol.wait
// (pdl_wait) before touching anything that kernel wrote. LUNELETTE_PDL=0 turns
// the attribute off for comparisons.
#pragma once
#include <cuda_runtime.h>
#include <stdlib.h>

namespace lun {

inline bool pdl_enabled()
{
    static const bool on = [] {
        const char *v = getenv("LUNELETTE_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

template <typename... Params, typename... Args>
cudaError_t launch(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

}  // namespace lun
