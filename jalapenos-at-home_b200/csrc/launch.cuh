// Kernel launches with programmatic dependent launch (PDL).
//
// Every kernel of a forward pass starts with griddepcontrol.wait before it
// touches activations, the KV cache or outputs, and signals
// griddepcontrol.launch_dependents once the next kernel may begin its own
// prologue.  Launched this way, a kernel's setup (barrier init, TMEM
// allocation, and for the tensor-core projections the first weight stages)
// overlaps the tail of the kernel before it.  Inside a captured CUDA graph
// the attribute becomes a programmatic dependency edge.
#pragma once

#include <cuda_runtime.h>

#include "jl_internal.h"

namespace jl {

template <typename... KArgs, typename... Args>
jl_status launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    JL_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
    return JL_OK;
}

}  // namespace jl
