// Kernel launch with programmatic dependent launch (PDL): the kernel may begin launching while the
// previous kernel in the stream is still running; it must execute griddepcontrol.wait before it touches
// memory the previous kernel writes or reads. Inside a captured CUDA graph this becomes a programmatic
// edge, so a dependent kernel's launch latency and prologue overlap its predecessor's tail.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace jb {

template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace jb
