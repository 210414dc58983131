// Kernel launch with programmatic dependent launch: the grid may be scheduled while the previous kernel on the
// stream is still running, so its prologue overlaps that kernel's tail. Every kernel launched this way executes
// griddepcontrol.wait (pdl_wait) in all of its CTAs before it reads what earlier kernels wrote, and before it exits,
// so that completion stays transitive along the stream.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace srhpm {

template <class... KArgs, class... Args>
cudaError_t launch_k_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                         Args &&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = grid;
    cfg.blockDim           = block;
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace srhpm
