// Kernel launch with an optional programmatic-dependent-launch attribute: with pdl set, the grid may
// begin launching before the previous kernel on the stream has completed (once every CTA of that kernel
// has executed grid_dep_launch or exited); the kernel must call grid_dep_wait before it reads anything
// the previous kernels wrote or writes anything they read. Captured into CUDA graphs as programmatic edges.
#pragma once

#include <cuda_runtime.h>

#include <utility>

#include "common/check.h"

namespace cudallm {

template <typename... KArgs, typename... Args>
void launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                   Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    CLLM_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

}  // namespace cudallm
