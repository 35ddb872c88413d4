// Programmatic dependent launch for back-to-back operators on one stream.
//
// A kernel launched with launch_dependent may be scheduled while the
// previous kernel of its stream is still draining; its first statement,
// pdl_enter(), waits until that kernel has completed and its memory is
// visible (so nothing is read or written early), then lets the next kernel
// be scheduled in turn.  What overlaps is the launch and CTA placement of
// one operator with the tail of the one before it.  Without the launch
// attribute (a plain <<< >>> launch, or a kernel that is first in its
// stream) both instructions return at once.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace emel {

__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... P, typename... A>
cudaError_t launch_dependent(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             A&&... args) {
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
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

}  // namespace emel
