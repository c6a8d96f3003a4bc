// Programmatic dependent launch for the latency-bound Transformer kernels.
//
// A kernel launched with launch_pdl() may be scheduled while its predecessor
// in the stream (or CUDA graph) is still running.  Every such kernel calls
// pdl_prologue() as its first statement: griddepcontrol.wait blocks until the
// predecessor grid has completed and its memory is visible (so no read or
// write of the kernel can race with it, and completion stays transitive down
// the chain), then griddepcontrol.launch_dependents lets the next kernel begin
// its own launch.  The overlap hides launch latency between the short
// dependent kernels of a decode step.  Without a programmatic predecessor both
// instructions are no-ops.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace tsacb::dev
{
__device__ __forceinline__ void pdl_prologue()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Split form for kernels that first read inputs no predecessor writes (model
// weights, scales, biases): pdl_release() lets the next kernel begin its own
// launch, the constant loads follow, and pdl_wait() then blocks until the
// predecessor grid has completed and its memory is visible, before anything
// it produced is read.
__device__ __forceinline__ void pdl_release()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <class... Params, class... Args>
void launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                cudaStream_t stream, Args&&... args)
{
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}
} // namespace tsacb::dev
