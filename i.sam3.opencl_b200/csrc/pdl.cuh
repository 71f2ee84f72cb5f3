// SPDX-License-Identifier: Unlicense
// Programmatic dependent launch (PDL). A kernel launched with the
// programmatic stream-serialization attribute may be scheduled while the
// previous kernel in its stream is still running. griddep_wait() blocks
// until that kernel has completed and its memory operations are visible (a
// no-op for a kernel launched without the attribute), so nothing before it
// may touch global memory the previous kernel reads or writes.
// griddep_launch() lets the next such kernel be scheduled once every CTA of
// this grid has executed it (or exited); that kernel still waits for this
// one's completion before its own accesses. The kernels that call both at
// their top are launched through launch_pdl, so a chain of short kernels
// overlaps each launch and setup with the previous kernel's tail.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace sam3 {

__device__ __forceinline__ void griddep_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void griddep_launch()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// kern<<<grid, block, smem, s>>>(args...) as a programmatic dependent of the
// previous kernel in s; returns the launch status.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      Args &&...args)
{
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace sam3
