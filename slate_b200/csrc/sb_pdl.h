/*
 * sb_pdl.h -- programmatic dependent launch for the kernels of the decode
 * step (internal, CUDA C++ only).
 *
 * A kernel launched with sb_launch_pdl may begin while the previous kernel of
 * its stream is still running (once that kernel has executed
 * griddepcontrol.launch_dependents in all its CTAs, which the step's kernels
 * do at their start), so its launch latency and set-up overlap that kernel's
 * tail.  Such a kernel must execute sb_grid_wait() (griddepcontrol.wait:
 * returns when the previous grid has completed and its memory is visible)
 * before it reads or writes anything the earlier kernels of the stream touch.
 * Because every kernel of the chain waits before it finishes, a completed
 * predecessor implies that all kernels before it completed too.  With a
 * memory copy or a non-PDL kernel before it, the launch is an ordinary one.
 */
#ifndef SB_PDL_H
#define SB_PDL_H

#include <cuda_runtime.h>
#include <utility>

__device__ __forceinline__ void sb_grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void sb_grid_release() { asm volatile("griddepcontrol.launch_dependents;"); }

template <typename... KArgs, typename... Args>
static inline cudaError_t sb_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                        size_t smem, cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#endif
