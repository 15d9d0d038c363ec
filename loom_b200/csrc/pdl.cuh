// pdl.cuh -- programmatic dependent launch for the model-step kernels: a
// kernel launched with launch_pdl may start while its predecessor on the
// stream is still running; it issues loads that do not depend on that
// predecessor (weights), then pdl_wait() blocks until the predecessor has
// completed and its writes are visible. Every kernel launched this way calls
// pdl_wait() on every path before it exits, so completion stays transitive
// along the stream; pdl_trigger() lets the successor start early.
#pragma once
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace loom {

__device__ __forceinline__ void pdl_wait_() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl_(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               Args... args) {
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
    count_launch();
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace loom
