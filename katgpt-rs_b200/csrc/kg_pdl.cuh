// kg_pdl.cuh — programmatic dependent launch for the forward's kernel chain.
//
// Launches carry cudaLaunchAttributeProgrammaticStreamSerialization, so the
// next kernel in a stream (or in a captured graph) is scheduled while the
// previous one drains. Every kernel launched this way calls pdl_wait() before
// its first global-memory access: griddepcontrol.wait blocks until the grids
// it depends on have completed and their memory is visible (a no-op after an
// ordinary launch or a memory operation).
#pragma once
#include <cuda_runtime.h>

namespace kg {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// kernel<<<grid, block, smem, s>>>(args...) with the programmatic-serialization
// attribute, as thread-block clusters of `cluster` when it is not 1 x 1 x 1.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                               dim3 cluster, Args &&...args) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute at[2];
    unsigned n = 0;
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
    if (cluster.x * cluster.y * cluster.z > 1) {
        at[n].id = cudaLaunchAttributeClusterDimension;
        at[n].val.clusterDim.x = cluster.x;
        at[n].val.clusterDim.y = cluster.y;
        at[n].val.clusterDim.z = cluster.z;
        ++n;
    }
    lc.attrs = at;
    lc.numAttrs = n;
    return cudaLaunchKernelEx(&lc, kernel, static_cast<Args &&>(args)...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args &&...args) {
    return launch_pdl_cluster(kernel, grid, block, smem, s, dim3(1, 1, 1), static_cast<Args &&>(args)...);
}

}  // namespace kg
