// Kernel launches with programmatic dependent launch (PDL).
//
// Every kernel of the library but the tcgen05 GEMM (wl_gemm.cu, launched plainly and never overlapped) is launched
// with programmatic stream serialisation allowed, and every such kernel starts
// with pdl_trigger() then pdl_wait(): the next kernel on the stream may be scheduled as soon as all CTAs of this one
// have started, and it waits in pdl_wait() until this one has completed and its writes are visible. A kernel does
// nothing before its pdl_wait() except work that reads no buffer another kernel writes (the weight copies of the
// matvec kernels). Because every kernel waits, the ordering stays transitive: kernel N+1 cannot complete before
// kernel N has. Outside a PDL launch (or after a memcpy/memset node) the two instructions are no-ops.
#pragma once
#include <utility>
#include <cuda_runtime.h>
#include "wl_common.h"

namespace wl {
namespace k {

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... P, typename... A>
inline void launch(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    WL_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...));
}

// The same with thread-block clusters of cluster_x CTAs along x (gridDim.x a multiple of cluster_x).
template <typename... P, typename... A>
inline void launch_cluster(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int cluster_x,
                           A&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    WL_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...));
}

}  // namespace k
}  // namespace wl
