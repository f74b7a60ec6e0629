// Scratch for wl_matvec_static: one file-scope device array per device, so the call allocates nothing.
//
// Callers that cannot allocate: a host runtime that plans all of its device memory up front (a serving process with a
// fixed memory budget, or a caller whose own allocator owns every byte of the device) cannot let a kernel export grow
// a private buffer with cudaMalloc behind its back, and a cudaMalloc/cudaFree pair inside a call also synchronises the
// device, which such callers schedule around. wl_matvec_static gives them the tensor-core matvec with its scratch
// (the error word and the prepared activations) in this module's own static array instead.
#include <mutex>
#include "wl_common.h"
#include "wl_kernels.h"

namespace wl {
namespace k {

static_assert(WL_MATVEC_STATIC_MAX_COLS == STATIC_MAX_COLS, "the header's limit and the scratch size disagree");

// [error word, padded to 256 bytes | prepared activations of 8 columns of up to STATIC_MAX_COLS values]
static __device__ __align__(256) uint8_t g_static_scratch[STATIC_SCRATCH_BYTES];

void* static_scratch()
{
    static std::mutex mu;
    static void* addr[64] = {};
    int dev = 0;
    WL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) WL_THROW(WL_EINVAL, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || !p)
            WL_THROW(WL_ECUDA, std::string("cudaGetSymbolAddress of the static matvec scratch failed: ") +
                               cudaGetErrorString(e));
        addr[dev] = p;
    }
    return addr[dev];
}

}  // namespace k
}  // namespace wl
