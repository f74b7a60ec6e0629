// Shared host-side plumbing of libwindlass_cuda: status codes, the thread-local error message, CUDA checks and the
// GGUF block layouts.
#pragma once
#include <cstdint>
#include <cstdio>
#include <string>
#include <cuda_runtime.h>
#include "../../include/windlass.h"

namespace wl {

// Sets the calling thread's error message (returned by wl_last_error) and returns the status.
int32_t fail(int32_t status, const std::string& msg);
void clear_error();

struct Error {
    int32_t status;
    std::string msg;
};

// Throws Error for a failed CUDA call; the C ABI turns it into WL_ECUDA (WL_ENOMEM for allocation failures).
void cuda_check(cudaError_t e, const char* what, const char* file, int line);
#define WL_CUDA(call) ::wl::cuda_check((call), #call, __FILE__, __LINE__)
#define WL_THROW(status, msg) throw ::wl::Error{(status), (msg)}

// Elements per block and bytes per block of a GGUF type (GgmlTypes.TryGetLayout, src/Gguf.cs:30-66).
bool layout(int type, int* block, int* bytes);
inline int64_t row_bytes_of(int type, int64_t cols)
{
    int b = 0, s = 0;
    layout(type, &b, &s);
    return b ? cols / b * s : 0;
}
// Quants.CanDecode (src/Quants.cs:11-21): the types every kernel of this library decodes.
bool can_decode(int type);
const char* type_name(int type);

}  // namespace wl
