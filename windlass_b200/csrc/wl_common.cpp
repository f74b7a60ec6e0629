// Status and error plumbing, block layouts.
#include "wl_common.h"
#include <string>

namespace wl {

static thread_local std::string t_error;

int32_t fail(int32_t status, const std::string& msg)
{
    t_error = msg;
    return status;
}

void clear_error() { t_error.clear(); }

const char* last_error_cstr() { return t_error.c_str(); }

void cuda_check(cudaError_t e, const char* what, const char* file, int line)
{
    if (e == cudaSuccess) return;
    cudaGetLastError();   // clear a non-sticky error so the context stays usable
    const int32_t status = (e == cudaErrorMemoryAllocation) ? WL_ENOMEM : WL_ECUDA;
    char buf[512];
    snprintf(buf, sizeof buf, "%s failed: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
    throw Error{status, buf};
}

// GgmlTypes.TryGetLayout (src/Gguf.cs:30-66).
bool layout(int t, int* bs, int* ts)
{
    int b = 0, s = 0;
    switch (t) {
    case 0: b = 1; s = 4; break;   case 1: b = 1; s = 2; break;   case 30: b = 1; s = 2; break;
    case 24: b = 1; s = 1; break;  case 25: b = 1; s = 2; break;  case 26: b = 1; s = 4; break;
    case 27: b = 1; s = 8; break;  case 28: b = 1; s = 8; break;
    case 2: b = 32; s = 18; break; case 3: b = 32; s = 20; break; case 6: b = 32; s = 22; break;
    case 7: b = 32; s = 24; break; case 8: b = 32; s = 34; break; case 9: b = 32; s = 36; break;
    case 10: b = 256; s = 84; break; case 11: b = 256; s = 110; break; case 12: b = 256; s = 144; break;
    case 13: b = 256; s = 176; break; case 14: b = 256; s = 210; break; case 15: b = 256; s = 292; break;
    case 16: b = 256; s = 66; break; case 17: b = 256; s = 74; break; case 18: b = 256; s = 98; break;
    case 19: b = 256; s = 50; break; case 20: b = 32; s = 18; break; case 21: b = 256; s = 110; break;
    case 22: b = 256; s = 82; break; case 23: b = 256; s = 136; break; case 29: b = 256; s = 56; break;
    default: if (bs) *bs = 0; if (ts) *ts = 0; return false;
    }
    if (bs) *bs = b;
    if (ts) *ts = s;
    return true;
}

bool can_decode(int t)
{
    switch (t) {
    case 0: case 1: case 30: case 2: case 3: case 6: case 7: case 8: case 10: case 11: case 12: case 13: case 14:
    case 16: case 17: case 18: case 19: case 20: case 21: case 22: case 23: case 29: return true;
    }
    return false;
}

const char* type_name(int t)
{
    switch (t) {
    case 0: return "f32"; case 1: return "f16"; case 30: return "bf16"; case 2: return "q4_0"; case 3: return "q4_1";
    case 6: return "q5_0"; case 7: return "q5_1"; case 8: return "q8_0"; case 10: return "q2_K"; case 11: return "q3_K";
    case 12: return "q4_K"; case 13: return "q5_K"; case 14: return "q6_K"; case 16: return "iq2_xxs";
    case 17: return "iq2_xs"; case 18: return "iq3_xxs"; case 19: return "iq1_s"; case 20: return "iq4_nl";
    case 21: return "iq3_s"; case 22: return "iq2_s"; case 23: return "iq4_xs"; case 29: return "iq1_m";
    }
    return "unknown";
}

}  // namespace wl
