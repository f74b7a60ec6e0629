// Activation prep of one 256-value superblock for the tensor-core matvecs, shared by every kernel that produces
// activations in that form (k_xprep, and the fused swiglu and attention-combine kernels).
//
// Layout of the XP_COL-byte block: three planes of signed 8-bit digits of the 256 values in natural order (pitch
// XP_DIGIT; 32 zero pad bytes each), then at XP_REC four (hi pair, lo pair) f16x2 words holding the sums of the eight
// 32-value sub-blocks, the float unit of the digits, and zeros up to XP_COL. X = round(x * 2^(20-e)) (|X| <= 2^20, e
// the exponent of the superblock's largest magnitude) is split into balanced base-128 digits X = X0*2^14 + X1*2^7 +
// X2, each in [-64, 64]. The sums are taken at 2^(10-e), where they fit f16 with a hi/lo split good to 2^-22.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include "wl_kernels.h"

namespace wl {
namespace k {

__device__ __forceinline__ uint32_t xp_h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Called by the 64 threads t = 0..63 of a 64-thread CTA (it synchronises the CTA); thread t holds values 4t..4t+3.
// scratch: two floats of shared memory.
__device__ __forceinline__ void xprep_sb(const float (&f)[4], int t, float* scratch, uint8_t* __restrict__ blk)
{
    float m = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((t & 31) == 0) scratch[t >> 5] = m;
    __syncthreads();
    m = fmaxf(scratch[0], scratch[1]);
    const bool finite = m <= 3.4e38f;          // false for inf and NaN
    int e = 0;
    if (m > 0.f && finite) frexpf(m, &e);
    e = e < -100 ? -100 : e > 100 ? 100 : e;
    const float up = ldexpf(1.0f, 20 - e);     // digit scale: |x| * up <= 2^20
    const float sup = ldexpf(1.0f, 10 - e);    // sum scale: |x| * sup < 2^10
    uint32_t dg0 = 0, dg1 = 0, dg2 = 0;
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) {
        const int X = finite ? __float2int_rn(f[k2] * up) : 0;
        const int x2 = ((X + 64) & 127) - 64;
        const int r = (X - x2) >> 7;
        const int x1 = ((r + 64) & 127) - 64;
        const int x0 = (r - x1) >> 7;
        dg0 |= (uint32_t)(x0 & 0xFF) << (8 * k2);
        dg1 |= (uint32_t)(x1 & 0xFF) << (8 * k2);
        dg2 |= (uint32_t)(x2 & 0xFF) << (8 * k2);
    }
    *reinterpret_cast<uint32_t*>(blk + 0 * XP_DIGIT + 4 * t) = dg0;
    *reinterpret_cast<uint32_t*>(blk + 1 * XP_DIGIT + 4 * t) = dg1;
    *reinterpret_cast<uint32_t*>(blk + 2 * XP_DIGIT + 4 * t) = dg2;
    if (t < 8) {
#pragma unroll
        for (int d = 0; d < 3; ++d) *reinterpret_cast<uint32_t*>(blk + d * XP_DIGIT + 256 + 4 * t) = 0u;
    }
    // sum of the 32 values of this thread's sub-block: 8 consecutive threads
    float s = (f[0] * sup + f[1] * sup) + (f[2] * sup + f[3] * sup);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    const float s_next = __shfl_down_sync(0xffffffffu, s, 8);
    uint32_t* rec = reinterpret_cast<uint32_t*>(blk + XP_REC);
    if ((t & 15) == 0) {
        const __half h0 = __float2half_rn(s), h1 = __float2half_rn(s_next);
        const __half l0 = __float2half_rn(s - __half2float(h0)), l1 = __float2half_rn(s_next - __half2float(h1));
        rec[2 * (t >> 4)] = xp_h2_bits(__halves2half2(h0, h1));
        rec[2 * (t >> 4) + 1] = xp_h2_bits(__halves2half2(l0, l1));
    }
    // digit unit (non-finite input makes it NaN, so the products are NaN as the fp32 dot would be), then zero padding
    if (t == 8) rec[8] = __float_as_uint(finite ? ldexpf(1.0f, e - 20) : __int_as_float(0x7fc00000));
    if (t >= 9 && t < (XP_COL - XP_REC) / 4) rec[t] = 0u;
}

}  // namespace k
}  // namespace wl
