// Activation prep of one 256-value superblock for the tensor-core matvecs, shared by every kernel that produces
// activations in that form (k_xprep, and the fused swiglu and attention-combine kernels).
//
// Layout of the XP_COL-byte block: three planes of signed 8-bit digits of the 256 values in natural order (pitch
// XP_DIGIT; 32 zero pad bytes each), then at XP_REC a record of f16 hi/lo sums of the 32-value and the 16-value
// sub-blocks and the float unit of the digits (word map below). X = round(x * 2^(20-e)) (|X| <= 2^20, e
// the exponent of the superblock's largest magnitude) is split into balanced base-128 digits X = X0*2^14 + X1*2^7 +
// X2, each in [-64, 64]. The sums are taken at 2^(10-e), where they fit f16 with a hi/lo split good to 2^-22.
// The 16-value sums serve Q6_K (16-value sub-blocks), the 32-value sums Q4_K.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include "wl_kernels.h"

namespace wl {
namespace k {

__device__ __forceinline__ uint32_t xp_h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Record words (32-bit, from XP_REC): 0..7 the 32-value sums as four (hi pair, lo pair) of sub-block pairs (2c, 2c+1);
// 8 the digit unit; XP_S16..XP_S16+15 the 16-value sums, for lane c four words [hi(2c, 2c+1), hi(2c+8, 2c+9),
// lo(2c, 2c+1), lo(2c+8, 2c+9)] (the B fragments of an m16n8k16 MMA over the 16 sub-blocks); the rest zero.
constexpr int XP_S16 = 12;

// f16 hi/lo split of two sums a, b into rec[hi_word] = (hi a, hi b), rec[lo_word] = (lo a, lo b).
__device__ __forceinline__ void xp_store_pair(uint32_t* rec, int hi_word, int lo_word, float a, float b)
{
    const __half h0 = __float2half_rn(a), h1 = __float2half_rn(b);
    const __half l0 = __float2half_rn(a - __half2float(h0)), l1 = __float2half_rn(b - __half2float(h1));
    rec[hi_word] = xp_h2_bits(__halves2half2(h0, h1));
    rec[lo_word] = xp_h2_bits(__halves2half2(l0, l1));
}

// Called by the 64 threads t = 0..63 of a 64-thread CTA (it synchronises the CTA), or with NAMED by 64 threads of a
// larger CTA (they synchronise on named barrier bar_id alone); thread t holds values 4t..4t+3. scratch: two floats of
// shared memory.
template <bool NAMED = false>
__device__ __forceinline__ void xprep_sb(const float (&f)[4], int t, float* scratch, uint8_t* __restrict__ blk,
                                         int bar_id = 1)
{
    float m = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((t & 31) == 0) scratch[t >> 5] = m;
    if (NAMED) asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
    else __syncthreads();
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
    // sums of the 16 values (4 consecutive threads) and 32 values (8) of this thread's sub-blocks
    float s = (f[0] * sup + f[1] * sup) + (f[2] * sup + f[3] * sup);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    const float s16 = s, s16_next = __shfl_down_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    const float s_next = __shfl_down_sync(0xffffffffu, s, 8);
    uint32_t* rec = reinterpret_cast<uint32_t*>(blk + XP_REC);
    if ((t & 15) == 0) xp_store_pair(rec, 2 * (t >> 4), 2 * (t >> 4) + 1, s, s_next);
    if ((t & 7) == 0) {
        const int p = t >> 3, c = p & 3, upper = p >> 2;
        xp_store_pair(rec, XP_S16 + 4 * c + upper, XP_S16 + 4 * c + 2 + upper, s16, s16_next);
    }
    // digit unit (non-finite input makes it NaN, so the products are NaN as the fp32 dot would be), then zero padding
    if (t == 8) rec[8] = __float_as_uint(finite ? ldexpf(1.0f, e - 20) : __int_as_float(0x7fc00000));
    if (t >= 9 && t < XP_S16) rec[t] = 0u;
    if (t >= XP_S16 + 16 && t < (XP_COL - XP_REC) / 4) rec[t] = 0u;
}

}  // namespace k
}  // namespace wl
