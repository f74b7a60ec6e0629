// Tensor-core decode matvec for the signed block formats Q8_0, IQ4_XS and IQ2_XXS (sm_100a): tile-major weights
// streamed into shared memory with 1-D bulk copies, decoded in registers to signed 8-bit values, integer mma.sync
// (s8 values x s8 activation digits, exact int32) for 1..8 activation columns.
//
// The structure is the Q4_K kernel's (wl_mmv.cu): a CTA owns 16 rows, warp w of its NW warps takes superblocks
// (256-value column groups) w, w + NW, ... of them through its own two-stage ring, each stage holding the 16 rows'
// tile of that superblock and the prepared activations of the same superblock (k_xprep's layout: three planes of
// balanced base-128 digits, so every integer MMA is exact). Lane (g, c) of a 32-value sub-block's MMA holds values
// 8c..8c+7 of rows g and g + 8 (the k order the activation layout is written in). Per format:
//   Q8_0     (src/Quants.cs:86-97)     the codes are the int8 values; each 32-value block's fp16 d is applied in fp32
//                                      to that block's int32 sums, per digit plane;
//   IQ4_XS   (src/IQuants.cs:61-80)    4-bit codes looked up in the IQ4_NL table with byte permutes; the 6-bit
//                                      sub-block scale ls - 32 is applied in integers, d in fp32 per superblock;
//   IQ2_XXS  (src/IQuants.cs:148-170)  each 8-value group is a grid row (8 magnitudes) with 7 sign bits and a parity
//                                      bit, read as two words of a table of every grid half-row under every four
//                                      signs (32 KB, in shared memory); the 4-bit scale s enters as the integer
//                                      2s + 1, d / 8 in fp32, since d * (0.5 + s) * 0.25 = d * (2s + 1) / 8.
// One or two columns pack (column, digit) pairs into the MMA's 8 columns; from three columns on each digit plane is
// its own MMA over the columns. Either way every (column, digit) goes through the same fp32 operations, and the
// planes are added ((0 + 1) + 2) and the warps in warp order, so a column's result does not depend on the other
// columns of the launch.
#include <cstdint>
#include <cstring>
#include <mutex>
#include <atomic>
#include <cuda_fp16.h>
#include "wl_common.h"
#include "wl_kernels.h"
#include "wl_launch.cuh"
#include "wl_mma.cuh"
#include "iq_tables.h"

namespace wl {
namespace k {

// IQ2_XXS grid rows with their signs applied, per half: [grid index][4 sign bits] -> the four signed values of bytes
// 0..3 (lo) or 4..7 (hi) of the grid row, so a lane's decode of an 8-value group is two table reads
__device__ uint32_t g_i8_iq2_lo[256 * 16], g_i8_iq2_hi[256 * 16];

namespace {

constexpr int I8_ROWS = 16;

// Tile layouts (16 rows x one 256-value superblock, 16-byte multiples):
//   Q8_0    [0, 256)     per row r at 16r: the eight blocks' fp16 d
//           [256, 4352)  per 32-value block j at 256 + 512j: lane L's 16 bytes at 16L: the 8 codes of values
//                        8c..8c+7 of row g, then of row g + 8 (L = 4g + c)
//   IQ4_XS  [0, 32)      per row r at 2r: fp16 d
//           [32, 160)    per row r at 32 + 8r: the eight sub-blocks' ls - 32 as int8
//           [160, 2208)  per sub-block pair p at 160 + 512p: lane L's four words at 16L: row g sub-block 2p, row g + 8
//                        sub-block 2p, row g sub-block 2p + 1, row g + 8 sub-block 2p + 1; nibble i of a word is the
//                        code of value 8c + i
//   IQ2_XXS [0, 32)      per row r at 2r: fp16 d
//           [32, 1056)   per sub-block j at 32 + 128j: per row r at 8r: the GGUF aux words (grid indices, then signs
//                        and scale)
template <int T> struct I8Fmt;
template <> struct I8Fmt<8> { static constexpr int TILE = 4352, SB_BYTES = 272; };
template <> struct I8Fmt<23> { static constexpr int TILE = 2208, SB_BYTES = 136; };
template <> struct I8Fmt<16> { static constexpr int TILE = 1056, SB_BYTES = 66; };

template <int T, int NC> struct I8Layout {
    static constexpr int X_OFF = (I8Fmt<T>::TILE + 127) / 128 * 128;
    static constexpr int STAGE = (X_OFF + NC * XP_COL + 127) / 128 * 128;
    static constexpr int TX = I8Fmt<T>::TILE + NC * XP_COL;
    static constexpr int STAGES = 2;
};

__device__ __forceinline__ void imma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%10,%10,%10,%10};\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// The IQ4_NL values of the 4-bit codes of a lane's word (nibble i the code of value i): values 0..3 (lo) or 4..7.
// The table's low half is negative and its high half positive, and a selector nibble with bit 3 set makes prmt
// replicate the sign of the byte it picks: prmt over the low half gives the value for codes < 8 and 0xFF for the rest;
// prmt over the complemented high half with bit 3 flipped gives ~value for codes >= 8 and 0xFF for the rest. Their AND
// is the value, or ~value where the code is >= 8, which an XOR with that byte mask undoes; the mask is one more
// sign-replicating prmt over the word and the word shifted by a nibble (bit 3 of nibble 2b sits at bit 7 of byte b of
// the shifted word, bit 3 of nibble 2b+1 at bit 7 of byte b of the word).
struct Iq4Lut {
    uint32_t lo0, lo1, nhi0, nhi1;
};
template <bool HI>
__device__ __forceinline__ uint32_t iq4_lookup(uint32_t w, uint32_t w4, const Iq4Lut& t)
{
    const uint32_t sel = HI ? w >> 16 : w;
    const uint32_t r1 = prmt(t.lo0, t.lo1, sel);
    const uint32_t r2 = prmt(t.nhi0, t.nhi1, sel ^ 0x8888u);
    const uint32_t m = prmt(w4, w, HI ? 0xFBEAu : 0xD9C8u);
    return (r1 & r2) ^ m;
}

template <int T, int NC, int NW>
__global__ void __launch_bounds__(32 * NW, (NC <= 2 ? 16 : 8) / NW) k_mmv_i8(const uint8_t* __restrict__ wt, int rows,
                                                                           int nsb, const uint8_t* xq, float* y,
                                                                           int64_t ldy, int* err, const Iq4Lut lut)
{
    using LY = I8Layout<T, NC>;
    constexpr int TILE = I8Fmt<T>::TILE;
    constexpr bool PACK = NC <= 2;
    constexpr int ND = PACK ? 1 : 3;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[NW][LY::STAGES];
    __shared__ __align__(16) uint32_t sgn_lo[T == 16 ? 4096 : 4], sgn_hi[T == 16 ? 4096 : 4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int r0 = blockIdx.x * I8_ROWS;
    uint8_t* ring = smem + warp * LY::STAGES * LY::STAGE;
    const int njobs = nsb > warp ? (nsb - warp + NW - 1) / NW : 0;

    pdl_trigger();
    if (T == 16)
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
            reinterpret_cast<uint4*>(sgn_lo)[i] = reinterpret_cast<const uint4*>(g_i8_iq2_lo)[i];
            reinterpret_cast<uint4*>(sgn_hi)[i] = reinterpret_cast<const uint4*>(g_i8_iq2_hi)[i];
        }
    if (lane == 0) {
        for (int s = 0; s < LY::STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    __syncwarp();
    auto issue_w = [&](int j, int s) {      // weights: written by no kernel, so they may stream before pdl_wait()
        mbar_expect_tx(&bars[warp][s], LY::TX);
        bulk_load(ring + s * LY::STAGE, wt + ((int64_t)blockIdx.x * nsb + warp + NW * j) * TILE, TILE, &bars[warp][s]);
    };
    auto issue_x = [&](int j, int s) {
        const int sb = warp + NW * j;
        uint8_t* st = ring + s * LY::STAGE;
#pragma unroll
        for (int n = 0; n < NC; ++n)
            bulk_load(st + LY::X_OFF + n * XP_COL, xq + ((int64_t)n * nsb + sb) * XP_COL, XP_COL, &bars[warp][s]);
    };
    if (lane == 0)
        for (int j = 0; j < LY::STAGES && j < njobs; ++j) issue_w(j, j);
    pdl_wait();
    if (lane == 0)
        for (int j = 0; j < LY::STAGES && j < njobs; ++j) issue_x(j, j);
    if (T == 16) __syncthreads();           // the signed grid tables are in place

    const bool b_ok = PACK ? g < 3 * NC : g < NC;
    const int b_off = LY::X_OFF + (PACK ? (g / 3) * XP_COL + (g % 3) * XP_DIGIT : g * XP_COL);
    int e_col[2], e_dig[2];
    bool e_ok[2];
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
        const int nn = 2 * c + k2;
        e_col[k2] = PACK ? nn / 3 : nn;
        e_dig[k2] = PACK ? nn % 3 : 0;
        e_ok[k2] = PACK ? nn < 3 * NC : nn < NC;
    }

    float facc[ND][4] = {};
    for (int j = 0; j < njobs; ++j) {
        const int s = j % LY::STAGES;
        const bool ok = mbar_wait_bounded(&bars[warp][s], (uint32_t)((j / LY::STAGES) & 1), err, 1);
        const uint8_t* st = ring + s * LY::STAGE;
        if (ok) {
            // (column, digit) factors of this lane's accumulator columns: the superblock's digit unit x 2^(14 - 7d)
            float f[ND][2];
#pragma unroll
            for (int k2 = 0; k2 < 2; ++k2) {
                const float unit = e_ok[k2] ? *reinterpret_cast<const float*>(st + LY::X_OFF + e_col[k2] * XP_COL + XP_REC + 32) : 0.f;
#pragma unroll
                for (int d = 0; d < ND; ++d) {
                    const int dig = PACK ? e_dig[k2] : d;
                    f[d][k2] = unit * (dig == 0 ? 16384.f : dig == 1 ? 128.f : 1.f);
                }
            }
            if (T == 8) {
#pragma unroll
                for (int jb = 0; jb < 8; ++jb) {
                    const uint4 v = lds128(st + 256 + jb * 512 + lane * 16);
                    const float dg = h2f_(*reinterpret_cast<const uint16_t*>(st + g * 16 + 2 * jb));
                    const float dg8 = h2f_(*reinterpret_cast<const uint16_t*>(st + (g + 8) * 16 + 2 * jb));
#pragma unroll
                    for (int d = 0; d < ND; ++d) {
                        const uint2 b = b_ok ? lds64(st + b_off + d * XP_DIGIT + 32 * jb + 8 * c) : make_uint2(0u, 0u);
                        int D[4];
                        imma_s8(D, v.x, v.z, v.y, v.w, b.x, b.y);
#pragma unroll
                        for (int k2 = 0; k2 < 2; ++k2) {
                            facc[d][k2] = fmaf((float)D[k2], dg * f[d][k2], facc[d][k2]);
                            facc[d][k2 + 2] = fmaf((float)D[k2 + 2], dg8 * f[d][k2], facc[d][k2 + 2]);
                        }
                    }
                }
            } else {
                int acc[ND][4] = {};
                float dg, dg8;
                if (T == 23) {
                    dg = h2f_(*reinterpret_cast<const uint16_t*>(st + 2 * g));
                    dg8 = h2f_(*reinterpret_cast<const uint16_t*>(st + 2 * (g + 8)));
                    const uint2 ha = lds64(st + 32 + 8 * g), hb = lds64(st + 32 + 8 * (g + 8));   // ls - 32, int8
                    const uint32_t sa0 = ha.x, sa1 = ha.y, sb0 = hb.x, sb1 = hb.y;
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const uint4 v = lds128(st + 160 + p * 512 + lane * 16);
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {
                            const int jb = 2 * p + hh;
                            const uint32_t wg = hh ? v.z : v.x, wg8 = hh ? v.w : v.y;
                            const uint32_t wg4 = wg << 4, wg84 = wg8 << 4;
                            const uint32_t a0 = iq4_lookup<false>(wg, wg4, lut), a2 = iq4_lookup<true>(wg, wg4, lut);
                            const uint32_t a1 = iq4_lookup<false>(wg8, wg84, lut), a3 = iq4_lookup<true>(wg8, wg84, lut);
                            const int sg = (int)(int8_t)(((jb < 4 ? sa0 : sa1) >> (8 * (jb & 3))) & 0xFF);
                            const int sg8 = (int)(int8_t)(((jb < 4 ? sb0 : sb1) >> (8 * (jb & 3))) & 0xFF);
#pragma unroll
                            for (int d = 0; d < ND; ++d) {
                                const uint2 b = b_ok ? lds64(st + b_off + d * XP_DIGIT + 32 * jb + 8 * c) : make_uint2(0u, 0u);
                                int D[4];
                                imma_s8(D, a0, a1, a2, a3, b.x, b.y);
                                acc[d][0] += sg * D[0];
                                acc[d][1] += sg * D[1];
                                acc[d][2] += sg8 * D[2];
                                acc[d][3] += sg8 * D[3];
                            }
                        }
                    }
                } else {    // IQ2_XXS
                    dg = h2f_(*reinterpret_cast<const uint16_t*>(st + 2 * g)) * 0.125f;
                    dg8 = h2f_(*reinterpret_cast<const uint16_t*>(st + 2 * (g + 8))) * 0.125f;
#pragma unroll
                    for (int jb = 0; jb < 8; ++jb) {
                        const uint2 q0 = lds64(st + 32 + jb * 128 + g * 8), q1 = lds64(st + 32 + jb * 128 + (g + 8) * 8);
                        uint32_t a[2][2];
                        int sc[2];
#pragma unroll
                        for (int rr = 0; rr < 2; ++rr) {
                            const uint2 q = rr ? q1 : q0;
                            const uint32_t gi = ((q.x >> (8 * c)) & 0xFFu) << 4;
                            const uint32_t s7 = (q.y >> (7 * c)) & 127u;
                            const uint32_t sg = s7 | ((__popc(s7) & 1u) << 7);    // the eighth bit: even parity
                            a[rr][0] = sgn_lo[gi | (sg & 0xFu)];
                            a[rr][1] = sgn_hi[gi | (sg >> 4)];
                            sc[rr] = 2 * (int)(q.y >> 28) + 1;
                        }
#pragma unroll
                        for (int d = 0; d < ND; ++d) {
                            const uint2 b = b_ok ? lds64(st + b_off + d * XP_DIGIT + 32 * jb + 8 * c) : make_uint2(0u, 0u);
                            int D[4];
                            imma_s8(D, a[0][0], a[1][0], a[0][1], a[1][1], b.x, b.y);
                            acc[d][0] += sc[0] * D[0];
                            acc[d][1] += sc[0] * D[1];
                            acc[d][2] += sc[1] * D[2];
                            acc[d][3] += sc[1] * D[3];
                        }
                    }
                }
#pragma unroll
                for (int d = 0; d < ND; ++d)
#pragma unroll
                    for (int k2 = 0; k2 < 2; ++k2) {
                        facc[d][k2] = fmaf((float)acc[d][k2], dg * f[d][k2], facc[d][k2]);
                        facc[d][k2 + 2] = fmaf((float)acc[d][k2 + 2], dg8 * f[d][k2], facc[d][k2 + 2]);
                    }
            }
        }
        __syncwarp();
        if (lane == 0 && j + LY::STAGES < njobs) {
            fence_proxy_async();        // the stage's generic reads are done before the copy engine rewrites it
            issue_w(j + LY::STAGES, s);
            issue_x(j + LY::STAGES, s);
        }
    }
    // per (row, column): (plane 0 + plane 1) + plane 2, then the warps in order, through each warp's own ring
    float* red = reinterpret_cast<float*>(ring);        // [I8_ROWS][9]
    if (PACK) {
#pragma unroll
        for (int e = 0; e < 4; ++e) red[(g + 8 * (e >> 1)) * 9 + 2 * c + (e & 1)] = facc[0][e];
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = g + 8 * (e >> 1), col = 2 * c + (e & 1);
            if (col < NC) red[row * 9 + col] = (facc[0][e] + facc[ND > 1 ? 1 : 0][e]) + facc[ND > 2 ? 2 : 0][e];
        }
    }
    __syncthreads();
    const int rl = threadIdx.x >> 3, col = threadIdx.x & 7;     // NW >= 4: every (row, column) has a thread
    if (col < NC && rl < I8_ROWS && r0 + rl < rows) {
        float sum = 0.f;
#pragma unroll
        for (int wv = 0; wv < NW; ++wv) {
            const float* rw = reinterpret_cast<const float*>(smem + wv * LY::STAGES * LY::STAGE) + rl * 9;
            sum += PACK ? (rw[3 * col] + rw[3 * col + 1]) + rw[3 * col + 2] : rw[col];
        }
        y[(int64_t)col * ldy + r0 + rl] = sum;
    }
}

// ---- repack of GGUF rows into the tiles above (once per matrix) ----
template <int T>
__global__ void k_i8_tile(const uint8_t* src, int rows, int nsb, int64_t row_bytes, uint8_t* dst)
{
    pdl_trigger();
    pdl_wait();
    constexpr int TILE = I8Fmt<T>::TILE, SBB = I8Fmt<T>::SB_BYTES;
    const int sb = blockIdx.x, rt = blockIdx.y;
    uint8_t* out = dst + ((int64_t)rt * nsb + sb) * TILE;
    for (int i = threadIdx.x; i < TILE; i += blockDim.x) {
        int r = 0;
        uint8_t v = 0;
        auto at = [&](int row, int off) -> uint8_t {
            const int gr = rt * I8_ROWS + row;
            return gr < rows ? src[(int64_t)gr * row_bytes + (int64_t)sb * SBB + off] : (uint8_t)0;
        };
        if (T == 8) {
            if (i < 256) {
                r = i >> 4;
                const int o = i & 15;
                v = at(r, (o >> 1) * 34 + (o & 1));
            } else {
                const int j = i - 256, blk = j >> 9, L = (j & 511) >> 4, b = j & 15;
                const int gg = L >> 2, cc = L & 3;
                r = b < 8 ? gg : gg + 8;
                v = at(r, blk * 34 + 2 + 8 * cc + (b & 7));
            }
        } else if (T == 23) {
            if (i < 32) {
                v = at(i >> 1, i & 1);
            } else if (i < 160) {
                r = (i - 32) >> 3;
                const int ib = (i - 32) & 7;
                const int sh = at(r, 2) | (at(r, 3) << 8), sl = at(r, 4 + ib / 2);
                const int ls = ((sl >> (4 * (ib & 1))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
                v = (uint8_t)(int8_t)(ls - 32);
            } else {
                const int j = i - 160, p = j >> 9, L = (j & 511) >> 4, b = j & 15;
                const int gg = L >> 2, cc = L & 3, wd = b >> 2, bb = b & 3;
                r = (wd & 1) ? gg + 8 : gg;
                const int ib = 2 * p + (wd >> 1);
                uint8_t nib[2];
                for (int h = 0; h < 2; ++h) {
                    const int val = 8 * cc + 2 * bb + h;    // value index within the 32-value sub-block
                    const uint8_t q = at(r, 8 + 16 * ib + (val & 15));
                    nib[h] = val < 16 ? (q & 0xF) : (q >> 4);
                }
                v = (uint8_t)(nib[0] | (nib[1] << 4));
            }
        } else {
            if (i < 32) {
                v = at(i >> 1, i & 1);
            } else {
                const int j = i - 32, ib = j >> 7;
                r = (j & 127) >> 3;
                v = at(r, 2 + 8 * ib + (j & 7));
            }
        }
        out[i] = v;
    }
}

template <int T, int NC, int NW> struct I8Attr {
    static std::atomic<bool> done[64];
};
template <int T, int NC, int NW> std::atomic<bool> I8Attr<T, NC, NW>::done[64];

template <int T, int NC, int NW>
void launch_i8(const uint8_t* tiles, int rows, int nsb, const XPrep& p, float* y, int64_t ldy, int* err, cudaStream_t s,
               const Iq4Lut& lut)
{
    constexpr int SMEM = NW * I8Layout<T, NC>::STAGES * I8Layout<T, NC>::STAGE;
    static std::mutex mu;
    int dev = 0;
    WL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) WL_THROW(WL_EINVAL, "device ordinal out of range");
    if (!I8Attr<T, NC, NW>::done[dev].load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lock(mu);
        if (!I8Attr<T, NC, NW>::done[dev].load(std::memory_order_relaxed)) {
            WL_CUDA(cudaFuncSetAttribute(k_mmv_i8<T, NC, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
            I8Attr<T, NC, NW>::done[dev].store(true, std::memory_order_release);
        }
    }
    launch(k_mmv_i8<T, NC, NW>, dim3((rows + I8_ROWS - 1) / I8_ROWS), dim3(32 * NW), SMEM, s, tiles, rows, nsb,
           (const uint8_t*)p.blocks, y, ldy, err, lut);
    note_launch();
}

template <int T, int NW>
void dispatch_i8_nc(const uint8_t* tiles, int rows, int nsb, const XPrep& p, float* y, int64_t ldy, int* err,
                    cudaStream_t s, const Iq4Lut& lut)
{
    switch (p.nc) {
    case 1: launch_i8<T, 1, NW>(tiles, rows, nsb, p, y, ldy, err, s, lut); break;
    case 2: launch_i8<T, 2, NW>(tiles, rows, nsb, p, y, ldy, err, s, lut); break;
    case 3: launch_i8<T, 3, NW>(tiles, rows, nsb, p, y, ldy, err, s, lut); break;
    case 4: launch_i8<T, 4, NW>(tiles, rows, nsb, p, y, ldy, err, s, lut); break;
    case 5: launch_i8<T, 5, NW>(tiles, rows, nsb, p, y, ldy, err, s, lut); break;
    case 6: launch_i8<T, 6, NW>(tiles, rows, nsb, p, y, ldy, err, s, lut); break;
    case 7: launch_i8<T, 7, NW>(tiles, rows, nsb, p, y, ldy, err, s, lut); break;
    default: launch_i8<T, 8, NW>(tiles, rows, nsb, p, y, ldy, err, s, lut); break;
    }
}

int sm_count_i8()
{
    static std::atomic<int> n{0};
    int v = n.load(std::memory_order_relaxed);
    if (!v) {
        int dev = 0;
        v = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        n.store(v, std::memory_order_relaxed);
    }
    return v;
}

// The IQ4_NL table as the permute tables iq4_lookup reads: the low half as is, the high half complemented.
Iq4Lut make_lut()
{
    Iq4Lut t;
    uint8_t b[16];
    for (int i = 0; i < 16; ++i) b[i] = (uint8_t)(i < 8 ? WL_KVALUES_IQ4NL[i] : ~WL_KVALUES_IQ4NL[i]);
    memcpy(&t.lo0, b, 4);
    memcpy(&t.lo1, b + 4, 4);
    memcpy(&t.nhi0, b + 8, 4);
    memcpy(&t.nhi1, b + 12, 4);
    return t;
}

}  // namespace

bool i8_tiles_supported(int type, int cols) { return (type == 8 || type == 23 || type == 16) && cols % 256 == 0; }

int64_t i8_tile_bytes(int type, int rows, int cols)
{
    const int tile = type == 8 ? I8Fmt<8>::TILE : type == 23 ? I8Fmt<23>::TILE : I8Fmt<16>::TILE;
    return (int64_t)((rows + I8_ROWS - 1) / I8_ROWS) * (cols / 256) * tile;
}

void init_i8_tables()
{
    // the IQ2_XXS grid rows with every combination of four signs applied, per half of the row
    static uint32_t lo[256 * 16], hi[256 * 16];
    for (int gi = 0; gi < 256; ++gi)
        for (int sg = 0; sg < 16; ++sg) {
            uint32_t l = 0, h = 0;
            for (int b = 0; b < 4; ++b) {
                const int ml = (int)((WL_IQ2XXS_GRID[gi] >> (8 * b)) & 0xFF), mh = (int)((WL_IQ2XXS_GRID[gi] >> (8 * (b + 4))) & 0xFF);
                l |= (uint32_t)(uint8_t)(int8_t)((sg >> b) & 1 ? -ml : ml) << (8 * b);
                h |= (uint32_t)(uint8_t)(int8_t)((sg >> b) & 1 ? -mh : mh) << (8 * b);
            }
            lo[gi * 16 + sg] = l;
            hi[gi * 16 + sg] = h;
        }
    WL_CUDA(cudaMemcpyToSymbol(g_i8_iq2_lo, lo, sizeof lo));
    WL_CUDA(cudaMemcpyToSymbol(g_i8_iq2_hi, hi, sizeof hi));
}

void make_i8_tiles(int type, const uint8_t* w, int rows, int cols, int64_t row_bytes, uint8_t* tiles, cudaStream_t s)
{
    if (!i8_tiles_supported(type, cols)) WL_THROW(WL_EUNSUPPORTED, "make_tiles: no tile layout for this type");
    const int sbb = type == 8 ? I8Fmt<8>::SB_BYTES : type == 23 ? I8Fmt<23>::SB_BYTES : I8Fmt<16>::SB_BYTES;
    if (row_bytes < (int64_t)(cols / 256) * sbb) WL_THROW(WL_EINVAL, "make_tiles: bad row size");
    if (rows <= 0) return;
    const dim3 grid(cols / 256, (rows + I8_ROWS - 1) / I8_ROWS);
    if (type == 8) launch(k_i8_tile<8>, grid, dim3(256), 0, s, w, rows, cols / 256, row_bytes, tiles);
    else if (type == 23) launch(k_i8_tile<23>, grid, dim3(256), 0, s, w, rows, cols / 256, row_bytes, tiles);
    else launch(k_i8_tile<16>, grid, dim3(256), 0, s, w, rows, cols / 256, row_bytes, tiles);
    note_launch();
}

// Eight warps per CTA up to 8 x SMs row tiles, four beyond (a choice that depends on the matrix alone, so a column's
// result never depends on the column count).
void matvec_i8_tiles(int type, const uint8_t* tiles, int rows, int cols, const XPrep& p, float* y, int64_t ldy, int* err,
                     cudaStream_t s)
{
    if (!i8_tiles_supported(type, cols) || p.cols != cols || p.nc < 1 || p.nc > 8)
        WL_THROW(WL_EINVAL, "matvec_tiles: activations do not match the tiles");
    if (rows <= 0) return;
    static const Iq4Lut lut = make_lut();
    const int nsb = cols / 256;
    const bool four = (rows + I8_ROWS - 1) / I8_ROWS >= 8 * sm_count_i8();
    if (type == 8) {
        if (four) dispatch_i8_nc<8, 4>(tiles, rows, nsb, p, y, ldy, err, s, lut);
        else dispatch_i8_nc<8, 8>(tiles, rows, nsb, p, y, ldy, err, s, lut);
    } else if (type == 23) {
        if (four) dispatch_i8_nc<23, 4>(tiles, rows, nsb, p, y, ldy, err, s, lut);
        else dispatch_i8_nc<23, 8>(tiles, rows, nsb, p, y, ldy, err, s, lut);
    } else {
        if (four) dispatch_i8_nc<16, 4>(tiles, rows, nsb, p, y, ldy, err, s, lut);
        else dispatch_i8_nc<16, 8>(tiles, rows, nsb, p, y, ldy, err, s, lut);
    }
}

}  // namespace k
}  // namespace wl
