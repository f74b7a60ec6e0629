// Device kernels of libwindlass_cuda (sm_100a). All device code of the library lives in this one translation unit.
//
// Decode matvec (the dominant cost of a decode step) is memory-bound: one warp owns one weight row, lanes stride
// over the row's units (64 values for Q4_K, 32 for the other formats) with 128-bit loads where the block layout
// allows, decode in registers and accumulate every activation column in fp32; the warp sums lanes with a fixed
// xor butterfly, so a column's result never depends on how many columns ran beside it (ForwardBatch rows are
// bit-identical to single runs, src/Transformer.cs:127-131).
#include <cstdint>
#include <cstdio>
#include <atomic>
#include <mutex>
#include <cuda_fp16.h>
#include "wl_common.h"
#include "wl_decode.cuh"
#include <algorithm>
#include "wl_kernels.h"
#include "wl_launch.cuh"
#include "wl_xprep.cuh"

namespace wl {

__device__ uint64_t g_iq2xxs_grid[256];
__device__ uint8_t g_ksigns[128];
__device__ int8_t g_kvalues[16];

namespace k {

// ------------------------------------------------------------------------------------------------------------------
// tables
// ------------------------------------------------------------------------------------------------------------------
void init_tables()
{
    static std::mutex mu;
    static uint64_t done = 0;   // bit per device ordinal
    int dev = 0;
    WL_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && (done >> dev) & 1) return;
    WL_CUDA(cudaMemcpyToSymbol(c_iq2xxs_grid, WL_IQ2XXS_GRID, sizeof(WL_IQ2XXS_GRID)));
    WL_CUDA(cudaMemcpyToSymbol(c_iq2xs_grid, WL_IQ2XS_GRID, sizeof(WL_IQ2XS_GRID)));
    WL_CUDA(cudaMemcpyToSymbol(c_iq2s_grid, WL_IQ2S_GRID, sizeof(WL_IQ2S_GRID)));
    WL_CUDA(cudaMemcpyToSymbol(c_iq1s_grid, WL_IQ1S_GRID, sizeof(WL_IQ1S_GRID)));
    WL_CUDA(cudaMemcpyToSymbol(c_iq3xxs_grid, WL_IQ3XXS_GRID, sizeof(WL_IQ3XXS_GRID)));
    WL_CUDA(cudaMemcpyToSymbol(c_iq3s_grid, WL_IQ3S_GRID, sizeof(WL_IQ3S_GRID)));
    WL_CUDA(cudaMemcpyToSymbol(c_ksigns, WL_KSIGNS_IQ2XS, sizeof(WL_KSIGNS_IQ2XS)));
    WL_CUDA(cudaMemcpyToSymbol(c_kvalues_iq4nl, WL_KVALUES_IQ4NL, sizeof(WL_KVALUES_IQ4NL)));
    WL_CUDA(cudaMemcpyToSymbol(g_iq2xxs_grid, WL_IQ2XXS_GRID, sizeof(WL_IQ2XXS_GRID)));
    WL_CUDA(cudaMemcpyToSymbol(g_ksigns, WL_KSIGNS_IQ2XS, sizeof(WL_KSIGNS_IQ2XS)));
    WL_CUDA(cudaMemcpyToSymbol(g_kvalues, WL_KVALUES_IQ4NL, sizeof(WL_KVALUES_IQ4NL)));
    init_i8_tables();
    if (dev < 64) done |= 1ull << dev;
}

static inline unsigned grid_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

static std::atomic<int64_t> g_launches{0};

// Checks the launch just made and counts it.
static inline void launched()
{
    WL_CUDA(cudaGetLastError());
    g_launches.fetch_add(1, std::memory_order_relaxed);
}

int64_t launches() { return g_launches.load(std::memory_order_relaxed); }

void note_launch() { launched(); }
void uncount_launches(int64_t n) { g_launches.fetch_sub(n, std::memory_order_relaxed); }

// ------------------------------------------------------------------------------------------------------------------
// dequant / embedding (bit-exact)
// ------------------------------------------------------------------------------------------------------------------
__global__ void k_dequant(int type, const uint8_t* blocks, int64_t n, float* out)
{
    pdl_trigger();
    pdl_wait();
    const int be = block_elems(type), bb = block_bytes(type);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = dq_elem(type, blocks + (i / be) * bb, (int)(i % be));
}

void dequant(int type, const void* blocks, int64_t n, float* out, cudaStream_t s)
{
    if (n <= 0) return;
    int64_t g = grid_for(n, 256);
    if (g > 148 * 64) g = 148 * 64;
    launch(k_dequant, dim3((unsigned)g), dim3(256), 0, s, type, (const uint8_t*)blocks, n, out);
    launched();
}

__global__ void k_embed(int type, const uint8_t* __restrict__ w, int64_t row_bytes, int rows, int cols,
                        const int32_t* tokens, float scale, float* x, int32_t* bad,
                        unsigned long long* epoch)
{
    pdl_trigger();
    pdl_wait();
    // a new step: the fused all-reduces of this step take sequence numbers from the next epoch (every later kernel
    // of the step reads it after its own wait, so after this kernel has completed)
    if (epoch && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *epoch += 1;
    const int t = blockIdx.y;
    const int be = block_elems(type), bb = block_bytes(type);
    const int tok = tokens[t];
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x) {
        float v = 0.0f;
        if (tok < 0 || tok >= rows) { if (c == 0) *bad = 1; }
        else {
            v = dq_elem(type, w + (int64_t)tok * row_bytes + (int64_t)(c / be) * bb, c % be);
            if (scale != 0.0f) v = __fmul_rn(v, scale);
        }
        x[(int64_t)t * cols + c] = v;
    }
}

void embed(int type, const uint8_t* w, int64_t row_bytes, int rows, int cols, const int32_t* tokens, int T,
           float scale, float* x, int32_t* bad, cudaStream_t s, unsigned long long* epoch)
{
    dim3 grid(grid_for(cols, 256), T);
    launch(k_embed, dim3(grid), dim3(256), 0, s, type, w, row_bytes, rows, cols, tokens, scale, x, bad, epoch);
    launched();
}

// ------------------------------------------------------------------------------------------------------------------
// decode matvec
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float4 ld4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Maximum over the block (any multiple of 32 threads); every thread gets the result.
__device__ __forceinline__ float block_max_f(float v, float* scratch)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float m = scratch[0];
    for (int i = 1; i < nw; ++i) m = fmaxf(m, scratch[i]);
    return m;
}

// Q4_K: a unit is one 64-value pair of sub-blocks (32 bytes of nibbles: low nibbles = values 0..31, high = 32..63).
// Per column: d*(s1*sum(q_lo*x) + s2*sum(q_hi*x)) - dmin*(m1*sum(x_lo) + m2*sum(x_hi)), the factoring of
// Quants.DotRow Q4_K (src/Quants.cs:110-133).
template <int NC>
__device__ __forceinline__ void unit_q4k(const uint8_t* __restrict__ row, int u, const float* __restrict__ x,
                                         int64_t ldx, float (&acc)[NC])
{
    const int sb = u >> 2, p = u & 3;
    const uint8_t* blk = row + (int64_t)sb * 144;
    const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(blk));
    const uint4 qa = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * p));
    const uint4 qb = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 32 * p));
    const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
    uint8_t sc[12];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sc[i] = (uint8_t)(hdr.y >> (8 * i)); sc[4 + i] = (uint8_t)(hdr.z >> (8 * i)); sc[8 + i] = (uint8_t)(hdr.w >> (8 * i));
    }
    int s1, m1, s2, m2;
    scale_min_k4(2 * p, sc, s1, m1);
    scale_min_k4(2 * p + 1, sc, s2, m2);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const float* xb = x + (int64_t)sb * 256 + 64 * p;
#pragma unroll
    for (int t = 0; t < NC; ++t) {
        const float* xt = xb + t * ldx;
        float a1 = 0.f, a2 = 0.f, x1 = 0.f, x2 = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const float4 lo = ld4(xt + 4 * w), hi = ld4(xt + 32 + 4 * w);
            const uint32_t qq = q[w];
            a1 += (float)(qq & 0xF) * lo.x + (float)((qq >> 8) & 0xF) * lo.y + (float)((qq >> 16) & 0xF) * lo.z + (float)((qq >> 24) & 0xF) * lo.w;
            a2 += (float)((qq >> 4) & 0xF) * hi.x + (float)((qq >> 12) & 0xF) * hi.y + (float)((qq >> 20) & 0xF) * hi.z + (float)(qq >> 28) * hi.w;
            x1 += (lo.x + lo.y) + (lo.z + lo.w);
            x2 += (hi.x + hi.y) + (hi.z + hi.w);
        }
        acc[t] += d * ((float)s1 * a1 + (float)s2 * a2) - dmin * ((float)m1 * x1 + (float)m2 * x2);
    }
}

// Q6_K: a unit is 32 values of one 128-value half: l in [8g, 8g+8) at offsets l, l+32, l+64, l+96
// (Quants.DotRow Q6_K, src/Quants.cs:159-184). Superblocks are 210 bytes, so loads are 16-bit.
template <int NC>
__device__ __forceinline__ void unit_q6k(const uint8_t* __restrict__ row, int u, const float* __restrict__ x,
                                         int64_t ldx, float (&acc)[NC])
{
    const int sb = u >> 3, sub = u & 7, kh = sub >> 2, g = sub & 3;
    const uint8_t* blk = row + (int64_t)sb * 210;
    const uint16_t* qlo = reinterpret_cast<const uint16_t*>(blk + 64 * kh + 8 * g);
    const uint16_t* qhi = reinterpret_cast<const uint16_t*>(blk + 64 * kh + 32 + 8 * g);
    const uint16_t* qhp = reinterpret_cast<const uint16_t*>(blk + 128 + 32 * kh + 8 * g);
    uint8_t lo[8], hi[8], hb[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint16_t a = __ldg(qlo + i), b = __ldg(qhi + i), c = __ldg(qhp + i);
        lo[2 * i] = (uint8_t)a; lo[2 * i + 1] = (uint8_t)(a >> 8);
        hi[2 * i] = (uint8_t)b; hi[2 * i + 1] = (uint8_t)(b >> 8);
        hb[2 * i] = (uint8_t)c; hb[2 * i + 1] = (uint8_t)(c >> 8);
    }
    const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * kh) + (g >> 1);
    const float sc0 = (float)__ldg(sc), sc2 = (float)__ldg(sc + 2), sc4 = (float)__ldg(sc + 4), sc6 = (float)__ldg(sc + 6);
    const float d = h2f(__ldg(reinterpret_cast<const uint16_t*>(blk + 208)));
    float q1[8], q2[8], q3[8], q4[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        q1[i] = (float)(((lo[i] & 0xF) | ((hb[i] & 3) << 4)) - 32);
        q2[i] = (float)(((hi[i] & 0xF) | (((hb[i] >> 2) & 3) << 4)) - 32);
        q3[i] = (float)(((lo[i] >> 4) | (((hb[i] >> 4) & 3) << 4)) - 32);
        q4[i] = (float)(((hi[i] >> 4) | (((hb[i] >> 6) & 3) << 4)) - 32);
    }
    const float* xb = x + (int64_t)sb * 256 + 128 * kh + 8 * g;
#pragma unroll
    for (int t = 0; t < NC; ++t) {
        const float* xt = xb + t * ldx;
        float a1 = 0.f, a2 = 0.f, a3 = 0.f, a4 = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float4 x1 = ld4(xt + 4 * h), x2 = ld4(xt + 32 + 4 * h), x3 = ld4(xt + 64 + 4 * h), x4 = ld4(xt + 96 + 4 * h);
            a1 += q1[4 * h] * x1.x + q1[4 * h + 1] * x1.y + q1[4 * h + 2] * x1.z + q1[4 * h + 3] * x1.w;
            a2 += q2[4 * h] * x2.x + q2[4 * h + 1] * x2.y + q2[4 * h + 2] * x2.z + q2[4 * h + 3] * x2.w;
            a3 += q3[4 * h] * x3.x + q3[4 * h + 1] * x3.y + q3[4 * h + 2] * x3.z + q3[4 * h + 3] * x3.w;
            a4 += q4[4 * h] * x4.x + q4[4 * h + 1] * x4.y + q4[4 * h + 2] * x4.z + q4[4 * h + 3] * x4.w;
        }
        acc[t] += d * ((sc0 * a1 + sc2 * a2) + (sc4 * a3 + sc6 * a4));
    }
}

// Q8_0: a unit is one 34-byte block of 32 int8 values with an fp16 scale (src/Quants.cs:86-97).
template <int NC>
__device__ __forceinline__ void unit_q8_0(const uint8_t* __restrict__ row, int u, const float* __restrict__ x,
                                          int64_t ldx, float (&acc)[NC])
{
    const uint8_t* blk = row + (int64_t)u * 34;
    const uint16_t* p = reinterpret_cast<const uint16_t*>(blk);
    const float d = h2f(__ldg(p));
    float q[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const uint16_t v = __ldg(p + 1 + i);
        q[2 * i] = (float)(int8_t)(v & 0xFF);
        q[2 * i + 1] = (float)(int8_t)(v >> 8);
    }
    const float* xb = x + (int64_t)u * 32;
#pragma unroll
    for (int t = 0; t < NC; ++t) {
        const float* xt = xb + t * ldx;
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const float4 v = ld4(xt + 4 * w);
            a += q[4 * w] * v.x + q[4 * w + 1] * v.y + q[4 * w + 2] * v.z + q[4 * w + 3] * v.w;
        }
        acc[t] += d * a;
    }
}

// IQ4_XS: a unit is one 32-value sub-block: dl = d*(ls-32), y = dl*kvalues[nibble] (src/IQuants.cs:61-80).
template <int NC>
__device__ __forceinline__ void unit_iq4xs(const uint8_t* __restrict__ row, int u, const float* __restrict__ x,
                                           int64_t ldx, float (&acc)[NC])
{
    const int sb = u >> 3, ib = u & 7;
    const uint8_t* blk = row + (int64_t)sb * 136;
    const uint16_t* hp = reinterpret_cast<const uint16_t*>(blk);
    const float d = h2f(__ldg(hp));
    const int sh = __ldg(hp + 1);
    const int sl = __ldg(blk + 4 + ib / 2);
    const int ls = ((sl >> (4 * (ib & 1))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
    const float dl = d * (float)(ls - 32);
    const uint2 qa = __ldg(reinterpret_cast<const uint2*>(blk + 8 + 16 * ib));
    const uint2 qb = __ldg(reinterpret_cast<const uint2*>(blk + 16 + 16 * ib));
    const uint32_t qw[4] = {qa.x, qa.y, qb.x, qb.y};
    float vlo[16], vhi[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int byte = (qw[i >> 2] >> (8 * (i & 3))) & 0xFF;
        vlo[i] = (float)g_kvalues[byte & 0xF];
        vhi[i] = (float)g_kvalues[byte >> 4];
    }
    const float* xb = x + (int64_t)sb * 256 + 32 * ib;
#pragma unroll
    for (int t = 0; t < NC; ++t) {
        const float* xt = xb + t * ldx;
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float4 l = ld4(xt + 4 * w), h = ld4(xt + 16 + 4 * w);
            a += vlo[4 * w] * l.x + vlo[4 * w + 1] * l.y + vlo[4 * w + 2] * l.z + vlo[4 * w + 3] * l.w;
            a += vhi[4 * w] * h.x + vhi[4 * w + 1] * h.y + vhi[4 * w + 2] * h.z + vhi[4 * w + 3] * h.w;
        }
        acc[t] += dl * a;
    }
}

// IQ2_XXS: a unit is one 32-value sub-block: four grid indices (aux0), four 7-bit sign indices and a 4-bit scale
// (aux1); db = d*(0.5+(aux1>>28))*0.25 (src/IQuants.cs:148-170).
template <int NC>
__device__ __forceinline__ void unit_iq2xxs(const uint8_t* __restrict__ row, int u, const float* __restrict__ x,
                                            int64_t ldx, float (&acc)[NC])
{
    const int sb = u >> 3, ib = u & 7;
    const uint8_t* blk = row + (int64_t)sb * 66;
    const uint16_t* p = reinterpret_cast<const uint16_t*>(blk);
    const float d = h2f(__ldg(p));
    const uint32_t aux0 = (uint32_t)__ldg(p + 1 + 4 * ib) | ((uint32_t)__ldg(p + 2 + 4 * ib) << 16);
    const uint32_t aux1 = (uint32_t)__ldg(p + 3 + 4 * ib) | ((uint32_t)__ldg(p + 4 + 4 * ib) << 16);
    const float db = d * (0.5f + (float)(aux1 >> 28)) * 0.25f;
    float v[32];
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint64_t g = g_iq2xxs_grid[(aux0 >> (8 * l)) & 0xFF];
        const int signs = g_ksigns[(aux1 >> (7 * l)) & 127];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float m = (float)((g >> (8 * j)) & 0xFF);
            v[8 * l + j] = (signs >> j) & 1 ? -m : m;
        }
    }
    const float* xb = x + (int64_t)sb * 256 + 32 * ib;
#pragma unroll
    for (int t = 0; t < NC; ++t) {
        const float* xt = xb + t * ldx;
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const float4 xv = ld4(xt + 4 * w);
            a += v[4 * w] * xv.x + v[4 * w + 1] * xv.y + v[4 * w + 2] * xv.z + v[4 * w + 3] * xv.w;
        }
        acc[t] += db * a;
    }
}

// F32 rows (the MoE router and other small float matrices): a unit is 32 consecutive values, read as eight 16-byte
// vectors; the products are summed in value order, as the generic path sums them.
template <int NC>
__device__ __forceinline__ void unit_f32(const uint8_t* __restrict__ row, int u, const float* __restrict__ x,
                                         int64_t ldx, float (&acc)[NC])
{
    const float* wr = reinterpret_cast<const float*>(row) + 32 * u;
    float w[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 v = ld4(wr + 4 * q);
        w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
    }
#pragma unroll
    for (int t = 0; t < NC; ++t) {
        const float* xt = x + t * ldx + 32 * u;
        float a = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 xv = ld4(xt + 4 * q);
            a += w[4 * q] * xv.x;
            a += w[4 * q + 1] * xv.y;
            a += w[4 * q + 2] * xv.z;
            a += w[4 * q + 3] * xv.w;
        }
        acc[t] += a;
    }
}

// Any decodable type, 32 values per unit, through the exact element decoder.
template <int NC>
__device__ __forceinline__ void unit_generic(int type, const uint8_t* __restrict__ row, int u, int cols,
                                             const float* __restrict__ x, int64_t ldx, float (&acc)[NC])
{
    const int be = block_elems(type), bb = block_bytes(type);
    float w[32];
    const int e0 = u * 32;
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
        const int e = e0 + i;
        w[i] = e < cols ? dq_elem(type, row + (int64_t)(e / be) * bb, e % be) : 0.0f;
    }
#pragma unroll
    for (int t = 0; t < NC; ++t) {
        const float* xt = x + t * ldx + e0;
        float a = 0.f;
        for (int i = 0; i < 32; ++i) if (e0 + i < cols) a += w[i] * xt[i];
        acc[t] += a;
    }
}

enum { MV_GENERIC = 0, MV_Q4K = 1, MV_Q6K = 2, MV_Q8_0 = 3, MV_IQ4XS = 4, MV_IQ2XXS = 5, MV_F32 = 6 };

template <int KIND, int NC>
__global__ void __launch_bounds__(128) k_matvec(int type, const uint8_t* __restrict__ w, int64_t row_bytes, int rows,
                                                int cols, const float* x, int64_t ldx,
                                                float* y, int64_t ldy)
{
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 4 + warp;
    if (row >= rows) return;
    const uint8_t* wr = w + (int64_t)row * row_bytes;
    float acc[NC];
#pragma unroll
    for (int t = 0; t < NC; ++t) acc[t] = 0.f;
    if (KIND == MV_Q4K) {
        const int units = cols >> 6;
        for (int u = lane; u < units; u += 32) unit_q4k<NC>(wr, u, x, ldx, acc);
    } else if (KIND == MV_Q6K) {
        const int units = cols >> 5;
        for (int u = lane; u < units; u += 32) unit_q6k<NC>(wr, u, x, ldx, acc);
    } else if (KIND == MV_Q8_0) {
        const int units = cols >> 5;
        for (int u = lane; u < units; u += 32) unit_q8_0<NC>(wr, u, x, ldx, acc);
    } else if (KIND == MV_IQ4XS) {
        const int units = cols >> 5;
        for (int u = lane; u < units; u += 32) unit_iq4xs<NC>(wr, u, x, ldx, acc);
    } else if (KIND == MV_IQ2XXS) {
        const int units = cols >> 5;
        for (int u = lane; u < units; u += 32) unit_iq2xxs<NC>(wr, u, x, ldx, acc);
    } else if (KIND == MV_F32) {
        const int units = cols >> 5;
        for (int u = lane; u < units; u += 32) unit_f32<NC>(wr, u, x, ldx, acc);
    } else {
        const int units = (cols + 31) >> 5;
        for (int u = lane; u < units; u += 32) unit_generic<NC>(type, wr, u, cols, x, ldx, acc);
    }
#pragma unroll
    for (int t = 0; t < NC; ++t) acc[t] = warp_sum(acc[t]);
    if (lane == 0) {
#pragma unroll
        for (int t = 0; t < NC; ++t) y[t * ldy + row] = acc[t];
    }
}

template <int KIND>
static void launch_mv(int nc, int type, const uint8_t* w, int64_t rb, int rows, int cols, const float* x, int64_t ldx,
                      float* y, int64_t ldy, cudaStream_t s)
{
    const unsigned g = grid_for(rows, 4);
    switch (nc) {
    case 1: launch(k_matvec<KIND, 1>, dim3(g), dim3(128), 0, s, type, w, rb, rows, cols, x, ldx, y, ldy); break;
    case 2: launch(k_matvec<KIND, 2>, dim3(g), dim3(128), 0, s, type, w, rb, rows, cols, x, ldx, y, ldy); break;
    case 3: launch(k_matvec<KIND, 3>, dim3(g), dim3(128), 0, s, type, w, rb, rows, cols, x, ldx, y, ldy); break;
    case 4: launch(k_matvec<KIND, 4>, dim3(g), dim3(128), 0, s, type, w, rb, rows, cols, x, ldx, y, ldy); break;
    case 5: launch(k_matvec<KIND, 5>, dim3(g), dim3(128), 0, s, type, w, rb, rows, cols, x, ldx, y, ldy); break;
    case 6: launch(k_matvec<KIND, 6>, dim3(g), dim3(128), 0, s, type, w, rb, rows, cols, x, ldx, y, ldy); break;
    case 7: launch(k_matvec<KIND, 7>, dim3(g), dim3(128), 0, s, type, w, rb, rows, cols, x, ldx, y, ldy); break;
    default: launch(k_matvec<KIND, 8>, dim3(g), dim3(128), 0, s, type, w, rb, rows, cols, x, ldx, y, ldy); break;
    }
}

// F32 matrices of few rows and a width that is a multiple of 1024 (the MoE router: experts x embedding): a CTA per
// row, thread t holding values 4t + 1024k, each column's products added in that order, then the CTA's partial sums by
// xor butterfly within warps and the warps in order; a column's arithmetic does not depend on the other columns.
template <int NC>
__global__ void __launch_bounds__(256) k_matvec_f32_row(const float* __restrict__ w, int64_t row_floats, int cols,
                                                        const float* x, int64_t ldx, float* y, int64_t ldy)
{
    pdl_trigger();
    pdl_wait();
    __shared__ float part[8][NC];
    const int row = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float* wr = w + (int64_t)row * row_floats;
    float acc[NC];
#pragma unroll
    for (int t = 0; t < NC; ++t) acc[t] = 0.f;
    for (int i = 4 * tid; i < cols; i += 1024) {
        const float4 wv = ld4(wr + i);
#pragma unroll
        for (int t = 0; t < NC; ++t) {
            const float4 xv = ld4(x + t * ldx + i);
            acc[t] += wv.x * xv.x;
            acc[t] += wv.y * xv.y;
            acc[t] += wv.z * xv.z;
            acc[t] += wv.w * xv.w;
        }
    }
#pragma unroll
    for (int t = 0; t < NC; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0) part[warp][t] = v;
    }
    __syncthreads();
    if (tid < NC) {
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) sum += part[k][tid];
        y[(int64_t)tid * ldy + row] = sum;
    }
}

static void launch_f32_rows(int nc, const uint8_t* w, int64_t row_bytes, int rows, int cols, const float* x,
                            int64_t ldx, float* y, int64_t ldy, cudaStream_t s)
{
    const float* wf = reinterpret_cast<const float*>(w);
    const int64_t rf = row_bytes / 4;
    switch (nc) {
    case 1: launch(k_matvec_f32_row<1>, dim3(rows), dim3(256), 0, s, wf, rf, cols, x, ldx, y, ldy); break;
    case 2: launch(k_matvec_f32_row<2>, dim3(rows), dim3(256), 0, s, wf, rf, cols, x, ldx, y, ldy); break;
    case 3: launch(k_matvec_f32_row<3>, dim3(rows), dim3(256), 0, s, wf, rf, cols, x, ldx, y, ldy); break;
    case 4: launch(k_matvec_f32_row<4>, dim3(rows), dim3(256), 0, s, wf, rf, cols, x, ldx, y, ldy); break;
    case 5: launch(k_matvec_f32_row<5>, dim3(rows), dim3(256), 0, s, wf, rf, cols, x, ldx, y, ldy); break;
    case 6: launch(k_matvec_f32_row<6>, dim3(rows), dim3(256), 0, s, wf, rf, cols, x, ldx, y, ldy); break;
    case 7: launch(k_matvec_f32_row<7>, dim3(rows), dim3(256), 0, s, wf, rf, cols, x, ldx, y, ldy); break;
    default: launch(k_matvec_f32_row<8>, dim3(rows), dim3(256), 0, s, wf, rf, cols, x, ldx, y, ldy); break;
    }
}

void matvec(int type, const uint8_t* w, int64_t row_bytes, int rows, int cols, const float* x, int64_t ldx,
            int ncols, float* y, int64_t ldy, cudaStream_t s)
{
    if (rows <= 0 || ncols <= 0) return;
    // The specialised kernels read x with 16-byte loads and the weights with 16/8/2-byte loads.
    const bool xa = ((uintptr_t)x % 16 == 0) && (ldx % 4 == 0);
    const bool w16 = ((uintptr_t)w % 16 == 0) && (row_bytes % 16 == 0);
    const bool w8 = ((uintptr_t)w % 8 == 0) && (row_bytes % 8 == 0);
    const bool w2 = ((uintptr_t)w % 2 == 0) && (row_bytes % 2 == 0);
    for (int c0 = 0; c0 < ncols; c0 += 8) {
        const int nc = ncols - c0 < 8 ? ncols - c0 : 8;
        const float* xc = x + c0 * ldx;
        float* yc = y + c0 * ldy;
        if (type == 12 && xa && w16 && cols % 256 == 0) launch_mv<MV_Q4K>(nc, type, w, row_bytes, rows, cols, xc, ldx, yc, ldy, s);
        else if (type == 14 && xa && w2 && cols % 256 == 0) launch_mv<MV_Q6K>(nc, type, w, row_bytes, rows, cols, xc, ldx, yc, ldy, s);
        else if (type == 8 && xa && w2 && cols % 32 == 0) launch_mv<MV_Q8_0>(nc, type, w, row_bytes, rows, cols, xc, ldx, yc, ldy, s);
        else if (type == 23 && xa && w8 && cols % 256 == 0) launch_mv<MV_IQ4XS>(nc, type, w, row_bytes, rows, cols, xc, ldx, yc, ldy, s);
        else if (type == 16 && xa && w2 && cols % 256 == 0) launch_mv<MV_IQ2XXS>(nc, type, w, row_bytes, rows, cols, xc, ldx, yc, ldy, s);
        else if (type == 0 && xa && w16 && cols % 1024 == 0 && rows <= 1024) launch_f32_rows(nc, w, row_bytes, rows, cols, xc, ldx, yc, ldy, s);
        else if (type == 0 && xa && w16 && cols % 32 == 0) launch_mv<MV_F32>(nc, type, w, row_bytes, rows, cols, xc, ldx, yc, ldy, s);
        else launch_mv<MV_GENERIC>(nc, type, w, row_bytes, rows, cols, xc, ldx, yc, ldy, s);
        launched();
    }
}

// ------------------------------------------------------------------------------------------------------------------
// normalisation, rope, bias, residual
// ------------------------------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T block_sum(T v, T* scratch)
{
    // Fixed-order reduction: warps in index order, lanes by xor butterfly.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    T s = 0;
    for (int i = 0; i < nw; ++i) s += scratch[i];
    return s;
}

__device__ __forceinline__ float block_max(float v, float* scratch)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float m = scratch[0];
    for (int i = 1; i < nw; ++i) m = fmaxf(m, scratch[i]);
    return m;
}

// RmsNormRows: sum of squares in double, scale = 1f / (float)sqrt((float)(sum/dim) + eps), y = (x*scale)*w.
__global__ void k_rmsnorm(const float* x, int dim, const float* __restrict__ w, float eps, float* y)
{
    pdl_trigger();
    pdl_wait();
    __shared__ double scratch[32];
    const float* xr = x + (int64_t)blockIdx.x * dim;
    float* yr = y + (int64_t)blockIdx.x * dim;
    double s = 0;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) { const double v = (double)xr[i]; s += v * v; }
    s = block_sum(s, scratch);
    const float mean = (float)(s / dim);
    const float scale = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(mean, eps)));
    __syncthreads();
    for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
}

// RmsNormRows for rows of at most 8192 values: every thread loads its (up to 8) values before the sum, so a row
// costs one memory round trip instead of one per loop iteration. Same arithmetic as k_rmsnorm.
__global__ void __launch_bounds__(1024) k_rmsnorm8(const float* x, int dim, const float* __restrict__ w, float eps,
                                                   float* y)
{
    pdl_trigger();
    pdl_wait();
    __shared__ double scratch[32];
    const float* xr = x + (int64_t)blockIdx.x * dim;
    float* yr = y + (int64_t)blockIdx.x * dim;
    float v[8];
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) {
        const int i = threadIdx.x + k2 * blockDim.x;
        v[k2] = i < dim ? xr[i] : 0.f;
    }
    double s = 0;
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) s += (double)v[k2] * (double)v[k2];
    s = block_sum(s, scratch);
    const float mean = (float)(s / dim);
    const float scale = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(mean, eps)));
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) {
        const int i = threadIdx.x + k2 * blockDim.x;
        if (i < dim) yr[i] = __fmul_rn(__fmul_rn(v[k2], scale), w[i]);
    }
}

void rmsnorm(const float* x, int n, int dim, const float* w, float eps, float* y, cudaStream_t s)
{
    if (n <= 0) return;
    if (dim <= 8 * 1024) {
        const int threads = std::min(1024, std::max(32, ((dim + 7) / 8 + 31) / 32 * 32));
        launch(k_rmsnorm8, dim3(n), dim3(threads), 0, s, x, dim, w, eps, y);
    } else {
        launch(k_rmsnorm, dim3(n), dim3(256), 0, s, x, dim, w, eps, y);
    }
    launched();
}

__global__ void k_add_bias(float* y, const float* __restrict__ b, int64_t total, int n)
{
    pdl_trigger();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], b[i % n]);
}

void add_bias(float* y, const float* b, int T, int n, cudaStream_t s)
{
    const int64_t total = (int64_t)T * n;
    if (total <= 0) return;
    int64_t g = grid_for(total, 256); if (g > 4096) g = 4096;
    launch(k_add_bias, dim3((unsigned)g), dim3(256), 0, s, y, b, total, n);
    launched();
}

__global__ void k_rope(float* x, int heads, int head_dim, int rope_dims, int neox, const int32_t* pos,
                       const float* __restrict__ table)
{
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y, half = rope_dims / 2;
    const int64_t base = (int64_t)t * heads * head_dim;
    const float* cs = table + (int64_t)pos[t] * rope_dims;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < heads * half; idx += gridDim.x * blockDim.x) {
        const int h = idx / half, i = idx % half;
        const int64_t o = base + (int64_t)h * head_dim;
        const int64_t a = neox ? o + i : o + 2 * i, b = neox ? o + i + half : o + 2 * i + 1;
        const float c = cs[2 * i], sn = cs[2 * i + 1];
        const float x0 = x[a], x1 = x[b];
        x[a] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        x[b] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
}

void rope(float* x, int T, int heads, int head_dim, int rope_dims, int neox, const int32_t* pos, const float* table,
          cudaStream_t s)
{
    if (T <= 0 || rope_dims <= 0) return;
    dim3 grid(grid_for((int64_t)heads * (rope_dims / 2), 256), T);
    launch(k_rope, dim3(grid), dim3(256), 0, s, x, heads, head_dim, rope_dims, neox, pos, table);
    launched();
}

__global__ void k_kv_append(const float* k, const float* v, int kd,
                            const RowKV* rows, int layer, const int32_t* pos)
{
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    uint16_t* kc = rows[t].k + layer * rows[t].layer_stride + (int64_t)pos[t] * kd;
    uint16_t* vc = rows[t].v + layer * rows[t].layer_stride + (int64_t)pos[t] * kd;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kd; i += gridDim.x * blockDim.x) {
        kc[i] = __half_as_ushort(__float2half_rn(k[(int64_t)t * kd + i]));
        vc[i] = __half_as_ushort(__float2half_rn(v[(int64_t)t * kd + i]));
    }
}

void kv_append(const float* k, const float* v, int T, int kd, const RowKV* rows, int layer, const int32_t* pos,
               cudaStream_t s)
{
    if (T <= 0) return;
    dim3 grid(grid_for(kd, 256), T);
    launch(k_kv_append, dim3(grid), dim3(256), 0, s, k, v, kd, rows, layer, pos);
    launched();
}

// RoPE of q and k plus the fp16 KV append, one kernel: work items are q's rotation pairs, then k's values (rotated
// pairs computed from both partners, unrotated dims copied), then v's values. The arithmetic is k_rope's.
__global__ void k_rope_append(float* q, const float* k, const float* v, int heads,
                              int kv_heads, int head_dim, int rope_dims, int neox, const int32_t* pos,
                              const float* __restrict__ table, const RowKV* rows, int layer)
{
    pdl_trigger();
    const int t = blockIdx.y, half = rope_dims / 2, kd = kv_heads * head_dim;
    const int nq = heads * half;
    // positions, cache rows and the rope table come from host copies, not from an earlier kernel
    const int p = pos[t];
    const float* cs = table + (int64_t)p * rope_dims;
    const RowKV rk = rows[t];
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    float c = 1.f, sn = 0.f;
    {
        const int d = idx < nq ? idx % half : idx < nq + kd ? (idx - nq) % head_dim : rope_dims;
        if (d < rope_dims) {
            const int i = idx < nq ? d : neox ? (d < half ? d : d - half) : d >> 1;
            c = cs[2 * i];
            sn = cs[2 * i + 1];
        }
    }
    pdl_wait();
    if (idx < nq) {
        const int h = idx / half, i = idx % half;
        float* x = q + (int64_t)t * heads * head_dim + (int64_t)h * head_dim;
        const int a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
        const float x0 = x[a], x1 = x[b];
        x[a] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        x[b] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    } else if (idx < nq + kd) {
        const int e = idx - nq, d = e % head_dim;
        const float* kr = k + (int64_t)t * kd + (e - d);
        float out = kr[d];
        if (d < rope_dims) {
            const bool first = neox ? d < half : (d & 1) == 0;
            const int i = neox ? (first ? d : d - half) : d >> 1;
            const int a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
            const float x0 = kr[a], x1 = kr[b];
            out = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        }
        rk.k[(int64_t)layer * rk.layer_stride + (int64_t)p * kd + e] = __half_as_ushort(__float2half_rn(out));
    } else if (idx < nq + 2 * kd) {
        const int e = idx - nq - kd;
        rk.v[(int64_t)layer * rk.layer_stride + (int64_t)p * kd + e] = __half_as_ushort(__float2half_rn(v[(int64_t)t * kd + e]));
    }
}

void rope_append(float* q, const float* k, const float* v, int T, int heads, int kv_heads, int head_dim, int rope_dims,
                 int neox, const int32_t* pos, const float* table, const RowKV* rows, int layer, cudaStream_t s)
{
    if (T <= 0) return;
    const int items = heads * (rope_dims / 2) + 2 * kv_heads * head_dim;
    launch(k_rope_append, dim3(grid_for(items, 256), T), dim3(256), 0, s, q, k, v, heads, kv_heads, head_dim, rope_dims,
           neox, pos, table, rows, layer);
    launched();
}

// Per-head QK-norm (Transformer.cs:197-201, RmsNormRows per head) fused with NEOX RoPE over the whole head and the
// KV append: one warp per (row, head), q heads first, then kv heads, whose warps also append the value head. Lane l
// holds values l, l + 32, ... of the head, the order k_rmsnorm8 gives them with 32 threads, and takes the same steps:
// the double sum of squares per lane in that order, the lanes by xor butterfly, the scale and the two rounded
// products; NEOX pairs (i, i + HD/2) then sit in one lane, rotated with k_rope_append's arithmetic. So q, the cache's K
// and V are bit for bit those of k_rmsnorm8 twice and k_rope_append.
template <int HD>
__global__ void __launch_bounds__(128) k_qknorm_rope_append(float* q, const float* k,
                                                            const float* v, int heads, int kv_heads,
                                                            const float* __restrict__ qw, const float* __restrict__ kw,
                                                            float eps, const int32_t* pos,
                                                            const float* __restrict__ table,
                                                            const RowKV* rows, int layer)
{
    constexpr int NV = HD / 32, NP = HD / 64, HALF = HD / 2;
    pdl_trigger();
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int hw = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (hw >= heads + kv_heads) {
        pdl_wait();
        return;
    }
    const bool isq = hw < heads;
    const int h = isq ? hw : hw - heads;
    // positions, cache rows, the rope table and the norm weights are written by no kernel: read them before the wait
    const int p = pos[t];
    const RowKV rk = rows[t];
    const float* cs = table + (int64_t)p * HD;
    const float* w = isq ? qw : kw;
    float wv[NV], c[NP], sn[NP];
#pragma unroll
    for (int j = 0; j < NV; ++j) wv[j] = w[lane + 32 * j];
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        c[j] = cs[2 * (lane + 32 * j)];
        sn[j] = cs[2 * (lane + 32 * j) + 1];
    }
    pdl_wait();
    const int kd = kv_heads * HD;
    const float* src = isq ? q + ((int64_t)t * heads + h) * HD : k + (int64_t)t * kd + (int64_t)h * HD;
    float x[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) x[j] = src[lane + 32 * j];
    double ss = 0;
#pragma unroll
    for (int j = 0; j < NV; ++j) ss += (double)x[j] * (double)x[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float mean = (float)(ss / HD);
    const float scale = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(mean, eps)));
    float y[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) y[j] = __fmul_rn(__fmul_rn(x[j], scale), wv[j]);
    float r[NV];
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        const float x0 = y[j], x1 = y[j + NP];
        r[j] = __fsub_rn(__fmul_rn(x0, c[j]), __fmul_rn(x1, sn[j]));
        r[j + NP] = __fadd_rn(__fmul_rn(x0, sn[j]), __fmul_rn(x1, c[j]));
    }
    static_assert(HALF == 32 * NP, "pairs (i, i + HD/2) must sit in one lane");
    if (isq) {
        float* dst = q + ((int64_t)t * heads + h) * HD;
#pragma unroll
        for (int j = 0; j < NV; ++j) dst[lane + 32 * j] = r[j];
    } else {
        const int64_t base = (int64_t)layer * rk.layer_stride + (int64_t)p * kd + (int64_t)h * HD;
        const float* vs = v + (int64_t)t * kd + (int64_t)h * HD;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            rk.k[base + lane + 32 * j] = __half_as_ushort(__float2half_rn(r[j]));
            rk.v[base + lane + 32 * j] = __half_as_ushort(__float2half_rn(vs[lane + 32 * j]));
        }
    }
}

bool qknorm_rope_append(float* q, const float* k, const float* v, int T, int heads, int kv_heads, int head_dim,
                        int rope_dims, int neox, const float* qw, const float* kw, float eps, const int32_t* pos,
                        const float* table, const RowKV* rows, int layer, cudaStream_t s)
{
    if (!neox || rope_dims != head_dim || (head_dim != 64 && head_dim != 128 && head_dim != 256)) return false;
    if (T <= 0) return true;
    const dim3 grid((unsigned)((heads + kv_heads + 3) / 4), (unsigned)T);
    if (head_dim == 64)
        launch(k_qknorm_rope_append<64>, grid, dim3(128), 0, s, q, k, v, heads, kv_heads, qw, kw, eps, pos, table, rows, layer);
    else if (head_dim == 128)
        launch(k_qknorm_rope_append<128>, grid, dim3(128), 0, s, q, k, v, heads, kv_heads, qw, kw, eps, pos, table, rows, layer);
    else
        launch(k_qknorm_rope_append<256>, grid, dim3(128), 0, s, q, k, v, heads, kv_heads, qw, kw, eps, pos, table, rows, layer);
    launched();
    return true;
}

// SwiGlu (k_swiglu's arithmetic) and the prepared activations of the result, one 256-value superblock per CTA.
__global__ void __launch_bounds__(64) k_swiglu_prep(float* g, const float* u, int F,
                                                    uint8_t* prep)
{
    pdl_trigger();
    pdl_wait();
    __shared__ float scratch[2];
    const int sb = blockIdx.x, t = blockIdx.y, tid = threadIdx.x;
    const int64_t i = (int64_t)t * F + sb * 256 + 4 * tid;
    const float4 a4 = *reinterpret_cast<const float4*>(g + i), u4 = *reinterpret_cast<const float4*>(u + i);
    const float a[4] = {a4.x, a4.y, a4.z, a4.w}, uu[4] = {u4.x, u4.y, u4.z, u4.w};
    float f[4];
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) {
        const float e = (float)exp(-(double)a[k2]);
        f[k2] = __fmul_rn(__fdiv_rn(a[k2], __fadd_rn(1.0f, e)), uu[k2]);
    }
    *reinterpret_cast<float4*>(g + i) = make_float4(f[0], f[1], f[2], f[3]);
    xprep_sb(f, tid, scratch, prep + ((int64_t)t * (F / 256) + sb) * XP_COL);
}

void swiglu_prep(float* g, const float* u, int T, int F, const XPrep& p, cudaStream_t s)
{
    if (T <= 0) return;
    if (F % 256 != 0 || p.cols != F || p.nc != T) WL_THROW(WL_EINVAL, "swiglu_prep: shape mismatch");
    launch(k_swiglu_prep, dim3(F / 256, T), dim3(64), 0, s, g, u, F, p.blocks);
    launched();
}

// ------------------------------------------------------------------------------------------------------------------
// attention
// ------------------------------------------------------------------------------------------------------------------
// Attention (Transformer.cs:351-395), split over positions (flash-decoding) and shared by the query heads of one KV
// head: CTA (range, kv head, row) stages its positions' fp16 keys and values in shared memory tile by tile (16-byte
// cp.async, all copies of a tile in flight at once) and uses them for all G = heads/kv_heads query heads. Scores keep
// the reference's four interleaved accumulators; exponentials are fp32 expf, the running sums double. Positions
// 0..pos[t] of row t are cut into S equal ranges by the row's own length, so a row's result does not depend on the
// other rows; each range keeps a running max m, sum l and unnormalised output o per head across its tiles. With
// S = 1 the CTA writes the normalised output; otherwise k_attn_combine merges the ranges in order. With ro.k (a
// one-row decode step) the kernel also does k_rope_append's work with its arithmetic: q is rotated as it is staged,
// and the CTA whose range holds the new position rotates k, writes k and v there in the cache and places them in its
// staged tile itself (only that CTA reads that position).
constexpr int ATT_P = 128;          // positions per tile (a range of a decode row up to 2048 positions is one tile)

__device__ __forceinline__ void cp_async16(void* dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// k_attn_combine's merge of the S ranges for 4 consecutive output values at value v of row t (same arithmetic and
// order: the maximum over the ranges, then NA accumulator sets of ranges s = a, a + NA, ... in range order, the
// sets added in set order), reading the partials through L2 (other CTAs wrote them).
template <int S>
__device__ __noinline__ void attn_merge4(const float* __restrict__ part, const float* __restrict__ ml, int t,
                                            int heads, int hd, int v, float (&f)[4])
{
    constexpr int NA = S > 16 ? 4 : 1;
    constexpr int SPT = S / NA;
    const int head = v / hd, d = v % hd;
    const float2* mlp = reinterpret_cast<const float2*>(ml + ((int64_t)t * heads + head) * S * 2);
    const float* pp = part + ((int64_t)t * heads + head) * S * hd + d;
    float M = -INFINITY;
#pragma unroll 16
    for (int s = 0; s < S; ++s) M = fmaxf(M, __ldcg(mlp + s).x);
    double Lt = 0.0, t0 = 0.0, t1 = 0.0, t2 = 0.0, t3 = 0.0;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
        double L = 0.0, o0 = 0.0, o1 = 0.0, o2 = 0.0, o3 = 0.0;
#pragma unroll 16
        for (int j = 0; j < SPT; ++j) {
            const int s = a + NA * j;
            const float2 m = __ldcg(mlp + s);
            const float4 ps = __ldcg(reinterpret_cast<const float4*>(pp + (int64_t)s * hd));
            const double w = m.y > 0.f ? (double)expf(m.x - M) : 0.0;
            L += w * (double)m.y;
            o0 += w * (double)ps.x;
            o1 += w * (double)ps.y;
            o2 += w * (double)ps.z;
            o3 += w * (double)ps.w;
        }
        if (a == 0) {
            Lt = L; t0 = o0; t1 = o1; t2 = o2; t3 = o3;
        } else {
            Lt += L; t0 += o0; t1 += o1; t2 += o2; t3 += o3;
        }
    }
    f[0] = (float)(t0 / Lt);
    f[1] = (float)(t1 / Lt);
    f[2] = (float)(t2 / Lt);
    f[3] = (float)(t3 / Lt);
}

// MERGE (S > 1, G * HD a multiple of 256): after writing its range's partials, each CTA takes a ticket on its row's
// counter for its KV head; the CTA that takes the last of the S tickets merges the S ranges of the group's G heads
// (attn_merge4: bit for bit k_attn_combine) and writes the output and, with prep, its prepared activations (the
// group's G * HD values are whole superblocks), then resets the counter for the next launch, so no combine launch is
// needed.
// Threads of an attention CTA: half a thread per (head, dim) of the group, 128 to 512, a multiple of 64, so that the
// positions of a tile times the G heads spread over every thread in the score phase and the G * HD outputs over
// every thread in the value phase (at decode a CTA is alone on its SM, and more warps hide more latency).
constexpr int attn_threads(int HD, int G)
{
    return (G * HD / 2) >= 512 ? 512 : (G * HD / 2) <= 128 ? 128 : (G * HD / 2) / 64 * 64;
}

template <int HD, int G, bool MERGE, int NT = attn_threads(HD, G)>
__global__ void __launch_bounds__(NT, NT == 256 ? 2 : 1) k_attn_part(const float* q, int heads, int kv_heads,
                                                  float scale, const RowKV* rows, int layer,
                                                  const int32_t* pos, int S,
                                                  float* out, float* part,
                                                  float* ml, int* tickets,
                                                  uint8_t* prep, const AttnRope ro)
{
    constexpr int KP = HD + 8;              // row pitch of the staged tiles in halves (16 bytes of padding)
    constexpr int CH = HD / 8;              // 16-byte chunks per row
    constexpr int HS = NT / ATT_P;          // score phase: a thread per position and heads hs, hs + HS, ...
    constexpr int GH = (G + HS - 1) / HS;
    constexpr int VI = G * HD;              // value phase: items (dim, head), item tid + NT * k of each thread
    constexpr int IPT = (VI + NT - 1) / NT;
    extern __shared__ __align__(16) uint8_t smraw[];
    uint16_t* ks = reinterpret_cast<uint16_t*>(smraw);           // [ATT_P][KP]
    uint16_t* vs = ks + ATT_P * KP;                               // [ATT_P][KP]
    float* qs = reinterpret_cast<float*>(vs + ATT_P * KP);       // [G][HD]
    __shared__ float sc[G][ATT_P];
    __shared__ float tmax[G], mrun[G], alpha[G];
    __shared__ double tsum[G], lrun[G];
    pdl_trigger();
    const int sp = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int QD = heads * HD, KD = kv_heads * HD;
    // positions and cache pointers come from host copies, not from an earlier kernel: read them before the wait
    const int n = pos[t] + 1;
    const RowKV rk = rows[t];
    pdl_wait();
    const int per = (n + S - 1) / S;
    const int start = sp * per, end = min(n, start + per);
    const float* qp = q + (int64_t)t * QD + (int64_t)kvh * G * HD;
    const uint16_t* K = rk.k + (int64_t)layer * rk.layer_stride + (int64_t)kvh * HD;
    const uint16_t* V = rk.v + (int64_t)layer * rk.layer_stride + (int64_t)kvh * HD;
    // with ro.k (one-row decode): RoPE here, k_rope_append's arithmetic, at the row's new position n - 1
    __shared__ uint16_t knew[HD], vnew[HD];
    const bool owns_new = ro.k && start <= n - 1 && n - 1 < end;
    if (ro.k) {
        const int half = ro.rope_dims / 2;
        const float* cs = ro.table + (int64_t)(n - 1) * ro.rope_dims;
        for (int e = tid; e < G * HD; e += NT) {
            const int hb = e - e % HD, d = e % HD;
            float val = qp[e];
            if (d < ro.rope_dims) {
                const bool first = ro.neox ? d < half : (d & 1) == 0;
                const int i = ro.neox ? (first ? d : d - half) : d >> 1;
                const int a = ro.neox ? i : 2 * i, b = ro.neox ? i + half : 2 * i + 1;
                const float x0 = qp[hb + a], x1 = qp[hb + b], c = cs[2 * i], sn = cs[2 * i + 1];
                val = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
            }
            qs[e] = val;
        }
        if (owns_new) {
            // this KV head's k (rotated) and v at the new position, into the cache and, below, into the staged tile
            const float* kr = ro.k + (int64_t)t * KD + (int64_t)kvh * HD;
            const float* vr = ro.v + (int64_t)t * KD + (int64_t)kvh * HD;
            uint16_t* Kw = rk.k + (int64_t)layer * rk.layer_stride + (int64_t)(n - 1) * KD + (int64_t)kvh * HD;
            uint16_t* Vw = rk.v + (int64_t)layer * rk.layer_stride + (int64_t)(n - 1) * KD + (int64_t)kvh * HD;
            for (int d = tid; d < HD; d += NT) {
                float kv = kr[d];
                if (d < ro.rope_dims) {
                    const bool first = ro.neox ? d < half : (d & 1) == 0;
                    const int i = ro.neox ? (first ? d : d - half) : d >> 1;
                    const int a = ro.neox ? i : 2 * i, b = ro.neox ? i + half : 2 * i + 1;
                    const float x0 = kr[a], x1 = kr[b], c = cs[2 * i], sn = cs[2 * i + 1];
                    kv = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
                }
                knew[d] = __half_as_ushort(__float2half_rn(kv));
                vnew[d] = __half_as_ushort(__float2half_rn(vr[d]));
                Kw[d] = knew[d];
                Vw[d] = vnew[d];
            }
        }
    } else {
        for (int i = tid; i < G * HD; i += NT) qs[i] = qp[i];
    }
    if (tid < G) { mrun[tid] = -INFINITY; lrun[tid] = 0.0; }
    float o[IPT];
    int od[IPT], oh[IPT];
#pragma unroll
    for (int k2 = 0; k2 < IPT; ++k2) {
        const int item = tid + NT * k2;
        od[k2] = item % HD;
        oh[k2] = item < VI ? item / HD : -1;
        o[k2] = 0.f;
    }
    const int pl = tid % ATT_P, hs = tid / ATT_P;
    for (int tile0 = start; tile0 < end; tile0 += ATT_P) {
        const int cnt = min(ATT_P, end - tile0);
        // (the new position's row, when this CTA wrote it, comes from knew/vnew: each thread places the values it
        // computed, so no barrier is needed before)
        const int rnew = owns_new && n - 1 < tile0 + cnt ? n - 1 - tile0 : -1;
        for (int i = tid; i < cnt * CH; i += NT) {
            const int r = i / CH, c = i % CH;
            if (r == rnew) continue;
            cp_async16(ks + r * KP + c * 8, K + (int64_t)(tile0 + r) * KD + c * 8);
            cp_async16(vs + r * KP + c * 8, V + (int64_t)(tile0 + r) * KD + c * 8);
        }
        if (rnew >= 0)
            for (int d = tid; d < HD; d += NT) {
                ks[rnew * KP + d] = knew[d];
                vs[rnew * KP + d] = vnew[d];
            }
        cp_async_wait_all();
        __syncthreads();
        // scores: the reference's four interleaved accumulators per (head, position), each on one thread
        {
            float s4[GH][4];
#pragma unroll
            for (int hh = 0; hh < GH; ++hh) s4[hh][0] = s4[hh][1] = s4[hh][2] = s4[hh][3] = 0.f;
            if (pl < cnt && hs < G) {
                const uint16_t* kr = ks + pl * KP;
#pragma unroll 2
                for (int d0 = 0; d0 < HD; d0 += 8) {
                    const uint4 kv8 = *reinterpret_cast<const uint4*>(kr + d0);
                    const uint16_t* kh = reinterpret_cast<const uint16_t*>(&kv8);
                    float kf[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) kf[e] = h2f(kh[e]);
#pragma unroll
                    for (int hh = 0; hh < GH; ++hh) {
                        const int h = hs + HS * hh;
                        if (h < G) {
                            const float4 qa = *reinterpret_cast<const float4*>(qs + h * HD + d0);
                            const float4 qb = *reinterpret_cast<const float4*>(qs + h * HD + d0 + 4);
                            const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
                            for (int e = 0; e < 8; ++e) s4[hh][e & 3] = __fadd_rn(s4[hh][e & 3], __fmul_rn(qv[e], kf[e]));
                        }
                    }
                }
            }
#pragma unroll
            for (int hh = 0; hh < GH; ++hh) {
                const int h = hs + HS * hh;
                if (h < G)
                    sc[h][pl] = pl < cnt ? __fmul_rn(__fadd_rn(__fadd_rn(s4[hh][0], s4[hh][1]), __fadd_rn(s4[hh][2], s4[hh][3])), scale)
                                         : -INFINITY;
            }
        }
        __syncthreads();
        for (int h = warp; h < G; h += NT / 32) {
            float m = sc[h][lane];
#pragma unroll
            for (int i = 1; i < ATT_P / 32; ++i) m = fmaxf(m, sc[h][lane + 32 * i]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
            if (lane == 0) {
                const float mn = fmaxf(m, mrun[h]);
                tmax[h] = mn;
                alpha[h] = expf(mrun[h] - mn);      // 0 while no position has been seen
            }
        }
        __syncthreads();
#pragma unroll
        for (int hh = 0; hh < GH; ++hh) {
            const int h = hs + HS * hh;
            if (h < G) sc[h][pl] = pl < cnt ? expf(__fsub_rn(sc[h][pl], tmax[h])) : 0.f;
        }
        __syncthreads();
        for (int h = warp; h < G; h += NT / 32) {
            double sum = (double)sc[h][lane];
#pragma unroll
            for (int i = 1; i < ATT_P / 32; ++i) sum += (double)sc[h][lane + 32 * i];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            if (lane == 0) tsum[h] = sum;
        }
        // o = o * e^(m_old - m_new) + sum_j p_j v_j per (dim, head) item, positions in order, from the staged values
        if constexpr (NT % HD == 0) {
            // a thread's items share their dimension (one V element a position, converted once for all its heads);
            // the items' sums advance together, each still adding the positions in order
            const int d = tid % HD;
            float acc[IPT];
#pragma unroll
            for (int k2 = 0; k2 < IPT; ++k2) acc[k2] = oh[k2] >= 0 ? __fmul_rn(o[k2], alpha[oh[k2]]) : 0.f;
#pragma unroll 2
            for (int j = 0; j < cnt; ++j) {
                const float vj = h2f(vs[j * KP + d]);
#pragma unroll
                for (int k2 = 0; k2 < IPT; ++k2)
                    if (oh[k2] >= 0) acc[k2] = __fadd_rn(acc[k2], __fmul_rn(sc[oh[k2]][j], vj));
            }
#pragma unroll
            for (int k2 = 0; k2 < IPT; ++k2)
                if (oh[k2] >= 0) o[k2] = acc[k2];
        } else {
#pragma unroll
            for (int k2 = 0; k2 < IPT; ++k2) {
                if (oh[k2] < 0) continue;
                const int d = od[k2], h = oh[k2];
                float acc = __fmul_rn(o[k2], alpha[h]);
#pragma unroll 4
                for (int j = 0; j < cnt; ++j) acc = __fadd_rn(acc, __fmul_rn(sc[h][j], h2f(vs[j * KP + d])));
                o[k2] = acc;
            }
        }
        __syncthreads();
        if (tid < G) {
            lrun[tid] = lrun[tid] * (double)alpha[tid] + tsum[tid];
            mrun[tid] = tmax[tid];
        }
        __syncthreads();
    }
#pragma unroll
    for (int k2 = 0; k2 < IPT; ++k2) {
        if (oh[k2] < 0) continue;
        const int d = od[k2], head = kvh * G + oh[k2];
        if (S == 1) out[(int64_t)t * QD + (int64_t)head * HD + d] = (float)((double)o[k2] / lrun[oh[k2]]);
        else part[(((int64_t)t * heads + head) * S + sp) * HD + d] = o[k2];
    }
    if (S > 1 && tid < G) {
        float* mlp = ml + (((int64_t)t * heads + kvh * G + tid) * S + sp) * 2;
        mlp[0] = mrun[tid];
        mlp[1] = (float)lrun[tid];
    }
    if (!MERGE || S == 1) return;
    constexpr int NG = NT / 64;     // 64-thread groups, a superblock each per round
    __shared__ int last;
    __shared__ float pscratch[NG][2];
    // the CTA's partials (written by many threads, ordered before thread 0 by the barrier) are released GPU-wide
    // with thread 0's ticket; the CTA that takes the last ticket acquires every range's partials with it
    __syncthreads();
    if (tid == 0) {
        int* ctr = tickets + t * kv_heads + kvh;
        int ticket;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(ticket) : "l"(ctr) : "memory");
        last = ticket == S - 1;
        if (last) *ctr = 0;         // every range has taken its ticket: ready for the next launch
    }
    __syncthreads();
    if (!last) return;
    constexpr int GV = G * HD;      // the group's values: GV / 256 whole superblocks
    const int v0 = kvh * GV, grp = tid >> 6, t64 = tid & 63;
    for (int r = 0; r < (GV / 256 + NG - 1) / NG; ++r) {
        const int sbl = NG * r + grp;                   // superblock of the group this 64-thread group serves
        if (sbl * 256 >= GV) continue;                  // (uniform per group)
        const int v = v0 + sbl * 256 + 4 * t64;
        float f[4];
        if (S == 16) attn_merge4<16>(part, ml, t, heads, HD, v, f);
        else if (S == 32) attn_merge4<32>(part, ml, t, heads, HD, v, f);
        else attn_merge4<64>(part, ml, t, heads, HD, v, f);
        *reinterpret_cast<float4*>(out + (int64_t)t * QD + v) = make_float4(f[0], f[1], f[2], f[3]);
        if (prep) xprep_sb<true>(f, t64, pscratch[grp], prep + ((int64_t)t * (QD / 256) + v / 256) * XP_COL, 1 + grp);
    }
}

// Merges the S position ranges of k_attn_part in range order for one 256-value superblock of a row's attention
// output: M = max m_s, w_s = e^(m_s - M), out = sum_s w_s o_s / sum_s w_s l_s, in double. Up to 16 ranges one
// thread per 4 consecutive values (64 threads) adds them in range order. Beyond 16, the ranges go to NA = 4
// accumulator sets (range s into set s % NA, each set in range order), which shortens the dependent chains of double
// adds: the four sets of a value run on four adjacent lanes (256 threads), each lane loading only its own ranges, and
// lane 0 of the four adds the sets in set order, so the result is fixed for a given S. With prep, the superblock is
// also written in the tensor-core matvec's activation layout. All loads of a thread are issued before their first use.
template <int S>
__global__ void __launch_bounds__(S > 16 ? 256 : 64) k_attn_combine(int heads, int hd, const float* part,
                                                                    const float* ml,
                                                                    float* out, uint8_t* prep)
{
    constexpr int NA = S > 16 ? 4 : 1;
    constexpr int SPT = S / NA;                 // ranges per thread
    pdl_trigger();
    pdl_wait();
    __shared__ float scratch[2];
    __shared__ float4 fs[NA > 1 ? 64 : 1];
    const int sb = blockIdx.x, t = blockIdx.y;
    const int vt = (int)threadIdx.x / NA, a = (int)threadIdx.x % NA;
    const int QD = heads * hd, v = sb * 256 + 4 * vt, head = v / hd, d = v % hd;
    const float2* mlp = reinterpret_cast<const float2*>(ml + ((int64_t)t * heads + head) * S * 2);
    const float* pp = part + ((int64_t)t * heads + head) * S * hd + d;
    float2 mls[SPT];
    float4 ps[SPT];
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        mls[j] = mlp[a + NA * j];
        ps[j] = *reinterpret_cast<const float4*>(pp + (int64_t)(a + NA * j) * hd);
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < SPT; ++j) M = fmaxf(M, mls[j].x);
    if (NA > 1) {
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
    }
    double L = 0.0, o0 = 0.0, o1 = 0.0, o2 = 0.0, o3 = 0.0;
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        const double w = mls[j].y > 0.f ? (double)expf(mls[j].x - M) : 0.0;
        L += w * (double)mls[j].y;
        o0 += w * (double)ps[j].x;
        o1 += w * (double)ps[j].y;
        o2 += w * (double)ps[j].z;
        o3 += w * (double)ps[j].w;
    }
    if (NA > 1) {
        double Ls[NA], a0[NA], a1[NA], a2[NA], a3[NA];
#pragma unroll
        for (int k2 = 1; k2 < NA; ++k2) {
            Ls[k2] = __shfl_down_sync(0xffffffffu, L, k2);
            a0[k2] = __shfl_down_sync(0xffffffffu, o0, k2);
            a1[k2] = __shfl_down_sync(0xffffffffu, o1, k2);
            a2[k2] = __shfl_down_sync(0xffffffffu, o2, k2);
            a3[k2] = __shfl_down_sync(0xffffffffu, o3, k2);
        }
#pragma unroll
        for (int k2 = 1; k2 < NA; ++k2) {
            L += Ls[k2];
            o0 += a0[k2];
            o1 += a1[k2];
            o2 += a2[k2];
            o3 += a3[k2];
        }
    }
    const float f[4] = {(float)(o0 / L), (float)(o1 / L), (float)(o2 / L), (float)(o3 / L)};
    if (a == 0) *reinterpret_cast<float4*>(out + (int64_t)t * QD + v) = make_float4(f[0], f[1], f[2], f[3]);
    if (!prep) return;
    uint8_t* blk = prep + ((int64_t)t * (QD / 256) + sb) * XP_COL;
    if (NA == 1) {
        xprep_sb(f, vt, scratch, blk);
        return;
    }
    if (a == 0) fs[vt] = make_float4(f[0], f[1], f[2], f[3]);
    __syncthreads();
    if (threadIdx.x < 64) {
        const float4 g = fs[threadIdx.x];
        const float fv[4] = {g.x, g.y, g.z, g.w};
        xprep_sb<true>(fv, (int)threadIdx.x, scratch, blk);
    }
}

int attention_splits(int T, int kv_heads)
{
    return T <= ATT_PART_ROWS ? attention_splits_for(kv_heads) : 1;
}

template <int HD, int G>
static void attn_launch(const float* q, int T, int heads, int kv_heads, float scale, const RowKV* rows, int layer,
                        const int32_t* pos, float* part, float* out, const XPrep* prep, cudaStream_t s,
                        const AttnRope& ro)
{
    const int S = attention_splits(T, kv_heads);
    const size_t smem = sizeof(uint16_t) * 2 * ATT_P * (HD + 8) + sizeof(float) * (size_t)G * HD;
    static std::mutex mu;
    static bool attr_set[64] = {false};
    int dev = 0;
    WL_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && !attr_set[dev]) {
            WL_CUDA(cudaFuncSetAttribute(k_attn_part<HD, G, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
            WL_CUDA(cudaFuncSetAttribute(k_attn_part<HD, G, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
            WL_CUDA(cudaFuncSetAttribute(k_attn_part<HD, G, false, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
            WL_CUDA(cudaFuncSetAttribute(k_attn_part<HD, G, true, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
            if (attn_threads(HD, G) > 256) {
                WL_CUDA(cudaFuncSetAttribute(k_attn_part<HD, G, false, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
                WL_CUDA(cudaFuncSetAttribute(k_attn_part<HD, G, true, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
            }
            attr_set[dev] = true;
        }
    }
    float* ml = part + (size_t)ATT_PART_ROWS * S * heads * HD;
    int* tickets = reinterpret_cast<int*>(part + (size_t)ATT_PART_ROWS * attention_splits_for(kv_heads) * heads * (HD + 2));
    // the merge runs in the last CTA of each KV head when the group's outputs are whole superblocks
    constexpr bool can_merge = (G * HD) % 256 == 0;
    constexpr int WIDE = attn_threads(HD, G);
    constexpr int MID = WIDE > 256 ? 256 : WIDE;
    // one CTA an SM when the grid fits the SMs about once or twice (a decode step of one row: the most threads per
    // CTA); two of up to 256 threads an SM for decode steps of 2 to 8 rows whose grid spans several waves (more CTAs
    // in flight hide each one's phases); otherwise 128 threads, several CTAs an SM. All give the same bits: every
    // score and every (dim, head) sum is one thread's.
    const int64_t ctas = (int64_t)S * kv_heads * T;
    const int width = ctas <= 2 * 148 ? WIDE : T <= 8 ? MID : 128;
    const dim3 grid(S, kv_heads, T);
    uint8_t* pb = prep ? prep->blocks : (uint8_t*)nullptr;
    if (S > 1 && can_merge) {
        if (width == WIDE) launch(k_attn_part<HD, G, true, WIDE>, grid, dim3(WIDE), smem, s, q, heads, kv_heads, scale,
                                  rows, layer, pos, S, out, part, ml, tickets, pb, ro);
        else if (width == MID) launch(k_attn_part<HD, G, true, MID>, grid, dim3(MID), smem, s, q, heads, kv_heads, scale,
                                      rows, layer, pos, S, out, part, ml, tickets, pb, ro);
        else launch(k_attn_part<HD, G, true, 128>, grid, dim3(128), smem, s, q, heads, kv_heads, scale, rows, layer, pos,
                    S, out, part, ml, tickets, pb, ro);
        launched();
        return;
    }
    if (width == WIDE) launch(k_attn_part<HD, G, false, WIDE>, grid, dim3(WIDE), smem, s, q, heads, kv_heads, scale, rows,
                              layer, pos, S, out, part, ml, tickets, (uint8_t*)nullptr, ro);
    else if (width == MID) launch(k_attn_part<HD, G, false, MID>, grid, dim3(MID), smem, s, q, heads, kv_heads, scale,
                                  rows, layer, pos, S, out, part, ml, tickets, (uint8_t*)nullptr, ro);
    else launch(k_attn_part<HD, G, false, 128>, grid, dim3(128), smem, s, q, heads, kv_heads, scale, rows, layer, pos, S,
                out, part, ml, tickets, (uint8_t*)nullptr, ro);
    launched();
    if (S > 1) {
        auto comb = S == 16 ? k_attn_combine<16> : S == 32 ? k_attn_combine<32> : k_attn_combine<64>;
        if (S != 16 && S != 32 && S != 64) WL_THROW(WL_EINVAL, "attention: unexpected range count");
        launch(comb, dim3(heads * HD / 256, T), dim3(S > 16 ? 256 : 64), 0, s, heads, (int)HD, (const float*)part,
               (const float*)ml, out, prep ? prep->blocks : (uint8_t*)nullptr);
        launched();
    }
}

template <int HD>
static void attn_launch_g(const float* q, int T, int heads, int kv_heads, float scale, const RowKV* rows, int layer,
                          const int32_t* pos, float* part, float* out, const XPrep* prep, cudaStream_t s,
                          const AttnRope& ro)
{
    switch (heads / kv_heads) {
    case 1: attn_launch<HD, 1>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    case 2: attn_launch<HD, 2>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    case 4: attn_launch<HD, 4>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    case 8: attn_launch<HD, 8>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    default: attn_launch<HD, 16>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    }
}

bool attention_supported(int heads, int kv_heads, int head_dim)
{
    const int g = kv_heads > 0 && heads % kv_heads == 0 ? heads / kv_heads : 0;
    return (g == 1 || g == 2 || g == 4 || g == 8 || g == 16) && (heads * head_dim) % 256 == 0 &&
           (head_dim == 64 || head_dim == 80 || head_dim == 96 || head_dim == 128 || head_dim == 256);
}

bool attention(const float* q, int T, int heads, int kv_heads, int head_dim, float scale, const RowKV* rows,
               int layer, const int32_t* pos, float* part, float* out, const XPrep* prep, cudaStream_t s,
               const AttnRope* rope)
{
    if (T <= 0) return false;
    const AttnRope ro = rope ? *rope : AttnRope{};
    if (ro.k && (T != 1 || !ro.v || !ro.table || ro.rope_dims < 2 || ro.rope_dims % 2 || ro.rope_dims > head_dim))
        WL_THROW(WL_EINVAL, "attention: RoPE in the attention serves one row, rope_dims even and at most head_dim");
    if (!attention_supported(heads, kv_heads, head_dim))
        WL_THROW(WL_EUNSUPPORTED, "attention: unsupported head layout (1, 2, 4, 8 or 16 query heads per KV head, head_dim 64, "
                                  "80, 96, 128 or 256, heads*head_dim a multiple of 256)");
    if (attention_splits(T, kv_heads) == 1) prep = nullptr;
    if (prep && (prep->cols != heads * head_dim || prep->nc != T)) WL_THROW(WL_EINVAL, "attention: prepared-activation view does not match");
    switch (head_dim) {
    case 64: attn_launch_g<64>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    case 80: attn_launch_g<80>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    case 96: attn_launch_g<96>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    case 128: attn_launch_g<128>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    default: attn_launch_g<256>(q, T, heads, kv_heads, scale, rows, layer, pos, part, out, prep, s, ro); break;
    }
    return prep != nullptr;
}

// ------------------------------------------------------------------------------------------------------------------
// elementwise
// ------------------------------------------------------------------------------------------------------------------
__global__ void k_swiglu(float* g, const float* u, int64_t n)
{
    pdl_trigger();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float a = g[i];
        const float e = (float)exp(-(double)a);
        g[i] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, e)), u[i]);
    }
}

void swiglu(float* g, const float* u, int64_t n, cudaStream_t s)
{
    if (n <= 0) return;
    int64_t gr = grid_for(n, 256); if (gr > 148 * 16) gr = 148 * 16;
    launch(k_swiglu, dim3((unsigned)gr), dim3(256), 0, s, g, u, n);
    launched();
}

__global__ void k_residual(float* x, const float* o, float rs, int64_t n)
{
    pdl_trigger();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], __fmul_rn(o[i], rs));
}

void residual(float* x, const float* o, float rs, int64_t n, cudaStream_t s)
{
    if (n <= 0) return;
    int64_t gr = grid_for(n, 256); if (gr > 148 * 16) gr = 148 * 16;
    launch(k_residual, dim3((unsigned)gr), dim3(256), 0, s, x, o, rs, n);
    launched();
}

__global__ void k_vocab_gather(const float* src, int n, int vp, int V, float* dst)
{
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < V; v += gridDim.x * blockDim.x) {
        const int g = v / vp;
        dst[(int64_t)t * V + v] = src[((int64_t)g * n + t) * vp + (v - g * vp)];
    }
}

void vocab_gather(const float* src, int G, int n, int vp, int V, float* dst, cudaStream_t s)
{
    if (n <= 0 || V <= 0) return;
    if ((int64_t)G * vp < V) WL_THROW(WL_EINVAL, "vocab_gather: parts do not cover the vocabulary");
    int64_t gr = grid_for(V, 256); if (gr > 148 * 4) gr = 148 * 4;
    launch(k_vocab_gather, dim3((unsigned)gr, (unsigned)n), dim3(256), 0, s, src, n, vp, V, dst);
    launched();
}

__global__ void k_scale(float* x, float f, int64_t n)
{
    pdl_trigger();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = __fmul_rn(x[i], f);
}

void scale(float* x, float f, int64_t n, cudaStream_t s)
{
    if (n <= 0) return;
    int64_t gr = grid_for(n, 256); if (gr > 148 * 16) gr = 148 * 16;
    launch(k_scale, dim3((unsigned)gr), dim3(256), 0, s, x, f, n);
    launched();
}

// ------------------------------------------------------------------------------------------------------------------
// greedy selection
// ------------------------------------------------------------------------------------------------------------------
// Sampler.Sample at temperature 0 (src/Engine.cs:356-360) and the guess-ahead check's Argmax (:329-334) scan
// best = 0; for i = 1..n-1: if (x[i] > x[best]) best = i. Its result is the lowest index of the largest non-NaN
// value, except that a NaN at index 0 is never replaced (every comparison with it is false), so the answer is 0 then;
// -0 and +0 compare equal. Here every candidate becomes one 64-bit key, ordered value above, inverted index below, so
// the largest key is the largest value at its lowest index: the blocks of a row each fold their range of the row
// and merge it into the row's key with atomicMax; the last block to finish (a counter per row) reads the key, applies
// the index-0 rule and resets key and counter for the next launch.
__device__ __forceinline__ unsigned long long argmax_key(float f, int v)
{
    unsigned b = __float_as_uint(f);
    if (b == 0x80000000u) b = 0u;                           // -0 compares equal to +0
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);         // order-preserving for every non-NaN float; never 0
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - (unsigned)v);
}

__global__ void __launch_bounds__(256) k_argmax(const float* logits, int V, int chunk,
                                                unsigned long long* key, unsigned* count, int32_t* ids,
                                                int32_t* next_tok, int32_t* next_pos)
{
    __shared__ unsigned long long red[8];
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.y;
    const float* x = logits + (int64_t)r * V;
    const int v0 = blockIdx.x * chunk, v1 = min(V, v0 + chunk);
    unsigned long long best = 0;                            // 0: no candidate (NaN or empty range)
    for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
        const float f = x[v];
        if (!isnan(f)) best = max(best, argmax_key(f, v));
    }
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = max(best, red[w]);
    if (best) atomicMax(&key[r], best);
    __threadfence();
    if (atomicAdd(&count[r], 1u) != gridDim.x - 1) return;
    __threadfence();
    const unsigned long long k = atomicExch(&key[r], 0ull);
    count[r] = 0u;
    const int id = (k == 0 || isnan(x[0])) ? 0 : (int)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFull));
    ids[r] = id;
    if (next_tok) {                                         // a chained decode step: the next token at the next position
        next_tok[r] = id;
        next_pos[r] += 1;
    }
}

int64_t argmax_blocks(int V, int n)
{
    const int64_t per_row = std::max<int64_t>(1, (2 * 148 + n - 1) / n);
    const int64_t chunk = std::max<int64_t>(2048, ((V + per_row - 1) / per_row + 255) / 256 * 256);
    return (V + chunk - 1) / chunk;
}

void argmax(const float* logits, int V, int n, unsigned long long* key, unsigned* count, int32_t* ids,
            int32_t* next_tok, int32_t* next_pos, cudaStream_t s)
{
    if (n <= 0 || V <= 0) return;
    if (n > 65535) WL_THROW(WL_EINVAL, "argmax: too many rows");
    const int64_t blocks = argmax_blocks(V, n);
    const int chunk = (int)((V + blocks - 1) / blocks);
    launch(k_argmax, dim3((unsigned)blocks, (unsigned)n), dim3(256), 0, s, logits, V, chunk, key, count, ids,
           next_tok, next_pos);
    launched();
}

// ------------------------------------------------------------------------------------------------------------------
// mixture of experts
// ------------------------------------------------------------------------------------------------------------------
// Route (Transformer.cs:315-340): one CTA per token, one thread per expert (n <= 256). The maximum (NaNs never win)
// and the exponentials are element-wise, so their results do not depend on the order; the double sum runs on one
// thread in expert order, as the reference's loop does. The reference's greedy top-k picks, among the experts not yet
// taken, the largest probability at its lowest id, so the expert of rank r under (probability descending, id
// ascending) is its pick number r: each thread counts the experts ranked before it and the k lowest ranks write
// their picks. (When the sum is NaN every probability is NaN, every comparison fails and the reference picks ids
// 0, 1, ... in order: NaNs rank by id.) The chosen sum is added in pick order and the renormalisation divides by it
// clamped at 6.103515625e-5, as the reference does.
__global__ void __launch_bounds__(256) k_route(const float* logits, int n, int k, int renorm,
                                               int32_t* sel, float* wts,
                                               unsigned long long* count)
{
    __shared__ float p[256];
    __shared__ float red[8];
    __shared__ float picked[32];
    __shared__ float inv_s;
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x, i = threadIdx.x, lane = i & 31, warp = i >> 5;
    const float v = i < n ? logits[(int64_t)t * n + i] : -INFINITY;
    float m = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float mx = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    if (i < n) p[i] = (float)exp((double)__fsub_rn(v, mx));
    __syncthreads();
    if (i == 0) {
        double sum = 0;
        for (int j = 0; j < n; ++j) sum += p[j];
        inv_s = (float)(1.0 / sum);
    }
    __syncthreads();
    const float pi = i < n ? __fmul_rn(p[i], inv_s) : 0.f;
    __syncthreads();
    if (i < n) p[i] = pi;
    __syncthreads();
    if (i < n) {
        const bool nan_i = isnan(pi);
        int rank = 0;
        for (int j = 0; j < n; ++j) {
            const float q = p[j];
            rank += (q > pi) || ((q == pi || nan_i) && j < i);
        }
        if (rank < k) {
            sel[(int64_t)t * k + rank] = i;
            picked[rank] = pi;
        }
    }
    __syncthreads();
    if (i == 0) {
        float chosen = 0.f;
        for (int j = 0; j < k; ++j) chosen = __fadd_rn(chosen, picked[j]);
        const float div = isnan(chosen) ? chosen : fmaxf(chosen, 6.103515625e-5f);
        for (int j = 0; j < k; ++j) wts[(int64_t)t * k + j] = renorm ? __fdiv_rn(picked[j], div) : picked[j];
        if (count) *count += (unsigned long long)k;     // one token: its k picks are k distinct experts
    }
}

void route(const float* logits, int T, int n, int k, int renorm, int32_t* sel, float* wts, cudaStream_t s,
           unsigned long long* count_one)
{
    if (T <= 0) return;
    if (n <= 0 || n > 256 || k <= 0 || k > 32 || k > n) WL_THROW(WL_EUNSUPPORTED, "route: 1..256 experts, 1..32 chosen");
    if (count_one && T != 1) WL_THROW(WL_EINVAL, "route: the expert count of one token only");
    launch(k_route, dim3((unsigned)T), dim3((unsigned)((n + 31) / 32 * 32)), 0, s, logits, n, k, renorm, sel, wts,
           count_one);
    launched();
}

__global__ void k_gather_rows(float* xe, const float* xn, const int32_t* toks, int n, int E)
{
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.y;
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < E; d += gridDim.x * blockDim.x)
        xe[(int64_t)i * E + d] = xn[(int64_t)toks[i] * E + d];
}

void gather_rows(float* xe, const float* xn, const int32_t* toks, int n, int E, cudaStream_t s)
{
    if (n <= 0) return;
    launch(k_gather_rows, dim3(dim3(grid_for(E, 256), n)), dim3(256), 0, s, xe, xn, toks, n, E);
    launched();
}

__global__ void k_scatter_add(float* outp, const float* ye, const int32_t* toks,
                              const float* w, int E)
{
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.y;
    float* o = outp + (int64_t)toks[i] * E;
    const float wi = w[i];
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < E; d += gridDim.x * blockDim.x)
        o[d] = __fadd_rn(o[d], __fmul_rn(wi, ye[(int64_t)i * E + d]));
}

void scatter_add(float* outp, const float* ye, const int32_t* toks, const float* w, int n, int E, cudaStream_t s)
{
    if (n <= 0) return;
    launch(k_scatter_add, dim3(dim3(grid_for(E, 256), n)), dim3(256), 0, s, outp, ye, toks, w, E);
    launched();
}

__global__ void k_moe_combine(const float* y, const int32_t* sel, const float* wts,
                              int K, int E, float* out, int e_lo, int e_n)
{
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    // token t's experts in ascending id order (the order the reference's per-expert loop adds them)
    int order[16];
    for (int j = 0; j < K; ++j) order[j] = j;
    for (int a = 1; a < K; ++a)
        for (int b = a; b > 0 && sel[t * K + order[b]] < sel[t * K + order[b - 1]]; --b) {
            const int tmp = order[b]; order[b] = order[b - 1]; order[b - 1] = tmp;
        }
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < E; d += gridDim.x * blockDim.x) {
        float o = 0.0f;
        for (int j = 0; j < K; ++j) {
            const int i = t * K + order[j];
            const int ex = sel[i] - e_lo;
            if (ex < 0 || ex >= e_n) continue;          // another GPU's expert
            o = __fadd_rn(o, __fmul_rn(wts[i], y[(int64_t)i * E + d]));
        }
        out[(int64_t)t * E + d] = o;
    }
}

void moe_combine(const float* y, const int32_t* sel, const float* wts, int T, int K, int E, float* out, cudaStream_t s,
                 int e_lo, int e_n)
{
    if (T <= 0) return;
    if (K < 1 || K > 16) WL_THROW(WL_EINVAL, "moe_combine: 1..16 experts per token");
    launch(k_moe_combine, dim3(grid_for(E, 256), T), dim3(256), 0, s, y, sel, wts, K, E, out, e_lo, e_n);
    launched();
}

__global__ void k_count_experts(const int32_t* sel, int n, unsigned long long* count)
{
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned int seen[8];
    if (threadIdx.x < 8) seen[threadIdx.x] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = sel[i];
        if (e >= 0 && e < 256) atomicOr(&seen[e >> 5], 1u << (e & 31));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long c = 0;
        for (int w = 0; w < 8; ++w) c += (unsigned long long)__popc(seen[w]);
        *count += c;
    }
}

void count_experts(const int32_t* sel, int n, unsigned long long* count, cudaStream_t s)
{
    if (n <= 0) return;
    launch(k_count_experts, dim3(1), dim3(128), 0, s, sel, n, count);
    launched();
}

__global__ void k_shared_expert_add(float* outp, const float* sh, const float* gl, int E)
{
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    const float f = gl ? __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)gl[t]))) : 1.0f;
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < E; d += gridDim.x * blockDim.x) {
        const int64_t o = (int64_t)t * E + d;
        outp[o] = __fadd_rn(outp[o], __fmul_rn(f, sh[o]));
    }
}

void shared_expert_add(float* outp, const float* sh, const float* gl, int T, int E, cudaStream_t s)
{
    if (T <= 0) return;
    launch(k_shared_expert_add, dim3(dim3(grid_for(E, 256), T)), dim3(256), 0, s, outp, sh, gl, E);
    launched();
}

// ------------------------------------------------------------------------------------------------------------------
// synthetic weights: bit-identical with the test oracle's CPU generator (or_gen.c). Every float operation below is
// one IEEE operation in the oracle's order; fp16 stores use the reference's round-to-nearest-even converter.
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t splitmix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float synth_normal(uint64_t base, int64_t i)
{
    const uint64_t h0 = splitmix64(base + 3 * (uint64_t)i), h1 = splitmix64(base + 3 * (uint64_t)i + 1),
                   h2 = splitmix64(base + 3 * (uint64_t)i + 2);
    int64_t s = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        s += (int64_t)((h0 >> (16 * k)) & 0xFFFF) + (int64_t)((h1 >> (16 * k)) & 0xFFFF) + (int64_t)((h2 >> (16 * k)) & 0xFFFF);
    return __fmul_rn((float)(s - 393210), 1.0f / 65536.0f);
}

// Half.FromFloat (src/Half.cs:29-57).
__device__ __forceinline__ uint16_t f2h_ref(float value)
{
    const uint32_t f = __float_as_uint(value);
    const uint32_t sign = (f >> 16) & 0x8000;
    const int e = (int)((f >> 23) & 0xFF);
    uint32_t m = f & 0x7FFFFF;
    if (e == 255) return (uint16_t)(sign | 0x7C00 | (m != 0 ? 0x200u : 0u));
    const int ne = e - 127 + 15;
    if (ne >= 31) return (uint16_t)(sign | 0x7C00);
    if (ne <= 0) {
        if (ne < -10) return (uint16_t)sign;
        m |= 0x800000;
        const int shift = 14 - ne;
        uint32_t hm = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1) != 0)) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)ne << 10) | (m >> 13);
    const uint32_t r = m & 0x1FFF;
    if (r > 0x1000 || (r == 0x1000 && (h & 1) != 0)) h++;
    return (uint16_t)h;
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

__device__ void quant_q8_0(const float* x, uint8_t* out)
{
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) { const float a = fabsf(x[j]); if (a > amax) amax = a; }
    const uint16_t dh = f2h_ref(__fdiv_rn(amax, 127.0f));
    const float d = h2f(dh);
    out[0] = (uint8_t)dh; out[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 32; ++j) out[2 + j] = (uint8_t)(int8_t)(d != 0.0f ? clampi((int)rintf(__fdiv_rn(x[j], d)), -127, 127) : 0);
}

__device__ void quant_q4_k(const float* x, uint8_t* out)
{
    float step[8], off[8];
    for (int j = 0; j < 8; ++j) {
        float lo = 0.f, hi = 0.f;
        for (int l = 0; l < 32; ++l) { const float v = x[32 * j + l]; if (v < lo) lo = v; if (v > hi) hi = v; }
        off[j] = -lo;
        step[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
    }
    float smax = 0.f, mmax = 0.f;
    for (int j = 0; j < 8; ++j) { if (step[j] > smax) smax = step[j]; if (off[j] > mmax) mmax = off[j]; }
    const uint16_t dh = f2h_ref(__fdiv_rn(smax, 63.0f)), mh = f2h_ref(__fdiv_rn(mmax, 63.0f));
    const float d = h2f(dh), dmin = h2f(mh);
    int sq[8], mq[8];
    for (int j = 0; j < 8; ++j) {
        sq[j] = d != 0.0f ? clampi((int)rintf(__fdiv_rn(step[j], d)), 0, 63) : 0;
        mq[j] = dmin != 0.0f ? clampi((int)rintf(__fdiv_rn(off[j], dmin)), 0, 63) : 0;
    }
    for (int i = 0; i < 144; ++i) out[i] = 0;
    out[0] = (uint8_t)dh; out[1] = (uint8_t)(dh >> 8); out[2] = (uint8_t)mh; out[3] = (uint8_t)(mh >> 8);
    uint8_t* sc = out + 4;
    for (int j = 0; j < 4; ++j) {
        sc[j] = (uint8_t)((sq[j] & 63) | ((sq[j + 4] >> 4) << 6));
        sc[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
        sc[j + 8] = (uint8_t)((sq[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
    }
    uint8_t* qs = out + 16;
    for (int pair = 0; pair < 4; ++pair)
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * pair + h;
            const float dj = __fmul_rn(d, (float)sq[j]), mj = __fmul_rn(dmin, (float)mq[j]);
            for (int l = 0; l < 32; ++l) {
                const int q = dj != 0.0f ? clampi((int)rintf(__fdiv_rn(__fadd_rn(x[32 * j + l], mj), dj)), 0, 15) : 0;
                qs[32 * pair + l] |= (uint8_t)(q << (4 * h));
            }
        }
}

__device__ void quant_q6_k(const float* x, uint8_t* out)
{
    float step[16];
    for (int g = 0; g < 16; ++g) {
        float amax = 0.f;
        for (int l = 0; l < 16; ++l) { const float a = fabsf(x[16 * g + l]); if (a > amax) amax = a; }
        step[g] = __fdiv_rn(amax, 32.0f);
    }
    float smax = 0.f;
    for (int g = 0; g < 16; ++g) if (step[g] > smax) smax = step[g];
    const uint16_t dh = f2h_ref(__fdiv_rn(smax, 127.0f));
    const float d = h2f(dh);
    int sc[16];
    for (int g = 0; g < 16; ++g) sc[g] = d != 0.0f ? clampi((int)rintf(__fdiv_rn(step[g], d)), -128, 127) : 0;
    for (int i = 0; i < 210; ++i) out[i] = 0;
    uint8_t* ql = out; uint8_t* qh = out + 128;
    for (int g = 0; g < 16; ++g) out[192 + g] = (uint8_t)(int8_t)sc[g];
    out[208] = (uint8_t)dh; out[209] = (uint8_t)(dh >> 8);
    for (int e = 0; e < 256; ++e) {
        const float dg = __fmul_rn(d, (float)sc[e / 16]);
        const int q = dg != 0.0f ? clampi((int)rintf(__fdiv_rn(x[e], dg)), -32, 31) : 0;
        const int u = q + 32;
        const int half = e / 128, w = e % 128, l = w % 32, quarter = w / 32;
        uint8_t* qlh = ql + 64 * half; uint8_t* qhh = qh + 32 * half;
        const int qli = (quarter & 1) ? l + 32 : l;
        qlh[qli] |= (uint8_t)((u & 0xF) << ((quarter >> 1) * 4));
        qhh[l] |= (uint8_t)(((u >> 4) & 3) << (2 * quarter));
    }
}

__global__ void k_synth(int type, uint64_t base, int64_t nblocks, float sigma, float offset, uint8_t* out)
{
    pdl_trigger();
    pdl_wait();
    const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    if (type == 0) { const float v = __fadd_rn(offset, __fmul_rn(sigma, synth_normal(base, b))); reinterpret_cast<float*>(out)[b] = v; return; }
    if (type == 1) { reinterpret_cast<uint16_t*>(out)[b] = f2h_ref(__fmul_rn(sigma, synth_normal(base, b))); return; }
    const int be = type == 8 ? 32 : 256, bb = block_bytes(type);
    float x[256];
    for (int j = 0; j < be; ++j) x[j] = __fmul_rn(sigma, synth_normal(base, b * be + j));
    uint8_t buf[210];
    if (type == 8) quant_q8_0(x, buf);
    else if (type == 12) quant_q4_k(x, buf);
    else quant_q6_k(x, buf);
    uint8_t* dst = out + b * bb;
    for (int i = 0; i < bb; ++i) dst[i] = buf[i];
}

static inline uint64_t splitmix64_host(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void synth(int type, uint64_t seed, uint32_t tid, int64_t rows, int64_t cols, float sigma, float offset, uint8_t* out,
           cudaStream_t s)
{
    const int be = block_elems(type);
    const int64_t nblocks = rows * cols / be;
    const uint64_t base = splitmix64_host(seed ^ ((uint64_t)tid * 0xD1B54A32D192ED03ull));
    if (nblocks <= 0) return;
    launch(k_synth, dim3(grid_for(nblocks, 128)), dim3(128), 0, s, type, base, nblocks, sigma, offset, out);
    launched();
}

}  // namespace k
}  // namespace wl
