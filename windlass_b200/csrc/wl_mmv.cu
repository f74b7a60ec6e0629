// Tensor-core decode matvec for Q4_K (sm_100a): TMA-staged weights, mma.sync m16n8k16 with f16 operands and fp32
// accumulation, for 1..8 activation columns.
//
// Weights. Each warp owns 32 rows and every eighth superblock of them; its lane 0 streams the [32 rows x 144 B]
// superblock tiles into a two-stage shared-memory ring with 2-D TMA copies (cp.async.bulk.tensor, no multicast),
// together with the activation chunks of the same superblock (1-D bulk copies), on one mbarrier per stage. The
// lanes then read their fragments from shared memory and turn the 4-bit codes into exact f16 A fragments: q*s, the
// code times its 6-bit sub-block scale (at most 945), made with one LOP3 and one HFMA2 per two values from the
// 0x6400|q bit pattern (high nibbles stay in place and use s/16).
//
// Activations. k_xprep writes, per column, an exact power-of-two scale and f16 hi/lo pairs of every value
// (x*2^k = hi + lo to 2^-22 relative), grouped so that one 16-byte shared-memory read gives a lane both B fragments
// of a k-step, plus the hi/lo sums of every 32 values for the Q4_K min term, which is one more MMA per superblock.
//
// Determinism. The eight warps of a CTA cover disjoint superblocks of the same 32 rows and are summed in warp order,
// so a column's result never depends on the other columns of the launch.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <mutex>
#include "wl_common.h"
#include "wl_kernels.h"

namespace wl {
namespace k {

namespace {

__device__ __forceinline__ float h2f_(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    // the suspend-time hint (ns) lets the warp sleep until the phase completes instead of spinning
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity; gives up after 4096 polls (each poll sleeps up to 1 ms, so at most a few
// seconds), records the failure in *err and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err, int code)
{
    for (uint32_t i = 0; i < 4096u; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(err, code);
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

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

// ScaleMinK4 (src/Quants.cs:322-330) on the 12 scale bytes held as three words (bytes 4..15 of the superblock).
__device__ __forceinline__ void scale_min_k4_words(int j, uint32_t y, uint32_t z, uint32_t w, int& s, int& m)
{
    const int sh = 8 * (j & 3);
    const int by = (y >> sh) & 0xFF, bz = (z >> sh) & 0xFF, bw = (w >> sh) & 0xFF;
    if (j < 4) { s = by & 63; m = bz & 63; }
    else { s = (bw & 0xF) | ((by >> 6) << 4); m = (bw >> 4) | ((bz >> 6) << 4); }
}

// Two 4-bit codes at bits [b, b+4) and [b+16, b+20) of w (b = 0 or 4) as f16x2 q*s, exact:
// (1024 + q*2^b)*(s/2^b) - 1024*(s/2^b).
__device__ __forceinline__ uint32_t q4_pair(uint32_t w, uint32_t mask, __half2 s2, __half2 ns2)
{
    return h2_bits(__hfma2(bits_h2((w & mask) | 0x64006400u), s2, ns2));
}

}  // namespace

// ------------------------------------------------------------------------------------------------------------------
// activation prep
// ------------------------------------------------------------------------------------------------------------------
// Chunk (16 bytes) of the 4 values 4v..4v+3 of a column: superblock sb = v/64, and inside it the lane group
// c = (v%64)/16, nibble half h = (v%16)/8, word i = v%8; stored at sb*64 + (h*8 + i)*4 + c so that, for a given
// (h, i), the four lanes of a row group read 64 contiguous bytes.
// One CTA of 64 threads per (superblock, column): each thread owns 4 values. The 256 values of the superblock are
// scaled by a power of two so their largest magnitude lies in [2^9, 2^10) (exact; the matvec multiplies the
// superblock's partial sums by the inverse), which keeps hi and the 32-value sums in f16 range and lo mostly clear of
// subnormals. Per (column, superblock) the sums record is 48 bytes: 4 x (hi pair, lo pair) of the eight 32-value sums,
// then the inverse scale.
__global__ void __launch_bounds__(64) k_xprep(const float* __restrict__ x, int64_t ldx, int nsb,
                                              uint4* __restrict__ groups, uint4* __restrict__ sums)
{
    __shared__ float scratch[2];
    const int sb = blockIdx.x, n = blockIdx.y, t = threadIdx.x;
    const float4 v4 = *reinterpret_cast<const float4*>(x + (int64_t)n * ldx + sb * 256 + 4 * t);
    float m = fmaxf(fmaxf(fabsf(v4.x), fabsf(v4.y)), fmaxf(fabsf(v4.z), fabsf(v4.w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((t & 31) == 0) scratch[t >> 5] = m;
    __syncthreads();
    m = fmaxf(scratch[0], scratch[1]);
    int e = 0;
    if (m > 0.f) frexpf(m, &e);
    e = e < -100 ? -100 : e > 100 ? 100 : e;
    const float scale = m > 0.f ? ldexpf(1.0f, 10 - e) : 1.0f;
    uint4* gc = groups + ((int64_t)n * nsb + sb) * 64;
    uint2* sc = reinterpret_cast<uint2*>(sums + ((int64_t)n * nsb + sb) * 3);
    {
        const int v = t;
        const float f[4] = {v4.x * scale, v4.y * scale, v4.z * scale, v4.w * scale};
        __half hi[4], lo[4];
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) {
            hi[k2] = __float2half_rn(f[k2]);
            lo[k2] = __float2half_rn(f[k2] - __half2float(hi[k2]));
        }
        const int c = (v >> 4) & 3, h = (v >> 3) & 1, i = v & 7;
        gc[(h * 8 + i) * 4 + c] =
            make_uint4(h2_bits(__halves2half2(hi[0], hi[2])), h2_bits(__halves2half2(hi[1], hi[3])),
                       h2_bits(__halves2half2(lo[0], lo[2])), h2_bits(__halves2half2(lo[1], lo[3])));
        // sum of the 32 values of this group's sub-block: 8 consecutive groups in 8 consecutive lanes
        float s = (f[0] + f[1]) + (f[2] + f[3]);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        const float s_next = __shfl_down_sync(0xffffffffu, s, 8);
        if ((v & 15) == 0) {
            const __half h0 = __float2half_rn(s), h1 = __float2half_rn(s_next);
            const __half l0 = __float2half_rn(s - __half2float(h0)), l1 = __float2half_rn(s_next - __half2float(h1));
            sc[v >> 4] = make_uint2(h2_bits(__halves2half2(h0, h1)), h2_bits(__halves2half2(l0, l1)));
        }
    }
    if (t == 0) {
        float* tail = reinterpret_cast<float*>(sc + 4);
        tail[0] = 1.0f / scale;
        tail[1] = tail[2] = tail[3] = 0.f;
    }
}

// ------------------------------------------------------------------------------------------------------------------
// Q4_K matvec
// ------------------------------------------------------------------------------------------------------------------
constexpr int Q4_ROWS = 16;                     // rows per CTA: one m16 row group per warp
constexpr int Q4_G = Q4_ROWS / 16, Q4_R = 2 * Q4_G;   // row groups per warp, rows per thread
// Stages of the per-warp copy ring: two, so three CTAs (24 warps) fit an SM at one activation column.
constexpr int Q4_TILE = Q4_ROWS * 144;          // weight bytes per stage
constexpr int Q4_XCOL = 1024 + 64;              // activation bytes per column per stage (+64: no bank conflicts)

template <int NC> struct Q4Layout {
    static constexpr int X_OFF = Q4_TILE;
    static constexpr int S_OFF = Q4_TILE + NC * Q4_XCOL;
    static constexpr int STAGE = (S_OFF + NC * 48 + 127) / 128 * 128;   // TMA destinations are 128-byte aligned
    static constexpr int TX = Q4_TILE + NC * 1024 + NC * 48;      // bytes the copies of one stage deliver
    static constexpr int STAGES = 2;
    static constexpr int SMEM = 8 * STAGES * STAGE;
};

template <int NC>
__global__ void __launch_bounds__(256, 3) k_mmv_q4k(const __grid_constant__ CUtensorMap wmap, int row_base, int rows,
                                                    int nsb, const uint4* __restrict__ xg,
                                                    const uint4* __restrict__ xs, float* __restrict__ y, int64_t ldy,
                                                    int* err)
{
    using LY = Q4Layout<NC>;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[8][3];
    __shared__ float red[8][Q4_ROWS][9];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int r0 = blockIdx.x * Q4_ROWS;
    uint8_t* ring = smem + warp * LY::STAGES * LY::STAGE;
    const int njobs = nsb > warp ? (nsb - warp + 7) / 8 : 0;

    if (lane == 0) {
        for (int s = 0; s < LY::STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    __syncwarp();
    auto issue = [&](int j, int s) {
        const int sb = warp + 8 * j;
        uint8_t* st = ring + s * LY::STAGE;
        mbar_expect_tx(&bars[warp][s], LY::TX);
        tma_load_2d(st, &wmap, sb * 144, row_base + r0, &bars[warp][s]);
#pragma unroll
        for (int n = 0; n < NC; ++n) {
            bulk_load(st + LY::X_OFF + n * Q4_XCOL, xg + ((int64_t)n * nsb + sb) * 64, 1024, &bars[warp][s]);
            bulk_load(st + LY::S_OFF + n * 48, xs + ((int64_t)n * nsb + sb) * 3, 48, &bars[warp][s]);
        }
    };
    if (lane == 0)
        for (int j = 0; j < LY::STAGES && j < njobs; ++j) issue(j, j);

    float dt[Q4_G][4] = {};
    const bool has_col = g < NC;
    for (int j = 0; j < njobs; ++j) {
        const int s = j % LY::STAGES;
        const bool ok = mbar_wait_bounded(&bars[warp][s], (uint32_t)((j / LY::STAGES) & 1), err, 1);
        const uint8_t* st = ring + s * LY::STAGE;
        if (ok) {
            uint4 hdr[Q4_R], qa[Q4_R], qb[Q4_R];
#pragma unroll
            for (int i = 0; i < Q4_R; ++i) {
                const uint8_t* row = st + (g + 8 * i) * 144;
                hdr[i] = lds128(row);
                qa[i] = lds128(row + 16 + 32 * c);
                qb[i] = lds128(row + 32 + 32 * c);
            }
            __half2 slo[Q4_R], nslo[Q4_R], shi[Q4_R], nshi[Q4_R];
            uint32_t mp[Q4_R];
            float dd[Q4_R], dm[Q4_R];
#pragma unroll
            for (int i = 0; i < Q4_R; ++i) {
                int s1, m1, s2, m2;
                scale_min_k4_words(2 * c, hdr[i].y, hdr[i].z, hdr[i].w, s1, m1);
                scale_min_k4_words(2 * c + 1, hdr[i].y, hdr[i].z, hdr[i].w, s2, m2);
                slo[i] = __float2half2_rn((float)s1);
                nslo[i] = __float2half2_rn(-1024.f * (float)s1);
                shi[i] = __float2half2_rn((float)s2 * 0.0625f);        // high nibble in place: value 16q
                nshi[i] = __float2half2_rn(-64.f * (float)s2);
                mp[i] = h2_bits(__floats2half2_rn((float)m1, (float)m2));
                dd[i] = h2f_((uint16_t)(hdr[i].x & 0xFFFF));
                dm[i] = h2f_((uint16_t)(hdr[i].x >> 16));
            }
            // independent accumulators per (row group, nibble half, hi/lo) keep eight MMA chains in flight
            float dq[Q4_G][2][2][4] = {};
            float dn[Q4_G][4] = {};
            const uint8_t* xst = st + LY::X_OFF + (has_col ? g : 0) * Q4_XCOL;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint32_t wa[Q4_R], ws[Q4_R];
#pragma unroll
                for (int r = 0; r < Q4_R; ++r) {
                    wa[r] = i < 4 ? (&qa[r].x)[i] : (&qb[r].x)[i - 4];
                    ws[r] = wa[r] >> 8;
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 b = has_col ? lds128(xst + ((h * 8 + i) * 4 + c) * 16) : make_uint4(0u, 0u, 0u, 0u);
                    const uint32_t mask = h ? 0x00F000F0u : 0x000F000Fu;
#pragma unroll
                    for (int G = 0; G < Q4_G; ++G) {
                        const int ra = 2 * G, rb = 2 * G + 1;
                        const __half2 sa = h ? shi[ra] : slo[ra], nsa = h ? nshi[ra] : nslo[ra];
                        const __half2 sv = h ? shi[rb] : slo[rb], nsv = h ? nshi[rb] : nslo[rb];
                        const uint32_t a0 = q4_pair(wa[ra], mask, sa, nsa);   // row g: values v0, v2
                        const uint32_t a2 = q4_pair(ws[ra], mask, sa, nsa);   // row g: values v1, v3
                        const uint32_t a1 = q4_pair(wa[rb], mask, sv, nsv);   // row g+8
                        const uint32_t a3 = q4_pair(ws[rb], mask, sv, nsv);
                        mma16816(dq[G][h][0], a0, a1, a2, a3, b.x, b.y);
                        mma16816(dq[G][h][1], a0, a1, a2, a3, b.z, b.w);
                    }
                }
            }
            const uint2 bs = has_col ? *reinterpret_cast<const uint2*>(st + LY::S_OFF + g * 48 + c * 8) : make_uint2(0u, 0u);
            // inverse scales of this superblock for the output columns 2c and 2c+1 of the D fragment
            const float is0 = 2 * c < NC ? *reinterpret_cast<const float*>(st + LY::S_OFF + (2 * c) * 48 + 32) : 0.f;
            const float is1 = 2 * c + 1 < NC ? *reinterpret_cast<const float*>(st + LY::S_OFF + (2 * c + 1) * 48 + 32) : 0.f;
#pragma unroll
            for (int G = 0; G < Q4_G; ++G) {
                mma16816(dn[G], mp[2 * G], mp[2 * G + 1], mp[2 * G], mp[2 * G + 1], bs.x, bs.y);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int rs = 2 * G + (e >> 1);
                    const float q = (dq[G][0][0][e] + dq[G][0][1][e]) + (dq[G][1][0][e] + dq[G][1][1][e]);
                    dt[G][e] += (dd[rs] * q - dm[rs] * dn[G][e]) * ((e & 1) ? is1 : is0);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && j + LY::STAGES < njobs) {
            fence_proxy_async();        // the stage's generic reads are done before the copy engine rewrites it
            issue(j + LY::STAGES, s);
        }
    }
#pragma unroll
    for (int G = 0; G < Q4_G; ++G)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][16 * G + g + 8 * (e >> 1)][2 * c + (e & 1)] = dt[G][e];
    __syncthreads();
    const int rl = threadIdx.x >> 3, col = threadIdx.x & 7;
    if (col < NC && rl < Q4_ROWS && r0 + rl < rows) {
        float sum = 0.f;
#pragma unroll
        for (int wv = 0; wv < 8; ++wv) sum += red[wv][rl][col];
        y[(int64_t)col * ldy + r0 + rl] = sum;
    }
}

// ------------------------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------------------------
size_t xprep_bytes(int cols, int nc)
{
    return (size_t)nc * ((size_t)cols * 4 + (size_t)(cols / 256) * 48) + 256;
}

XPrep xprep_view(void* scratch, int cols, int nc)
{
    XPrep p;
    uint8_t* b = (uint8_t*)scratch;
    p.groups = (uint4*)b;
    b += (size_t)nc * cols * 4;
    p.sums = (uint4*)b;
    p.cols = cols;
    p.nc = nc;
    return p;
}

void xprep(const float* x, int64_t ldx, int cols, int nc, const XPrep& p, cudaStream_t s)
{
    k_xprep<<<dim3(cols / 256, nc), 64, 0, s>>>(x, ldx, cols / 256, p.groups, p.sums);
    note_launch();
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static std::mutex mu;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        WL_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (!p || q != cudaDriverEntryPointSuccess) WL_THROW(WL_ECUDA, "cuTensorMapEncodeTiled is unavailable");
        fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

bool mma_supported(int type, const uint8_t* w, int64_t row_bytes, int cols)
{
    return type == 12 && cols % 256 == 0 && (uintptr_t)w % 16 == 0 && row_bytes % 16 == 0;
}

// A 2-D byte tensor map over `rows_total` rows of `row_bytes` bytes with boxes of one superblock x 32 rows.
void make_weight_map(int type, const uint8_t* w, int64_t rows_total, int64_t row_bytes, WeightMap* out)
{
    if (type != 12) WL_THROW(WL_EUNSUPPORTED, "no tensor map layout for this type");
    CUtensorMap* map = reinterpret_cast<CUtensorMap*>(out->bytes);
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows_total};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {144, Q4_ROWS};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)w, dims, strides, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) WL_THROW(WL_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    out->valid = true;
}

template <int NC>
static void launch_q4k(const WeightMap& map, int row_base, int rows, int nsb, const XPrep& p, float* y, int64_t ldy,
                       int* err, cudaStream_t s)
{
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        WL_CUDA(cudaFuncSetAttribute(k_mmv_q4k<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, Q4Layout<NC>::SMEM));
        attr[dev] = true;
    }
    const CUtensorMap& m = *reinterpret_cast<const CUtensorMap*>(map.bytes);
    k_mmv_q4k<NC><<<(rows + Q4_ROWS - 1) / Q4_ROWS, 256, Q4Layout<NC>::SMEM, s>>>(m, row_base, rows, nsb, p.groups,
                                                                                  p.sums, y, ldy, err);
    note_launch();
}

void matvec_mma(int type, const WeightMap& map, int row_base, int rows, int cols, const XPrep& p, float* y, int64_t ldy,
                int* err, cudaStream_t s)
{
    (void)type;
    const int nsb = cols / 256;
    switch (p.nc) {
    case 1: launch_q4k<1>(map, row_base, rows, nsb, p, y, ldy, err, s); break;
    case 2: launch_q4k<2>(map, row_base, rows, nsb, p, y, ldy, err, s); break;
    case 3: launch_q4k<3>(map, row_base, rows, nsb, p, y, ldy, err, s); break;
    case 4: launch_q4k<4>(map, row_base, rows, nsb, p, y, ldy, err, s); break;
    case 5: launch_q4k<5>(map, row_base, rows, nsb, p, y, ldy, err, s); break;
    case 6: launch_q4k<6>(map, row_base, rows, nsb, p, y, ldy, err, s); break;
    case 7: launch_q4k<7>(map, row_base, rows, nsb, p, y, ldy, err, s); break;
    default: launch_q4k<8>(map, row_base, rows, nsb, p, y, ldy, err, s); break;
    }
}

}  // namespace k
}  // namespace wl
