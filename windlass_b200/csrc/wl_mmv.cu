// Tensor-core decode matvec for Q4_K (sm_100a): TMA-staged weights, integer mma.sync (u8 codes x s8 activation
// digits, int32 accumulate) for 1..8 activation columns.
//
// Weights. A CTA owns 16 rows; warp w streams superblocks w, w+8, ... of them ([16 rows x 144 B] tiles, 2-D TMA copies
// with no multicast) into its own shared-memory ring, together with the prepared activations of the same superblock
// (1-D bulk copies), on one mbarrier per stage. A lane's fragment of a 32-value sub-block is two words of code bytes
// masked to the low nibbles (codes q) or the high nibbles (16q, in place).
//
// Activations. k_xprep writes each superblock of each column as three planes of balanced base-128 digits of
// round(x * 2^(20-e)) (21 bits below the superblock's largest magnitude), so the integer MMAs are exact, plus the
// hi/lo f16 sums of every 32 values for the Q4_K min term, which is one f16 MMA per superblock.
//
// Determinism. The eight warps of a CTA cover disjoint superblocks of the same rows and are summed in warp order,
// and every column goes through the same fp32 operations whatever the number of columns beside it, so a column's
// result never depends on the other columns of the launch.
#include <atomic>
#include <climits>
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <cstring>
#include <mutex>
#include "wl_common.h"
#include "wl_kernels.h"
#include "wl_launch.cuh"
#include "wl_xprep.cuh"
#include "wl_mma.cuh"

namespace wl {
namespace k {

namespace {

// Fixed-order block sum: lanes by xor butterfly, then the warps in index order.
__device__ __forceinline__ double block_sum_d(double v, double* scratch)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    double s = 0;
    for (int i = 0; i < nw; ++i) s += scratch[i];
    return s;
}

// ---- thread-block cluster helpers ----
__device__ __forceinline__ void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// A double in the shared memory of CTA `rank` of this cluster, at the address p has in this CTA.
__device__ __forceinline__ double ld_cluster_f64(const double* p, uint32_t rank)
{
    uint32_t ra;
    double v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(ra) : "memory");
    return v;
}

// ---- fused tensor-parallel all-reduce (layout and protocol in wl_kernels.h) ----
__device__ __forceinline__ unsigned long long ar_seq(const unsigned long long* epoch, int idx)
{
    return *epoch * (unsigned long long)AR_STEP + (unsigned long long)idx;
}

// The flag of sequence number q's elements: its low 31 bits with the top bit set, so a zeroed buffer matches no flag
// (a slot is rewritten every AR_SLOTS all-reduces, far within the 2^31 period).
__device__ __forceinline__ uint32_t ar_flag(unsigned long long q) { return (uint32_t)(q & 0x7FFFFFFFull) | 0x80000000u; }

__device__ __forceinline__ size_t ar_elem(unsigned long long q, int src, int col, int E)
{
    return (((size_t)(q % AR_SLOTS) * AR_MAX_RANKS + src) * AR_COLS + col) * (size_t)E;
}

// One element {value, flag}: a single 8-byte store, so value and flag arrive together.
__device__ __forceinline__ void st_elem(unsigned long long* p, float v, uint32_t flag)
{
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(flag) : "memory");
}
// Two elements in one 16-byte store.
__device__ __forceinline__ void st_elem2(unsigned long long* p, float v0, float v1, uint32_t flag)
{
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(__float_as_uint(v0)), "r"(flag),
                 "r"(__float_as_uint(v1)), "r"(flag) : "memory");
}
// Two elements (x, z the values, y, w the flags); each 8-byte half is read whole.
__device__ __forceinline__ uint4 ld_elem2(const unsigned long long* p)
{
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p) : "memory");
    return v;
}

// Element (col, row) of this rank's partial of all-reduce ao.idx, pushed into every rank's buffer. Out of line: the
// Q4_K matvec that calls it from its epilogue then keeps the main loop's register allocation.
__device__ __noinline__ void ar_push_elem(const ArOut& ao, int col, int row, float v)
{
    const unsigned long long q = ar_seq(ao.epoch, ao.idx);
    const uint32_t fl = ar_flag(q);
    const size_t off = ar_elem(q, ao.rank, col, ao.E) + row;
#pragma unroll
    for (int g = 0; g < AR_MAX_RANKS; ++g)
        if (g < ao.G) st_elem(ao.ll[g] + off, v, fl);
}

// Polls two elements until both carry `flag`, for up to ar.wait_ns of %globaltimer time; then records code 2 in *err
// and returns what it read (the sums are then garbage and the host reports WL_ETIMEDOUT), so a rank that never pushes
// cannot hang the GPU. Once any wait of this rank has given up, later waits return at once.
__device__ __noinline__ uint4 ar_wait_elem2(const unsigned long long* p, uint32_t flag, const ArIn ar)
{
    const unsigned long long t0 = globaltimer_ns();
    for (uint32_t n = 0;; ++n) {
        const uint4 v = ld_elem2(p);
        if (v.y == flag && v.w == flag) return v;
        if (n >= 32) {
            if (*(volatile int*)ar.err != 0) return v;
            if ((long long)(globaltimer_ns() - t0) > ar.wait_ns) { atomicExch(ar.err, 2); return v; }
            __nanosleep(64);
        }
    }
}

}  // namespace

// ------------------------------------------------------------------------------------------------------------------
// activation prep
// ------------------------------------------------------------------------------------------------------------------
// One CTA of 64 threads per (superblock, column); each thread owns 4 consecutive values (layout in wl_xprep.cuh).
__global__ void __launch_bounds__(64) k_xprep(const float* x, int64_t ldx, int nsb, uint8_t* out)
{
    pdl_trigger();
    pdl_wait();
    __shared__ float scratch[2];
    const int sb = blockIdx.x, n = blockIdx.y, t = threadIdx.x;
    const float4 v4 = *reinterpret_cast<const float4*>(x + (int64_t)n * ldx + sb * 256 + 4 * t);
    const float f[4] = {v4.x, v4.y, v4.z, v4.w};
    xprep_sb(f, t, scratch, out + ((int64_t)n * nsb + sb) * XP_COL);
}

// ------------------------------------------------------------------------------------------------------------------
// residual + RmsNorm + activation prep in one pass
// ------------------------------------------------------------------------------------------------------------------
// A cluster of gridDim.x CTAs per row (row blockIdx.y): CTA r of the cluster owns superblocks r*W .. r*W+W-1 of the
// row (W = blockDim.x / 32), warp w superblock r*W + w, a lane 8 consecutive values. Spreading a row over several SMs
// spreads its loads, and under tensor parallelism each CTA polls only its own slice of the ranks' pushed partials.
// x += o * rs (Transformer.cs:225,231) when o is given; y = RmsNormRows(x) * w (Transformer.cs:454-464, sum of squares
// in double: lanes by xor butterfly, then warps in order, then the cluster's CTAs in order, through distributed
// shared memory, so every CTA of the row gets the same sum); when prep is given, y's superblocks are also written in
// k_xprep's layout with the same arithmetic (same maximum, digits, and the same association of the 32-value sums),
// so the result is bit-identical to rmsnorm followed by k_xprep.
// MOE: o is not read; each row's o is instead the mixture-of-experts combine of its K chosen experts' outputs (moe.y
// rows t*K + j, weights moe.wts), added in ascending expert id one rounded multiply and add at a time from zero,
// k_moe_combine's arithmetic, so the combine needs no launch of its own.
template <bool RES, bool PREP, bool MOE>
__global__ void __launch_bounds__(256) k_norm_prep(float* x, const float* o, float rs,
                                                   int E, const float* __restrict__ w, float eps, float* y,
                                                   uint8_t* prep, const ArIn ar, const MoeIn moe)
{
    pdl_trigger();
    __shared__ double wsum[8];
    __shared__ double cta_sum, row_sum;
    const int t = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int C = gridDim.x, sb = blockIdx.x * nw + warp;
    const int i0 = sb * 256 + lane * 8;
    // the norm weights are written by no kernel: fetch them before waiting for the previous one
    const float4 wa = *reinterpret_cast<const float4*>(w + i0), wb = *reinterpret_cast<const float4*>(w + i0 + 4);
    pdl_wait();
    float* xr = x + (int64_t)t * E + i0;
    float4 a = *reinterpret_cast<const float4*>(xr), b = *reinterpret_cast<const float4*>(xr + 4);
    if (RES) {
        float4 oa, ob;
        if (MOE) {
            const int K = moe.K;
            int order[16];
            for (int j = 0; j < K; ++j) order[j] = j;
            for (int a2 = 1; a2 < K; ++a2)
                for (int b2 = a2; b2 > 0 && moe.sel[t * K + order[b2]] < moe.sel[t * K + order[b2 - 1]]; --b2) {
                    const int tmp = order[b2]; order[b2] = order[b2 - 1]; order[b2 - 1] = tmp;
                }
            float ov[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int j = 0; j < K; ++j) {
                const int i = t * K + order[j];
                const float wt = moe.wts[i];
                const float* yr = moe.y + (int64_t)i * E + i0;
                const float4 ya = *reinterpret_cast<const float4*>(yr), yb = *reinterpret_cast<const float4*>(yr + 4);
                const float yv[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) ov[e] = __fadd_rn(ov[e], __fmul_rn(wt, yv[e]));
            }
            oa = make_float4(ov[0], ov[1], ov[2], ov[3]);
            ob = make_float4(ov[4], ov[5], ov[6], ov[7]);
        } else if (ar.G > 0) {
            // the fused all-reduce: every rank's partial of this row, pushed into this rank's buffer, summed in rank
            // order; each rank's four 16-byte loads are issued before any is checked
            const unsigned long long q = ar_seq(ar.epoch, ar.idx);
            const uint32_t fl = ar_flag(q);
            float ov[8];
#pragma unroll
            for (int h = 0; h < AR_MAX_RANKS; h += 4) {
                uint4 ln[4][4];
#pragma unroll
                for (int src = h; src < h + 4; ++src)
                    if (src < ar.G) {
                        const unsigned long long* pe = ar.ll + ar_elem(q, src, ar.row0 + t, E) + i0;
#pragma unroll
                        for (int k4 = 0; k4 < 4; ++k4) ln[src - h][k4] = ld_elem2(pe + 2 * k4);
                    }
#pragma unroll
                for (int src = h; src < h + 4; ++src)
                    if (src < ar.G) {
                        const unsigned long long* pe = ar.ll + ar_elem(q, src, ar.row0 + t, E) + i0;
#pragma unroll
                        for (int k4 = 0; k4 < 4; ++k4) {
                            uint4 v = ln[src - h][k4];
                            if (v.y != fl || v.w != fl) v = ar_wait_elem2(pe + 2 * k4, fl, ar);
                            const float v0 = __uint_as_float(v.x), v1 = __uint_as_float(v.z);
                            ov[2 * k4] = src == 0 ? v0 : __fadd_rn(ov[2 * k4], v0);
                            ov[2 * k4 + 1] = src == 0 ? v1 : __fadd_rn(ov[2 * k4 + 1], v1);
                        }
                    }
            }
            oa = make_float4(ov[0], ov[1], ov[2], ov[3]);
            ob = make_float4(ov[4], ov[5], ov[6], ov[7]);
        } else {
            const float* orow = o + (int64_t)t * E + i0;
            oa = *reinterpret_cast<const float4*>(orow);
            ob = *reinterpret_cast<const float4*>(orow + 4);
        }
        a = make_float4(__fadd_rn(a.x, __fmul_rn(oa.x, rs)), __fadd_rn(a.y, __fmul_rn(oa.y, rs)),
                        __fadd_rn(a.z, __fmul_rn(oa.z, rs)), __fadd_rn(a.w, __fmul_rn(oa.w, rs)));
        b = make_float4(__fadd_rn(b.x, __fmul_rn(ob.x, rs)), __fadd_rn(b.y, __fmul_rn(ob.y, rs)),
                        __fadd_rn(b.z, __fmul_rn(ob.z, rs)), __fadd_rn(b.w, __fmul_rn(ob.w, rs)));
        *reinterpret_cast<float4*>(xr) = a;
        *reinterpret_cast<float4*>(xr + 4) = b;
    }
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    double ss = 0;
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) ss += (double)v[k2] * (double)v[k2];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) wsum[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double cs = 0;
        for (int i = 0; i < nw; ++i) cs += wsum[i];
        cta_sum = cs;
    }
    // every CTA's partial in place (and every CTA of the cluster running) before any reads another's
    cluster_arrive_release();
    cluster_wait_acquire();
    if (threadIdx.x == 0) {
        double tot = 0;
        for (int r = 0; r < C; ++r) tot += ld_cluster_f64(&cta_sum, (uint32_t)r);
        row_sum = tot;
    }
    cluster_arrive_relaxed();       // this CTA is done with the others' shared memory (waited for before exit)
    __syncthreads();
    const float mean = (float)(row_sum / E);
    const float scale = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(mean, eps)));
    const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    float f[8];
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) f[k2] = __fmul_rn(__fmul_rn(v[k2], scale), wv[k2]);
    float* yr = y + (int64_t)t * E + i0;
    *reinterpret_cast<float4*>(yr) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(yr + 4) = make_float4(f[4], f[5], f[6], f[7]);
    if (PREP) {
        float m = 0.f;
#pragma unroll
        for (int k2 = 0; k2 < 8; ++k2) m = fmaxf(m, fabsf(f[k2]));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        const bool finite = m <= 3.4e38f;
        int e = 0;
        if (m > 0.f && finite) frexpf(m, &e);
        e = e < -100 ? -100 : e > 100 ? 100 : e;
        const float up = ldexpf(1.0f, 20 - e), sup = ldexpf(1.0f, 10 - e);
        const int nsb = E / 256;
        uint8_t* blk = prep + ((int64_t)t * nsb + sb) * XP_COL;
        uint32_t dg[3][2] = {};
#pragma unroll
        for (int k2 = 0; k2 < 8; ++k2) {
            const int X = finite ? __float2int_rn(f[k2] * up) : 0;
            const int x2 = ((X + 64) & 127) - 64;
            const int r = (X - x2) >> 7;
            const int x1 = ((r + 64) & 127) - 64;
            const int x0 = (r - x1) >> 7;
            dg[0][k2 >> 2] |= (uint32_t)(x0 & 0xFF) << (8 * (k2 & 3));
            dg[1][k2 >> 2] |= (uint32_t)(x1 & 0xFF) << (8 * (k2 & 3));
            dg[2][k2 >> 2] |= (uint32_t)(x2 & 0xFF) << (8 * (k2 & 3));
        }
#pragma unroll
        for (int d = 0; d < 3; ++d) *reinterpret_cast<uint2*>(blk + d * XP_DIGIT + 8 * lane) = make_uint2(dg[d][0], dg[d][1]);
        if (lane < 8) {
#pragma unroll
            for (int d = 0; d < 3; ++d) *reinterpret_cast<uint32_t*>(blk + d * XP_DIGIT + 256 + 4 * lane) = 0u;
        }
        // 16- and 32-value sums with k_xprep's association: (g0+g1) per lane, then lanes xor 1 (16 values), then xor 2
        float sm = __fadd_rn(__fadd_rn(f[0] * sup, f[1] * sup), __fadd_rn(f[2] * sup, f[3] * sup));
        const float s1 = __fadd_rn(__fadd_rn(f[4] * sup, f[5] * sup), __fadd_rn(f[6] * sup, f[7] * sup));
        sm = __fadd_rn(sm, s1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        const float s16 = sm, s16_next = __shfl_down_sync(0xffffffffu, sm, 2);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        const float s_next = __shfl_down_sync(0xffffffffu, sm, 4);
        uint32_t* rec = reinterpret_cast<uint32_t*>(blk + XP_REC);
        if ((lane & 7) == 0) xp_store_pair(rec, 2 * (lane >> 3), 2 * (lane >> 3) + 1, sm, s_next);
        if ((lane & 3) == 0) {
            const int p = lane >> 2, c = p & 3, upper = p >> 2;
            xp_store_pair(rec, XP_S16 + 4 * c + upper, XP_S16 + 4 * c + 2 + upper, s16, s16_next);
        }
        if (lane == 8) rec[8] = __float_as_uint(finite ? ldexpf(1.0f, e - 20) : __int_as_float(0x7fc00000));
        if (lane >= 9 && lane < XP_S16) rec[lane] = 0u;
        if (lane >= XP_S16 + 16) rec[lane] = 0u;
    }
    cluster_wait_acquire();         // no CTA leaves while another may still read its partial
}

// ------------------------------------------------------------------------------------------------------------------
// Q4_K matvec
// ------------------------------------------------------------------------------------------------------------------
constexpr int Q4_ROWS = 16;                     // rows per CTA: one m16 row group, shared by the eight warps
constexpr int Q4_TILE = Q4_ROWS * 144;          // weight bytes per stage
// Tile-major Q4_K (k_q4k_tile): per tile of 16 rows x one superblock, the 16 rows' 16-byte headers (d, dmin, scales),
// then per 32-byte run r of codes 512 bytes in which lane (g, c) finds at lane*16 its 8 code bytes of row g and
// then of row g+8 (raw bytes 16 + 32r + 8c ..+8), one conflict-free 16-byte read per run.
constexpr int Q4_HDRS = Q4_ROWS * 16;

template <int NC, int NW = 8> struct Q4Layout {
    static constexpr int X_OFF = Q4_TILE;       // 2304, a multiple of 128
    static constexpr int STAGE = (X_OFF + NC * XP_COL + 127) / 128 * 128;   // TMA destinations are 128-byte aligned
    static constexpr int TX = Q4_TILE + NC * XP_COL;                         // bytes the copies of one stage deliver
    static constexpr int STAGES = 2;
    static constexpr int SMEM = NW * STAGES * STAGE;
};

// The second matrix of a two-matrix Q4_K matvec launch (same columns and activations as the first).
struct MvSeg {
    const uint8_t* wt;
    int row_base, rows;
    int first_ctas;             // CTAs of the first matrix; INT_MAX: one matrix
    float* y;
    int64_t ldy;
    // pair mode (sel != nullptr): the mixture-of-experts grouped matvec. CTA b serves pair b / tiles_per_pair (a
    // token and one of its K chosen experts) and that expert's row tile b % tiles_per_pair; the expert id is
    // sel[pair] (written by the router kernel), its rows start at row_base + id * rows, the activations are column
    // pair / K (x_per_token) or column pair of the prepared input, and the output row is y + pair * ldy.
    const int32_t* sel;
    int K, tiles_per_pair, x_per_token;
    // under tensor parallelism a GPU holds experts e_lo .. e_lo + e_n - 1 only (stacked from row_base): a pair whose
    // expert lives on another GPU is skipped (its CTAs return at once)
    int e_lo = 0, e_n = INT_MAX;
};

__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%10,%10,%10,%10};\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// One CTA per 16 rows; warp w of its NW warps takes superblocks w, w+NW, ... of those rows. Per superblock and 32-value sub-block
// one integer MMA (u8 codes x s8 activation digits, exact int32) gives sum(q*X); the 6-bit sub-block scales are
// applied in integers; the superblock's d and the digit unit are applied in fp32 per digit plane; the min term
// dmin * sum_j m_j * sum(x_j) is one f16 MMA over the hi/lo sub-block sums.
// Up to two columns, the 8 MMA columns hold (column, digit) pairs (one MMA per sub-block); from three columns on,
// one MMA per digit plane holds the columns. Both orders give every column the same fp32 operations, so a column's
// result does not depend on how many columns share the launch.
// PAIRS: the grouped-expert form (seg.sel set), compiled apart so that the dense matvec carries none of its code.
// The launch bound's CTA count is what fits an SM: four (NW = 8) or eight (NW = 4) at one column, two or four from
// three columns on; at two columns the stages leave room for only three or six (228 KB of shared memory an SM, 1 KB
// of it reserved per CTA), and the bound says so, so that the compiler keeps the two-column loop in registers.
constexpr int ctas_by_smem(int bytes) { return 228 * 1024 / (bytes + 1024); }
template <int NC, int NW> constexpr int q4_min_ctas()
{
    return NC == 2 ? (ctas_by_smem(Q4Layout<NC, NW>::SMEM) < 32 / NW ? ctas_by_smem(Q4Layout<NC, NW>::SMEM) : 32 / NW)
                   : (NC <= 2 ? 32 : 16) / NW;
}

template <int NC, bool TILED, bool PAIRS, int NW = 8, bool AR = false>
__global__ void __launch_bounds__(32 * NW, q4_min_ctas<NC, NW>()) k_mmv_q4k(const __grid_constant__ CUtensorMap wmap,
                                                    const uint8_t* __restrict__ wt_a, int row_base_a, int rows_a, int nsb,
                                                    const uint8_t* xq, float* y_a,
                                                    int64_t ldy_a, int* err, const MvSeg seg, const ArOut ao)
{
    using LY = Q4Layout<NC, NW>;
    constexpr bool PACK = NC <= 2;
    constexpr int ND = PACK ? 1 : 3;            // MMAs per sub-block
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[NW][LY::STAGES];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    // two matrices with the same input in one launch: CTAs past the first matrix's row tiles take the second's
    const bool second = TILED && !seg.sel && (int)blockIdx.x >= seg.first_ctas;
    int bx = second ? (int)blockIdx.x - seg.first_ctas : (int)blockIdx.x;
    const uint8_t* __restrict__ wt = second ? seg.wt : wt_a;
    int row_base = second ? seg.row_base : row_base_a;
    const int rows = second ? seg.rows : rows_a;
    float* y = second ? seg.y : y_a;
    const int64_t ldy = second ? seg.ldy : ldy_a;
    if (TILED && seg.sel && !PAIRS) {
        // (the single-matrix grouped form; launches use the PAIRS instantiation below, this keeps the dense
        // instantiation's code, and so its register allocation, as it was)
        pdl_wait();
        const int pair = (int)blockIdx.x / seg.tiles_per_pair;
        bx = (int)blockIdx.x % seg.tiles_per_pair;
        row_base = row_base_a + seg.sel[pair] * rows_a;
        xq += (int64_t)(seg.x_per_token ? pair / seg.K : pair) * nsb * XP_COL;
        y = y_a + (int64_t)pair * ldy_a;
    }
    if (TILED && PAIRS) {
        // grouped experts: the expert ids come from the router kernel, so wait for it before the first weight copy.
        // With seg.wt the launch covers a second stacked matrix of the same shape (up after gate): its CTAs follow
        // the first matrix's and write seg.y.
        pdl_wait();
        int b = (int)blockIdx.x;
        const int per = seg.first_ctas * seg.tiles_per_pair;
        const bool up = seg.wt && b >= per;
        if (up) b -= per;
        const int pair = b / seg.tiles_per_pair;
        bx = b % seg.tiles_per_pair;
        if (up) wt = seg.wt;
        const int ex = seg.sel[pair] - seg.e_lo;
        if (ex < 0 || ex >= seg.e_n) return;        // an expert of another GPU
        row_base = row_base_a + ex * rows_a;
        xq += (int64_t)(seg.x_per_token ? pair / seg.K : pair) * nsb * XP_COL;
        y = (up ? seg.y : y_a) + (int64_t)pair * (up ? seg.ldy : ldy_a);
    }
    const int r0 = bx * Q4_ROWS;
    uint8_t* ring = smem + warp * LY::STAGES * LY::STAGE;
    const int njobs = nsb > warp ? (nsb - warp + NW - 1) / NW : 0;

    pdl_trigger();
    if (lane == 0) {
        for (int s = 0; s < LY::STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    __syncwarp();
    auto issue_w = [&](int j, int s) {      // weights: written by no kernel, so they may stream before pdl_wait()
        uint8_t* st = ring + s * LY::STAGE;
        mbar_expect_tx(&bars[warp][s], LY::TX);
        if (TILED)
            bulk_load(st, wt + ((int64_t)(row_base / Q4_ROWS + bx) * nsb + warp + NW * j) * Q4_TILE, Q4_TILE,
                      &bars[warp][s]);
        else
            tma_load_2d(st, &wmap, (warp + NW * j) * 144, row_base + r0, &bars[warp][s]);
    };
    auto issue_x = [&](int j, int s) {      // prepared activations of the same superblock, on the same barrier
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

    // B operand of this lane: MMA column g is (column g/3, digit g%3) when packed, else column g
    const bool b_ok = PACK ? g < 3 * NC : g < NC;
    const int b_off = LY::X_OFF + (PACK ? (g / 3) * XP_COL + (g % 3) * XP_DIGIT : g * XP_COL);
    // D columns 2c, 2c+1 of this lane: (column, digit) pairs when packed, else columns
    int e_col[2], e_dig[2];
    bool e_ok[2];
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
        const int nn = 2 * c + k2;
        e_col[k2] = PACK ? nn / 3 : nn;
        e_dig[k2] = PACK ? nn % 3 : 0;
        e_ok[k2] = PACK ? nn < 3 * NC : nn < NC;
    }
    const bool m_ok0 = 2 * c < NC, m_ok1 = 2 * c + 1 < NC;   // columns of the min-term MMA's D fragment
    // the mins of sub-blocks 2c, 2c+1 as f16 1024+m: bytes (2c)&3, (2c+1)&3 of the mins word, 0x64 above each
    const uint32_t msel = (uint32_t)((2 * c) & 3) | (4u << 4) | ((uint32_t)((2 * c + 1) & 3) << 8) | (4u << 12);
    const __half2 k1024 = __float2half2_rn(1024.f);

    float facc[ND][4] = {};     // per digit plane: d * unit * sum_j s_j sum(q X)
    float macc[4] = {};         // dmin * unit * sum_j m_j sum(x)
    for (int j = 0; j < njobs; ++j) {
        const int s = j % LY::STAGES;
        const bool ok = mbar_wait_bounded(&bars[warp][s], (uint32_t)((j / LY::STAGES) & 1), err, 1);
        const uint8_t* st = ring + s * LY::STAGE;
        if (ok) {
            const uint8_t* row0 = st + g * (TILED ? 16 : 144);
            const uint8_t* row1 = st + (g + 8) * (TILED ? 16 : 144);
            const uint4 h0 = lds128(row0), h1 = lds128(row1);
            // ScaleMinK4 for all eight sub-blocks at once: scales and mins as bytes
            const uint32_t s0lo = h0.y & 0x3F3F3F3Fu, s0hi = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
            const uint32_t s1lo = h1.y & 0x3F3F3F3Fu, s1hi = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
            int acc_lo[ND][4] = {}, acc_hi[ND][4] = {};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                uint2 w0, w1;
                if (TILED) {
                    const uint4 wv = lds128(st + Q4_HDRS + r * 512 + lane * 16);
                    w0 = make_uint2(wv.x, wv.y);
                    w1 = make_uint2(wv.z, wv.w);
                } else {
                    w0 = lds64(row0 + 16 + 32 * r + 8 * c);
                    w1 = lds64(row1 + 16 + 32 * r + 8 * c);
                }
                const uint32_t sw0 = r < 2 ? s0lo : s0hi, sw1 = r < 2 ? s1lo : s1hi;
                const int kb = (2 * r) & 3;
                const int sl0 = (int)((sw0 >> (8 * kb)) & 0xFFu), sh0 = (int)((sw0 >> (8 * kb + 8)) & 0xFFu);
                const int sl1 = (int)((sw1 >> (8 * kb)) & 0xFFu), sh1 = (int)((sw1 >> (8 * kb + 8)) & 0xFFu);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const uint32_t mask = hh ? 0xF0F0F0F0u : 0x0F0F0F0Fu;   // high nibbles stay in place: 16q
                    const uint32_t a0 = w0.x & mask, a1 = w1.x & mask, a2 = w0.y & mask, a3 = w1.y & mask;
                    const int sa = hh ? sh0 : sl0, sb2 = hh ? sh1 : sl1;
#pragma unroll
                    for (int d = 0; d < ND; ++d) {
                        const uint2 b = b_ok ? lds64(st + b_off + d * XP_DIGIT + 32 * (2 * r + hh) + 8 * c)
                                             : make_uint2(0u, 0u);
                        int D[4];
                        imma16832(D, a0, a1, a2, a3, b.x, b.y);
                        int (&acc)[4] = hh ? acc_hi[d] : acc_lo[d];
                        acc[0] += sa * D[0];
                        acc[1] += sa * D[1];
                        acc[2] += sb2 * D[2];
                        acc[3] += sb2 * D[3];
                    }
                }
            }
            const float dd0 = h2f_((uint16_t)(h0.x & 0xFFFF)), dm0 = h2f_((uint16_t)(h0.x >> 16));
            const float dd1 = h2f_((uint16_t)(h1.x & 0xFFFF)), dm1 = h2f_((uint16_t)(h1.x >> 16));
            // digit planes: 16 * sum_j s_j sum(q X) = 16 acc_lo + acc_hi (exact); unit * 2^(14 - 7 digit) / 16
#pragma unroll
            for (int k2 = 0; k2 < 2; ++k2) {
                const float unit = e_ok[k2] ? *reinterpret_cast<const float*>(st + LY::X_OFF + e_col[k2] * XP_COL + XP_REC + 32) : 0.f;
#pragma unroll
                for (int d = 0; d < ND; ++d) {
                    const int dig = PACK ? e_dig[k2] : d;
                    const float f = unit * (dig == 0 ? 1024.f : dig == 1 ? 8.f : 0.0625f);
                    facc[d][k2] = fmaf((float)(acc_lo[d][k2] * 16 + acc_hi[d][k2]), dd0 * f, facc[d][k2]);
                    facc[d][k2 + 2] = fmaf((float)(acc_lo[d][k2 + 2] * 16 + acc_hi[d][k2 + 2]), dd1 * f, facc[d][k2 + 2]);
                }
            }
            // min term: A = the mins of sub-blocks 2c, 2c+1 (k slots 2c, 2c+1 and again 2c+8, 2c+9), B = hi sums in
            // slots 0..7 and lo sums in 8..15 of the lane's column
            const uint32_t m0lo = h0.z & 0x3F3F3F3Fu, m0hi = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
            const uint32_t m1lo = h1.z & 0x3F3F3F3Fu, m1hi = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
            const uint32_t mp0 = h2_bits(__hsub2(bits_h2(__byte_perm(c < 2 ? m0lo : m0hi, 0x64646464u, msel)), k1024));
            const uint32_t mp1 = h2_bits(__hsub2(bits_h2(__byte_perm(c < 2 ? m1lo : m1hi, 0x64646464u, msel)), k1024));
            const uint2 bs = g < NC ? lds64(st + LY::X_OFF + g * XP_COL + XP_REC + 8 * c) : make_uint2(0u, 0u);
            float dn[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(dn, mp0, mp1, mp0, mp1, bs.x, bs.y);
            const float mu0 = m_ok0 ? *reinterpret_cast<const float*>(st + LY::X_OFF + (2 * c) * XP_COL + XP_REC + 32) * 1024.f : 0.f;
            const float mu1 = m_ok1 ? *reinterpret_cast<const float*>(st + LY::X_OFF + (2 * c + 1) * XP_COL + XP_REC + 32) * 1024.f : 0.f;
            macc[0] = fmaf(dn[0], dm0 * mu0, macc[0]);
            macc[1] = fmaf(dn[1], dm0 * mu1, macc[1]);
            macc[2] = fmaf(dn[2], dm1 * mu0, macc[2]);
            macc[3] = fmaf(dn[3], dm1 * mu1, macc[3]);
        }
        __syncwarp();
        if (lane == 0 && j + LY::STAGES < njobs) {
            fence_proxy_async();        // the stage's generic reads are done before the copy engine rewrites it
            issue_w(j + LY::STAGES, s);
            issue_x(j + LY::STAGES, s);
        }
    }
    // per (row, column): ((plane 0 + plane 1) + plane 2) - min term, then the warps in order. Each warp's partials
    // go to the start of its own ring, whose stages it has finished with.
    float* red = reinterpret_cast<float*>(ring);        // [Q4_ROWS][9]
    if (PACK) {
#pragma unroll
        for (int e = 0; e < 4; ++e) red[(g + 8 * (e >> 1)) * 9 + 2 * c + (e & 1)] = facc[0][e];
        if (c == 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e) red[(g + 8 * (e >> 1)) * 9 + 6 + (e & 1)] = macc[e];
        }
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = g + 8 * (e >> 1), col = 2 * c + (e & 1);
            if (col < NC) red[row * 9 + col] = ((facc[0][e] + facc[ND > 1 ? 1 : 0][e]) + facc[ND > 2 ? 2 : 0][e]) - macc[e];
        }
    }
    __syncthreads();
    const int rl = threadIdx.x >> 3, col = threadIdx.x & 7;     // NW >= 4: every (row, column) has a thread
    if (col < NC && rl < Q4_ROWS && r0 + rl < rows) {
        float sum = 0.f;
#pragma unroll
        for (int wv = 0; wv < NW; ++wv) {
            const float* rw = reinterpret_cast<const float*>(smem + wv * LY::STAGES * LY::STAGE) + rl * 9;
            const float v = PACK ? ((rw[3 * col] + rw[3 * col + 1]) + rw[3 * col + 2]) - rw[6 + col] : rw[col];
            sum += v;
        }
        if constexpr (AR) {
            ar_push_elem(ao, col, r0 + rl, sum);     // a fused all-reduce's partial: pushed into every rank's buffer
        } else {
            y[(int64_t)col * ldy + r0 + rl] = sum;
        }
    }
}

// ---- the persistent form (six to eight columns) ----
// At many columns, a 16-row CTA that streams every superblock's prepared activations for NC columns (992 bytes
// each) next to 2304 bytes of weights is bound by its stage count and the CTAs resident per SM rather than by HBM:
// 8192 x 8192 at 8 columns took 20 us in four partial waves. Here a grid of as many CTAs as fit at once walks the row
// tiles in pairs (pair p = tiles 2p, 2p + 1 of one matrix; a matrix with an odd tile count ends in a single), CTA b
// taking pairs b, b + gridDim.x, ...: each stage holds both tiles of one superblock and the activations once, every
// warp's ring runs on across pairs, and the activation fragments of a sub-block serve both tiles. Warp w still takes
// superblocks w, w + NW, ... of every row, each tile's arithmetic is k_mmv_q4k's (the same integer MMAs, fp32
// operations and order, planes added ((0 + 1) + 2) - min, warps in order), so every row equals k_mmv_q4k's bit for bit.
template <int NC, int NW> struct Q4LayoutP {
    static constexpr int X_OFF = 2 * Q4_TILE;
    static constexpr int STAGE = (X_OFF + NC * XP_COL + 127) / 128 * 128;
    static constexpr int STAGES = 2;
    static constexpr int RED = NW * 2 * Q4_ROWS * 9 * 4;
    static constexpr int SMEM = NW * STAGES * STAGE + RED;
};

template <int NC, int NW>
__global__ void __launch_bounds__(32 * NW, 1) k_mmv_q4kp(const uint8_t* __restrict__ wt_a, int row_base_a, int rows_a,
                                                        int nsb, const uint8_t* xq, float* y_a, int64_t ldy_a,
                                                        int* err, const MvSeg seg)
{
    static_assert(NC >= 3 && NC <= 8, "the persistent form serves three to eight columns");
    using LY = Q4LayoutP<NC, NW>;
    constexpr int ND = 3;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[NW][LY::STAGES];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int tiles_a = (rows_a + Q4_ROWS - 1) / Q4_ROWS;
    const int pairs_a = (tiles_a + 1) / 2;
    const int tiles_b = seg.wt ? (seg.rows + Q4_ROWS - 1) / Q4_ROWS : 0;
    const int pairs = pairs_a + (tiles_b + 1) / 2;
    const int G = (int)gridDim.x;
    const int npair = pairs > (int)blockIdx.x ? (pairs - (int)blockIdx.x + G - 1) / G : 0;
    const int per = nsb > warp ? (nsb - warp + NW - 1) / NW : 0;     // this warp's superblocks of a row
    const int njobs = npair * per;
    uint8_t* ring = smem + warp * LY::STAGES * LY::STAGE;
    float* red = reinterpret_cast<float*>(smem + NW * LY::STAGES * LY::STAGE);     // [NW][2][Q4_ROWS][9]

    // pair q (global index): its matrix, first tile (in that matrix's tile numbering) and tile count
    struct PairOf {
        const uint8_t* wt;
        int tile0, ntile, rows;
        float* y;
        int64_t ldy;
    };
    auto pair_of = [&](int q) -> PairOf {
        PairOf r;
        if (q < pairs_a) {
            r.wt = wt_a; r.tile0 = row_base_a / Q4_ROWS + 2 * q; r.ntile = min(2, tiles_a - 2 * q);
            r.rows = rows_a - 2 * q * Q4_ROWS; r.y = y_a + 2 * q * Q4_ROWS; r.ldy = ldy_a;
        } else {
            const int qb = q - pairs_a;
            r.wt = seg.wt; r.tile0 = seg.row_base / Q4_ROWS + 2 * qb; r.ntile = min(2, tiles_b - 2 * qb);
            r.rows = seg.rows - 2 * qb * Q4_ROWS; r.y = seg.y + 2 * qb * Q4_ROWS; r.ldy = seg.ldy;
        }
        return r;
    };
    auto issue_w = [&](int j, int s) {      // weights: written by no kernel, so they may stream before pdl_wait()
        const int k = j / per, sb = warp + NW * (j - k * per);
        const PairOf pr = pair_of((int)blockIdx.x + k * G);
        uint8_t* st = ring + s * LY::STAGE;
        mbar_expect_tx(&bars[warp][s], pr.ntile * Q4_TILE + NC * XP_COL);
        for (int q = 0; q < pr.ntile; ++q)
            bulk_load(st + q * Q4_TILE, pr.wt + ((int64_t)(pr.tile0 + q) * nsb + sb) * Q4_TILE, Q4_TILE, &bars[warp][s]);
    };
    auto issue_x = [&](int j, int s) {      // the superblock's prepared activations, on the same barrier
        const int sb = warp + NW * (j % per);
        uint8_t* st = ring + s * LY::STAGE;
#pragma unroll
        for (int n = 0; n < NC; ++n)
            bulk_load(st + LY::X_OFF + n * XP_COL, xq + ((int64_t)n * nsb + sb) * XP_COL, XP_COL, &bars[warp][s]);
    };

    pdl_trigger();
    if (lane == 0) {
        for (int s = 0; s < LY::STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    __syncwarp();
    if (lane == 0)
        for (int j = 0; j < LY::STAGES && j < njobs; ++j) issue_w(j, j);
    pdl_wait();
    if (lane == 0)
        for (int j = 0; j < LY::STAGES && j < njobs; ++j) issue_x(j, j);

    const bool b_ok = g < NC;
    const int b_off = LY::X_OFF + g * XP_COL;
    const bool m_ok0 = 2 * c < NC, m_ok1 = 2 * c + 1 < NC;
    const uint32_t msel = (uint32_t)((2 * c) & 3) | (4u << 4) | ((uint32_t)((2 * c + 1) & 3) << 8) | (4u << 12);
    const __half2 k1024 = __float2half2_rn(1024.f);

    int j = 0;
    for (int k = 0; k < npair; ++k) {
        const PairOf pr = pair_of((int)blockIdx.x + k * G);
        float facc[2][ND][4] = {};
        float macc[2][4] = {};
        for (int i = 0; i < per; ++i, ++j) {
            const int s = j % LY::STAGES;
            const bool ok = mbar_wait_bounded(&bars[warp][s], (uint32_t)((j / LY::STAGES) & 1), err, 1);
            const uint8_t* st = ring + s * LY::STAGE;
            if (ok) {
                uint4 h0[2], h1[2];
                uint32_t s0lo[2], s0hi[2], s1lo[2], s1hi[2];
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    if (q < pr.ntile) {
                        h0[q] = lds128(st + q * Q4_TILE + g * 16);
                        h1[q] = lds128(st + q * Q4_TILE + (g + 8) * 16);
                    } else {
                        h0[q] = make_uint4(0u, 0u, 0u, 0u);
                        h1[q] = h0[q];
                    }
                    s0lo[q] = h0[q].y & 0x3F3F3F3Fu;
                    s0hi[q] = (h0[q].w & 0x0F0F0F0Fu) | ((h0[q].y >> 2) & 0x30303030u);
                    s1lo[q] = h1[q].y & 0x3F3F3F3Fu;
                    s1hi[q] = (h1[q].w & 0x0F0F0F0Fu) | ((h1[q].y >> 2) & 0x30303030u);
                }
                int acc_lo[2][ND][4] = {}, acc_hi[2][ND][4] = {};
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    uint2 bf[2][ND];
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                        for (int d = 0; d < ND; ++d)
                            bf[hh][d] = b_ok ? lds64(st + b_off + d * XP_DIGIT + 32 * (2 * r + hh) + 8 * c) : make_uint2(0u, 0u);
                    const int kb = (2 * r) & 3;
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        if (q >= pr.ntile) break;
                        const uint4 wv = lds128(st + q * Q4_TILE + Q4_HDRS + r * 512 + lane * 16);
                        const uint32_t sw0 = r < 2 ? s0lo[q] : s0hi[q], sw1 = r < 2 ? s1lo[q] : s1hi[q];
                        const int sl0 = (int)((sw0 >> (8 * kb)) & 0xFFu), sh0 = (int)((sw0 >> (8 * kb + 8)) & 0xFFu);
                        const int sl1 = (int)((sw1 >> (8 * kb)) & 0xFFu), sh1 = (int)((sw1 >> (8 * kb + 8)) & 0xFFu);
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {
                            const uint32_t mask = hh ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
                            const uint32_t a0 = wv.x & mask, a1 = wv.z & mask, a2 = wv.y & mask, a3 = wv.w & mask;
                            const int sa = hh ? sh0 : sl0, sb2 = hh ? sh1 : sl1;
#pragma unroll
                            for (int d = 0; d < ND; ++d) {
                                int D[4];
                                imma16832(D, a0, a1, a2, a3, bf[hh][d].x, bf[hh][d].y);
                                int (&acc)[4] = hh ? acc_hi[q][d] : acc_lo[q][d];
                                acc[0] += sa * D[0];
                                acc[1] += sa * D[1];
                                acc[2] += sb2 * D[2];
                                acc[3] += sb2 * D[3];
                            }
                        }
                    }
                }
                // digit planes: unit * 2^(14 - 7 digit) / 16 per (column, digit), as k_mmv_q4k forms it
                float fu[2][ND];
#pragma unroll
                for (int k2 = 0; k2 < 2; ++k2) {
                    const int col = 2 * c + k2;
                    const float unit = col < NC ? *reinterpret_cast<const float*>(st + LY::X_OFF + col * XP_COL + XP_REC + 32) : 0.f;
#pragma unroll
                    for (int d = 0; d < ND; ++d) fu[k2][d] = unit * (d == 0 ? 1024.f : d == 1 ? 8.f : 0.0625f);
                }
                const uint2 bs = g < NC ? lds64(st + LY::X_OFF + g * XP_COL + XP_REC + 8 * c) : make_uint2(0u, 0u);
                const float mu0 = m_ok0 ? *reinterpret_cast<const float*>(st + LY::X_OFF + (2 * c) * XP_COL + XP_REC + 32) * 1024.f : 0.f;
                const float mu1 = m_ok1 ? *reinterpret_cast<const float*>(st + LY::X_OFF + (2 * c + 1) * XP_COL + XP_REC + 32) * 1024.f : 0.f;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    if (q >= pr.ntile) break;
                    const float dd0 = h2f_((uint16_t)(h0[q].x & 0xFFFF)), dm0 = h2f_((uint16_t)(h0[q].x >> 16));
                    const float dd1 = h2f_((uint16_t)(h1[q].x & 0xFFFF)), dm1 = h2f_((uint16_t)(h1[q].x >> 16));
#pragma unroll
                    for (int k2 = 0; k2 < 2; ++k2)
#pragma unroll
                        for (int d = 0; d < ND; ++d) {
                            facc[q][d][k2] = fmaf((float)(acc_lo[q][d][k2] * 16 + acc_hi[q][d][k2]), dd0 * fu[k2][d],
                                                  facc[q][d][k2]);
                            facc[q][d][k2 + 2] = fmaf((float)(acc_lo[q][d][k2 + 2] * 16 + acc_hi[q][d][k2 + 2]),
                                                      dd1 * fu[k2][d], facc[q][d][k2 + 2]);
                        }
                    const uint32_t m0lo = h0[q].z & 0x3F3F3F3Fu;
                    const uint32_t m0hi = ((h0[q].w >> 4) & 0x0F0F0F0Fu) | ((h0[q].z >> 2) & 0x30303030u);
                    const uint32_t m1lo = h1[q].z & 0x3F3F3F3Fu;
                    const uint32_t m1hi = ((h1[q].w >> 4) & 0x0F0F0F0Fu) | ((h1[q].z >> 2) & 0x30303030u);
                    const uint32_t mp0 = h2_bits(__hsub2(bits_h2(__byte_perm(c < 2 ? m0lo : m0hi, 0x64646464u, msel)), k1024));
                    const uint32_t mp1 = h2_bits(__hsub2(bits_h2(__byte_perm(c < 2 ? m1lo : m1hi, 0x64646464u, msel)), k1024));
                    float dn[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(dn, mp0, mp1, mp0, mp1, bs.x, bs.y);
                    macc[q][0] = fmaf(dn[0], dm0 * mu0, macc[q][0]);
                    macc[q][1] = fmaf(dn[1], dm0 * mu1, macc[q][1]);
                    macc[q][2] = fmaf(dn[2], dm1 * mu0, macc[q][2]);
                    macc[q][3] = fmaf(dn[3], dm1 * mu1, macc[q][3]);
                }
            }
            __syncwarp();
            if (lane == 0 && j + LY::STAGES < njobs) {
                fence_proxy_async();        // the stage's generic reads are done before the copy engine rewrites it
                issue_w(j + LY::STAGES, s);
                issue_x(j + LY::STAGES, s);
            }
        }
        // this warp's sums of the pair: ((plane 0 + plane 1) + plane 2) - min per (row, column)
        float* rw = red + warp * 2 * Q4_ROWS * 9;
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = g + 8 * (e >> 1), col = 2 * c + (e & 1);
                if (col < NC) rw[(q * Q4_ROWS + row) * 9 + col] = ((facc[q][0][e] + facc[q][1][e]) + facc[q][2][e]) - macc[q][e];
            }
        __syncthreads();
        for (int idx = threadIdx.x; idx < 2 * Q4_ROWS * 8; idx += 32 * NW) {
            const int rl = idx >> 3, col = idx & 7;     // rl: row 0..31 of the pair
            if (col < NC && rl < pr.ntile * Q4_ROWS && rl < pr.rows) {
                float sum = 0.f;
#pragma unroll
                for (int wv = 0; wv < NW; ++wv) sum += red[(wv * 2 * Q4_ROWS + rl) * 9 + col];
                pr.y[(int64_t)col * pr.ldy + rl] = sum;
            }
        }
        __syncthreads();                            // the red area is free for the next pair
    }
}

// Repacks rows [0, rows) of a Q4_K matrix into the tile-major layout above; rows past the end are zero. One CTA per tile.
__global__ void k_q4k_tile(const uint8_t* src, int rows, int nsb, int64_t row_bytes,
                           uint8_t* dst)
{
    pdl_trigger();
    pdl_wait();
    const int sb = blockIdx.x, rt = blockIdx.y;
    uint8_t* out = dst + ((int64_t)rt * nsb + sb) * Q4_TILE;
    for (int i = threadIdx.x; i < Q4_TILE; i += blockDim.x) {
        int r, off;
        if (i < Q4_HDRS) {
            r = i >> 4;
            off = i & 15;
        } else {
            const int j = i - Q4_HDRS, run = j >> 9, ln = (j & 511) >> 4, b = j & 15;
            const int gg = ln >> 2, cc = ln & 3;
            r = b < 8 ? gg : gg + 8;
            off = 16 + 32 * run + 8 * cc + (b & 7);
        }
        const int row = rt * Q4_ROWS + r;
        out[i] = row < rows ? src[(int64_t)row * row_bytes + (int64_t)sb * 144 + off] : (uint8_t)0;
    }
}

// ------------------------------------------------------------------------------------------------------------------
// Q6_K matvec
// ------------------------------------------------------------------------------------------------------------------
// Q6_K superblocks are 210 bytes, so a row's superblocks are only 2-byte aligned and cannot be copied by TMA. The
// weights are therefore repacked once (k_q6k_tile) into tiles of 16 rows x one superblock (Q6_TILE = 3360 bytes,
// 16-byte aligned), tile (r, b) at ((r * nsb) + b) * Q6_TILE, each laid out for conflict-free fragment reads:
//   [0, 2048)     ql: per row 128 bytes; lane c's eight words (word h*4 + kk*2 + is = ql bytes 64h + 32kk + 16is +
//                 4c..+3) sit at c*32, the two 16-byte halves swapped on odd rows
//   [2048, 3072)  qh: per row 64 bytes; lane c's four words (word h*2 + is = qh bytes 32h + 16is + 4c..+3) at c*16
//   [3072, 3328)  the 16 int8 sub-block scales of each row
//   [3328, 3360)  the fp16 d of each row
// Sub-block j (16 values 16j..16j+15: half h = j/8, quarter k = (j/2)%4, is = j%2) is one m16n8k16 integer MMA whose
// A bytes are the 6-bit codes q (u8: ql nibble k/2, qh bits 2k..2k+1), B the activation digits; the sub-block scale
// is applied in integers, d and the digit unit in fp32, and the -32 offset of the codes as
// -32 * d * sum_j sc_j * sum16_j, one f16 MMA pair (hi, lo) over the 16-value sums.
constexpr int Q6_TILE = Q6K_TILE;
constexpr int Q6_QH = 2048, Q6_SC = 3072, Q6_D = 3328;

template <int NC> struct Q6Layout {
    static constexpr int X_OFF = (Q6_TILE + 127) / 128 * 128;   // 3456
    static constexpr int STAGE = (X_OFF + NC * XP_COL + 127) / 128 * 128;
    static constexpr int TX = Q6_TILE + NC * XP_COL;
    static constexpr int STAGES = 2;
    static constexpr int SMEM = 8 * STAGES * STAGE;
};

// Three CTAs an SM at one column; from two columns on the stages leave room for two, and the launch bound says so.
template <int NC> constexpr int q6_min_ctas()
{
    return ctas_by_smem(Q6Layout<NC>::SMEM) < 3 ? ctas_by_smem(Q6Layout<NC>::SMEM) : 3;
}

__device__ __forceinline__ void imma16816(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// int8 scale pair (bytes i0, i1 of w) as exact f16x2: (sc ^ 0x80) under the 0x64 exponent is 1152 + sc.
__device__ __forceinline__ uint32_t sc_pair_h2(uint32_t w, uint32_t sel, __half2 k1152)
{
    return h2_bits(__hsub2(bits_h2(__byte_perm(w ^ 0x80808080u, 0x64646464u, sel)), k1152));
}

template <int NC>
__global__ void __launch_bounds__(256, q6_min_ctas<NC>()) k_mmv_q6k(const uint8_t* __restrict__ wt, int rows, int nsb,
                                                    const uint8_t* xq, float* y, int64_t ldy,
                                                    int* err)
{
    using LY = Q6Layout<NC>;
    constexpr bool PACK = NC <= 2;
    constexpr int ND = PACK ? 1 : 3;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[8][LY::STAGES];
    __shared__ float red[8][16][9];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int rt = blockIdx.x, r0 = rt * 16;
    uint8_t* ring = smem + warp * LY::STAGES * LY::STAGE;
    const int njobs = nsb > warp ? (nsb - warp + 7) / 8 : 0;

    pdl_trigger();
    if (lane == 0) {
        for (int s = 0; s < LY::STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    __syncwarp();
    auto issue_w = [&](int j, int s) {      // weights: written by no kernel, so they may stream before pdl_wait()
        uint8_t* st = ring + s * LY::STAGE;
        mbar_expect_tx(&bars[warp][s], LY::TX);
        bulk_load(st, wt + ((int64_t)rt * nsb + warp + 8 * j) * Q6_TILE, Q6_TILE, &bars[warp][s]);
    };
    auto issue_x = [&](int j, int s) {
        const int sb = warp + 8 * j;
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
    const bool m_ok0 = 2 * c < NC, m_ok1 = 2 * c + 1 < NC;
    // scale bytes 2c, 2c+1 (and 2c+8, 2c+9 from the second word pair) of a row's 16 scales
    const uint32_t ssel = (uint32_t)((2 * c) & 3) | (4u << 4) | ((uint32_t)((2 * c + 1) & 3) << 8) | (4u << 12);
    const __half2 k1152 = __float2half2_rn(1152.f);
    const int par = (g & 1) << 4;           // odd rows keep their ql halves swapped

    float facc[ND][4] = {};
    float macc[4] = {};
    for (int j = 0; j < njobs; ++j) {
        const int s = j % LY::STAGES;
        const bool ok = mbar_wait_bounded(&bars[warp][s], (uint32_t)((j / LY::STAGES) & 1), err, 1);
        const uint8_t* st = ring + s * LY::STAGE;
        if (ok) {
            uint32_t qa[8], qb[8], ha[4], hb[4];
            {
                const uint8_t* la = st + g * 128 + c * 32;
                const uint8_t* lb = st + (g + 8) * 128 + c * 32;
                const uint4 a_lo = lds128(la + par), a_hi = lds128(la + (par ^ 16));
                const uint4 b_lo = lds128(lb + par), b_hi = lds128(lb + (par ^ 16));
                qa[0] = a_lo.x; qa[1] = a_lo.y; qa[2] = a_lo.z; qa[3] = a_lo.w;
                qa[4] = a_hi.x; qa[5] = a_hi.y; qa[6] = a_hi.z; qa[7] = a_hi.w;
                qb[0] = b_lo.x; qb[1] = b_lo.y; qb[2] = b_lo.z; qb[3] = b_lo.w;
                qb[4] = b_hi.x; qb[5] = b_hi.y; qb[6] = b_hi.z; qb[7] = b_hi.w;
                const uint4 h0 = lds128(st + Q6_QH + g * 64 + c * 16), h1 = lds128(st + Q6_QH + (g + 8) * 64 + c * 16);
                ha[0] = h0.x; ha[1] = h0.y; ha[2] = h0.z; ha[3] = h0.w;
                hb[0] = h1.x; hb[1] = h1.y; hb[2] = h1.z; hb[3] = h1.w;
            }
            const uint4 sa = lds128(st + Q6_SC + g * 16), sb4 = lds128(st + Q6_SC + (g + 8) * 16);
            const uint32_t swa[4] = {sa.x, sa.y, sa.z, sa.w}, swb[4] = {sb4.x, sb4.y, sb4.z, sb4.w};
            int acc[ND][4] = {};
#pragma unroll
            for (int sbj = 0; sbj < 16; ++sbj) {
                const int h = sbj >> 3, kq = (sbj >> 1) & 3, is = sbj & 1;
                const int wi = h * 4 + (kq & 1) * 2 + is, hi = h * 2 + is;
                const int nsh = 4 * (kq >> 1), hsh = 2 * kq;
                const uint32_t a0 = ((qa[wi] >> nsh) & 0x0F0F0F0Fu) | (((ha[hi] >> hsh) & 0x03030303u) << 4);
                const uint32_t a1 = ((qb[wi] >> nsh) & 0x0F0F0F0Fu) | (((hb[hi] >> hsh) & 0x03030303u) << 4);
                const int s0 = (int)(int8_t)((swa[sbj >> 2] >> (8 * (sbj & 3))) & 0xFFu);
                const int s1 = (int)(int8_t)((swb[sbj >> 2] >> (8 * (sbj & 3))) & 0xFFu);
#pragma unroll
                for (int d = 0; d < ND; ++d) {
                    const uint32_t b = b_ok ? *reinterpret_cast<const uint32_t*>(st + b_off + d * XP_DIGIT + 16 * sbj + 4 * c) : 0u;
                    int D[4];
                    imma16816(D, a0, a1, b);
                    acc[d][0] += s0 * D[0];
                    acc[d][1] += s0 * D[1];
                    acc[d][2] += s1 * D[2];
                    acc[d][3] += s1 * D[3];
                }
            }
            const float dd0 = h2f_(*reinterpret_cast<const uint16_t*>(st + Q6_D + 2 * g));
            const float dd1 = h2f_(*reinterpret_cast<const uint16_t*>(st + Q6_D + 2 * (g + 8)));
#pragma unroll
            for (int k2 = 0; k2 < 2; ++k2) {
                const float unit = e_ok[k2] ? *reinterpret_cast<const float*>(st + LY::X_OFF + e_col[k2] * XP_COL + XP_REC + 32) : 0.f;
#pragma unroll
                for (int d = 0; d < ND; ++d) {
                    const int dig = PACK ? e_dig[k2] : d;
                    const float f = unit * (dig == 0 ? 16384.f : dig == 1 ? 128.f : 1.f);
                    facc[d][k2] = fmaf((float)acc[d][k2], dd0 * f, facc[d][k2]);
                    facc[d][k2 + 2] = fmaf((float)acc[d][k2 + 2], dd1 * f, facc[d][k2 + 2]);
                }
            }
            // offset term: sum_j sc_j * sum16_j, A = the scales of sub-blocks 2c, 2c+1 (k slots 2c, 2c+1) and
            // 2c+8, 2c+9 (slots 2c+8, 2c+9), B = the hi sums, then the lo sums, of the lane's column
            const bool hi_c = c >= 2;           // scales 2c, 2c+1 sit in word c/2, scales 2c+8, 2c+9 in word 2 + c/2
            const uint32_t wA0 = hi_c ? sa.y : sa.x, wA1 = hi_c ? sa.w : sa.z;
            const uint32_t wB0 = hi_c ? sb4.y : sb4.x, wB1 = hi_c ? sb4.w : sb4.z;
            const uint32_t p00 = sc_pair_h2(wA0, ssel, k1152), p01 = sc_pair_h2(wA1, ssel, k1152);
            const uint32_t p10 = sc_pair_h2(wB0, ssel, k1152), p11 = sc_pair_h2(wB1, ssel, k1152);
            const uint4 bs = g < NC ? lds128(st + LY::X_OFF + g * XP_COL + XP_REC + 4 * (XP_S16 + 4 * c)) : make_uint4(0u, 0u, 0u, 0u);
            float dn[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(dn, p00, p10, p01, p11, bs.x, bs.y);
            mma16816(dn, p00, p10, p01, p11, bs.z, bs.w);
            const float mu0 = m_ok0 ? *reinterpret_cast<const float*>(st + LY::X_OFF + (2 * c) * XP_COL + XP_REC + 32) * 32768.f : 0.f;
            const float mu1 = m_ok1 ? *reinterpret_cast<const float*>(st + LY::X_OFF + (2 * c + 1) * XP_COL + XP_REC + 32) * 32768.f : 0.f;
            macc[0] = fmaf(dn[0], dd0 * mu0, macc[0]);
            macc[1] = fmaf(dn[1], dd0 * mu1, macc[1]);
            macc[2] = fmaf(dn[2], dd1 * mu0, macc[2]);
            macc[3] = fmaf(dn[3], dd1 * mu1, macc[3]);
        }
        __syncwarp();
        if (lane == 0 && j + LY::STAGES < njobs) {
            fence_proxy_async();
            issue_w(j + LY::STAGES, s);
            issue_x(j + LY::STAGES, s);
        }
    }
    if (PACK) {
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][g + 8 * (e >> 1)][2 * c + (e & 1)] = facc[0][e];
        if (c == 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e) red[warp][g + 8 * (e >> 1)][6 + (e & 1)] = macc[e];
        }
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = g + 8 * (e >> 1), col = 2 * c + (e & 1);
            if (col < NC) red[warp][row][col] = ((facc[0][e] + facc[ND > 1 ? 1 : 0][e]) + facc[ND > 2 ? 2 : 0][e]) - macc[e];
        }
    }
    __syncthreads();
    const int rl = threadIdx.x >> 3, col = threadIdx.x & 7;
    if (col < NC && rl < 16 && r0 + rl < rows) {
        float sum = 0.f;
#pragma unroll
        for (int wv = 0; wv < 8; ++wv) {
            const float v = PACK ? ((red[wv][rl][3 * col] + red[wv][rl][3 * col + 1]) + red[wv][rl][3 * col + 2]) - red[wv][rl][6 + col]
                                 : red[wv][rl][col];
            sum += v;
        }
        y[(int64_t)col * ldy + r0 + rl] = sum;
    }
}

// Repacks rows [0, rows) of a Q6_K matrix (row_bytes apart, nsb superblocks each) into the tile layout above; rows past
// the end of the last tile are zero. One CTA per tile.
__global__ void k_q6k_tile(const uint8_t* src, int rows, int nsb, int64_t row_bytes,
                           uint8_t* dst)
{
    pdl_trigger();
    pdl_wait();
    const int sb = blockIdx.x, rt = blockIdx.y;
    uint8_t* out = dst + ((int64_t)rt * nsb + sb) * Q6_TILE;
    for (int i = threadIdx.x; i < Q6_TILE; i += blockDim.x) {
        int r, off;
        if (i < Q6_QH) {
            r = i >> 7;
            const int pidx = i & 127, c = pidx >> 5, q = (pidx & 31) ^ ((r & 1) << 4);
            const int wi = q >> 2, b = q & 3, h = wi >> 2, kk = (wi >> 1) & 1, is = wi & 1;
            off = 64 * h + 32 * kk + 16 * is + 4 * c + b;
        } else if (i < Q6_SC) {
            r = (i - Q6_QH) >> 6;
            const int pidx = (i - Q6_QH) & 63, c = pidx >> 4, q = pidx & 15;
            const int wi = q >> 2, b = q & 3, h = wi >> 1, is = wi & 1;
            off = 128 + 32 * h + 16 * is + 4 * c + b;
        } else if (i < Q6_D) {
            r = (i - Q6_SC) >> 4;
            off = 192 + ((i - Q6_SC) & 15);
        } else {
            r = (i - Q6_D) >> 1;
            off = 208 + ((i - Q6_D) & 1);
        }
        const int row = rt * 16 + r;
        out[i] = row < rows ? src[(int64_t)row * row_bytes + (int64_t)sb * 210 + off] : (uint8_t)0;
    }
}

// ------------------------------------------------------------------------------------------------------------------
// the fused all-reduce's push for producers other than the Q4_K decode matvec
// ------------------------------------------------------------------------------------------------------------------
// Row blockIdx.y of src (E floats) into every rank's elements of all-reduce ao.idx, source ao.rank: a thread per two
// consecutive values, one 16-byte store per rank.
__global__ void __launch_bounds__(128) k_ar_push(const float* src, const ArOut ao)
{
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y, i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    const float2 v = *reinterpret_cast<const float2*>(src + (int64_t)t * ao.E + i);
    const unsigned long long q = ar_seq(ao.epoch, ao.idx);
    const uint32_t fl = ar_flag(q);
    const size_t off = ar_elem(q, ao.rank, t, ao.E) + i;
#pragma unroll
    for (int g = 0; g < AR_MAX_RANKS; ++g)
        if (g < ao.G) st_elem2(ao.ll[g] + off, v.x, v.y, fl);
}

// ------------------------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------------------------
size_t xprep_bytes(int cols, int nc) { return xprep_bytes_c(cols, nc); }

bool norm_prep_supported(int E) { return E % 256 == 0 && E <= 8192; }

void norm_prep(float* x, const float* o, float rs, int T, int E, const float* w, float eps, float* y, const XPrep* p,
               cudaStream_t s, const ArIn* ar, const MoeIn* moe)
{
    if (moe && (ar || !moe->y || !moe->sel || !moe->wts || moe->K < 1 || moe->K > 16))
        WL_THROW(WL_EINVAL, "norm_prep: the expert combine takes 1..16 experts per row and no all-reduce");
    if (T <= 0) return;
    if (!norm_prep_supported(E)) WL_THROW(WL_EUNSUPPORTED, "norm_prep: the row length must be a multiple of 256, at most 8192");
    if (p && (p->cols != E || p->nc != T)) WL_THROW(WL_EINVAL, "norm_prep: prepared-activation view does not match");
    ArIn in{};
    if (ar) {
        if (ar->E != E || ar->row0 < 0 || ar->row0 + T > AR_COLS || ar->G < 1 || ar->G > AR_MAX_RANKS || ar->rank < 0 ||
            ar->rank >= ar->G || ar->idx < 0 || ar->idx >= AR_STEP)
            WL_THROW(WL_EINVAL, "norm_prep: all-reduce slot does not match");
        in = *ar;
    }
    uint8_t* pb = p ? p->blocks : nullptr;
    // a cluster of C CTAs per row, C the largest divisor of the row's superblock count up to 8 (the portable cluster
    // size), each CTA a warp per superblock
    const int nsb = E / 256;
    int C = 1;
    for (int c = 8; c >= 1; --c)
        if (nsb % c == 0) { C = c; break; }
    const dim3 grid(C, T), block(32 * (nsb / C));
    const MoeIn mi = moe ? *moe : MoeIn{};
    if (moe) {
        if (p) launch_cluster(k_norm_prep<true, true, true>, grid, block, 0, s, C, x, o, rs, E, w, eps, y, pb, in, mi);
        else launch_cluster(k_norm_prep<true, false, true>, grid, block, 0, s, C, x, o, rs, E, w, eps, y, pb, in, mi);
    } else if (o || ar) {
        if (p) launch_cluster(k_norm_prep<true, true, false>, grid, block, 0, s, C, x, o, rs, E, w, eps, y, pb, in, mi);
        else launch_cluster(k_norm_prep<true, false, false>, grid, block, 0, s, C, x, o, rs, E, w, eps, y, pb, in, mi);
    } else {
        if (p) launch_cluster(k_norm_prep<false, true, false>, grid, block, 0, s, C, x, o, rs, E, w, eps, y, pb, in, mi);
        else launch_cluster(k_norm_prep<false, false, false>, grid, block, 0, s, C, x, o, rs, E, w, eps, y, pb, in, mi);
    }
    note_launch();
}

int selftest_ar_wait(long long wait_ns)
{
    // one row of 256 values, the all-reduce of two ranks where this GPU is rank 0 and rank 1 never runs: rank 0 pushes
    // its own elements of the current sequence number (epoch 1, index 0) into its buffer, and the consumer's wait for
    // rank 1's elements can only run out
    const int E = 256;
    const size_t arb = ar_buffer_bytes(E);
    uint8_t* buf = nullptr;
    float *x = nullptr, *w = nullptr, *y = nullptr;
    int* err = nullptr;
    int code = -1;
    WL_CUDA(cudaMalloc(&buf, arb));
    try {
        WL_CUDA(cudaMalloc(&x, 3 * E * sizeof(float)));
        w = x + E;
        y = w + E;
        WL_CUDA(cudaMalloc(&err, sizeof(int)));
        WL_CUDA(cudaMemset(buf, 0, arb));
        WL_CUDA(cudaMemset(x, 0, 3 * E * sizeof(float)));
        WL_CUDA(cudaMemset(err, 0, sizeof(int)));
        const unsigned long long epoch = 1;
        WL_CUDA(cudaMemcpy(buf + AR_EPOCH, &epoch, sizeof epoch, cudaMemcpyHostToDevice));
        unsigned long long* ll = reinterpret_cast<unsigned long long*>(buf + ar_ll_offset(E));
        ArOut out{};
        out.ll[0] = ll;
        out.epoch = reinterpret_cast<const unsigned long long*>(buf + AR_EPOCH);
        out.idx = 0; out.G = 1; out.rank = 0; out.E = E;
        ar_push(x, 1, out, 0);
        ArIn in{};
        in.ll = ll;
        in.epoch = out.epoch;
        in.err = err;
        in.idx = 0; in.G = 2; in.rank = 0; in.E = E; in.row0 = 0;
        in.wait_ns = wait_ns;
        norm_prep(x, nullptr, 1.0f, 1, E, w, 1e-5f, y, nullptr, 0, &in);
        WL_CUDA(cudaDeviceSynchronize());
        WL_CUDA(cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost));
    } catch (...) {
        cudaFree(buf); if (x) cudaFree(x); if (err) cudaFree(err);
        throw;
    }
    cudaFree(buf); cudaFree(x); cudaFree(err);
    return code;
}

void ar_push(const float* src, int T, const ArOut& ao, cudaStream_t s)
{
    if (T <= 0) return;
    if (T > AR_COLS || ao.G < 1 || ao.G > AR_MAX_RANKS || ao.rank < 0 || ao.rank >= ao.G || ao.E % 256 != 0 ||
        ao.idx < 0 || ao.idx >= AR_STEP)
        WL_THROW(WL_EINVAL, "ar_push: all-reduce slot does not match");
    launch(k_ar_push, dim3(ao.E / 256, T), dim3(128), 0, s, src, ao);
    note_launch();
}

XPrep xprep_view(void* scratch, int cols, int nc)
{
    XPrep p;
    p.blocks = (uint8_t*)scratch;
    p.cols = cols;
    p.nc = nc;
    return p;
}

void xprep(const float* x, int64_t ldx, int cols, int nc, const XPrep& p, cudaStream_t s)
{
    launch(k_xprep, dim3(dim3(cols / 256, nc)), dim3(64), 0, s, x, ldx, cols / 256, p.blocks);
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

// Raises a kernel's dynamic shared-memory limit once per device; `done` is that kernel's own per-device flags (one
// set per template instantiation, so kernels of the same signature do not share them). Safe from several host threads.
template <typename Kernel>
static void ensure_smem_attr(Kernel kernel, int bytes, std::atomic<bool> (&done)[64])
{
    static std::mutex mu;
    int dev = 0;
    WL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) WL_THROW(WL_EINVAL, "device ordinal out of range");
    if (done[dev].load(std::memory_order_acquire)) return;
    std::lock_guard<std::mutex> lock(mu);
    if (done[dev].load(std::memory_order_relaxed)) return;
    WL_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[dev].store(true, std::memory_order_release);
}

template <int NC, bool TILED, bool PAIRS, int NW = 8, bool AR = false> struct Q4Attr {
    static std::atomic<bool> done[64];
    static void ensure() { ensure_smem_attr(k_mmv_q4k<NC, TILED, PAIRS, NW, AR>, Q4Layout<NC, NW>::SMEM, done); }
};
template <int NC, bool TILED, bool PAIRS, int NW, bool AR> std::atomic<bool> Q4Attr<NC, TILED, PAIRS, NW, AR>::done[64];
template <int NC> struct Q6Attr {
    static std::atomic<bool> done[64];
    static void ensure() { ensure_smem_attr(k_mmv_q6k<NC>, Q6Layout<NC>::SMEM, done); }
};
template <int NC> std::atomic<bool> Q6Attr<NC>::done[64];

static int sm_count();

// The persistent form's grid: as many CTAs as fit on the GPU at once (per device, from the occupancy query), at most
// one per tile pair.
template <int NC, int NW> struct Q4AttrP {
    static std::atomic<bool> done[64];
    static std::atomic<int> per_sm[64];
    static int ensure()
    {
        ensure_smem_attr(k_mmv_q4kp<NC, NW>, Q4LayoutP<NC, NW>::SMEM, done);
        int dev = 0;
        WL_CUDA(cudaGetDevice(&dev));
        int n = per_sm[dev].load(std::memory_order_relaxed);
        if (!n) {
            WL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_mmv_q4kp<NC, NW>, 32 * NW, Q4LayoutP<NC, NW>::SMEM));
            if (n < 1) WL_THROW(WL_ECUDA, "matvec: the persistent Q4_K kernel does not fit an SM");
            per_sm[dev].store(n, std::memory_order_relaxed);
        }
        return n;
    }
};
template <int NC, int NW> std::atomic<bool> Q4AttrP<NC, NW>::done[64];
template <int NC, int NW> std::atomic<int> Q4AttrP<NC, NW>::per_sm[64];

template <int NC, int NW>
static void launch_q4kp(const uint8_t* tiles, int row_base, int rows, int nsb, const XPrep& p, float* y, int64_t ldy,
                        int* err, cudaStream_t s, const MvSeg& seg)
{
    const int per_sm = Q4AttrP<NC, NW>::ensure();
    const int pairs = ((rows + Q4_ROWS - 1) / Q4_ROWS + 1) / 2 + (seg.wt ? ((seg.rows + Q4_ROWS - 1) / Q4_ROWS + 1) / 2 : 0);
    const int grid = std::max(1, std::min(pairs, sm_count() * per_sm));
    launch(k_mmv_q4kp<NC, NW>, dim3(grid), dim3(32 * NW), Q4LayoutP<NC, NW>::SMEM, s, tiles, row_base, rows, nsb,
           (const uint8_t*)p.blocks, y, ldy, err, seg);
    note_launch();
}

template <int NC, bool TILED, bool PAIRS = false, int NW = 8>
static void launch_q4k(const CUtensorMap& m, const uint8_t* tiles, int row_base, int rows, int nsb, const XPrep& p,
                       float* y, int64_t ldy, int* err, cudaStream_t s, const MvSeg& seg, const ArOut& ao = ArOut{})
{
    if constexpr (TILED && !PAIRS && NC >= 6) {
        // six or more columns on tile-major weights: the persistent paired-tile form (same bits per row; measured on
        // 8192 x 8192: 16.4 against 20.0 us at 8 columns, while at 3 and 4 columns, where the 16-row form fits two
        // CTAs an SM and this one a single, 15.6 against 13.5 us)
        if (ao.G == 0 && !seg.sel) {
            launch_q4kp<NC, NW>(tiles, row_base, rows, nsb, p, y, ldy, err, s, seg);
            return;
        }
    }
    if (TILED && !PAIRS && ao.G > 0) {
        // the fused all-reduce's producer: its own instantiation, so the one-GPU kernels keep their register allocation
        Q4Attr<NC, true, false, NW, true>::ensure();
        launch(k_mmv_q4k<NC, true, false, NW, true>, dim3((rows + Q4_ROWS - 1) / Q4_ROWS), dim3(32 * NW),
               Q4Layout<NC, NW>::SMEM, s, m, tiles, row_base, rows, nsb, (const uint8_t*)p.blocks, y, ldy, err, seg, ao);
        note_launch();
        return;
    }
    Q4Attr<NC, TILED, PAIRS, NW>::ensure();
    const int ctas = seg.sel ? seg.tiles_per_pair * seg.first_ctas * (seg.wt ? 2 : 1)
                             : (rows + Q4_ROWS - 1) / Q4_ROWS + (seg.wt ? (seg.rows + Q4_ROWS - 1) / Q4_ROWS : 0);
    if (PAIRS != (seg.sel != nullptr)) WL_THROW(WL_EINVAL, "matvec: the grouped-expert form needs the expert ids");
    launch(k_mmv_q4k<NC, TILED, PAIRS, NW>, dim3(ctas), dim3(32 * NW), Q4Layout<NC, NW>::SMEM, s, m, tiles, row_base,
           rows, nsb, (const uint8_t*)p.blocks, y, ldy, err, seg, ao);
    note_launch();
}

template <bool TILED, int NW = 8>
static void dispatch_q4k(const CUtensorMap& m, const uint8_t* tiles, int row_base, int rows, int nsb, const XPrep& p,
                         float* y, int64_t ldy, int* err, cudaStream_t s, const MvSeg& seg, const ArOut& ao = ArOut{})
{
    switch (p.nc) {
    case 1: launch_q4k<1, TILED, false, NW>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao); break;
    case 2: launch_q4k<2, TILED, false, NW>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao); break;
    case 3: launch_q4k<3, TILED, false, NW>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao); break;
    case 4: launch_q4k<4, TILED, false, NW>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao); break;
    case 5: launch_q4k<5, TILED, false, NW>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao); break;
    case 6: launch_q4k<6, TILED, false, NW>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao); break;
    case 7: launch_q4k<7, TILED, false, NW>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao); break;
    default: launch_q4k<8, TILED, false, NW>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao); break;
    }
}

// The GPU's SM count (per process, from the current device).
static int sm_count()
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

// The model's decode matvec on tile-major Q4_K: one 16-row CTA per row tile. In a decode step every matvec follows a
// small kernel, and CTAs this size start under programmatic dependent launch while that kernel still runs (four fit
// beside it on an SM) and stream their first stages meanwhile; a 32-row form (a warp on two tiles of the same
// superblocks), faster back to back, lost 6 % of the 70B step for that reason and was dropped. Eight warps per CTA for up to 8 x SMs row tiles at one or two columns; four warps
// (twice the superblocks per warp, twice the CTAs per SM) for taller matrices. The warp count fixes how a row's
// superblocks are grouped and added, so it depends on the matrix alone, never on the column count: a decode step's
// rows then equal single-sequence steps bit for bit. (An earlier version took four warps for every matrix from three
// columns on, 8 % faster at 8 columns, but its 8192-row matrices then grouped a row's superblocks by four where a
// single-sequence step groups them by eight.)
static void dispatch_q4k16(const CUtensorMap& m, const uint8_t* tiles, int row_base, int rows, int nsb, const XPrep& p,
                           float* y, int64_t ldy, int* err, cudaStream_t s, const MvSeg& seg, const ArOut& ao = ArOut{})
{
    const int tiles_n = (rows + Q4_ROWS - 1) / Q4_ROWS + (seg.wt ? (seg.rows + Q4_ROWS - 1) / Q4_ROWS : 0);
    const int nw = tiles_n >= 8 * sm_count() ? 4 : 8;
    if (nw == 4)
        dispatch_q4k<true, 4>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao);
    else
        dispatch_q4k<true, 8>(m, tiles, row_base, rows, nsb, p, y, ldy, err, s, seg, ao);
}

void prepare_matvec_mma()
{
    Q4Attr<1, false, false>::ensure();
    Q4Attr<2, false, false>::ensure();
    Q4Attr<3, false, false>::ensure();
    Q4Attr<4, false, false>::ensure();
    Q4Attr<5, false, false>::ensure();
    Q4Attr<6, false, false>::ensure();
    Q4Attr<7, false, false>::ensure();
    Q4Attr<8, false, false>::ensure();
}

void matvec_mma(int type, const WeightMap& map, int row_base, int rows, int cols, const XPrep& p, float* y, int64_t ldy,
                int* err, cudaStream_t s)
{
    (void)type;
    dispatch_q4k<false>(*reinterpret_cast<const CUtensorMap*>(map.bytes), nullptr, row_base, rows, cols / 256, p, y,
                        ldy, err, s, MvSeg{nullptr, 0, 0, INT_MAX, nullptr, 0, nullptr, 0, 1, 0});
}


bool tiles_supported(int type, int cols)
{
    return ((type == 12 || type == 14) && cols % 256 == 0) || i8_tiles_supported(type, cols);
}

int64_t tile_bytes(int type, int rows, int cols)
{
    if (i8_tiles_supported(type, cols)) return i8_tile_bytes(type, rows, cols);
    return (int64_t)((rows + 15) / 16) * (cols / 256) * (type == 12 ? Q4_TILE : Q6_TILE);
}

void make_tiles(int type, const uint8_t* w, int rows, int cols, int64_t row_bytes, uint8_t* tiles, cudaStream_t s)
{
    if (i8_tiles_supported(type, cols)) {
        make_i8_tiles(type, w, rows, cols, row_bytes, tiles, s);
        return;
    }
    if (!tiles_supported(type, cols)) WL_THROW(WL_EUNSUPPORTED, "make_tiles: no tile layout for this type");
    if (row_bytes < (int64_t)(cols / 256) * (type == 12 ? 144 : 210)) WL_THROW(WL_EINVAL, "make_tiles: bad row size");
    if (rows <= 0) return;
    const dim3 grid(cols / 256, (rows + 15) / 16);
    if (type == 12) launch(k_q4k_tile, grid, dim3(256), 0, s, w, rows, cols / 256, row_bytes, tiles);
    else launch(k_q6k_tile, grid, dim3(256), 0, s, w, rows, cols / 256, row_bytes, tiles);
    note_launch();
}

template <int NC>
static void launch_q6k(const uint8_t* tiles, int rows, int nsb, const XPrep& p, float* y, int64_t ldy, int* err,
                       cudaStream_t s)
{
    Q6Attr<NC>::ensure();
    launch(k_mmv_q6k<NC>, dim3((rows + 15) / 16), dim3(256), Q6Layout<NC>::SMEM, s, tiles, rows, nsb,
           (const uint8_t*)p.blocks, y, ldy, err);
    note_launch();
}

static void matvec_q6k(const uint8_t* tiles, int rows, int cols, const XPrep& p, float* y, int64_t ldy, int* err,
                       cudaStream_t s)
{
    const int nsb = cols / 256;
    switch (p.nc) {
    case 1: launch_q6k<1>(tiles, rows, nsb, p, y, ldy, err, s); break;
    case 2: launch_q6k<2>(tiles, rows, nsb, p, y, ldy, err, s); break;
    case 3: launch_q6k<3>(tiles, rows, nsb, p, y, ldy, err, s); break;
    case 4: launch_q6k<4>(tiles, rows, nsb, p, y, ldy, err, s); break;
    case 5: launch_q6k<5>(tiles, rows, nsb, p, y, ldy, err, s); break;
    case 6: launch_q6k<6>(tiles, rows, nsb, p, y, ldy, err, s); break;
    case 7: launch_q6k<7>(tiles, rows, nsb, p, y, ldy, err, s); break;
    default: launch_q6k<8>(tiles, rows, nsb, p, y, ldy, err, s); break;
    }
}

void matvec_tiles2(const uint8_t* tiles_a, int row_base_a, int rows_a, float* y_a, int64_t ldy_a, const uint8_t* tiles_b,
                   int row_base_b, int rows_b, float* y_b, int64_t ldy_b, int cols, const XPrep& p, int* err,
                   cudaStream_t s)
{
    if ((uintptr_t)tiles_a % 16 != 0 || (uintptr_t)tiles_b % 16 != 0 || row_base_a % 16 != 0 || row_base_b % 16 != 0)
        WL_THROW(WL_EINVAL, "matvec_tiles2: misaligned tiles");
    if (!tiles_supported(12, cols)) WL_THROW(WL_EUNSUPPORTED, "matvec_tiles2: Q4_K with cols a multiple of 256 only");
    CUtensorMap none;
    memset(&none, 0, sizeof none);
    const MvSeg seg{tiles_b, row_base_b, rows_b, (rows_a + Q4_ROWS - 1) / Q4_ROWS, y_b, ldy_b, nullptr, 0, 1, 0};
    dispatch_q4k16(none, tiles_a, row_base_a, rows_a, cols / 256, p, y_a, ldy_a, err, s, seg);
}

void matvec_pairs(const uint8_t* tiles, int row_base, int expert_rows, int cols, const int32_t* sel, int npairs, int K,
                  bool x_per_token, const XPrep& p, float* y, int64_t ldy, int* err, cudaStream_t s, int e_lo, int e_n)
{
    if ((uintptr_t)tiles % 16 != 0 || row_base % 16 != 0 || expert_rows % 16 != 0)
        WL_THROW(WL_EINVAL, "matvec_pairs: experts must start on 16-row tiles");
    if (!tiles_supported(12, cols) || p.cols != cols) WL_THROW(WL_EUNSUPPORTED, "matvec_pairs: Q4_K with matching activations only");
    if (npairs <= 0) return;
    if (x_per_token ? (npairs + K - 1) / K > p.nc : npairs > p.nc) WL_THROW(WL_EINVAL, "matvec_pairs: too few activation columns");
    CUtensorMap none;
    memset(&none, 0, sizeof none);
    const int tiles_per_pair = expert_rows / Q4_ROWS;
    // first_ctas carries the pair count (the CTA count is pairs x tiles per pair)
    const MvSeg seg{nullptr, 0, 0, npairs, nullptr, 0, sel, K, tiles_per_pair, x_per_token ? 1 : 0, e_lo, e_n};
    launch_q4k<1, true, true>(none, tiles, row_base, expert_rows, cols / 256, p, y, ldy, err, s, seg);
}

void matvec_pairs2(const uint8_t* tiles_a, const uint8_t* tiles_b, int expert_rows, int cols, const int32_t* sel,
                   int npairs, int K, const XPrep& p, float* ya, float* yb, int64_t ldy, int* err, cudaStream_t s,
                   int e_lo, int e_n)
{
    if ((uintptr_t)tiles_a % 16 != 0 || (uintptr_t)tiles_b % 16 != 0 || expert_rows % 16 != 0)
        WL_THROW(WL_EINVAL, "matvec_pairs2: experts must start on 16-row tiles");
    if (!tiles_supported(12, cols) || p.cols != cols) WL_THROW(WL_EUNSUPPORTED, "matvec_pairs2: Q4_K with matching activations only");
    if (npairs <= 0) return;
    if ((npairs + K - 1) / K > p.nc) WL_THROW(WL_EINVAL, "matvec_pairs2: too few activation columns");
    CUtensorMap none;
    memset(&none, 0, sizeof none);
    const int tiles_per_pair = expert_rows / Q4_ROWS;
    const MvSeg seg{tiles_b, 0, expert_rows, npairs, yb, ldy, sel, K, tiles_per_pair, 1, e_lo, e_n};
    launch_q4k<1, true, true>(none, tiles_a, 0, expert_rows, cols / 256, p, ya, ldy, err, s, seg);
}

void matvec_tiles(int type, const uint8_t* tiles, int row_base, int rows, int cols, const XPrep& p, float* y,
                  int64_t ldy, int* err, cudaStream_t s, const ArOut* ao)
{
    if ((uintptr_t)tiles % 16 != 0 || row_base % 16 != 0) WL_THROW(WL_EINVAL, "matvec_tiles: misaligned tiles");
    if (!tiles_supported(type, cols)) WL_THROW(WL_EUNSUPPORTED, "matvec_tiles: no tile layout for this type");
    if (ao && (type != 12 || ao->G < 1 || ao->G > AR_MAX_RANKS || ao->rank < 0 || ao->rank >= ao->G ||
               ao->E != rows || p.nc > AR_COLS || ao->idx < 0 || ao->idx >= AR_STEP))
        WL_THROW(WL_EINVAL, "matvec_tiles: the all-reduce push does not match");
    if (i8_tiles_supported(type, cols)) {
        const int64_t tb = i8_tile_bytes(type, 16, cols);
        matvec_i8_tiles(type, tiles + (int64_t)(row_base / 16) * tb, rows, cols, p, y, ldy, err, s);
        return;
    }
    if (type == 12) {
        CUtensorMap none;
        memset(&none, 0, sizeof none);
        dispatch_q4k16(none, tiles, row_base, rows, cols / 256, p, y, ldy, err, s,
                       MvSeg{nullptr, 0, 0, INT_MAX, nullptr, 0, nullptr, 0, 1, 0}, ao ? *ao : ArOut{});
    } else {
        matvec_q6k(tiles + (int64_t)(row_base / 16) * (cols / 256) * Q6_TILE, rows, cols, p, y, ldy, err, s);
    }
}

}  // namespace k
}  // namespace wl
