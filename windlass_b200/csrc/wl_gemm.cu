// Prefill / batched GEMM for Q4_K weights on the 5th-generation tensor cores (tcgen05, sm_100a):
// y[t*ldy + r] = W[r] . x[t] for T > 8 activation rows (FastMath.Block's job in the reference, src/FastMath.cs:218-264).
//
// One CTA computes a 128-row x BN-token tile of y (BN = 128, or 256 for Q4_K prompts of more than 128 rows, so that
// each weight is dequantized once per 256 tokens); its fp32 accumulator lives in tensor memory (BN TMEM columns).
// Per K step of 64 values, in a shared-memory ring (3 stages of 64 KB at BN = 128, 2 of 96 KB at 256) fed by a
// 4-stage ring of raw weights:
//   - one warp copies the step's raw Q4_K bytes of the CTA's eight 16-row tiles (each tile's 256 header bytes and the
//     512 code bytes of the step's 64 values) into the raw ring with 1-D bulk copies, ahead of their use;
//   - 8 dequantizing warps read those bytes from shared memory (two threads per row, one 32-value sub-block each),
//     rebuild every weight exactly as the reference does (d1 = d*s, m1 = dmin*m, w = d1*q - m1, each rounded in fp32)
//     and store it as two bf16 planes, w_hi = bf16(w) and w_lo = bf16(w - w_hi), in the 128-byte-swizzled K-major
//     layout the MMA reads;
//   - one warp loads the tokens' bf16 planes x_hi, x_lo (written by k_split_bf16) with 2-D TMA copies (no multicast);
//   - one thread issues tcgen05.mma kind::f16 (bf16 x bf16 -> fp32) per 16-value slice:
//     w_hi.x_hi + w_hi.x_lo + w_lo.x_hi. The dropped w_lo.x_lo term is below 2^-16 of each product, so the result
//     carries fp32-level accuracy (a plain bf16 GEMM would carry 2^-9 relative error per weight);
//   - tcgen05.commit frees each stage when its MMAs have read it; a final commit releases the epilogue.
// The four epilogue warps (warp w owns TMEM lanes 32w..32w+31 = tile rows) read the accumulator with tcgen05.ld and
// store y rows, coalesced along the weight rows. Every wait is bounded: a stuck wait records a code in *err (host:
// WL_ETIMEDOUT) and the kernel runs on to its TMEM release and returns.
#include <cstdint>
#include <cstring>
#include <mutex>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include "wl_common.h"
#include "wl_kernels.h"
#include "wl_launch.cuh"

namespace wl {
namespace k {

namespace {

constexpr int G_BM = 128;                  // weight rows per CTA (MMA M)
constexpr int G_BK = 64;                   // values per K step: one 128-byte swizzle atom of bf16
constexpr int G_A_BYTES = G_BM * G_BK * 2;             // one bf16 plane of the weight tile: 16 KB
template <int BN> constexpr int g_b_bytes() { return BN * G_BK * 2; }                 // one bf16 plane: 16 or 32 KB
template <int BN> constexpr int g_stage() { return 2 * G_A_BYTES + 2 * g_b_bytes<BN>(); } // 64 or 96 KB
constexpr int G_DQ_WARPS = 8, G_TMA_WARP = 8, G_RAW_WARP = 9, G_MMA_WARP = 10, G_THREADS = 352;
constexpr int Q4T = 2304;                               // bytes of a 16-row x one-superblock Q4_K tile
constexpr int Q6T = 3360;                               // bytes of a 16-row x one-superblock Q6_K tile

// Per weight format: the A/B ring depth and the raw ring. Q4_K stages one K step of each 16-row tile at a time (its
// 256 header bytes and the step's 512 code bytes); Q6_K stages whole tiles (one superblock = four K steps), its
// quarter-superblock bytes being interleaved across the tile for the matvec's fragment reads.
template <int WT, int BN> struct GemmFmt;
template <int BN> struct GemmFmt<12, BN> {
    static constexpr int STAGES = BN == 128 ? 3 : 2, RAW_STAGES = 4, STEPS_PER_RAW = 1;
    static constexpr int RAW_TILE = 256 + 512, TILE = Q4T;
    static constexpr int RAW_STAGE = (G_BM / 16) * RAW_TILE;                          // 6 KB
    static constexpr int SMEM = STAGES * g_stage<BN>() + RAW_STAGES * RAW_STAGE + 1024; // + 1024-byte alignment slack
};
template <int BN> struct GemmFmt<14, BN> {
    static_assert(BN == 128, "Q6_K's whole-tile raw ring leaves room for 128-token stages only");
    static constexpr int STAGES = 2, RAW_STAGES = 2, STEPS_PER_RAW = 4;
    static constexpr int RAW_TILE = Q6T, TILE = Q6T;
    static constexpr int RAW_STAGE = (G_BM / 16) * RAW_TILE;                          // 26.25 KB
    static constexpr int SMEM = STAGES * g_stage<BN>() + RAW_STAGES * RAW_STAGE + 1024;
};
static_assert(GemmFmt<12, 256>::SMEM <= 227 * 1024, "Q4_K 256-token stages must fit one CTA's shared memory");

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long gtime_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded by time: gives up after 2 s of %globaltimer (a poll may return well before its sleep hint, so the limit is
// not a poll count), records `code` in *err and raises the CTA's abort flag, after which every later wait of the CTA
// returns at once, so a broken pipeline ends in seconds, not minutes, and a slow one never gives up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort)
{
    if (*abort) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtime_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (gtime_ns() - t0 > 2000000000ull) {
            atomicExch(err, code);
            *abort = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

// Shared-memory matrix descriptor (sm100): K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc(const void* p)
{
    const uint64_t addr = smem_u32(p);
    return ((addr & 0x3FFFFull) >> 4)        // start address, 16-byte units
           | (1ull << 16)                    // leading byte offset (unused for swizzled K-major; canonical 1)
           | ((1024ull >> 4) << 32)          // stride byte offset: next 8-row group
           | (1ull << 46)                    // descriptor version (sm100)
           | (2ull << 61);                   // layout: 128-byte swizzle
}

// Instruction descriptor: kind::f16, A and B bf16, D fp32, both K-major, M = 128, N = BN.
template <int BN> constexpr uint32_t g_idesc()
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(G_BM >> 4) << 24);
}

template <int BN>
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate)
{
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                 ::"r"(tmem_d), "l"(a), "l"(b), "r"(g_idesc<BN>()), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }

// The 64 fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64])
{
    uint32_t r[64];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,"
                 "%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,"
                 "%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
                   "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
                   "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
                   "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
                   "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Two weights to their bf16 hi and lo planes, packed as element pairs (lower address first).
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo)
{
    const __nv_bfloat16 ah = __float2bfloat16_rn(a), bh = __float2bfloat16_rn(b);
    const __nv_bfloat16 al = __float2bfloat16_rn(__fsub_rn(a, __bfloat162float(ah)));
    const __nv_bfloat16 bl = __float2bfloat16_rn(__fsub_rn(b, __bfloat162float(bh)));
    hi = (uint32_t)__bfloat16_as_ushort(ah) | ((uint32_t)__bfloat16_as_ushort(bh) << 16);
    lo = (uint32_t)__bfloat16_as_ushort(al) | ((uint32_t)__bfloat16_as_ushort(bl) << 16);
}

template <int WT, int BN>
__global__ void __launch_bounds__(G_THREADS, 1) k_gemm(const __grid_constant__ CUtensorMap xh_map,
                                                            const __grid_constant__ CUtensorMap xl_map,
                                                            const uint8_t* __restrict__ tiles, int row_base, int rows,
                                                            int nsb, int T, float* __restrict__ y, int64_t ldy, int* err)
{
    using F = GemmFmt<WT, BN>;
    constexpr int G_STAGES = F::STAGES, G_RAW_STAGES = F::RAW_STAGES, G_RAW_STAGE = F::RAW_STAGE;
    constexpr int G_STAGE = g_stage<BN>(), G_B_BYTES = g_b_bytes<BN>();
    constexpr int G_TMEM_COLS = BN;             // the fp32 accumulator: BN columns x 128 lanes
    constexpr int SPR = F::STEPS_PER_RAW;
    extern __shared__ uint8_t g_smem_raw[];
    __shared__ __align__(8) uint64_t full_a[G_STAGES], full_b[G_STAGES], empty[G_STAGES], acc_full;
    __shared__ __align__(8) uint64_t raw_full[G_RAW_STAGES], raw_empty[G_RAW_STAGES];
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    uint8_t* smem = (uint8_t*)(((uintptr_t)g_smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* raw = smem + G_STAGES * G_STAGE;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * G_BM, n0 = blockIdx.y * BN;
    const int nk = nsb * 4;                 // K steps of 64 values
    // 16-row weight tiles of this CTA that exist (the last CTA of a matrix may have fewer than eight)
    const int live_tiles = min(G_BM / 16, (rows + 15) / 16 - m0 / 16);

    if (threadIdx.x == 0) {
        for (int s = 0; s < G_STAGES; ++s) {
            mbar_init(&full_a[s], G_DQ_WARPS * 32);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < G_RAW_STAGES; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], G_DQ_WARPS * 32);
        }
        mbar_init(&acc_full, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {                        // the accumulator: BN TMEM columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_base)), "r"(G_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp < G_DQ_WARPS) {
        // ---- dequantizers: thread -> (row m, half h); per K step 32 values of the row: 32h .. 32h+31
        const int t = threadIdx.x, m = t >> 1, h = t & 1;
        const bool live = (m >> 4) < live_tiles;
        const int r16 = m & 15, tile_off = (m >> 4) * F::RAW_TILE;
        const int swz = m & 7;
        uint8_t* arow = smem + (m >> 3) * 1024 + swz * 128;
        for (int i = 0; i < nk; ++i) {
            const int s = i % G_STAGES, rstep = i / SPR, rs = rstep % G_RAW_STAGES;
            const int p = i & 3;
            uint32_t hi[16], lo[16];
            if (i % SPR == 0) mbar_wait(&raw_full[rs], (uint32_t)((rstep / G_RAW_STAGES) & 1), err, 16, &abort_flag);
            const uint8_t* rb = raw + rs * G_RAW_STAGE + tile_off;
            float wv[32];
            if (WT == 12) {
                // Q4_K (src/Quants.cs:333-350): the step's run of the row holds values 64p .. 64p+63; this thread's
                // 32 are sub-block 2p+h (low nibbles for h = 0, high for h = 1) of code bytes 32p .. 32p+31
                uint4 hv = make_uint4(0u, 0u, 0u, 0u);
                uint2 cv[4] = {};
                if (live) {
                    hv = *reinterpret_cast<const uint4*>(rb + r16 * 16);
                    const int code = 256 + ((r16 & 7) * 4) * 16 + (r16 >> 3) * 8;
#pragma unroll
                    for (int c = 0; c < 4; ++c) cv[c] = *reinterpret_cast<const uint2*>(rb + code + c * 16);
                }
                // ScaleMinK4 (src/Quants.cs:322-330) of sub-block j = 2p + h; scale byte b is byte b & 3 of word
                // hv.y / hv.z / hv.w for b in 0-3 / 4-7 / 8-11
                const int j = 2 * p + h, sh8 = 8 * (j & 3);
                int s6, m6;
                if (j < 4) {
                    s6 = (int)((hv.y >> sh8) & 63u);
                    m6 = (int)((hv.z >> sh8) & 63u);
                } else {
                    const uint32_t bj4 = (hv.w >> sh8) & 0xFFu, bjm4 = (hv.y >> sh8) & 0xFFu, bj = (hv.z >> sh8) & 0xFFu;
                    s6 = (int)((bj4 & 0xFu) | ((bjm4 >> 6) << 4));
                    m6 = (int)((bj4 >> 4) | ((bj >> 6) << 4));
                }
                const float d1 = __fmul_rn(h2f(hv.x & 0xFFFF), (float)s6), mm1 = __fmul_rn(h2f(hv.x >> 16), (float)m6);
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int b = 0; b < 8; ++b) {
                        const uint32_t word = b < 4 ? cv[c].x : cv[c].y;
                        const int q = (int)((word >> (8 * (b & 3) + (h ? 4 : 0))) & 15u);
                        wv[c * 8 + b] = __fsub_rn(__fmul_rn(d1, (float)q), mm1);
                    }
            } else {
                // Q6_K (src/Quants.cs:373-396): the step covers quarters 2(p&1), 2(p&1)+1 of half k = p/2; this
                // thread's 32 values are quarter Q = 2(p&1) + h: value l (0..31) has the low code bits in nibble p&1
                // of ql byte 64k + 32h + l, the high two in bits 2Q of qh byte 32k + l, the scale sc[8k + l/16 + 2Q].
                // In the tile, ql byte 64k + 32kk + 16is + 4c + b of row r is at r*128 + c*32 + 4*((4k + 2kk + is)
                // ^ 4(r&1)) + b, qh byte 32k + 16is + 4c + b at 2048 + r*64 + c*16 + 4*(2k + is) + b.
                const int k = p >> 1, Q = 2 * (p & 1) + h;
                uint32_t qlw[2][4] = {}, qhw[2][4] = {};
                int sc0 = 0, sc1 = 0;
                float d = 0.f;
                if (live) {
#pragma unroll
                    for (int is = 0; is < 2; ++is)
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            qlw[is][c] = *reinterpret_cast<const uint32_t*>(rb + r16 * 128 + c * 32 + 4 * ((4 * k + 2 * h + is) ^ ((r16 & 1) << 2)));
                            qhw[is][c] = *reinterpret_cast<const uint32_t*>(rb + 2048 + r16 * 64 + c * 16 + 4 * (2 * k + is));
                        }
                    const int8_t* sc = reinterpret_cast<const int8_t*>(rb + 3072 + r16 * 16 + 8 * k + 2 * Q);
                    sc0 = sc[0];
                    sc1 = sc[1];
                    d = h2f(*reinterpret_cast<const uint16_t*>(rb + 3328 + r16 * 2));
                }
                const float ds[2] = {__fmul_rn(d, (float)sc0), __fmul_rn(d, (float)sc1)};
#pragma unroll
                for (int is = 0; is < 2; ++is)
#pragma unroll
                    for (int c = 0; c < 4; ++c)
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const int lo4 = (int)((qlw[is][c] >> (8 * b + 4 * (p & 1))) & 15u);
                            const int hi2 = (int)((qhw[is][c] >> (8 * b + 2 * Q)) & 3u);
                            wv[16 * is + 4 * c + b] = __fmul_rn(ds[is], (float)((lo4 | (hi2 << 4)) - 32));
                        }
            }
            if (i >= G_STAGES) mbar_wait(&empty[s], (uint32_t)(((i / G_STAGES) + 1) & 1), err, 11, &abort_flag);
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                if (live) split2(wv[2 * q], wv[2 * q + 1], hi[q], lo[q]);
                else hi[q] = lo[q] = 0u;
            }
            // values 32h .. 32h+31 of the row: 16-byte chunks 4h .. 4h+3, swizzled by the row within its 8-row group
            uint8_t* ah = arow + (size_t)s * G_STAGE;
            uint8_t* al = ah + G_A_BYTES;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int chunk = (4 * h + c) ^ swz;
                *reinterpret_cast<uint4*>(ah + chunk * 16) = make_uint4(hi[4 * c], hi[4 * c + 1], hi[4 * c + 2], hi[4 * c + 3]);
                *reinterpret_cast<uint4*>(al + chunk * 16) = make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
            }
            // the generic-proxy accesses of this step (the stores above, the raw reads before them) are ordered
            // before the async proxy's: the tensor cores read the planes, the bulk copies refill the raw slot
            fence_async_shared();
            mbar_arrive(&full_a[s]);
            if (i % SPR == SPR - 1) mbar_arrive(&raw_empty[rs]);
        }
    } else if (warp == G_RAW_WARP) {
        // ---- raw weights into the raw ring: Q4_K per K step and live 16-row tile its headers and the step's 512
        // code bytes; Q6_K per superblock the live tiles whole
        if (lane == 0) {
            const uint8_t* t0 = tiles + ((int64_t)(row_base / 16 + m0 / 16) * nsb) * F::TILE;
            const int nraw = nk / SPR;
            for (int r = 0; r < nraw; ++r) {
                const int rs = r % G_RAW_STAGES;
                if (r >= G_RAW_STAGES) {
                    mbar_wait(&raw_empty[rs], (uint32_t)(((r / G_RAW_STAGES) + 1) & 1), err, 17, &abort_flag);
                    fence_async_shared();   // the dequantizers' reads of the slot before the copy engine rewrites it
                }
                uint8_t* dst = raw + rs * G_RAW_STAGE;
                mbar_expect_tx(&raw_full[rs], (uint32_t)(live_tiles * F::RAW_TILE));
                for (int tt = 0; tt < live_tiles; ++tt) {
                    if (WT == 12) {
                        const int sb = r >> 2, p = r & 3;
                        const uint8_t* tb = t0 + ((int64_t)tt * nsb + sb) * F::TILE;
                        bulk_load(dst + tt * F::RAW_TILE, tb, 256, &raw_full[rs]);
                        bulk_load(dst + tt * F::RAW_TILE + 256, tb + 256 + p * 512, 512, &raw_full[rs]);
                    } else {
                        bulk_load(dst + tt * F::RAW_TILE, t0 + ((int64_t)tt * nsb + r) * F::TILE, F::TILE, &raw_full[rs]);
                    }
                }
            }
        }
    } else if (warp == G_TMA_WARP) {
        // ---- the tokens' bf16 planes, one 64-value x BN-token box each per K step (rows past T read as zeros)
        if (lane == 0) {
            for (int i = 0; i < nk; ++i) {
                const int s = i % G_STAGES;
                if (i >= G_STAGES) mbar_wait(&empty[s], (uint32_t)(((i / G_STAGES) + 1) & 1), err, 12, &abort_flag);
                uint8_t* st = smem + (size_t)s * G_STAGE + 2 * G_A_BYTES;
                mbar_expect_tx(&full_b[s], 2 * G_B_BYTES);
                tma_load_2d(st, &xh_map, i * G_BK, n0, &full_b[s]);
                tma_load_2d(st + G_B_BYTES, &xl_map, i * G_BK, n0, &full_b[s]);
            }
        }
    } else {
        // ---- one thread issues the MMAs
        if (lane == 0) {
            for (int i = 0; i < nk; ++i) {
                const int s = i % G_STAGES;
                const uint32_t par = (uint32_t)((i / G_STAGES) & 1);
                mbar_wait(&full_a[s], par, err, 13, &abort_flag);
                mbar_wait(&full_b[s], par, err, 14, &abort_flag);
                tc_fence_after();
                const uint8_t* st = smem + (size_t)s * G_STAGE;
#pragma unroll
                for (int kk = 0; kk < G_BK / 16; ++kk) {
                    const uint64_t ah = sdesc(st + kk * 32), al = sdesc(st + G_A_BYTES + kk * 32);
                    const uint64_t bh = sdesc(st + 2 * G_A_BYTES + kk * 32), bl = sdesc(st + 2 * G_A_BYTES + G_B_BYTES + kk * 32);
                    umma_bf16<BN>(tmem, ah, bh, (i > 0 || kk > 0) ? 1u : 0u);
                    umma_bf16<BN>(tmem, ah, bl, 1u);
                    umma_bf16<BN>(tmem, al, bh, 1u);
                }
                umma_commit(&empty[s]);     // the stage is free once these MMAs have read it
            }
            umma_commit(&acc_full);
        }
    }

    // ---- epilogue: warps 0-3, warp w reads TMEM lanes 32w .. 32w+31 (tile rows), BN token columns 64 at a time
    if (warp < 4) {
        mbar_wait(&acc_full, 0u, err, 15, &abort_flag);
        tc_fence_after();
        const int r = m0 + 32 * warp + lane;
#pragma unroll
        for (int half = 0; half < BN / 64; ++half) {
            float v[64];
            tmem_ld64(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(64 * half), v);
            if (r < rows) {
#pragma unroll
                for (int j = 0; j < 64; ++j) {
                    const int n = n0 + 64 * half + j;
                    if (n < T) y[(int64_t)n * ldy + r] = v[j];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G_TMEM_COLS) : "memory");
    }
}

// x (T rows of K fp32, ldx apart) to its bf16 planes hi = bf16(x), lo = bf16(x - hi), each [T][K].
__global__ void k_split_bf16(const float* x, int64_t ldx, int K, int64_t n, __nv_bfloat16* hi,
                             __nv_bfloat16* lo)
{
    pdl_trigger();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / K, c = i - t * K;
        const float v = x[t * ldx + c];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled()
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

// A [T][K] bf16 plane as 64-value x bn-token boxes with the 128-byte swizzle the MMA descriptors expect.
CUtensorMap plane_map(const void* base, int T, int K, int bn)
{
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {G_BK, (cuuint32_t)bn};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_tiled()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) WL_THROW(WL_ECUDA, "cuTensorMapEncodeTiled (activation planes) failed (" + std::to_string((int)r) + ")");
    return map;
}

}  // namespace

bool gemm_supported(int type, int cols) { return (type == 12 || type == 14) && cols % 256 == 0; }

int gemm_min_rows(int type) { return type == 14 ? 57 : 81; }

size_t gemm_scratch_bytes(int T, int cols) { return (size_t)2 * T * cols * 2 + 256; }

void gemm_tiles(int type, const uint8_t* tiles, int row_base, int rows, int cols, const float* x, int64_t ldx, int T,
                float* y, int64_t ldy, void* scratch, int* err, cudaStream_t s)
{
    if (!gemm_supported(type, cols)) WL_THROW(WL_EUNSUPPORTED, "gemm_tiles: Q4_K or Q6_K with cols a multiple of 256 only");
    if ((uintptr_t)tiles % 16 != 0 || row_base % 16 != 0) WL_THROW(WL_EINVAL, "gemm_tiles: misaligned tiles");
    if (T <= 0 || rows <= 0) return;
    __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(((uintptr_t)scratch + 255) & ~(uintptr_t)255);
    __nv_bfloat16* lo = hi + (size_t)T * cols;
    const int64_t n = (int64_t)T * cols;
    int64_t gr = (n + 255) / 256;
    if (gr > 148 * 8) gr = 148 * 8;
    launch(k_split_bf16, dim3((unsigned)gr), dim3(256), 0, s, x, ldx, cols, n, hi, lo);
    note_launch();
    // Q4_K prompts of more than 128 rows: 256-token tiles, so each weight is dequantized once per 256 tokens and each
    // stage of dequantized weights feeds twice the MMA work
    const int bn = (type == 12 && T > 128) ? 256 : 128;
    const CUtensorMap mh = plane_map(hi, T, cols, bn), ml = plane_map(lo, T, cols, bn);
    static std::mutex mu;
    static bool attr[64] = {false};
    int dev = 0;
    WL_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && !attr[dev]) {
            WL_CUDA(cudaFuncSetAttribute(k_gemm<12, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmFmt<12, 128>::SMEM));
            WL_CUDA(cudaFuncSetAttribute(k_gemm<12, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmFmt<12, 256>::SMEM));
            WL_CUDA(cudaFuncSetAttribute(k_gemm<14, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmFmt<14, 128>::SMEM));
            attr[dev] = true;
        }
    }
    const dim3 grid((rows + G_BM - 1) / G_BM, (T + bn - 1) / bn);
    // A plain launch, and the kernel does not trigger its dependents: no other kernel overlaps a GEMM. With programmatic
    // dependent launch on both sides, consecutive GEMMs (each with its own activation-plane tensor maps) overlapped
    // and gave wrong sums now and then (1-3 % relative error in a 2-layer prefill, never with either side serialised).
    if (type == 12 && bn == 256)
        k_gemm<12, 256><<<grid, G_THREADS, GemmFmt<12, 256>::SMEM, s>>>(mh, ml, tiles, row_base, rows, cols / 256, T, y, ldy, err);
    else if (type == 12)
        k_gemm<12, 128><<<grid, G_THREADS, GemmFmt<12, 128>::SMEM, s>>>(mh, ml, tiles, row_base, rows, cols / 256, T, y, ldy, err);
    else
        k_gemm<14, 128><<<grid, G_THREADS, GemmFmt<14, 128>::SMEM, s>>>(mh, ml, tiles, row_base, rows, cols / 256, T, y, ldy, err);
    WL_CUDA(cudaGetLastError());
    note_launch();
}

}  // namespace k
}  // namespace wl
