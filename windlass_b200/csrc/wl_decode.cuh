// Device-side GGUF block decoding, bit-exact with the reference's CPU decoders (src/Quants.cs:189-396,
// src/IQuants.cs:136-369): every product and sum is a separately rounded IEEE operation (__fmul_rn, __fadd_rn,
// __fsub_rn), in the reference's order, so the compiler cannot contract them into fused multiply-adds.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include "iq_tables.h"

namespace wl {

// All device code of the library is compiled in one translation unit (wl_kernels.cu), so the tables are defined
// here. Total ~33 KB of constant memory.
__constant__ uint64_t c_iq2xxs_grid[256];
__constant__ uint64_t c_iq2xs_grid[512];
__constant__ uint64_t c_iq2s_grid[1024];
__constant__ uint64_t c_iq1s_grid[2048];
__constant__ uint32_t c_iq3xxs_grid[256];
__constant__ uint32_t c_iq3s_grid[512];
__constant__ uint8_t c_ksigns[128];
__constant__ int8_t c_kvalues_iq4nl[16];

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__device__ __forceinline__ float ldh(const uint8_t* p) { return h2f(ld_u16(p)); }

// ScaleMinK4 (src/Quants.cs:322-330).
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& m)
{
    if (j < 4) { sc = q[j] & 63; m = q[j + 4] & 63; }
    else { sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4); m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
}

__device__ __forceinline__ float sgn(int signs, int j) { return (signs >> j) & 1 ? -1.0f : 1.0f; }

// Value of element e (0 <= e < block size) of the block at b, exactly as the reference decodes it.
__device__ inline float dq_elem(int type, const uint8_t* b, int e)
{
    switch (type) {
    case 0: { uint32_t v = ld_u32(b + 4 * e); return __uint_as_float(v); }                      // F32
    case 1: return ldh(b + 2 * e);                                                               // F16
    case 30: return __uint_as_float((uint32_t)ld_u16(b + 2 * e) << 16);                          // BF16
    case 2: {                                                                                     // Q4_0
        float d = ldh(b); int j = e & 15; int q = e < 16 ? (b[2 + j] & 0xF) : (b[2 + j] >> 4);
        return __fmul_rn((float)(q - 8), d);
    }
    case 3: {                                                                                     // Q4_1
        float d = ldh(b), m = ldh(b + 2); int j = e & 15; int q = e < 16 ? (b[4 + j] & 0xF) : (b[4 + j] >> 4);
        return __fadd_rn(__fmul_rn((float)q, d), m);
    }
    case 6: {                                                                                     // Q5_0
        float d = ldh(b); uint32_t qh = ld_u32(b + 2); int j = e & 15; int v;
        if (e < 16) v = (b[6 + j] & 0xF) | (int)(((qh >> j) << 4) & 0x10);
        else v = (b[6 + j] >> 4) | (int)((qh >> (j + 12)) & 0x10);
        return __fmul_rn((float)(v - 16), d);
    }
    case 7: {                                                                                     // Q5_1
        float d = ldh(b), m = ldh(b + 2); uint32_t qh = ld_u32(b + 4); int j = e & 15; int v;
        if (e < 16) v = (b[8 + j] & 0xF) | (int)(((qh >> j) << 4) & 0x10);
        else v = (b[8 + j] >> 4) | (int)((qh >> (j + 12)) & 0x10);
        return __fadd_rn(__fmul_rn((float)v, d), m);
    }
    case 8: return __fmul_rn((float)(int8_t)b[2 + e], ldh(b));                                   // Q8_0
    case 10: {                                                                                    // Q2_K
        int k = e >> 7, e2 = e & 127, j = e2 >> 5, part = (e2 >> 4) & 1, l = e2 & 15;
        int s = b[k * 8 + 2 * j + part];
        float d = ldh(b + 80), mn = ldh(b + 82);
        float dl = __fmul_rn(d, (float)(s & 0xF)), ml = __fmul_rn(mn, (float)(s >> 4));
        int q = (b[16 + 32 * k + 16 * part + l] >> (2 * j)) & 3;
        return __fsub_rn(__fmul_rn(dl, (float)q), ml);
    }
    case 11: {                                                                                    // Q3_K
        const uint8_t* s12 = b + 96;
        uint32_t a0 = ld_u32(s12), a1 = ld_u32(s12 + 4), tmp = ld_u32(s12 + 8);
        const uint32_t km1 = 0x03030303u, km2 = 0x0f0f0f0fu;
        uint32_t aux[4];
        aux[2] = ((a0 >> 4) & km2) | (((tmp >> 4) & km1) << 4);
        aux[3] = ((a1 >> 4) & km2) | (((tmp >> 6) & km1) << 4);
        aux[0] = (a0 & km2) | (((tmp >> 0) & km1) << 4);
        aux[1] = (a1 & km2) | (((tmp >> 2) & km1) << 4);
        int k = e >> 7, e2 = e & 127, j = e2 >> 5, part = (e2 >> 4) & 1, l = e2 & 15;
        int idx = k * 8 + 2 * j + part;
        int sc = (int8_t)((aux[idx >> 2] >> (8 * (idx & 3))) & 0xFF);
        float dl = __fmul_rn(ldh(b + 108), (float)(sc - 32));
        int m = 1 << (k * 4 + j);
        int q = (b[32 + 32 * k + 16 * part + l] >> (2 * j)) & 3;
        int hm = b[16 * part + l];
        return __fmul_rn(dl, (float)(q - ((hm & m) != 0 ? 0 : 4)));
    }
    case 12: {                                                                                    // Q4_K
        int p = e >> 6, h = (e >> 5) & 1, l = e & 31, s, m;
        scale_min_k4(2 * p + h, b + 4, s, m);
        float d1 = __fmul_rn(ldh(b), (float)s), m1 = __fmul_rn(ldh(b + 2), (float)m);
        int q = h ? (b[16 + 32 * p + l] >> 4) : (b[16 + 32 * p + l] & 0xF);
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case 13: {                                                                                    // Q5_K
        int p = e >> 6, h = (e >> 5) & 1, l = e & 31, s, m;
        scale_min_k4(2 * p + h, b + 4, s, m);
        float d1 = __fmul_rn(ldh(b), (float)s), m1 = __fmul_rn(ldh(b + 2), (float)m);
        int ql = b[48 + 32 * p + l];
        int u = 1 << (2 * p + h);
        int q = (h ? (ql >> 4) : (ql & 0xF)) + ((b[16 + l] & u) != 0 ? 16 : 0);
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case 14: {                                                                                    // Q6_K
        int k = e >> 7, e2 = e & 127, quarter = e2 >> 5, l = e2 & 31;
        const uint8_t* ql = b + 64 * k; const uint8_t* qh = b + 128 + 32 * k; const int8_t* sc = (const int8_t*)(b + 192 + 8 * k);
        int lo = (quarter & 1) ? ql[l + 32] : ql[l];
        lo = (quarter & 2) ? (lo >> 4) : (lo & 0xF);
        int q = (lo | (((qh[l] >> (2 * quarter)) & 3) << 4)) - 32;
        float ds = __fmul_rn(ldh(b + 208), (float)sc[(l >> 4) + 2 * quarter]);
        return __fmul_rn(ds, (float)q);
    }
    case 20: {                                                                                    // IQ4_NL
        int j = e & 15; int nib = e < 16 ? (b[2 + j] & 0xF) : (b[2 + j] >> 4);
        return __fmul_rn(ldh(b), (float)c_kvalues_iq4nl[nib]);
    }
    case 23: {                                                                                    // IQ4_XS
        int ib = e >> 5, j = e & 31;
        int sh = ld_u16(b + 2);
        int ls = ((b[4 + ib / 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
        float dl = __fmul_rn(ldh(b), (float)(ls - 32));
        int nib = j < 16 ? (b[8 + 16 * ib + j] & 0xF) : (b[8 + 16 * ib + j - 16] >> 4);
        return __fmul_rn(dl, (float)c_kvalues_iq4nl[nib]);
    }
    case 18: {                                                                                    // IQ3_XXS
        int ib = e >> 5, w = e & 31, l = w >> 3, jj = w & 7;
        uint32_t aux32 = ld_u32(b + 2 + 64 + 4 * ib);
        float db = __fmul_rn(__fmul_rn(ldh(b), __fadd_rn(0.5f, (float)(aux32 >> 28))), 0.5f);
        int signs = c_ksigns[(aux32 >> (7 * l)) & 127];
        const uint8_t* qs = b + 2 + 8 * ib;
        uint32_t g = c_iq3xxs_grid[jj < 4 ? qs[2 * l] : qs[2 * l + 1]];
        float v = (float)((g >> (8 * (jj & 3))) & 0xFF);
        return __fmul_rn(__fmul_rn(db, v), sgn(signs, jj));
    }
    case 21: {                                                                                    // IQ3_S
        int ib = e >> 5, w = e & 31, l = w >> 3, jj = w & 7;
        int sc = b[106 + ib / 2];
        float db = __fmul_rn(ldh(b), (float)(1 + 2 * ((ib & 1) ? (sc >> 4) : (sc & 0xF))));
        int h = b[66 + ib];
        const uint8_t* qs = b + 2 + 8 * ib;
        int gi = jj < 4 ? (qs[2 * l] | ((h << (8 - 2 * l)) & 256)) : (qs[2 * l + 1] | ((h << (7 - 2 * l)) & 256));
        uint32_t g = c_iq3s_grid[gi];
        float v = (float)((g >> (8 * (jj & 3))) & 0xFF);
        int signs = b[74 + 4 * ib + l];
        return __fmul_rn(__fmul_rn(db, v), sgn(signs, jj));
    }
    case 16: {                                                                                    // IQ2_XXS
        int ib = e >> 5, w = e & 31, l = w >> 3, jj = w & 7;
        uint32_t aux0 = ld_u32(b + 2 + 8 * ib), aux1 = ld_u32(b + 2 + 8 * ib + 4);
        float db = __fmul_rn(__fmul_rn(ldh(b), __fadd_rn(0.5f, (float)(aux1 >> 28))), 0.25f);
        uint64_t g = c_iq2xxs_grid[(aux0 >> (8 * l)) & 0xFF];
        int signs = c_ksigns[(aux1 >> (7 * l)) & 127];
        float v = (float)((g >> (8 * jj)) & 0xFF);
        return __fmul_rn(__fmul_rn(db, v), sgn(signs, jj));
    }
    case 17: {                                                                                    // IQ2_XS
        int ib = e >> 5, w = e & 31, l = w >> 3, jj = w & 7;
        int sc = b[66 + ib];
        float db = __fmul_rn(__fmul_rn(ldh(b), __fadd_rn(0.5f, (float)(l < 2 ? (sc & 0xF) : (sc >> 4)))), 0.25f);
        uint16_t qv = ld_u16(b + 2 + 2 * (4 * ib + l));
        uint64_t g = c_iq2xs_grid[qv & 511];
        int signs = c_ksigns[qv >> 9];
        float v = (float)((g >> (8 * jj)) & 0xFF);
        return __fmul_rn(__fmul_rn(db, v), sgn(signs, jj));
    }
    case 22: {                                                                                    // IQ2_S
        int ib = e >> 5, w = e & 31, l = w >> 3, jj = w & 7;
        int sc = b[74 + ib];
        float db = __fmul_rn(__fmul_rn(ldh(b), __fadd_rn(0.5f, (float)(l < 2 ? (sc & 0xF) : (sc >> 4)))), 0.25f);
        int qh = b[66 + ib];
        uint64_t g = c_iq2s_grid[b[2 + 4 * ib + l] | ((qh << (8 - 2 * l)) & 0x300)];
        int signs = b[2 + 32 + 4 * ib + l];
        float v = (float)((g >> (8 * jj)) & 0xFF);
        return __fmul_rn(__fmul_rn(db, v), sgn(signs, jj));
    }
    case 19: {                                                                                    // IQ1_S
        int ib = e >> 5, w = e & 31, l = w >> 3, jj = w & 7;
        uint16_t qh = ld_u16(b + 34 + 2 * ib);
        float dl = __fmul_rn(ldh(b), (float)(2 * ((qh >> 12) & 7) + 1));
        float delta = (qh & 0x8000) != 0 ? -0.125f : 0.125f;
        uint64_t g = c_iq1s_grid[b[2 + 4 * ib + l] | (((qh >> (3 * l)) & 7) << 8)];
        float v = (float)(int8_t)(uint8_t)((g >> (8 * jj)) & 0xFF);
        return __fmul_rn(dl, __fadd_rn(v, delta));
    }
    case 29: {                                                                                    // IQ1_M
        int ib = e >> 5, w = e & 31, l = w >> 3, jj = w & 7;
        uint16_t sc0 = ld_u16(b + 48), sc1 = ld_u16(b + 50), sc2 = ld_u16(b + 52), sc3 = ld_u16(b + 54);
        uint16_t s16 = (uint16_t)((sc0 >> 12) | ((sc1 >> 8) & 0x00F0) | ((sc2 >> 4) & 0x0F00) | (sc3 & 0xF000));
        float d = h2f(s16);
        uint16_t scw = ld_u16(b + 48 + 2 * (ib / 2));
        int shift = 6 * (ib % 2) + (l < 2 ? 0 : 3);
        float dl = __fmul_rn(d, (float)(2 * ((scw >> shift) & 7) + 1));
        const uint8_t* qs = b + 4 * ib; const uint8_t* qh = b + 32 + 2 * ib;
        int hb = qh[l >> 1];
        int gi = (l & 1) ? (qs[l] | ((hb << 4) & 0x700)) : (qs[l] | ((hb << 8) & 0x700));
        float delta = ((l & 1) ? (hb & 0x80) : (hb & 0x08)) != 0 ? -0.125f : 0.125f;
        uint64_t g = c_iq1s_grid[gi];
        float v = (float)(int8_t)(uint8_t)((g >> (8 * jj)) & 0xFF);
        return __fmul_rn(dl, __fadd_rn(v, delta));
    }
    }
    return 0.0f;
}

__host__ __device__ constexpr int block_elems(int type)
{
    return (type == 0 || type == 1 || type == 30) ? 1
         : (type == 2 || type == 3 || type == 6 || type == 7 || type == 8 || type == 20) ? 32 : 256;
}
__host__ __device__ constexpr int block_bytes(int type)
{
    return type == 0 ? 4 : type == 1 ? 2 : type == 30 ? 2 : type == 2 ? 18 : type == 3 ? 20 : type == 6 ? 22
         : type == 7 ? 24 : type == 8 ? 34 : type == 10 ? 84 : type == 11 ? 110 : type == 12 ? 144 : type == 13 ? 176
         : type == 14 ? 210 : type == 16 ? 66 : type == 17 ? 74 : type == 18 ? 98 : type == 19 ? 50 : type == 20 ? 18
         : type == 21 ? 110 : type == 22 ? 82 : type == 23 ? 136 : type == 29 ? 56 : 0;
}

}  // namespace wl
