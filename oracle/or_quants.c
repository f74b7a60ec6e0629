/* Oracle numerics: fp16, block layouts, row decoders, fused row dots and the blocked float kernel.
 * Test infrastructure only (see oracle.h). Each function names the reference lines it restates. */
#include "oracle.h"
#include "../windlass_b200/csrc/iq_tables.h"
#include <string.h>
#include <stdlib.h>

/* Half.Decode (Half.cs:59-89): exact fp16 -> fp32. */
float or_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    int exp = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF, bits;
    if (exp == 0) {
        if (mant == 0) bits = sign;
        else {
            int e = -1;
            do { e++; mant <<= 1; } while ((mant & 0x400) == 0);
            mant &= 0x3FF;
            bits = sign | (uint32_t)(127 - 15 - e) << 23 | mant << 13;
        }
    } else if (exp == 31) bits = sign | 0x7F800000u | mant << 13;
    else bits = sign | (uint32_t)(exp - 15 + 127) << 23 | mant << 13;
    float f; memcpy(&f, &bits, 4); return f;
}

/* Half.FromFloat (Half.cs:29-57): fp32 -> fp16, round to nearest even, NaN keeps a quiet payload bit. */
uint16_t or_float_to_half(float value)
{
    uint32_t f; memcpy(&f, &value, 4);
    uint32_t sign = (f >> 16) & 0x8000;
    int e = (int)((f >> 23) & 0xFF);
    uint32_t m = f & 0x7FFFFF;
    if (e == 255) return (uint16_t)(sign | 0x7C00 | (m != 0 ? 0x200u : 0u));
    int ne = e - 127 + 15;
    if (ne >= 31) return (uint16_t)(sign | 0x7C00);
    if (ne <= 0) {
        if (ne < -10) return (uint16_t)sign;
        m |= 0x800000;
        int shift = 14 - ne;
        uint32_t hm = m >> shift, rem = m & ((1u << shift) - 1), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1) != 0)) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)ne << 10) | (m >> 13), r = m & 0x1FFF;
    if (r > 0x1000 || (r == 0x1000 && (h & 1) != 0)) h++;
    return (uint16_t)h;
}

static inline float H(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return or_half_to_float(v); }
static inline uint32_t U32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }
static inline uint16_t U16(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return v; }
static inline float BF16(uint16_t v) { uint32_t b = (uint32_t)v << 16; float f; memcpy(&f, &b, 4); return f; }

/* GgmlTypes.TryGetLayout (Gguf.cs:30-66). */
int or_layout(int t, int* bs, int* ts)
{
    int b = 0, s = 0;
    switch (t) {
    case OR_F32: b = 1; s = 4; break;   case OR_F16: b = 1; s = 2; break;   case OR_BF16: b = 1; s = 2; break;
    case OR_I8: b = 1; s = 1; break;    case OR_I16: b = 1; s = 2; break;   case OR_I32: b = 1; s = 4; break;
    case OR_I64: b = 1; s = 8; break;   case OR_F64: b = 1; s = 8; break;
    case OR_Q4_0: b = 32; s = 18; break; case OR_Q4_1: b = 32; s = 20; break; case OR_Q5_0: b = 32; s = 22; break;
    case OR_Q5_1: b = 32; s = 24; break; case OR_Q8_0: b = 32; s = 34; break; case OR_Q8_1: b = 32; s = 36; break;
    case OR_Q2_K: b = 256; s = 84; break; case OR_Q3_K: b = 256; s = 110; break; case OR_Q4_K: b = 256; s = 144; break;
    case OR_Q5_K: b = 256; s = 176; break; case OR_Q6_K: b = 256; s = 210; break; case OR_Q8_K: b = 256; s = 292; break;
    case OR_IQ2_XXS: b = 256; s = 66; break; case OR_IQ2_XS: b = 256; s = 74; break; case OR_IQ3_XXS: b = 256; s = 98; break;
    case OR_IQ1_S: b = 256; s = 50; break; case OR_IQ4_NL: b = 32; s = 18; break; case OR_IQ3_S: b = 256; s = 110; break;
    case OR_IQ2_S: b = 256; s = 82; break; case OR_IQ4_XS: b = 256; s = 136; break; case OR_IQ1_M: b = 256; s = 56; break;
    default: if (bs) *bs = 0; if (ts) *ts = 0; return 0;
    }
    if (bs) *bs = b;
    if (ts) *ts = s;
    return 1;
}

static int is_iquant(int t)
{
    return t == OR_IQ4_NL || t == OR_IQ4_XS || t == OR_IQ3_XXS || t == OR_IQ3_S || t == OR_IQ2_XXS ||
           t == OR_IQ2_XS || t == OR_IQ2_S || t == OR_IQ1_S || t == OR_IQ1_M;
}

/* Quants.CanDecode (Quants.cs:11-21). */
int or_can_decode(int t)
{
    switch (t) {
    case OR_F32: case OR_F16: case OR_BF16: case OR_Q4_0: case OR_Q4_1: case OR_Q5_0: case OR_Q5_1: case OR_Q8_0:
    case OR_Q2_K: case OR_Q3_K: case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: return 1;
    }
    return is_iquant(t);
}

/* Quants.CanDot (Quants.cs:56-65). */
int or_can_dot(int t)
{
    switch (t) {
    case OR_F32: case OR_F16: case OR_BF16: case OR_Q4_0: case OR_Q8_0: case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: return 1;
    }
    return 0;
}

/* ScaleMinK4 (Quants.cs:322-330). */
static inline void scale_min_k4(int j, const uint8_t* q, int* sc, int* m)
{
    if (j < 4) { *sc = q[j] & 63; *m = q[j + 4] & 63; }
    else { *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4); *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
}

/* ---------- legacy and K-quant decoders, Quants.cs:189-396 ---------- */
static void dec_q4_0(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 32; i++, b += 18, y += 32) {
        float d = H(b); const uint8_t* q = b + 2;
        for (int j = 0; j < 16; j++) { y[j] = ((q[j] & 0xF) - 8) * d; y[j + 16] = ((q[j] >> 4) - 8) * d; }
    }
}
static void dec_q4_1(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 32; i++, b += 20, y += 32) {
        float d = H(b), m = H(b + 2); const uint8_t* q = b + 4;
        for (int j = 0; j < 16; j++) { y[j] = (q[j] & 0xF) * d + m; y[j + 16] = (q[j] >> 4) * d + m; }
    }
}
static void dec_q5_0(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 32; i++, b += 22, y += 32) {
        float d = H(b); uint32_t qh = U32(b + 2); const uint8_t* q = b + 6;
        for (int j = 0; j < 16; j++) {
            int h0 = (int)(((qh >> j) << 4) & 0x10), h1 = (int)((qh >> (j + 12)) & 0x10);
            y[j] = (((q[j] & 0xF) | h0) - 16) * d; y[j + 16] = (((q[j] >> 4) | h1) - 16) * d;
        }
    }
}
static void dec_q5_1(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 32; i++, b += 24, y += 32) {
        float d = H(b), m = H(b + 2); uint32_t qh = U32(b + 4); const uint8_t* q = b + 8;
        for (int j = 0; j < 16; j++) {
            int h0 = (int)(((qh >> j) << 4) & 0x10), h1 = (int)((qh >> (j + 12)) & 0x10);
            y[j] = ((q[j] & 0xF) | h0) * d + m; y[j + 16] = ((q[j] >> 4) | h1) * d + m;
        }
    }
}
static void dec_q8_0(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 32; i++, b += 34, y += 32) {
        float d = H(b); const int8_t* q = (const int8_t*)(b + 2);
        for (int j = 0; j < 32; j++) y[j] = q[j] * d;
    }
}
static void dec_q2_k(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 84) {
        const uint8_t* sc = b; const uint8_t* q = b + 16;
        float d = H(b + 80), mn = H(b + 82);
        int idx = 0;
        for (int k = 0; k < 256; k += 128) {
            int shift = 0;
            for (int j = 0; j < 4; j++) {
                int s = sc[idx++];
                float dl = d * (s & 0xF), ml = mn * (s >> 4);
                for (int l = 0; l < 16; l++) *y++ = dl * ((q[l] >> shift) & 3) - ml;
                s = sc[idx++];
                dl = d * (s & 0xF); ml = mn * (s >> 4);
                for (int l = 0; l < 16; l++) *y++ = dl * ((q[l + 16] >> shift) & 3) - ml;
                shift += 2;
            }
            q += 32;
        }
    }
}
static void dec_q3_k(const uint8_t* b, int64_t n, float* y)
{
    const uint32_t kmask1 = 0x03030303, kmask2 = 0x0f0f0f0f;
    uint32_t aux[4];
    for (int64_t i = 0; i < n / 256; i++, b += 110) {
        const uint8_t* hm = b; const uint8_t* q = b + 32; const uint8_t* s12 = b + 96;
        float dAll = H(b + 108);
        aux[0] = U32(s12); aux[1] = U32(s12 + 4); aux[2] = U32(s12 + 8);
        uint32_t tmp = aux[2];
        aux[2] = ((aux[0] >> 4) & kmask2) | (((tmp >> 4) & kmask1) << 4);
        aux[3] = ((aux[1] >> 4) & kmask2) | (((tmp >> 6) & kmask1) << 4);
        aux[0] = (aux[0] & kmask2) | (((tmp >> 0) & kmask1) << 4);
        aux[1] = (aux[1] & kmask2) | (((tmp >> 2) & kmask1) << 4);
        const int8_t* scales = (const int8_t*)aux;
        int idx = 0, m = 1;
        for (int k = 0; k < 256; k += 128) {
            int shift = 0;
            for (int j = 0; j < 4; j++) {
                float dl = dAll * (scales[idx++] - 32);
                for (int l = 0; l < 16; l++) *y++ = dl * (((q[l] >> shift) & 3) - ((hm[l] & m) != 0 ? 0 : 4));
                dl = dAll * (scales[idx++] - 32);
                for (int l = 0; l < 16; l++) *y++ = dl * (((q[l + 16] >> shift) & 3) - ((hm[l + 16] & m) != 0 ? 0 : 4));
                shift += 2; m <<= 1;
            }
            q += 32;
        }
    }
}
/* Quants.Q4_K (Quants.cs:333-350): y = (d*s)*q - (dmin*m), each product rounded separately. */
static void dec_q4_k(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 144) {
        float d = H(b), mn = H(b + 2);
        const uint8_t* sc = b + 4; const uint8_t* q = b + 16;
        int idx = 0;
        for (int j = 0; j < 256; j += 64) {
            int s, m;
            scale_min_k4(idx, sc, &s, &m); float d1 = d * s, m1 = mn * m;
            scale_min_k4(idx + 1, sc, &s, &m); float d2 = d * s, m2 = mn * m;
            for (int l = 0; l < 32; l++) *y++ = d1 * (q[l] & 0xF) - m1;
            for (int l = 0; l < 32; l++) *y++ = d2 * (q[l] >> 4) - m2;
            q += 32; idx += 2;
        }
    }
}
static void dec_q5_k(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 176) {
        float d = H(b), mn = H(b + 2);
        const uint8_t* sc = b + 4; const uint8_t* qh = b + 16; const uint8_t* ql = b + 48;
        int idx = 0, u1 = 1, u2 = 2;
        for (int j = 0; j < 256; j += 64) {
            int s, m;
            scale_min_k4(idx, sc, &s, &m); float d1 = d * s, m1 = mn * m;
            scale_min_k4(idx + 1, sc, &s, &m); float d2 = d * s, m2 = mn * m;
            for (int l = 0; l < 32; l++) *y++ = d1 * ((ql[l] & 0xF) + ((qh[l] & u1) != 0 ? 16 : 0)) - m1;
            for (int l = 0; l < 32; l++) *y++ = d2 * ((ql[l] >> 4) + ((qh[l] & u2) != 0 ? 16 : 0)) - m2;
            ql += 32; idx += 2; u1 <<= 2; u2 <<= 2;
        }
    }
}
/* Quants.Q6_K (Quants.cs:373-396): y = (d*sc)*q. */
static void dec_q6_k(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 210) {
        float d = H(b + 208);
        const uint8_t* ql = b; const uint8_t* qh = b + 128; const int8_t* sc = (const int8_t*)(b + 192);
        for (int k = 0; k < 256; k += 128) {
            for (int l = 0; l < 32; l++) {
                int s = l / 16;
                int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l] = d * sc[s] * q1; y[l + 32] = d * sc[s + 2] * q2;
                y[l + 64] = d * sc[s + 4] * q3; y[l + 96] = d * sc[s + 6] * q4;
            }
            y += 128; ql += 64; qh += 32; sc += 8;
        }
    }
}

/* ---------- I-quant decoders, IQuants.cs:136-369 ---------- */
static void dec_iq4_nl(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 32; i++, b += 18, y += 32) {
        float d = H(b); const uint8_t* q = b + 2;
        for (int j = 0; j < 16; j++) { y[j] = d * WL_KVALUES_IQ4NL[q[j] & 0xF]; y[j + 16] = d * WL_KVALUES_IQ4NL[q[j] >> 4]; }
    }
}
/* IQuants.IQ4_XS (IQuants.cs:61-80): dl = d*(ls-32); y = dl*kvalues[nibble]. */
static void dec_iq4_xs(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 136) {
        float d = H(b); int scalesH = U16(b + 2);
        const uint8_t* scalesL = b + 4; const uint8_t* q = b + 8;
        for (int ib = 0; ib < 8; ib++, q += 16, y += 32) {
            int ls = ((scalesL[ib / 2] >> (4 * (ib % 2))) & 0xF) | (((scalesH >> (2 * ib)) & 3) << 4);
            float dl = d * (ls - 32);
            for (int j = 0; j < 16; j++) { y[j] = dl * WL_KVALUES_IQ4NL[q[j] & 0xF]; y[j + 16] = dl * WL_KVALUES_IQ4NL[q[j] >> 4]; }
        }
    }
}
static void dec_iq3_xxs(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 98) {
        float d = H(b); const uint8_t* qs = b + 2; const uint8_t* ss = qs + 64;
        for (int ib = 0; ib < 8; ib++) {
            uint32_t aux32 = U32(ss + 4 * ib);
            float db = d * (0.5f + (float)(aux32 >> 28)) * 0.5f;
            for (int l = 0; l < 4; l++) {
                int signs = WL_KSIGNS_IQ2XS[(aux32 >> (7 * l)) & 127];
                uint32_t g1 = WL_IQ3XXS_GRID[qs[2 * l]], g2 = WL_IQ3XXS_GRID[qs[2 * l + 1]];
                for (int j = 0; j < 4; j++) {
                    y[j] = db * (float)(uint8_t)(g1 >> (8 * j)) * ((signs & WL_KMASK_IQ2XS[j]) != 0 ? -1.f : 1.f);
                    y[j + 4] = db * (float)(uint8_t)(g2 >> (8 * j)) * ((signs & WL_KMASK_IQ2XS[j + 4]) != 0 ? -1.f : 1.f);
                }
                y += 8;
            }
            qs += 8;
        }
    }
}
static void dec_iq3_s(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 110) {
        float d = H(b);
        const uint8_t* qs = b + 2; const uint8_t* qh = b + 66; const uint8_t* signs = b + 74; const uint8_t* scales = b + 106;
        for (int ib = 0; ib < 8; ib += 2) {
            float db1 = d * (1 + 2 * (scales[ib / 2] & 0xF));
            float db2 = d * (1 + 2 * (scales[ib / 2] >> 4));
            for (int half = 0; half < 2; half++) {
                float db = half == 0 ? db1 : db2;
                int h = qh[half];
                for (int l = 0; l < 4; l++) {
                    uint32_t g1 = WL_IQ3S_GRID[qs[2 * l] | ((h << (8 - 2 * l)) & 256)];
                    uint32_t g2 = WL_IQ3S_GRID[qs[2 * l + 1] | ((h << (7 - 2 * l)) & 256)];
                    for (int j = 0; j < 4; j++) {
                        y[j] = db * (float)(uint8_t)(g1 >> (8 * j)) * ((signs[l] & WL_KMASK_IQ2XS[j]) != 0 ? -1.f : 1.f);
                        y[j + 4] = db * (float)(uint8_t)(g2 >> (8 * j)) * ((signs[l] & WL_KMASK_IQ2XS[j + 4]) != 0 ? -1.f : 1.f);
                    }
                    y += 8;
                }
                qs += 8; signs += 4;
            }
            qh += 2;
        }
    }
}
/* IQuants.IQ2_XXS (IQuants.cs:148-170): db = d*(0.5+(aux1>>28))*0.25; y = db*grid_byte*(+-1). */
static void dec_iq2_xxs(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 66) {
        float d = H(b); const uint8_t* qs = b + 2;
        for (int ib = 0; ib < 8; ib++) {
            uint32_t aux0 = U32(qs + 8 * ib), aux1 = U32(qs + 8 * ib + 4);
            float db = d * (0.5f + (float)(aux1 >> 28)) * 0.25f;
            for (int l = 0; l < 4; l++) {
                uint64_t g = WL_IQ2XXS_GRID[(aux0 >> (8 * l)) & 0xFF];
                int signs = WL_KSIGNS_IQ2XS[(aux1 >> (7 * l)) & 127];
                for (int j = 0; j < 8; j++)
                    y[j] = db * (float)(uint8_t)(g >> (8 * j)) * ((signs & WL_KMASK_IQ2XS[j]) != 0 ? -1.f : 1.f);
                y += 8;
            }
        }
    }
}
static void dec_iq2_xs(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 74) {
        float d = H(b); const uint8_t* qs = b + 2; const uint8_t* scales = b + 66;
        for (int ib = 0; ib < 8; ib++) {
            float db0 = d * (0.5f + (float)(scales[ib] & 0xF)) * 0.25f;
            float db1 = d * (0.5f + (float)(scales[ib] >> 4)) * 0.25f;
            for (int l = 0; l < 4; l++) {
                uint16_t qv = U16(qs + 2 * (4 * ib + l));
                uint64_t g = WL_IQ2XS_GRID[qv & 511];
                int signs = WL_KSIGNS_IQ2XS[qv >> 9];
                float db = l < 2 ? db0 : db1;
                for (int j = 0; j < 8; j++)
                    y[j] = db * (float)(uint8_t)(g >> (8 * j)) * ((signs & WL_KMASK_IQ2XS[j]) != 0 ? -1.f : 1.f);
                y += 8;
            }
        }
    }
}
static void dec_iq2_s(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 82) {
        float d = H(b);
        const uint8_t* qs = b + 2; const uint8_t* signs = qs + 32; const uint8_t* qh = b + 66; const uint8_t* scales = b + 74;
        for (int ib = 0; ib < 8; ib++) {
            float db0 = d * (0.5f + (float)(scales[ib] & 0xF)) * 0.25f;
            float db1 = d * (0.5f + (float)(scales[ib] >> 4)) * 0.25f;
            for (int l = 0; l < 4; l++) {
                float dl = l < 2 ? db0 : db1;
                uint64_t g = WL_IQ2S_GRID[qs[l] | ((qh[ib] << (8 - 2 * l)) & 0x300)];
                for (int j = 0; j < 8; j++)
                    y[j] = dl * (float)(uint8_t)(g >> (8 * j)) * ((signs[l] & WL_KMASK_IQ2XS[j]) != 0 ? -1.f : 1.f);
                y += 8;
            }
            qs += 4; signs += 4;
        }
    }
}
static void dec_iq1_s(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 50) {
        float d = H(b); const uint8_t* qs = b + 2; const uint8_t* qhp = b + 34;
        for (int ib = 0; ib < 8; ib++) {
            uint16_t qh = U16(qhp + 2 * ib);
            float dl = d * (2 * ((qh >> 12) & 7) + 1);
            float delta = (qh & 0x8000) != 0 ? -0.125f : 0.125f;
            for (int l = 0; l < 4; l++) {
                uint64_t g = WL_IQ1S_GRID[qs[l] | (((qh >> (3 * l)) & 7) << 8)];
                for (int j = 0; j < 8; j++) y[j] = dl * ((float)(int8_t)(uint8_t)(g >> (8 * j)) + delta);
                y += 8;
            }
            qs += 4;
        }
    }
}
static void dec_iq1_m(const uint8_t* b, int64_t n, float* y)
{
    for (int64_t i = 0; i < n / 256; i++, b += 56) {
        uint16_t sc[4];
        for (int k = 0; k < 4; k++) sc[k] = U16(b + 48 + 2 * k);
        uint16_t scale16 = (uint16_t)((sc[0] >> 12) | ((sc[1] >> 8) & 0x00F0) | ((sc[2] >> 4) & 0x0F00) | (sc[3] & 0xF000));
        float d = or_half_to_float(scale16);
        const uint8_t* qs = b; const uint8_t* qh = b + 32;
        for (int ib = 0; ib < 8; ib++) {
            float dl1 = d * (2 * ((sc[ib / 2] >> (6 * (ib % 2) + 0)) & 7) + 1);
            float dl2 = d * (2 * ((sc[ib / 2] >> (6 * (ib % 2) + 3)) & 7) + 1);
            int i0 = qs[0] | ((qh[0] << 8) & 0x700), i1 = qs[1] | ((qh[0] << 4) & 0x700);
            int i2 = qs[2] | ((qh[1] << 8) & 0x700), i3 = qs[3] | ((qh[1] << 4) & 0x700);
            float d0 = (qh[0] & 0x08) != 0 ? -0.125f : 0.125f, d1 = (qh[0] & 0x80) != 0 ? -0.125f : 0.125f;
            float d2 = (qh[1] & 0x08) != 0 ? -0.125f : 0.125f, d3 = (qh[1] & 0x80) != 0 ? -0.125f : 0.125f;
            for (int j = 0; j < 8; j++) y[j] = dl1 * ((float)(int8_t)(uint8_t)(WL_IQ1S_GRID[i0] >> (8 * j)) + d0);
            y += 8;
            for (int j = 0; j < 8; j++) y[j] = dl1 * ((float)(int8_t)(uint8_t)(WL_IQ1S_GRID[i1] >> (8 * j)) + d1);
            y += 8;
            for (int j = 0; j < 8; j++) y[j] = dl2 * ((float)(int8_t)(uint8_t)(WL_IQ1S_GRID[i2] >> (8 * j)) + d2);
            y += 8;
            for (int j = 0; j < 8; j++) y[j] = dl2 * ((float)(int8_t)(uint8_t)(WL_IQ1S_GRID[i3] >> (8 * j)) + d3);
            y += 8;
            qs += 4; qh += 2;
        }
    }
}

/* Quants.DecodeRow (Quants.cs:32-52) and IQuants.DecodeRow (IQuants.cs:27-42). */
int or_decode_row(int t, const uint8_t* src, int64_t n, float* dst)
{
    switch (t) {
    case OR_F32: memcpy(dst, src, (size_t)n * 4); return 0;
    case OR_F16: for (int64_t i = 0; i < n; i++) dst[i] = or_half_to_float(U16(src + 2 * i)); return 0;
    case OR_BF16: for (int64_t i = 0; i < n; i++) dst[i] = BF16(U16(src + 2 * i)); return 0;
    case OR_Q4_0: dec_q4_0(src, n, dst); return 0;
    case OR_Q4_1: dec_q4_1(src, n, dst); return 0;
    case OR_Q5_0: dec_q5_0(src, n, dst); return 0;
    case OR_Q5_1: dec_q5_1(src, n, dst); return 0;
    case OR_Q8_0: dec_q8_0(src, n, dst); return 0;
    case OR_Q2_K: dec_q2_k(src, n, dst); return 0;
    case OR_Q3_K: dec_q3_k(src, n, dst); return 0;
    case OR_Q4_K: dec_q4_k(src, n, dst); return 0;
    case OR_Q5_K: dec_q5_k(src, n, dst); return 0;
    case OR_Q6_K: dec_q6_k(src, n, dst); return 0;
    case OR_IQ4_NL: dec_iq4_nl(src, n, dst); return 0;
    case OR_IQ4_XS: dec_iq4_xs(src, n, dst); return 0;
    case OR_IQ3_XXS: dec_iq3_xxs(src, n, dst); return 0;
    case OR_IQ3_S: dec_iq3_s(src, n, dst); return 0;
    case OR_IQ2_XXS: dec_iq2_xxs(src, n, dst); return 0;
    case OR_IQ2_XS: dec_iq2_xs(src, n, dst); return 0;
    case OR_IQ2_S: dec_iq2_s(src, n, dst); return 0;
    case OR_IQ1_S: dec_iq1_s(src, n, dst); return 0;
    case OR_IQ1_M: dec_iq1_m(src, n, dst); return 0;
    }
    return -1;
}

/* Transformer.Dot (Transformer.cs:466-477): four accumulators, combined pairwise. */
float or_dot_f32(const float* a, const float* b, int n)
{
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int i = 0;
    for (; i + 4 <= n; i += 4) { s0 += a[i] * b[i]; s1 += a[i + 1] * b[i + 1]; s2 += a[i + 2] * b[i + 2]; s3 += a[i + 3] * b[i + 3]; }
    for (; i < n; i++) s0 += a[i] * b[i];
    return (s0 + s1) + (s2 + s3);
}

/* Quants.DotRow (Quants.cs:67-187): fused decode and dot of one row, in the reference's accumulation order. */
float or_dot_row(int t, const uint8_t* b, const float* x, int n)
{
    switch (t) {
    case OR_F32: return or_dot_f32((const float*)b, x, n);
    case OR_F16: {
        float s0 = 0, s1 = 0;
        for (int i = 0; i < n; i += 2) { s0 += or_half_to_float(U16(b + 2 * i)) * x[i]; s1 += or_half_to_float(U16(b + 2 * i + 2)) * x[i + 1]; }
        return s0 + s1;
    }
    case OR_BF16: {
        float s0 = 0, s1 = 0;
        for (int i = 0; i < n; i += 2) { s0 += BF16(U16(b + 2 * i)) * x[i]; s1 += BF16(U16(b + 2 * i + 2)) * x[i + 1]; }
        return s0 + s1;
    }
    case OR_Q8_0: {
        float sum = 0;
        for (int i = 0; i < n / 32; i++, b += 34, x += 32) {
            const int8_t* q = (const int8_t*)(b + 2);
            float s0 = 0, s1 = 0;
            for (int j = 0; j < 32; j += 2) { s0 += q[j] * x[j]; s1 += q[j + 1] * x[j + 1]; }
            sum += H(b) * (s0 + s1);
        }
        return sum;
    }
    case OR_Q4_0: {
        float sum = 0;
        for (int i = 0; i < n / 32; i++, b += 18, x += 32) {
            const uint8_t* q = b + 2;
            float s0 = 0, s1 = 0;
            for (int j = 0; j < 16; j++) { s0 += ((q[j] & 0xF) - 8) * x[j]; s1 += ((q[j] >> 4) - 8) * x[j + 16]; }
            sum += H(b) * (s0 + s1);
        }
        return sum;
    }
    case OR_Q4_K: {
        float sum = 0;
        for (int i = 0; i < n / 256; i++, b += 144) {
            float d = H(b), mn = H(b + 2);
            const uint8_t* sc = b + 4; const uint8_t* q = b + 16;
            for (int j = 0; j < 4; j++, q += 32, x += 64) {
                int s1, m1, s2, m2;
                scale_min_k4(2 * j, sc, &s1, &m1);
                scale_min_k4(2 * j + 1, sc, &s2, &m2);
                float a1 = 0, a2 = 0, x1 = 0, x2 = 0;
                for (int l = 0; l < 32; l++) {
                    float xl = x[l], xh = x[l + 32];
                    a1 += (q[l] & 0xF) * xl; x1 += xl;
                    a2 += (q[l] >> 4) * xh; x2 += xh;
                }
                sum += d * (s1 * a1 + s2 * a2) - mn * (m1 * x1 + m2 * x2);
            }
        }
        return sum;
    }
    case OR_Q5_K: {
        float sum = 0;
        for (int i = 0; i < n / 256; i++, b += 176) {
            float d = H(b), mn = H(b + 2);
            const uint8_t* sc = b + 4; const uint8_t* qh = b + 16; const uint8_t* ql = b + 48;
            int u1 = 1, u2 = 2;
            for (int j = 0; j < 4; j++, ql += 32, x += 64, u1 <<= 2, u2 <<= 2) {
                int s1, m1, s2, m2;
                scale_min_k4(2 * j, sc, &s1, &m1);
                scale_min_k4(2 * j + 1, sc, &s2, &m2);
                float a1 = 0, a2 = 0, x1 = 0, x2 = 0;
                for (int l = 0; l < 32; l++) {
                    float xl = x[l], xh = x[l + 32];
                    a1 += ((ql[l] & 0xF) + ((qh[l] & u1) != 0 ? 16 : 0)) * xl; x1 += xl;
                    a2 += ((ql[l] >> 4) + ((qh[l] & u2) != 0 ? 16 : 0)) * xh; x2 += xh;
                }
                sum += d * (s1 * a1 + s2 * a2) - mn * (m1 * x1 + m2 * x2);
            }
        }
        return sum;
    }
    case OR_Q6_K: {
        float sum = 0, acc[8];
        for (int i = 0; i < n / 256; i++, b += 210) {
            float d = H(b + 208);
            const uint8_t* ql = b; const uint8_t* qh = b + 128; const int8_t* sc = (const int8_t*)(b + 192);
            for (int k = 0; k < 2; k++, ql += 64, qh += 32, sc += 8, x += 128) {
                for (int g = 0; g < 8; g++) acc[g] = 0;
                for (int l = 0; l < 32; l++) {
                    int s = l >> 4;
                    acc[s] += (((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32) * x[l];
                    acc[s + 2] += (((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32) * x[l + 32];
                    acc[s + 4] += (((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32) * x[l + 64];
                    acc[s + 6] += (((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32) * x[l + 96];
                }
                float part = 0;
                for (int g = 0; g < 8; g++) part += sc[g] * acc[g];
                sum += d * part;
            }
        }
        return sum;
    }
    }
    return 0.0f;
}

/* FastMath.Block (FastMath.cs:218-264): 4 weight rows x 2 tokens register blocking; one accumulator chain per
 * (row, token) summed in index order. */
void or_block(const float* w, int ws, int nr, const float* x, int xs, int nt, int cols, float* y, int ystride)
{
    int r = 0;
    for (; r + 4 <= nr; r += 4) {
        const float *w0 = w + (int64_t)r * ws, *w1 = w0 + ws, *w2 = w1 + ws, *w3 = w2 + ws;
        int t = 0;
        for (; t + 2 <= nt; t += 2) {
            const float *xa = x + (int64_t)t * xs, *xb = xa + xs;
            float a0 = 0, a1 = 0, a2 = 0, a3 = 0, b0 = 0, b1 = 0, b2 = 0, b3 = 0;
            for (int i = 0; i < cols; i++) {
                float va = xa[i], vb = xb[i];
                float u0 = w0[i], u1 = w1[i], u2 = w2[i], u3 = w3[i];
                a0 += u0 * va; a1 += u1 * va; a2 += u2 * va; a3 += u3 * va;
                b0 += u0 * vb; b1 += u1 * vb; b2 += u2 * vb; b3 += u3 * vb;
            }
            float *ya = y + (int64_t)t * ystride + r, *yb = ya + ystride;
            ya[0] = a0; ya[1] = a1; ya[2] = a2; ya[3] = a3;
            yb[0] = b0; yb[1] = b1; yb[2] = b2; yb[3] = b3;
        }
        for (; t < nt; t++) {
            const float* xa = x + (int64_t)t * xs;
            float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
            for (int i = 0; i < cols; i++) {
                float va = xa[i];
                a0 += w0[i] * va; a1 += w1[i] * va; a2 += w2[i] * va; a3 += w3[i] * va;
            }
            float* ya = y + (int64_t)t * ystride + r;
            ya[0] = a0; ya[1] = a1; ya[2] = a2; ya[3] = a3;
        }
    }
    for (; r < nr; r++) {
        const float* wr = w + (int64_t)r * ws;
        for (int t = 0; t < nt; t++) {
            const float* xa = x + (int64_t)t * xs;
            float s = 0;
            for (int i = 0; i < cols; i++) s += wr[i] * xa[i];
            y[(int64_t)t * ystride + r] = s;
        }
    }
}

/* ---------- Transformer.MatMul / MatMulEach (Transformer.cs:483-561), the float paths ---------- */
#define ROW_TILE 32
typedef struct {
    int type, rows, cols, T, mode;   /* mode 0: fused T==1, 1: each-token, 2: decode tile + Block */
    int64_t row_bytes;
    const uint8_t* w; const float* x; float* y;
} mm_ctx;

static void mm_task(void* vctx, int64_t begin, int64_t end)
{
    mm_ctx* c = (mm_ctx*)vctx;
    float* scratch = NULL;
    if (c->mode == 2) scratch = (float*)malloc(sizeof(float) * ROW_TILE * (size_t)c->cols);
    for (int64_t tile = begin; tile < end; tile++) {
        int r0 = (int)tile * ROW_TILE, r1 = r0 + ROW_TILE < c->rows ? r0 + ROW_TILE : c->rows;
        if (c->mode == 0) {
            for (int r = r0; r < r1; r++) c->y[r] = or_dot_row(c->type, c->w + r * c->row_bytes, c->x, c->cols);
        } else if (c->mode == 1) {
            for (int r = r0; r < r1; r++)
                for (int t = 0; t < c->T; t++)
                    c->y[(int64_t)t * c->rows + r] = or_dot_row(c->type, c->w + r * c->row_bytes, c->x + (int64_t)t * c->cols, c->cols);
        } else {
            for (int r = r0; r < r1; r++) or_decode_row(c->type, c->w + r * c->row_bytes, c->cols, scratch + (int64_t)(r - r0) * c->cols);
            or_block(scratch, c->cols, r1 - r0, c->x, c->cols, c->T, c->cols, c->y + r0, c->rows);
        }
    }
    free(scratch);
}

int or_matmul(int type, const uint8_t* w, int rows, int cols, int64_t row_bytes, const float* x, int T, float* y,
              int each_token, int threads)
{
    if (!or_can_decode(type)) return -1;
    mm_ctx c;
    c.type = type; c.rows = rows; c.cols = cols; c.T = T; c.row_bytes = row_bytes; c.w = w; c.x = x; c.y = y;
    if (each_token && T > 1 && or_can_dot(type)) c.mode = 1;
    else if (T == 1 && or_can_dot(type)) c.mode = 0;
    else c.mode = 2;
    int tiles = (rows + ROW_TILE - 1) / ROW_TILE;
    or_parallel_for(tiles, threads, mm_task, &c);
    return 0;
}
