/*
 * q35_oracle.c -- CPU restatement of the reference's numerics (formats,
 * quantizers, dequantizers, scalar dots, elementwise ops).  TEST
 * INFRASTRUCTURE ONLY: see q35_oracle.h for the rules and for the list of
 * reference locations each function follows.
 *
 * Compiled with -ffp-contract=off: every `a*b + c` below is two roundings,
 * exactly as the reference's scalar C (and Zig, which never contracts without
 * an explicit float mode) evaluates it.
 */
#include "q35_oracle.h"

#include <math.h>
#include <string.h>
#include <stdlib.h>

/* ====================================================================== */
/* f16 <-> f32 (src/kernels/x86/kernels32.c:46-101)                        */
/* ====================================================================== */

float q35o_f16_to_f32(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (uint32_t)(h >> 10) & 0x1Fu;
    const uint32_t m = (uint32_t)(h & 0x3FFu);
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            /* subnormal: m * 2^-24, normalised into [512, 1024) */
            uint32_t mm = m, lz = 0;
            while (mm < 0x200u) { mm <<= 1; lz++; }
            bits = sign | ((112u - lz) << 23) | ((mm & 0x1FFu) << 14);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* f32 -> f16 bits, round-to-nearest-even, inf/nan -> inf.  `sub_carry` is
 * the bit pattern written when a subnormal rounds up into the smallest
 * normal: IEEE gives 0x0400 (2^-14); the reference's activation quantizer
 * (kernels32.c:95, k32_f32_to_f16bits) writes 0x0380, and that value is kept
 * for it so the quantized activation bytes match the reference exactly. */
static uint16_t f32_to_f16_impl(float x, uint16_t sub_carry)
{
    uint32_t u;
    memcpy(&u, &x, 4);
    const uint32_t sign = (u & 0x80000000u) >> 16;
    const uint32_t e = (u >> 23) & 0xFFu;
    const uint32_t m = u & 0x7FFFFFu;
    if (e == 255u) return (uint16_t)(0x7C00u | sign);
    if (e >= 143u) return (uint16_t)(0x7C00u | sign);
    if (e >= 113u) {
        uint32_t keep = m >> 13;
        const uint32_t drop = m & 0x1FFFu;
        const uint32_t up = (drop > 0x1000u) || (drop == 0x1000u && (keep & 1u));
        keep += up;
        uint32_t e16 = e - 112u;
        if (keep >= 0x400u) { keep = 0; e16 += 1; }
        if (e16 > 30u) return (uint16_t)(0x7C00u | sign);
        return (uint16_t)(sign | (e16 << 10) | keep);
    }
    {
        const uint32_t t = m | 0x800000u;
        const int s = (int)(126u - e);
        if (s >= 25) return (uint16_t)sign;
        uint32_t keep = t >> s;
        const uint32_t drop = t & ((1u << s) - 1u);
        const uint32_t mid = 1u << (s - 1);
        const uint32_t up = (drop > mid) || (drop == mid && (keep & 1u));
        keep += up;
        if (keep >= 0x400u) return (uint16_t)(sub_carry | sign);
        return (uint16_t)(sign | keep);
    }
}

/* IEEE conversion (Zig @floatCast, used by the weight quantizer) */
uint16_t q35o_f32_to_f16(float x) { return f32_to_f16_impl(x, 0x0400u); }
/* the reference C activation quantizer's conversion */
static uint16_t f32_to_f16_act(float x) { return f32_to_f16_impl(x, 0x0380u); }

static inline float f16at(const uint8_t *p)
{
    return q35o_f16_to_f32((uint16_t)(p[0] | ((uint16_t)p[1] << 8)));
}
static inline float f32at(const uint8_t *p)
{
    float f;
    memcpy(&f, p, 4);
    return f;
}
static inline int32_t i16at(const uint8_t *p)
{
    int16_t v;
    memcpy(&v, p, 2);
    return (int32_t)v;
}

/* ====================================================================== */
/* geometry (src/gguf.zig:185-215)                                         */
/* ====================================================================== */

int q35o_block_geom(int ttype, int *elems, int *bytes)
{
    int e = 0, b = 0;
    switch (ttype) {
    case Q35O_TT_Q8_0: e = 32; b = 34; break;
    case Q35O_TT_Q4_0: e = 32; b = 18; break;
    case Q35O_TT_Q4_1: e = 32; b = 20; break;
    case Q35O_TT_Q5_0: e = 32; b = 22; break;
    case Q35O_TT_Q5_1: e = 32; b = 24; break;
    case Q35O_TT_IQ4_NL: e = 32; b = 18; break;
    case Q35O_TT_Q4_K: e = 256; b = 144; break;
    case Q35O_TT_Q5_K: e = 256; b = 176; break;
    case Q35O_TT_Q6_K: e = 256; b = 210; break;
    case Q35O_TT_IQ4_XS: e = 256; b = 136; break;
    case Q35O_TT_Q8_K: e = 256; b = 292; break;
    default: return 0;
    }
    if (elems) *elems = e;
    if (bytes) *bytes = b;
    return 1;
}

/* src/backend_cpu.zig:42-50 (actFamily) */
int q35o_act_block_elems(int ttype)
{
    int e;
    if (!q35o_block_geom(ttype, &e, NULL) || ttype == Q35O_TT_Q8_K) return 0;
    return e == 32 ? 32 : 256;
}

size_t q35o_row_bytes(int ttype, int cols)
{
    int e, b;
    if (!q35o_block_geom(ttype, &e, &b)) return 0;
    return (size_t)(cols / e) * (size_t)b;
}

size_t q35o_act_row_bytes(int ttype, int cols)
{
    const int f = q35o_act_block_elems(ttype);
    if (f == 32) return (size_t)(cols / 32) * 34u;
    if (f == 256) return (size_t)(cols / 256) * 292u;
    return 0;
}

/* ====================================================================== */
/* activation quantizers                                                   */
/* ====================================================================== */

/* kernels32.c:1064-1090: amax/127 stored f16; q = trunc(v +- 0.5). */
void q35o_quantize_q8_0(int n, const float *x, uint8_t *out)
{
    for (int ib = 0; ib < n / 32; ib++) {
        const float *xb = x + ib * 32;
        uint8_t *yb = out + ib * 34;
        float amax = 0.0f;
        for (int k = 0; k < 32; k++) {
            const float a = xb[k] < 0.0f ? -xb[k] : xb[k];
            if (a > amax) amax = a;
        }
        const float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
        const float inv = amax > 0.0f ? 1.0f / scale : 0.0f;
        const uint16_t sb = f32_to_f16_act(scale);
        yb[0] = (uint8_t)(sb & 0xFF);
        yb[1] = (uint8_t)(sb >> 8);
        for (int k = 0; k < 32; k++) {
            const float v = xb[k] * inv;
            int q = (int)(v + (v >= 0.0f ? 0.5f : -0.5f));
            if (q > 127) q = 127;
            if (q < -128) q = -128;
            yb[2 + k] = (uint8_t)(int8_t)q;
        }
    }
}

/* kernels256.c:865-900: f32 scale, roundf, clamp [-127,127], bsums. */
void q35o_quantize_q8_K(int n, const float *x, uint8_t *out)
{
    for (int i = 0; i < n; i += 256) {
        uint8_t *o = out + (size_t)(i / 256) * 292;
        float amax = 0.0f;
        for (int j = 0; j < 256; j++) {
            const float a = x[i + j] < 0.0f ? -x[i + j] : x[i + j];
            if (a > amax) amax = a;
        }
        const float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
        const float inv = amax > 0.0f ? 1.0f / scale : 0.0f;
        memcpy(o, &scale, 4);
        int16_t gsum[16] = {0};
        for (int k = 0; k < 256; k++) {
            float r = roundf(x[i + k] * inv);
            if (r < -127.0f) r = -127.0f;
            if (r > 127.0f) r = 127.0f;
            if (!(r >= -127.0f)) r = 127.0f;
            const int8_t q = (int8_t)(int32_t)r;
            o[4 + k] = (uint8_t)q;
            gsum[k / 16] = (int16_t)(gsum[k / 16] + (int32_t)q);
        }
        for (int g = 0; g < 16; g++) memcpy(o + 260 + g * 2, &gsum[g], 2);
    }
}

void q35o_quantize_act(int ttype, int n, const float *x, uint8_t *out)
{
    if (q35o_act_block_elems(ttype) == 32)
        q35o_quantize_q8_0(n, x, out);
    else
        q35o_quantize_q8_K(n, x, out);
}

/* ====================================================================== */
/* weight quantizers                                                       */
/* ====================================================================== */

/* src/quant_dequant.zig:1404-1425.  scale32 = max/127, stored as f16;
 * q = round(x / scale32) (half away from zero).  An all-zero block divides
 * 0 by 0 in the reference (undefined); here it encodes q = 0. */
void q35o_quantize_weight_q8_0(int n, const float *x, uint8_t *out)
{
    for (int ib = 0; ib < n / 32; ib++) {
        const float *xb = x + ib * 32;
        uint8_t *yb = out + ib * 34;
        float mx = 0.0f;
        for (int k = 0; k < 32; k++) {
            const float v = fabsf(xb[k]);
            if (v > mx) mx = v;
        }
        const float scale32 = mx / 127.0f;
        const uint16_t sb = q35o_f32_to_f16(scale32);
        yb[0] = (uint8_t)(sb & 0xFF);
        yb[1] = (uint8_t)(sb >> 8);
        for (int k = 0; k < 32; k++) {
            int q = 0;
            if (scale32 > 0.0f) q = (int)roundf(xb[k] / scale32);
            if (q > 127) q = 127;
            if (q < -128) q = -128;
            yb[2 + k] = (uint8_t)(int8_t)q;
        }
    }
}

static const int8_t kIq4nl[16] = {
    -127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113,
};

static inline int clampi(int v, int lo, int hi)
{
    return v < lo ? lo : (v > hi ? hi : v);
}

/* IQ4_NL, one 32-element block: scale maps the largest-magnitude element to
 * codebook entry 0 (-127); every element takes the nearest codebook value
 * (first of equals). */
static void wq_iq4_nl_block(const float *x, uint8_t *y)
{
    float amax = 0.0f, vmax = 0.0f;
    for (int i = 0; i < 32; i++) {
        const float a = fabsf(x[i]);
        if (a > amax) { amax = a; vmax = x[i]; }
    }
    const float d = vmax / -127.0f;
    const uint16_t dh = q35o_f32_to_f16(d);
    const float dr = q35o_f16_to_f32(dh);
    const float id = dr != 0.0f ? 1.0f / dr : 0.0f;
    y[0] = (uint8_t)(dh & 0xFF);
    y[1] = (uint8_t)(dh >> 8);
    uint8_t idx[32];
    for (int i = 0; i < 32; i++) {
        const float v = x[i] * id;
        int best = 0;
        float berr = fabsf(v - (float)kIq4nl[0]);
        for (int k = 1; k < 16; k++) {
            const float e = fabsf(v - (float)kIq4nl[k]);
            if (e < berr) { berr = e; best = k; }
        }
        idx[i] = (uint8_t)best;
    }
    for (int j = 0; j < 16; j++) y[2 + j] = (uint8_t)(idx[j] | (idx[j + 16] << 4));
}

/* Q4_0 / Q5_0 (symmetric, 2^(bits-1) levels either side) and Q4_1 / Q5_1
 * (affine over [min, max]) encoders of this project, one 32-element block:
 * d from the value of largest magnitude (or the range) rounded to f16, the
 * elements quantized against the rounded scale.  GGUF layout: element j < 16
 * in the low nibble of qs[j], element j + 16 in the high nibble; Q5 keeps bit
 * 4 of element j in bit j of qh. */
static void wq_legacy_block(int tt, const float *x, uint8_t *y)
{
    const int affine = tt == Q35O_TT_Q4_1 || tt == Q35O_TT_Q5_1;
    const int five = tt == Q35O_TT_Q5_0 || tt == Q35O_TT_Q5_1;
    const int qmax = five ? 31 : 15;
    uint8_t q[32];
    if (affine) {
        float mn = x[0], mx = x[0];
        for (int i = 1; i < 32; i++) {
            if (x[i] < mn) mn = x[i];
            if (x[i] > mx) mx = x[i];
        }
        const uint16_t dh = q35o_f32_to_f16((mx - mn) / (float)qmax), mh = q35o_f32_to_f16(mn);
        const float dr = q35o_f16_to_f32(dh), mr = q35o_f16_to_f32(mh);
        const float id = dr != 0.0f ? 1.0f / dr : 0.0f;
        for (int i = 0; i < 32; i++) {
            int v = (int)((x[i] - mr) * id + 0.5f);
            q[i] = (uint8_t)(v < 0 ? 0 : (v > qmax ? qmax : v));
        }
        y[0] = (uint8_t)(dh & 0xFF); y[1] = (uint8_t)(dh >> 8);
        y[2] = (uint8_t)(mh & 0xFF); y[3] = (uint8_t)(mh >> 8);
    } else {
        float amax = 0.0f, vmax = 0.0f;
        for (int i = 0; i < 32; i++) {
            const float a = fabsf(x[i]);
            if (a > amax) { amax = a; vmax = x[i]; }
        }
        const float half = five ? 16.0f : 8.0f;
        const uint16_t dh = q35o_f32_to_f16(vmax / -half);
        const float dr = q35o_f16_to_f32(dh);
        const float id = dr != 0.0f ? 1.0f / dr : 0.0f;
        for (int i = 0; i < 32; i++) {
            int v = (int)(x[i] * id + (half + 0.5f));
            q[i] = (uint8_t)(v < 0 ? 0 : (v > qmax ? qmax : v));
        }
        y[0] = (uint8_t)(dh & 0xFF); y[1] = (uint8_t)(dh >> 8);
    }
    const int qs_off = affine ? (five ? 8 : 4) : (five ? 6 : 2);
    if (five) {
        uint32_t qh = 0;
        for (int j = 0; j < 32; j++) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
        uint8_t *h = y + (affine ? 4 : 2);
        h[0] = (uint8_t)qh; h[1] = (uint8_t)(qh >> 8); h[2] = (uint8_t)(qh >> 16); h[3] = (uint8_t)(qh >> 24);
    }
    for (int j = 0; j < 16; j++) y[qs_off + j] = (uint8_t)((q[j] & 0x0F) | ((q[j + 16] & 0x0F) << 4));
}

/* Q4_K / Q5_K, one 256-element super-block.  Each 32-element sub-block gets
 * an affine range [mn, mx] with mn <= 0; its scale (mx-mn)/L and offset -mn
 * are quantized to 6 bits against f16 super-scales, and the elements are
 * re-quantized against the rounded pair.  L = 15 (Q4_K) or 31 (Q5_K). */
static void wq_kq_block(const float *x, uint8_t *y, int bits5)
{
    const float L = bits5 ? 31.0f : 15.0f;
    const int qmax = bits5 ? 31 : 15;
    float sc[8], mnv[8];
    float max_sc = 0.0f, max_mn = 0.0f;
    for (int j = 0; j < 8; j++) {
        float mn = x[j * 32], mx = x[j * 32];
        for (int i = 1; i < 32; i++) {
            const float v = x[j * 32 + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        sc[j] = (mx - mn) / L;
        mnv[j] = -mn;
        if (sc[j] > max_sc) max_sc = sc[j];
        if (mnv[j] > max_mn) max_mn = mnv[j];
    }
    const uint16_t dh = q35o_f32_to_f16(max_sc / 63.0f);
    const uint16_t mh = q35o_f32_to_f16(max_mn / 63.0f);
    const float dr = q35o_f16_to_f32(dh);
    const float mr = q35o_f16_to_f32(mh);
    int ls[8], lm[8];
    for (int j = 0; j < 8; j++) {
        ls[j] = dr > 0.0f ? clampi((int)roundf(sc[j] / dr), 0, 63) : 0;
        lm[j] = mr > 0.0f ? clampi((int)roundf(mnv[j] / mr), 0, 63) : 0;
    }
    y[0] = (uint8_t)(dh & 0xFF);
    y[1] = (uint8_t)(dh >> 8);
    y[2] = (uint8_t)(mh & 0xFF);
    y[3] = (uint8_t)(mh >> 8);
    uint8_t *s = y + 4;
    memset(s, 0, 12);
    /* inverse of get_scale_min_k4 (quant_dequant.zig:43-52) */
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(ls[j] & 63);
        s[j + 4] = (uint8_t)(lm[j] & 63);
    }
    for (int j = 4; j < 8; j++) {
        s[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
        s[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
        s[j] |= (uint8_t)((lm[j] >> 4) << 6);
    }
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
        const float ed = dr * (float)ls[j];
        const float em = mr * (float)lm[j];
        for (int i = 0; i < 32; i++) {
            int v = 0;
            if (ed > 0.0f) v = clampi((int)roundf((x[j * 32 + i] + em) / ed), 0, qmax);
            q[j * 32 + i] = (uint8_t)v;
        }
    }
    if (!bits5) {
        uint8_t *qs = y + 16;
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++)
                qs[c * 32 + l] = (uint8_t)((q[c * 64 + l] & 0xF) | ((q[c * 64 + 32 + l] & 0xF) << 4));
    } else {
        uint8_t *qh = y + 16;
        uint8_t *ql = y + 48;
        memset(qh, 0, 32);
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++) {
                const int lo = q[c * 64 + l], hi = q[c * 64 + 32 + l];
                ql[c * 32 + l] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
                qh[l] |= (uint8_t)(((lo >> 4) & 1) << (2 * c));
                qh[l] |= (uint8_t)(((hi >> 4) & 1) << (2 * c + 1));
            }
    }
}

/* Q6_K, one 256-element super-block: 16 sub-blocks of 16 with signed int8
 * scales against one f16 super-scale; values in [-32, 31] stored +32. */
static void wq_q6_k_block(const float *x, uint8_t *y)
{
    float sc[16];
    float max_abs = 0.0f;
    for (int j = 0; j < 16; j++) {
        float amax = 0.0f, vmax = 0.0f;
        for (int i = 0; i < 16; i++) {
            const float a = fabsf(x[j * 16 + i]);
            if (a > amax) { amax = a; vmax = x[j * 16 + i]; }
        }
        sc[j] = vmax / -32.0f;
        const float as = fabsf(sc[j]);
        if (as > max_abs) max_abs = as;
    }
    const uint16_t dh = q35o_f32_to_f16(max_abs / 127.0f);
    const float dr = q35o_f16_to_f32(dh);
    int8_t isc[16];
    for (int j = 0; j < 16; j++)
        isc[j] = (int8_t)(dr > 0.0f ? clampi((int)roundf(sc[j] / dr), -128, 127) : 0);
    uint8_t u[256];
    for (int j = 0; j < 16; j++) {
        const float ed = dr * (float)isc[j];
        for (int i = 0; i < 16; i++) {
            int v = 0;
            if (ed != 0.0f) v = clampi((int)roundf(x[j * 16 + i] / ed), -32, 31);
            u[j * 16 + i] = (uint8_t)(v + 32);
        }
    }
    uint8_t *ql = y, *qh = y + 128;
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            const uint8_t u0 = u[h * 128 + l], u1 = u[h * 128 + 32 + l];
            const uint8_t u2 = u[h * 128 + 64 + l], u3 = u[h * 128 + 96 + l];
            ql[h * 64 + l] = (uint8_t)((u0 & 0xF) | ((u2 & 0xF) << 4));
            ql[h * 64 + l + 32] = (uint8_t)((u1 & 0xF) | ((u3 & 0xF) << 4));
            qh[h * 32 + l] = (uint8_t)((u0 >> 4) | ((u1 >> 4) << 2) | ((u2 >> 4) << 4) | ((u3 >> 4) << 6));
        }
    for (int j = 0; j < 16; j++) y[192 + j] = (uint8_t)isc[j];
    y[208] = (uint8_t)(dh & 0xFF);
    y[209] = (uint8_t)(dh >> 8);
}

void q35o_quantize_weight(int ttype, int n, const float *x, uint8_t *out)
{
    switch (ttype) {
    case Q35O_TT_Q8_0: q35o_quantize_weight_q8_0(n, x, out); break;
    case Q35O_TT_Q4_0:
    case Q35O_TT_Q4_1:
    case Q35O_TT_Q5_0:
    case Q35O_TT_Q5_1: {
        int e, b;
        q35o_block_geom(ttype, &e, &b);
        for (int i = 0; i < n / 32; i++) wq_legacy_block(ttype, x + i * 32, out + (size_t)i * b);
        break;
    }
    case Q35O_TT_IQ4_NL:
        for (int b = 0; b < n / 32; b++) wq_iq4_nl_block(x + b * 32, out + b * 18);
        break;
    case Q35O_TT_Q4_K:
        for (int b = 0; b < n / 256; b++) wq_kq_block(x + b * 256, out + b * 144, 0);
        break;
    case Q35O_TT_Q5_K:
        for (int b = 0; b < n / 256; b++) wq_kq_block(x + b * 256, out + b * 176, 1);
        break;
    case Q35O_TT_Q6_K:
        for (int b = 0; b < n / 256; b++) wq_q6_k_block(x + b * 256, out + b * 210);
        break;
    default: break;
    }
}

/* ====================================================================== */
/* dequantizers (src/quant_dequant.zig)                                    */
/* ====================================================================== */

/* quant_dequant.zig:43-52 */
static void scale_min_k4(int j, const uint8_t *s, int *sc, int *m)
{
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* one native block; out gets block_elems floats */
static void dequant_block(int ttype, const uint8_t *x, float *out)
{
    switch (ttype) {
    case Q35O_TT_Q8_0: { /* quant_dequant.zig:1388-1402 */
        const float d = f16at(x);
        for (int j = 0; j < 32; j++) out[j] = d * (float)(int8_t)x[2 + j];
        break;
    }
    case Q35O_TT_Q4_0: { /* quant_dequant.zig:78-90 */
        const float d = f16at(x);
        for (int j = 0; j < 16; j++) {
            out[j] = ((float)(x[2 + j] & 0x0F) - 8.0f) * d;
            out[j + 16] = ((float)(x[2 + j] >> 4) - 8.0f) * d;
        }
        break;
    }
    case Q35O_TT_Q4_1: { /* quant_dequant.zig:92-103 */
        const float d = f16at(x), m = f16at(x + 2);
        for (int j = 0; j < 16; j++) {
            out[j] = (float)(x[4 + j] & 0x0F) * d + m;
            out[j + 16] = (float)(x[4 + j] >> 4) * d + m;
        }
        break;
    }
    case Q35O_TT_Q5_0:
    case Q35O_TT_Q5_1: { /* GGUF layout: low nibbles 0..15, high 16..31, bit 4 from qh */
        const int aff = ttype == Q35O_TT_Q5_1;
        const float d = f16at(x), m = aff ? f16at(x + 2) : 0.0f;
        const uint32_t qh = (uint32_t)x[aff ? 4 : 2] | ((uint32_t)x[aff ? 5 : 3] << 8) |
                            ((uint32_t)x[aff ? 6 : 4] << 16) | ((uint32_t)x[aff ? 7 : 5] << 24);
        const uint8_t *qs = x + (aff ? 8 : 6);
        for (int j = 0; j < 32; j++) {
            const int q = (j < 16 ? (qs[j] & 0x0F) : (qs[j - 16] >> 4)) | (int)(((qh >> j) & 1u) << 4);
            out[j] = aff ? (float)q * d + m : ((float)q - 16.0f) * d;
        }
        break;
    }
    case Q35O_TT_IQ4_NL: { /* quant_dequant.zig:347-360 */
        const float d = f16at(x);
        for (int j = 0; j < 16; j++) {
            out[j] = d * (float)kIq4nl[x[2 + j] & 0x0F];
            out[j + 16] = d * (float)kIq4nl[x[2 + j] >> 4];
        }
        break;
    }
    case Q35O_TT_IQ4_XS: { /* quant_dequant.zig:323-345: dl = d * (ls - 32) per 32 */
        const float d = f16at(x);
        const int sh = x[2] | (x[3] << 8);
        for (int ib = 0; ib < 8; ib++) {
            const int ls = ((x[4 + ib / 2] >> (4 * (ib % 2))) & 0x0F) | (((sh >> (2 * ib)) & 3) << 4);
            const float dl = d * (float)(ls - 32);
            const uint8_t *qs = x + 8 + 16 * ib;
            for (int j = 0; j < 16; j++) {
                out[32 * ib + j] = dl * (float)kIq4nl[qs[j] & 0x0F];
                out[32 * ib + 16 + j] = dl * (float)kIq4nl[qs[j] >> 4];
            }
        }
        break;
    }
    case Q35O_TT_Q4_K:
    case Q35O_TT_Q5_K: { /* quant_dequant.zig:54-76, 188-220 */
        const int q5 = ttype == Q35O_TT_Q5_K;
        const float d = f16at(x), mn = f16at(x + 2);
        const uint8_t *s = x + 4;
        const uint8_t *qh = x + 16;
        const uint8_t *q = q5 ? x + 48 : x + 16;
        int y = 0;
        uint8_t bm1 = 1, bm2 = 2;
        for (int c = 0; c < 4; c++) {
            int sc, m;
            scale_min_k4(2 * c, s, &sc, &m);
            const float d1 = d * (float)sc, m1 = mn * (float)m;
            scale_min_k4(2 * c + 1, s, &sc, &m);
            const float d2 = d * (float)sc, m2 = mn * (float)m;
            for (int l = 0; l < 32; l++) {
                const int hi = q5 ? ((qh[l] & bm1) ? 16 : 0) : 0;
                out[y + l] = d1 * (float)((q[l] & 0x0F) | hi) - m1;
            }
            for (int l = 0; l < 32; l++) {
                const int hi = q5 ? ((qh[l] & bm2) ? 16 : 0) : 0;
                out[y + 32 + l] = d2 * (float)((q[l] >> 4) | hi) - m2;
            }
            y += 64;
            q += 32;
            bm1 = (uint8_t)(bm1 << 2);
            bm2 = (uint8_t)(bm2 << 2);
        }
        break;
    }
    case Q35O_TT_Q6_K: { /* quant_dequant.zig:222-250 */
        const float d = f16at(x + 208);
        const uint8_t *ql = x, *qh = x + 128;
        const int8_t *sc = (const int8_t *)(x + 192);
        for (int n = 0; n < 256; n += 128) {
            const int qlb = n / 2, qhb = n / 4, scb = n / 16;
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const int q1 = (int)(int8_t)((ql[qlb + l] & 0x0F) | (((qh[qhb + l] >> 0) & 3) << 4)) - 32;
                const int q2 = (int)(int8_t)((ql[qlb + l + 32] & 0x0F) | (((qh[qhb + l] >> 2) & 3) << 4)) - 32;
                const int q3 = (int)(int8_t)((ql[qlb + l] >> 4) | (((qh[qhb + l] >> 4) & 3) << 4)) - 32;
                const int q4 = (int)(int8_t)((ql[qlb + l + 32] >> 4) | (((qh[qhb + l] >> 6) & 3) << 4)) - 32;
                out[n + l] = d * (float)sc[scb + is + 0] * (float)q1;
                out[n + l + 32] = d * (float)sc[scb + is + 2] * (float)q2;
                out[n + l + 64] = d * (float)sc[scb + is + 4] * (float)q3;
                out[n + l + 96] = d * (float)sc[scb + is + 6] * (float)q4;
            }
        }
        break;
    }
    default: break;
    }
}

void q35o_dequant_row(int ttype, const uint8_t *row, float *out, int cols)
{
    int e, b;
    if (!q35o_block_geom(ttype, &e, &b)) return;
    for (int i = 0; i < cols / e; i++) dequant_block(ttype, row + (size_t)i * b, out + (size_t)i * e);
}

/* ====================================================================== */
/* scalar block dots                                                       */
/* ====================================================================== */

/* integer dot of one 32-block: Q8_0 (kernels32.c:447-466), IQ4_NL
 * (kernels32.c:342-365), Q4_0 */
static int32_t isum32(int ttype, const uint8_t *xb, const uint8_t *yb)
{
    int32_t s = 0;
    if (ttype == Q35O_TT_Q8_0) {
        for (int j = 0; j < 32; j++) s += (int32_t)(int8_t)xb[2 + j] * (int32_t)(int8_t)yb[2 + j];
    } else if (ttype == Q35O_TT_IQ4_NL) {
        for (int j = 0; j < 16; j++) {
            s += (int32_t)kIq4nl[xb[2 + j] & 0x0F] * (int32_t)(int8_t)yb[2 + j];
            s += (int32_t)kIq4nl[xb[2 + j] >> 4] * (int32_t)(int8_t)yb[2 + 16 + j];
        }
    } else if (ttype == Q35O_TT_Q4_0) { /* kernels32.c:297-316 */
        for (int j = 0; j < 16; j++) {
            s += ((int32_t)(xb[2 + j] & 0x0F) - 8) * (int32_t)(int8_t)yb[2 + j];
            s += ((int32_t)(xb[2 + j] >> 4) - 8) * (int32_t)(int8_t)yb[2 + 16 + j];
        }
    } else if (ttype == Q35O_TT_Q4_1) { /* kernels32.c:318-340 */
        for (int j = 0; j < 16; j++) {
            s += (int32_t)(xb[4 + j] & 0x0F) * (int32_t)(int8_t)yb[2 + j];
            s += (int32_t)(xb[4 + j] >> 4) * (int32_t)(int8_t)yb[2 + 16 + j];
        }
    } else if (ttype == Q35O_TT_Q5_0 || ttype == Q35O_TT_Q5_1) {
        /* kernels32.c:546-566, 628-652 arithmetic; the GGUF nibble layout
         * (the reference's AVX2 unpack, kernels32.c:485-509) */
        const int aff = ttype == Q35O_TT_Q5_1;
        const uint8_t *h = xb + (aff ? 4 : 2), *qs = xb + (aff ? 8 : 6);
        const uint32_t qh = (uint32_t)h[0] | ((uint32_t)h[1] << 8) | ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
        for (int j = 0; j < 32; j++) {
            const int32_t q = (j < 16 ? (qs[j] & 0x0F) : (qs[j - 16] >> 4)) | (int32_t)(((qh >> j) & 1u) << 4);
            s += (aff ? q : q - 16) * (int32_t)(int8_t)yb[2 + j];
        }
    }
    return s;
}

/* sum of the 32 activation values of a Q8_0 block (the min term of Q4_1 /
 * Q5_1, kernels32.c:336, 646) */
static int32_t sumy32(const uint8_t *yb)
{
    int32_t s = 0;
    for (int j = 0; j < 32; j++) s += (int32_t)(int8_t)yb[2 + j];
    return s;
}

/* kernels256.c:185-230 (aux8 builders) + dot256 (kernels256.c:217-228) */
static void kq_aux8(int ttype, const uint8_t *x, int8_t *a8)
{
    if (ttype == Q35O_TT_Q4_K) {
        const uint8_t *q4 = x + 16;
        for (int c = 0; c < 4; c++) {
            for (int l = 0; l < 32; l++) a8[c * 64 + l] = (int8_t)(q4[c * 32 + l] & 0x0F);
            for (int l = 0; l < 32; l++) a8[c * 64 + 32 + l] = (int8_t)(q4[c * 32 + l] >> 4);
        }
    } else if (ttype == Q35O_TT_Q5_K) {
        const uint8_t *q4 = x + 48, *hm = x + 16;
        int m = 1;
        for (int c = 0; c < 4; c++) {
            for (int l = 0; l < 32; l++) a8[c * 64 + l] = (int8_t)((q4[c * 32 + l] & 0x0F) + ((hm[l] & m) ? 16 : 0));
            for (int l = 0; l < 32; l++) a8[c * 64 + 32 + l] = (int8_t)((q4[c * 32 + l] >> 4) + ((hm[l] & (m << 1)) ? 16 : 0));
            m <<= 2;
        }
    } else { /* Q6_K */
        const uint8_t *q4 = x, *qh = x + 128;
        for (int h = 0; h < 2; h++)
            for (int l = 0; l < 32; l++) {
                a8[h * 128 + l + 0] = (int8_t)(((q4[h * 64 + l] & 0x0F) | (((qh[h * 32 + l] >> 0) & 3) << 4)) - 32);
                a8[h * 128 + l + 32] = (int8_t)(((q4[h * 64 + l + 32] & 0x0F) | (((qh[h * 32 + l] >> 2) & 3) << 4)) - 32);
                a8[h * 128 + l + 64] = (int8_t)(((q4[h * 64 + l] >> 4) | (((qh[h * 32 + l] >> 4) & 3) << 4)) - 32);
                a8[h * 128 + l + 96] = (int8_t)(((q4[h * 64 + l + 32] >> 4) | (((qh[h * 32 + l] >> 6) & 3) << 4)) - 32);
            }
    }
}

static int32_t dot256(const int8_t *a8, const uint8_t *q8, const int32_t *sc)
{
    int32_t isum = 0;
    for (int g = 0; g < 16; g++) {
        int32_t sub = 0;
        for (int l = 0; l < 16; l++) sub += (int32_t)a8[g * 16 + l] * (int32_t)(int8_t)q8[g * 16 + l];
        isum += sc[g] * sub;
    }
    return isum;
}

/* K-quant block: scaled integer sum and (Q4_K/Q5_K) the min-term integer sum */
static void kq_isums(int ttype, const uint8_t *x, const uint8_t *y, int32_t *isum, int32_t *msum)
{
    int8_t a8[256];
    int32_t scv[16];
    kq_aux8(ttype, x, a8);
    *msum = 0;
    if (ttype == Q35O_TT_Q6_K) {
        const int8_t *sc = (const int8_t *)(x + 192);
        for (int g = 0; g < 16; g++) scv[g] = (int32_t)sc[g];
    } else {
        int sm[16];
        for (int j = 0; j < 8; j++) scale_min_k4(j, x + 4, &sm[j], &sm[8 + j]);
        int32_t s = 0;
        for (int j = 0; j < 16; j++) s += i16at(y + 260 + j * 2) * (int32_t)sm[8 + j / 2];
        *msum = s;
        for (int g = 0; g < 16; g++) scv[g] = (int32_t)sm[g / 2];
    }
    *isum = dot256(a8, y + 4, scv);
}

int32_t q35o_block_isum(int ttype, const uint8_t *wblk, const uint8_t *xblk)
{
    int32_t is, ms;
    if (q35o_act_block_elems(ttype) == 32) return isum32(ttype, wblk, xblk);
    kq_isums(ttype, wblk, xblk, &is, &ms);
    return is;
}

/* Strict block-order f32 fold, the reference scalar tier:
 *   Q8_0 / IQ4_NL: sumf += dx*dy*(float)isum     (kernels32.c:361, 462)
 *   Q4_K / Q5_K  : sumf += d*(float)isum - dmin*(float)sumi, d = dy*dw
 *                                                 (kernels256.c:494, 625)
 *   Q6_K         : sumf += dw*dy*(float)isum      (kernels256.c:735) */
float q35o_vec_dot(int ttype, int n, const uint8_t *w, const uint8_t *xq)
{
    float sumf = 0.0f;
    if (q35o_act_block_elems(ttype) == 32) {
        int e, b;
        q35o_block_geom(ttype, &e, &b);
        const int aff = ttype == Q35O_TT_Q4_1 || ttype == Q35O_TT_Q5_1;
        for (int ib = 0; ib < n / 32; ib++) {
            const uint8_t *xb = w + (size_t)ib * b, *yb = xq + (size_t)ib * 34;
            const float dx = f16at(xb), dy = f16at(yb);
            const int32_t s = isum32(ttype, xb, yb);
            if (aff) /* kernels32.c:338, 648: sumf += dx*dy*sumi + mx*dy*sumy */
                sumf += dx * dy * (float)s + f16at(xb + 2) * dy * (float)sumy32(yb);
            else
                sumf += dx * dy * (float)s;
        }
        return sumf;
    }
    int e, b;
    q35o_block_geom(ttype, &e, &b);
    if (ttype == Q35O_TT_IQ4_XS) {
        /* iq_kernels.c:967-1000 (scalar tier): d4d8 = d * dy; per 32-element
         * sub-block d1 = d4d8 * (ls - 32), sumf += d1 * (sumi1 + sumi2) */
        for (int i = 0; i < n / 256; i++) {
            const uint8_t *x = w + (size_t)i * b, *y = xq + (size_t)i * 292;
            const float d4d8 = f16at(x) * f32at(y);
            const int sh = x[2] | (x[3] << 8);
            const int8_t *q8 = (const int8_t *)(y + 4);
            for (int ib = 0; ib < 8; ib++) {
                const int ls = ((x[4 + ib / 2] >> (4 * (ib % 2))) & 0x0F) | (((sh >> (2 * ib)) & 3) << 4);
                const float d1 = d4d8 * (float)(ls - 32);
                const uint8_t *qs = x + 8 + 16 * ib;
                int32_t s1 = 0, s2 = 0;
                for (int j = 0; j < 16; j++) {
                    s1 += (int32_t)q8[32 * ib + j] * (int32_t)kIq4nl[qs[j] & 0x0F];
                    s2 += (int32_t)q8[32 * ib + 16 + j] * (int32_t)kIq4nl[qs[j] >> 4];
                }
                sumf += d1 * (float)(s1 + s2);
            }
        }
        return sumf;
    }
    for (int i = 0; i < n / 256; i++) {
        const uint8_t *x = w + (size_t)i * b, *y = xq + (size_t)i * 292;
        int32_t isum, msum;
        kq_isums(ttype, x, y, &isum, &msum);
        const float dy = f32at(y);
        if (ttype == Q35O_TT_Q6_K) {
            sumf += f16at(x + 208) * dy * (float)isum;
        } else {
            const float d = dy * f16at(x);
            const float dmin = dy * f16at(x + 2);
            sumf += d * (float)isum - dmin * (float)msum;
        }
    }
    return sumf;
}

void q35o_matvec_f32(const float *w, const float *x, float *out, int rows, int cols, int tokens)
{
    for (int t = 0; t < tokens; t++)
        for (int r = 0; r < rows; r++) {
            float acc = 0.0f;
            for (int c = 0; c < cols; c++) acc = fmaf(w[(size_t)r * cols + c], x[(size_t)t * cols + c], acc);
            out[(size_t)t * rows + r] = acc;
        }
}

void q35o_matvec_w16(int ttype, const uint16_t *w, const float *x, float *out, int rows, int cols, int tokens)
{
    for (int t = 0; t < tokens; t++)
        for (int r = 0; r < rows; r++) {
            float acc = 0.0f;
            for (int c = 0; c < cols; c++) {
                const uint16_t h = w[(size_t)r * cols + c];
                float wv;
                if (ttype == 30) {
                    const uint32_t bits = (uint32_t)h << 16;
                    memcpy(&wv, &bits, 4);
                } else {
                    wv = q35o_f16_to_f32(h);
                }
                acc = fmaf(wv, x[(size_t)t * cols + c], acc);
            }
            out[(size_t)t * rows + r] = acc;
        }
}

void q35o_matvec_q(int ttype, const uint8_t *w, const uint8_t *xq, float *out,
                   int rows, int cols, int tokens)
{
    const size_t rb = q35o_row_bytes(ttype, cols);
    const size_t ab = q35o_act_row_bytes(ttype, cols);
    for (int t = 0; t < tokens; t++)
        for (int r = 0; r < rows; r++)
            out[(size_t)t * rows + r] = q35o_vec_dot(ttype, cols, w + (size_t)r * rb, xq + (size_t)t * ab);
}

void q35o_matvec(int ttype, const uint8_t *w, const float *x, float *out,
                 int rows, int cols, int tokens)
{
    const size_t ab = q35o_act_row_bytes(ttype, cols);
    uint8_t *xq = (uint8_t *)malloc(ab * (size_t)tokens + 1);
    for (int t = 0; t < tokens; t++) q35o_quantize_act(ttype, cols, x + (size_t)t * cols, xq + (size_t)t * ab);
    q35o_matvec_q(ttype, w, xq, out, rows, cols, tokens);
    free(xq);
}

/* ====================================================================== */
/* elementwise (src/elementwise.zig)                                       */
/* ====================================================================== */

/* elementwise.zig:43-57: serial sum of squares; out = x*scale*w */
void q35o_rmsnorm(float *out, const float *x, const float *w, int n, float eps)
{
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

void q35o_rmsnorm_rows(float *out, const float *x, const float *w, int rows, int n, float eps)
{
    for (int r = 0; r < rows; r++) q35o_rmsnorm(out + (size_t)r * n, x + (size_t)r * n, w, n, eps);
}

/* elementwise.zig:100-105 */
void q35o_l2norm(float *x, int n)
{
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss + 1e-6f);
    for (int i = 0; i < n; i++) x[i] *= inv;
}

void q35o_scale_vec(float *x, int n, float s)
{
    for (int i = 0; i < n; i++) x[i] *= s;
}

/* backend_cpu.zig:935-942: l2norm every q row, every k row, then q *= qscale */
void q35o_l2norm_qk_scale(float *x, int nk, int kd, int k_offset, float qscale)
{
    for (int r = 0; r < nk; r++) q35o_l2norm(x + (size_t)r * kd, kd);
    for (int r = 0; r < nk; r++) q35o_l2norm(x + k_offset + (size_t)r * kd, kd);
    q35o_scale_vec(x, nk * kd, qscale);
}

float q35o_silu(float x) { return x / (1.0f + Q35O_EXPF(-x)); }
float q35o_sigmoid(float x) { return 1.0f / (1.0f + Q35O_EXPF(-x)); }
/* elementwise.zig:89-91 (threshold 20) */
float q35o_softplus(float x) { return x > 20.0f ? x : Q35O_LOG1PF(Q35O_EXPF(x)); }

void q35o_silu_vec(float *x, int n)
{
    for (int i = 0; i < n; i++) x[i] = x[i] / (1.0f + Q35O_EXPF(-x[i]));
}

void q35o_mul_silu(float *out, const float *gate, int n)
{
    for (int i = 0; i < n; i++) {
        const float g = gate[i];
        out[i] = out[i] * (g / (1.0f + Q35O_EXPF(-g)));
    }
}

void q35o_mul_sigmoid(float *out, const float *gate, int n)
{
    for (int i = 0; i < n; i++) out[i] = out[i] * (1.0f / (1.0f + Q35O_EXPF(-gate[i])));
}

/* elementwise.zig:27 bufSwiglu: g = silu(g) * u */
void q35o_swiglu(float *gate, const float *up, int n)
{
    for (int i = 0; i < n; i++) gate[i] = q35o_silu(gate[i]) * up[i];
}

/* elementwise.zig:93-102 */
void q35o_softmax(float *x, int n)
{
    float mx = -3.40282347e38f;
    for (int i = 0; i < n; i++) mx = x[i] > mx ? x[i] : mx;
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = Q35O_EXPF(x[i] - mx);
        sum += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

void q35o_add_resid(float *dst, const float *src, int n)
{
    for (int i = 0; i < n; i++) dst[i] += src[i];
}

/* elementwise.zig:306-318: dims 0..63 of one head, pairs (j, j+32),
 * theta = (f32)pos * base^(-(2j)/64).  The reference evaluates the power with
 * Zig's std.math.pow; this restatement uses the C library's powf. */
void q35o_rope64(float *x, int pos, float base)
{
    for (int j = 0; j < 32; j++) {
        const float theta = (float)pos * powf(base, -(float)(2 * j) / 64.0f);
        const float c = cosf(theta), s = sinf(theta);
        const float a = x[j], b = x[j + 32];
        x[j] = a * c - b * s;
        x[j + 32] = a * s + b * c;
    }
}

/* Every head of every row is rotated: the semantics of the reference's
 * device kernel (src/kernels/cuda/rope.cu:81-110) and of the per-head loop
 * engine.zig:1980-1995 describes.  (The reference CPU backend's
 * vRope64Rows, backend_cpu.zig:893-899, hands the whole row to applyRope64,
 * which only touches its first 64 floats, i.e. the first head.) */
void q35o_rope64_rows(float *x, int rows, int heads, int hd, int pos0, float base)
{
    for (int r = 0; r < rows; r++)
        for (int h = 0; h < heads; h++) q35o_rope64(x + ((size_t)r * heads + h) * hd, pos0 + r, base);
}

/* elementwise.zig:322-342: y = ((h0*w0 + h1*w1) + h2*w2) + x*w3, shift, silu */
void q35o_conv_step(float *conv, float *y, const float *w, int n)
{
    for (int i = 0; i < n; i++) {
        float *h = conv + (size_t)i * 3;
        const float cur = y[i];
        const float p0 = h[0] * w[i * 4], p1 = h[1] * w[i * 4 + 1];
        const float p2 = h[2] * w[i * 4 + 2], p3 = cur * w[i * 4 + 3];
        y[i] = p0 + p1 + p2 + p3;
        h[0] = h[1];
        h[1] = h[2];
        h[2] = cur;
    }
    q35o_silu_vec(y, n);
}

/* elementwise.zig:378-384 */
void q35o_gdn_gamma(const float *a_raw, float *b_raw, const float *ssm_a,
                    const float *dt_bias, float *gamma, int nv)
{
    for (int h = 0; h < nv; h++) {
        b_raw[h] = q35o_sigmoid(b_raw[h]);
        const float g = ssm_a[h] * q35o_softplus(a_raw[h] + dt_bias[h]);
        gamma[h] = Q35O_EXPF(g);
    }
}

/* elementwise.zig:221-278 (gdnFused, vd == 128 path; the same per-element
 * order serves any vd):
 *   pass 1: km[j] = (sum_i S[i][j]*k[i]) * gamma
 *   delta[j] = (v[j] - km[j]) * beta
 *   pass 2: S[i][j] = S[i][j]*gamma + k[i]*delta[j]; out[j] += S[i][j]*q[i] */
void q35o_gdn_fused(float *S, const float *k, const float *v, const float *q,
                    float *km, float *delta, float *out, float gamma, float beta,
                    int kd, int vd)
{
    for (int j = 0; j < vd; j++) {
        float acc = 0.0f;
        for (int i = 0; i < kd; i++) acc += S[(size_t)i * vd + j] * k[i];
        km[j] = acc * gamma;
    }
    for (int j = 0; j < vd; j++) delta[j] = (v[j] - km[j]) * beta;
    for (int j = 0; j < vd; j++) out[j] = 0.0f;
    for (int i = 0; i < kd; i++)
        for (int j = 0; j < vd; j++) {
            const float r = S[(size_t)i * vd + j] * gamma + k[i] * delta[j];
            S[(size_t)i * vd + j] = r;
            out[j] += r * q[i];
        }
}

/* backend_cpu.zig:983-1017: value head h uses k/q head h % nk */
void q35o_gdn_step_rows(float *state, const float *k, const float *v,
                        const float *q, float *km, float *delta, float *out,
                        const float *gamma, const float *beta, int heads,
                        int nk, int kd, int vd)
{
    for (int h = 0; h < heads; h++) {
        const int kh = h % nk;
        q35o_gdn_fused(state + (size_t)h * kd * vd, k + (size_t)kh * kd, v + (size_t)h * vd,
                       q + (size_t)kh * kd, km + (size_t)h * vd, delta + (size_t)h * vd,
                       out + (size_t)h * vd, gamma[h], beta[h], kd, vd);
    }
}

/* elementwise.zig:428-433 */
void q35o_deinterleave_qg(float *q, float *gate, const float *src, int heads, int hd)
{
    for (int h = 0; h < heads; h++) {
        memcpy(q + (size_t)h * hd, src + (size_t)h * 2 * hd, (size_t)hd * 4);
        memcpy(gate + (size_t)h * hd, src + (size_t)h * 2 * hd + hd, (size_t)hd * 4);
    }
}

/* elementwise.zig:349-372 */
void q35o_attn_decode(const float *q, const float *gate, const float *kcache,
                      const float *vcache, float *att, float *gout, int slot,
                      int heads, int gqa, int hd, int kv_dim, float scale)
{
    float accv[512];
    for (int h = 0; h < heads; h++) {
        const int kvh = h / gqa;
        const float *qs = q + (size_t)h * hd;
        for (int t = 0; t <= slot; t++) {
            const float *ks = kcache + (size_t)t * kv_dim + (size_t)kvh * hd;
            float acc = 0.0f;
            for (int j = 0; j < hd; j++) acc += qs[j] * ks[j];
            att[t] = acc * scale;
        }
        q35o_softmax(att, slot + 1);
        for (int j = 0; j < hd; j++) accv[j] = 0.0f;
        for (int t = 0; t <= slot; t++) {
            const float w = att[t];
            const float *vs = vcache + (size_t)t * kv_dim + (size_t)kvh * hd;
            for (int j = 0; j < hd; j++) accv[j] += w * vs[j];
        }
        memcpy(gout + (size_t)h * hd, accv, (size_t)hd * 4);
    }
    q35o_mul_sigmoid(gout, gate, heads * hd);
}

/* elementwise.zig:395-405: first index of the strict maximum */
int q35o_argmax(const float *x, int n)
{
    int best = 0;
    float bv = -INFINITY;
    for (int i = 0; i < n; i++)
        if (x[i] > bv) { bv = x[i]; best = i; }
    return best;
}

/* ====================================================================== */
/* seeded synthetic values (the library's q35b_synth_fill, restated):      */
/* splitmix64 finalizer over key*0x9E37.. + i*0xD1B5.., the four 16-bit    */
/* fields summed (Irwin-Hall n = 4) and centred, one f32 multiply by k.    */
/* Not part of the reference: it builds benchmark weights on the host.     */
/* ====================================================================== */
void q35o_synth_fill(uint64_t key, long long n, float k, float *dst)
{
    for (long long i = 0; i < n; i++) {
        uint64_t z = key * 0x9E3779B97F4A7C15ull + (uint64_t)i * 0xD1B54A32D192ED03ull;
        z ^= z >> 30;
        z *= 0xBF58476D1CE4E5B9ull;
        z ^= z >> 27;
        z *= 0x94D049BB133111EBull;
        z ^= z >> 31;
        const int sum = (int)(z & 0xffff) + (int)((z >> 16) & 0xffff) + (int)((z >> 32) & 0xffff) + (int)(z >> 48);
        dst[i] = (float)(sum - 131070) * k;
    }
}

/* ====================================================================== */
/* sampler (src/sampler.zig:60-190, Sampler.nextU64 / nextF32 / sample)    */
/* ====================================================================== */
static uint64_t o_xs64(uint64_t *s)
{
    uint64_t x = *s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 0x2545F4914F6CDD1DULL;
}

static int o_cmp_desc(const void *a, const void *b)
{
    const float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

/* the k-th largest value (0-based rank), sampler.zig:196-255: any exact
 * selection gives the same value; a descending sort here */
float q35o_kth_largest(float *a, int n, int rank)
{
    qsort(a, (size_t)n, sizeof(float), o_cmp_desc);
    return a[rank];
}

int q35o_sample(const float *logits, int n, float temperature, int top_k, float top_p, uint64_t *state,
                float *scratch)
{
    if (!(temperature > 0)) { /* :71-80 greedy, ties to the lowest index */
        int best = 0;
        float bv = -3.402823466e38f;
        for (int i = 0; i < n; i++)
            if (logits[i] > bv) {
                bv = logits[i];
                best = i;
            }
        return best;
    }
    const float t = temperature;
    float maxv = logits[0];
    for (int i = 1; i < n; i++)
        if (logits[i] > maxv) maxv = logits[i];
    float thresh = -3.402823466e38f;
    if (top_k > 0 && top_k < n) { /* :93-99 */
        memcpy(scratch, logits, (size_t)n * sizeof(float));
        thresh = q35o_kth_largest(scratch, n, top_k - 1);
    }
    if (top_p > 0 && top_p < 1) { /* :125-165 */
        double total = 0;
        for (int i = 0; i < n; i++)
            if (logits[i] >= thresh) total += (double)Q35O_EXPF((logits[i] - maxv) / t);
        if (total > 0) {
            const double target = total * (double)top_p;
            int ns = 0;
            for (int i = 0; i < n; i++)
                if (!(logits[i] < thresh)) scratch[ns++] = logits[i];
            qsort(scratch, (size_t)ns, sizeof(float), o_cmp_desc);
            double acc = 0;
            float cut = thresh;
            for (int i = 0; i < ns; i++) {
                acc += (double)Q35O_EXPF((scratch[i] - maxv) / t);
                if (acc >= target) {
                    cut = scratch[i];
                    break;
                }
            }
            if (cut > thresh) thresh = cut;
        }
    }
    double sum = 0; /* :167-172 */
    for (int i = 0; i < n; i++)
        if (logits[i] >= thresh) sum += (double)Q35O_EXPF((logits[i] - maxv) / t);
    if (*state == 0) *state = 0x9E3779B97F4A7C15ULL;
    const double coin = (double)((float)(o_xs64(state) >> 40) / 16777216.0f);
    double acc = 0;
    for (int i = 0; i < n; i++) { /* :174-184 */
        if (logits[i] < thresh) continue;
        acc += (double)Q35O_EXPF((logits[i] - maxv) / t);
        if (coin < acc / sum) return i;
    }
    for (int i = n; i > 0; i--) /* :185-189 */
        if (logits[i - 1] >= thresh) return i - 1;
    return 0;
}
