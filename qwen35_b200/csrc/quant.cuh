// quant.cuh -- activation quantizers, weight encoders and row dequantizers.
//
// Activation quantizers are bit-exact with the reference's CPU quantizers
// (src/kernels/x86/kernels32.c:1064-1090 quantize_q8_0,
//  src/kernels/x86/kernels256.c:865-900 quantize_q8_K): the max is order
// independent, and every scale / inverse / rounding is the same IEEE
// operation the C code performs.
#pragma once
#include "common.cuh"

namespace q35 {

// ---------------------------------------------------------------------------
// Q8_0 activation block (34 B / 32): one warp per block, lane = element.
// ---------------------------------------------------------------------------
Q35_DEV void quant_q8_0_warp(float v, uint8_t *yb, int lane) {
    const float amax = warp_max(fabsf(v));
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = amax > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    if (lane == 0) {
        const uint16_t sb = f32_to_f16_bits(scale, 0x0380u);
        yb[0] = (uint8_t)(sb & 0xFF);
        yb[1] = (uint8_t)(sb >> 8);
    }
    const float x = __fmul_rn(v, inv);
    int q = __float2int_rz(__fadd_rn(x, x >= 0.0f ? 0.5f : -0.5f));
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    yb[2 + lane] = (uint8_t)(int8_t)q;
}

__global__ void k_quantize_q8_0(const float *__restrict__ x, uint8_t *__restrict__ out, int nblocks) {
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    quant_q8_0_warp(x[(size_t)b * 32 + lane], out + (size_t)b * 34, lane);
}

// ---------------------------------------------------------------------------
// Q8_K activation block (292 B / 256): one warp per block, 8 values a lane.
// Lane l owns elements [8l, 8l+8); bsum group g = elements [16g, 16g+16) is
// lanes 2g and 2g+1.
// ---------------------------------------------------------------------------
Q35_DEV void quant_q8_K_warp(const float (&v)[8], uint8_t *o, int lane) {
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) a = fmaxf(a, fabsf(v[i]));
    const float amax = warp_max(a);
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = amax > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    if (lane == 0) *reinterpret_cast<float *>(o) = scale;
    int s = 0;
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float r = roundf(__fmul_rn(v[i], inv));
        if (r < -127.0f) r = -127.0f;
        if (r > 127.0f) r = 127.0f;
        if (!(r >= -127.0f)) r = 127.0f;
        const int q = (int)r;
        s += q;
        if (i < 4)
            w0 |= (uint32_t)(q & 0xFF) << (8 * i);
        else
            w1 |= (uint32_t)(q & 0xFF) << (8 * (i - 4));
    }
    uint32_t *qs = reinterpret_cast<uint32_t *>(o + 4);
    qs[lane * 2] = w0;
    qs[lane * 2 + 1] = w1;
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if ((lane & 1) == 0) *reinterpret_cast<int16_t *>(o + 260 + lane) = (int16_t)s;
}

__global__ void k_quantize_q8_K(const float *__restrict__ x, uint8_t *__restrict__ out, int nblocks) {
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    float v[8];
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)b * 256 + lane * 8);
    const float4 a = src[0], c = src[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    quant_q8_K_warp(v, out + (size_t)b * 292, lane);
}

// ---------------------------------------------------------------------------
// Row dequantizers (embedding lookup): src/quant_dequant.zig:54-76 (Q4_K),
// 188-220 (Q5_K), 222-250 (Q6_K), 347-360 (IQ4_NL), 1388-1402 (Q8_0).
// One thread per output element; bit-exact (same products in the same order).
// ---------------------------------------------------------------------------
Q35_DEV void kq_scale_min(int j, const uint8_t *s, int &sc, int &m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

__device__ __constant__ int8_t c_iq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                              1,    13,   25,  38,  53,  69,  89,  113};

Q35_DEV float dequant_elem(int tt, const uint8_t *row, int i) {
    switch (tt) {
    case TT_Q8_0: {
        const uint8_t *x = row + (i / 32) * 34;
        return __fmul_rn(f16_to_f32(ld_u16(x)), (float)(int8_t)x[2 + (i & 31)]);
    }
    case TT_IQ4_NL: {
        const uint8_t *x = row + (i / 32) * 18;
        const int j = i & 31;
        const int nib = j < 16 ? (x[2 + j] & 0xF) : (x[2 + j - 16] >> 4);
        return __fmul_rn(f16_to_f32(ld_u16(x)), (float)c_iq4nl[nib]);
    }
    case TT_IQ4_XS: {
        // quant_dequant.zig:323-345: dl = d * (ls - 32) per 32-element sub-block
        const uint8_t *x = row + (i / 256) * 136;
        const int k = i & 255, ib = k >> 5, j = k & 31;
        const int ls = iq4xs_ls(x[4 + (ib >> 1)], ld_u16(x + 2), ib);
        const float dl = __fmul_rn(f16_to_f32(ld_u16(x)), (float)(ls - 32));
        const uint8_t *qs = x + 8 + 16 * ib;
        const int nib = j < 16 ? (qs[j] & 0xF) : (qs[j - 16] >> 4);
        return __fmul_rn(dl, (float)c_iq4nl[nib]);
    }
    case TT_Q4_0:
    case TT_Q4_1:
    case TT_Q5_0:
    case TT_Q5_1: {
        // quant_dequant.zig:78-103 (Q4_0: (q - 8) * d; Q4_1: q * d + m); Q5
        // likewise with 5-bit q, centred at 16 for Q5_0
        const uint8_t *x = row + (i / 32) * geom_of(tt).bytes;
        const int j = i & 31;
        const uint8_t *qs = x + legacy_qs_off(tt);
        int q = j < 16 ? (qs[j] & 0xF) : (qs[j - 16] >> 4);
        if (legacy_five(tt)) {
            const uint8_t *h = x + legacy_qh_off(tt);
            q |= ((h[j >> 3] >> (j & 7)) & 1) << 4;
        }
        const float d = f16_to_f32(ld_u16(x));
        if (legacy_affine(tt)) return __fadd_rn(__fmul_rn((float)q, d), f16_to_f32(ld_u16(x + 2)));
        return __fmul_rn(__fsub_rn((float)q, legacy_five(tt) ? 16.0f : 8.0f), d);
    }
    case TT_Q4_K:
    case TT_Q5_K: {
        const bool q5 = tt == TT_Q5_K;
        const uint8_t *x = row + (i / 256) * (q5 ? 176 : 144);
        const int e = i & 255, c = e / 64, hi = (e & 63) >= 32, l = e & 31;
        int sc, m;
        kq_scale_min(2 * c + hi, x + 4, sc, m);
        const float d1 = __fmul_rn(f16_to_f32(ld_u16(x)), (float)sc);
        const float m1 = __fmul_rn(f16_to_f32(ld_u16(x + 2)), (float)m);
        const uint8_t *q = (q5 ? x + 48 : x + 16) + c * 32;
        int v = hi ? (q[l] >> 4) : (q[l] & 0xF);
        if (q5 && (x[16 + l] & (1 << (2 * c + hi)))) v |= 16;
        return __fsub_rn(__fmul_rn(d1, (float)v), m1);
    }
    case TT_Q6_K: {
        const uint8_t *x = row + (i / 256) * 210;
        const int e = i & 255, n = e / 128, r = e & 127, quarter = r / 32, l = r & 31;
        const uint8_t *ql = x + n * 64, *qh = x + 128 + n * 32;
        const int8_t *sc = reinterpret_cast<const int8_t *>(x + 192) + n * 8;
        const int lo4 = (quarter & 1) ? ql[l + 32] : ql[l];
        const int nib = (quarter >= 2) ? (lo4 >> 4) : (lo4 & 0xF);
        const int h2 = (qh[l] >> (2 * quarter)) & 3;
        const int q = (int)(int8_t)(nib | (h2 << 4)) - 32;
        const float d = f16_to_f32(ld_u16(x + 208));
        return __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * quarter]), (float)q);
    }
    default: return 0.0f;
    }
}

__global__ void k_dequant_row(int tt, const uint8_t *__restrict__ row, float *__restrict__ out, int cols) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < cols) out[i] = dequant_elem(tt, row, i);
}

// rows gathered by token id: out[t*cols + i] = dequant(W[tokens[t]])[i]
// token ids outside [0, vocab) read row 0 and record error 160
__global__ void k_embed_rows(int tt, const uint8_t *__restrict__ w, size_t row_bytes,
                             const int *__restrict__ tokens, float *__restrict__ out, int cols, long long vocab) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    long long tok = tokens[t];
    if (tok < 0 || tok >= vocab) {
        if (blockIdx.x == 0 && threadIdx.x == 0) set_error(160);
        tok = 0;
    }
    const uint8_t *row = w + (size_t)tok * row_bytes;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x)
        out[(size_t)t * cols + i] = dequant_elem(tt, row, i);
}

// ---------------------------------------------------------------------------
// Weight encoders.  Q8_0 is the reference's own weight quantizer
// (src/quant_dequant.zig:1404-1425); the reference has none for IQ4_NL and
// the K-quants, so those are this library's deterministic encoders (the same
// algorithms as the CPU checker's, operation for operation).  One thread
// per native block.
// ---------------------------------------------------------------------------
Q35_DEV int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
Q35_DEV uint16_t f16_ieee(float x) { return f32_to_f16_bits(x, 0x0400u); }

Q35_DEV void wq_q8_0(const float *x, uint8_t *y) {
    float mx = 0.0f;
    for (int k = 0; k < 32; k++) {
        const float v = fabsf(x[k]);
        if (v > mx) mx = v;
    }
    const float s = __fdiv_rn(mx, 127.0f);
    const uint16_t sb = f16_ieee(s);
    y[0] = (uint8_t)(sb & 0xFF);
    y[1] = (uint8_t)(sb >> 8);
    for (int k = 0; k < 32; k++) {
        int q = 0;
        if (s > 0.0f) q = (int)roundf(__fdiv_rn(x[k], s));
        y[2 + k] = (uint8_t)(int8_t)clampi(q, -128, 127);
    }
}

Q35_DEV void wq_iq4_nl(const float *x, uint8_t *y) {
    float amax = 0.0f, vmax = 0.0f;
    for (int i = 0; i < 32; i++) {
        const float a = fabsf(x[i]);
        if (a > amax) { amax = a; vmax = x[i]; }
    }
    const uint16_t dh = f16_ieee(__fdiv_rn(vmax, -127.0f));
    const float dr = f16_to_f32(dh);
    const float id = dr != 0.0f ? __fdiv_rn(1.0f, dr) : 0.0f;
    y[0] = (uint8_t)(dh & 0xFF);
    y[1] = (uint8_t)(dh >> 8);
    uint8_t idx[32];
    for (int i = 0; i < 32; i++) {
        const float v = __fmul_rn(x[i], id);
        int best = 0;
        float berr = fabsf(__fsub_rn(v, (float)c_iq4nl[0]));
        for (int k = 1; k < 16; k++) {
            const float e = fabsf(__fsub_rn(v, (float)c_iq4nl[k]));
            if (e < berr) { berr = e; best = k; }
        }
        idx[i] = (uint8_t)best;
    }
    for (int j = 0; j < 16; j++) y[2 + j] = (uint8_t)(idx[j] | (idx[j + 16] << 4));
}

// Q4_0 / Q4_1 / Q5_0 / Q5_1 encoders of this project (the oracle's
// wq_legacy_block, operation for operation): d from the value of largest
// magnitude (Q4_0 / Q5_0) or the range (Q4_1 / Q5_1), rounded to f16, the
// elements quantized against the rounded scale, GGUF nibble / qh layout
Q35_DEV void wq_legacy(int tt, const float *x, uint8_t *y) {
    const bool affine = legacy_affine(tt), five = legacy_five(tt);
    const int qmax = five ? 31 : 15;
    uint8_t q[32];
    if (affine) {
        float mn = x[0], mx = x[0];
        for (int i = 1; i < 32; i++) {
            if (x[i] < mn) mn = x[i];
            if (x[i] > mx) mx = x[i];
        }
        const uint16_t dh = f16_ieee(__fdiv_rn(__fsub_rn(mx, mn), (float)qmax)), mh = f16_ieee(mn);
        const float dr = f16_to_f32(dh), mr = f16_to_f32(mh);
        const float id = dr != 0.0f ? __fdiv_rn(1.0f, dr) : 0.0f;
        for (int i = 0; i < 32; i++) {
            const int v = (int)__fadd_rn(__fmul_rn(__fsub_rn(x[i], mr), id), 0.5f);
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
        const uint16_t dh = f16_ieee(__fdiv_rn(vmax, -half));
        const float dr = f16_to_f32(dh);
        const float id = dr != 0.0f ? __fdiv_rn(1.0f, dr) : 0.0f;
        for (int i = 0; i < 32; i++) {
            const int v = (int)__fadd_rn(__fmul_rn(x[i], id), __fadd_rn(half, 0.5f));
            q[i] = (uint8_t)(v < 0 ? 0 : (v > qmax ? qmax : v));
        }
        y[0] = (uint8_t)(dh & 0xFF); y[1] = (uint8_t)(dh >> 8);
    }
    if (five) {
        uint32_t qh = 0;
        for (int j = 0; j < 32; j++) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
        uint8_t *h = y + legacy_qh_off(tt);
        h[0] = (uint8_t)qh; h[1] = (uint8_t)(qh >> 8); h[2] = (uint8_t)(qh >> 16); h[3] = (uint8_t)(qh >> 24);
    }
    uint8_t *qs = y + legacy_qs_off(tt);
    for (int j = 0; j < 16; j++) qs[j] = (uint8_t)((q[j] & 0x0F) | ((q[j + 16] & 0x0F) << 4));
}

Q35_DEV void wq_kq(const float *x, uint8_t *y, bool q5) {
    const float L = q5 ? 31.0f : 15.0f;
    const int qmax = q5 ? 31 : 15;
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
        sc[j] = __fdiv_rn(__fsub_rn(mx, mn), L);
        mnv[j] = -mn;
        if (sc[j] > max_sc) max_sc = sc[j];
        if (mnv[j] > max_mn) max_mn = mnv[j];
    }
    const uint16_t dh = f16_ieee(__fdiv_rn(max_sc, 63.0f));
    const uint16_t mh = f16_ieee(__fdiv_rn(max_mn, 63.0f));
    const float dr = f16_to_f32(dh), mr = f16_to_f32(mh);
    int ls[8], lm[8];
    for (int j = 0; j < 8; j++) {
        ls[j] = dr > 0.0f ? clampi((int)roundf(__fdiv_rn(sc[j], dr)), 0, 63) : 0;
        lm[j] = mr > 0.0f ? clampi((int)roundf(__fdiv_rn(mnv[j], mr)), 0, 63) : 0;
    }
    y[0] = (uint8_t)(dh & 0xFF);
    y[1] = (uint8_t)(dh >> 8);
    y[2] = (uint8_t)(mh & 0xFF);
    y[3] = (uint8_t)(mh >> 8);
    uint8_t *s = y + 4;
    for (int j = 0; j < 12; j++) s[j] = 0;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(ls[j] & 63);
        s[j + 4] = (uint8_t)(lm[j] & 63);
    }
    for (int j = 4; j < 8; j++) {
        s[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
        s[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
        s[j] |= (uint8_t)((lm[j] >> 4) << 6);
    }
    uint8_t *qh = y + 16;
    uint8_t *ql = q5 ? y + 48 : y + 16;
    if (q5)
        for (int l = 0; l < 32; l++) qh[l] = 0;
    for (int c = 0; c < 4; c++) {
        const float ed0 = __fmul_rn(dr, (float)ls[2 * c]), em0 = __fmul_rn(mr, (float)lm[2 * c]);
        const float ed1 = __fmul_rn(dr, (float)ls[2 * c + 1]), em1 = __fmul_rn(mr, (float)lm[2 * c + 1]);
        for (int l = 0; l < 32; l++) {
            int lo = 0, hi = 0;
            if (ed0 > 0.0f) lo = clampi((int)roundf(__fdiv_rn(__fadd_rn(x[c * 64 + l], em0), ed0)), 0, qmax);
            if (ed1 > 0.0f) hi = clampi((int)roundf(__fdiv_rn(__fadd_rn(x[c * 64 + 32 + l], em1), ed1)), 0, qmax);
            ql[c * 32 + l] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
            if (q5) {
                qh[l] |= (uint8_t)(((lo >> 4) & 1) << (2 * c));
                qh[l] |= (uint8_t)(((hi >> 4) & 1) << (2 * c + 1));
            }
        }
    }
}

Q35_DEV void wq_q6_k(const float *x, uint8_t *y) {
    float sc[16];
    float max_abs = 0.0f;
    for (int j = 0; j < 16; j++) {
        float amax = 0.0f, vmax = 0.0f;
        for (int i = 0; i < 16; i++) {
            const float a = fabsf(x[j * 16 + i]);
            if (a > amax) { amax = a; vmax = x[j * 16 + i]; }
        }
        sc[j] = __fdiv_rn(vmax, -32.0f);
        const float as = fabsf(sc[j]);
        if (as > max_abs) max_abs = as;
    }
    const uint16_t dh = f16_ieee(__fdiv_rn(max_abs, 127.0f));
    const float dr = f16_to_f32(dh);
    int8_t isc[16];
    for (int j = 0; j < 16; j++)
        isc[j] = (int8_t)(dr > 0.0f ? clampi((int)roundf(__fdiv_rn(sc[j], dr)), -128, 127) : 0);
    uint8_t *ql = y, *qh = y + 128;
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            uint8_t u[4];
            for (int k = 0; k < 4; k++) {
                const int e = h * 128 + 32 * k + l;
                const float ed = __fmul_rn(dr, (float)isc[e / 16]);
                int v = 0;
                if (ed != 0.0f) v = clampi((int)roundf(__fdiv_rn(x[e], ed)), -32, 31);
                u[k] = (uint8_t)(v + 32);
            }
            ql[h * 64 + l] = (uint8_t)((u[0] & 0xF) | ((u[2] & 0xF) << 4));
            ql[h * 64 + l + 32] = (uint8_t)((u[1] & 0xF) | ((u[3] & 0xF) << 4));
            qh[h * 32 + l] = (uint8_t)((u[0] >> 4) | ((u[1] >> 4) << 2) | ((u[2] >> 4) << 4) | ((u[3] >> 4) << 6));
        }
    for (int j = 0; j < 16; j++) y[192 + j] = (uint8_t)isc[j];
    y[208] = (uint8_t)(dh & 0xFF);
    y[209] = (uint8_t)(dh >> 8);
}

__global__ void k_quantize_weight(int tt, const float *__restrict__ x, uint8_t *__restrict__ y, long long nblocks) {
    const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const Geom g = geom_of(tt);
    const float *xb = x + b * g.elems;
    uint8_t *yb = y + b * g.bytes;
    switch (tt) {
    case TT_Q8_0: wq_q8_0(xb, yb); break;
    case TT_IQ4_NL: wq_iq4_nl(xb, yb); break;
    case TT_Q4_0:
    case TT_Q4_1:
    case TT_Q5_0:
    case TT_Q5_1: wq_legacy(tt, xb, yb); break;
    case TT_Q4_K: wq_kq(xb, yb, false); break;
    case TT_Q5_K: wq_kq(xb, yb, true); break;
    case TT_Q6_K: wq_q6_k(xb, yb); break;
    default: break;
    }
}

// Seeded synthetic values for benchmark / test weights, identical on the CPU
// (the same integer steps in C or numpy): element i of stream `key` hashes
// the counter (splitmix64's finalizer, Steele, Lea & Flood 2014) and sums
// the four 16-bit fields of the hash (Irwin-Hall with n = 4: mean 131070,
// standard deviation 37837.23), so the centred sum is an exact integer and
// its one rounded product with k (scale / 37837.23, formed by the caller)
// gives the same f32 bits on any IEEE machine.
Q35_DEV uint64_t synth_hash(uint64_t key, uint64_t i) {
    uint64_t z = key * 0x9E3779B97F4A7C15ull + i * 0xD1B54A32D192ED03ull;
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}

__global__ void k_synth_fill(uint64_t key, long long n, float k, float *__restrict__ y) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const uint64_t z = synth_hash(key, (uint64_t)i);
        const int s = (int)(z & 0xffff) + (int)((z >> 16) & 0xffff) + (int)((z >> 32) & 0xffff) + (int)(z >> 48);
        y[i] = __fmul_rn((float)(s - 131070), k);
    }
}

// Q6_K blocks from the GGUF 210-byte layout to the 224-byte one (14 zero
// bytes after d), whose rows are 16-byte multiples for the TMA / MMQ paths;
// one thread per 16-bit word
__global__ void k_repack_q6k(const uint8_t *src, uint8_t *dst, long long nblk) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= nblk * 112) return;
    const long long b = i / 112;
    const int hw = (int)(i - b * 112);
    const uint16_t v = hw < 105 ? reinterpret_cast<const uint16_t *>(src + b * 210)[hw] : (uint16_t)0;
    reinterpret_cast<uint16_t *>(dst + b * 224)[hw] = v;
}

}  // namespace q35
