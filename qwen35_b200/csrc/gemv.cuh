// gemv.cuh -- quantized matrix-vector product over raw GGUF blocks, for a
// handful of tokens (decode).  sm_100a design:
//
//   * Weights are streamed, never gathered: the rows of one tile are a
//     contiguous byte range, copied global -> shared by one elected thread
//     with cp.async.bulk (the TMA bulk engine) into a 4-stage mbarrier ring,
//     so HBM sees only full 16-byte-aligned bursts whatever the block size
//     (34 B Q8_0, 18 B IQ4_NL, 210 B Q6_K are not 16-byte aligned).
//   * The quantized activation of every token is converted once per CTA into
//     an aligned shared layout (int8 plane + f32 scales + int32 bsums), so the
//     inner loop reads it with 128-bit shared loads.
//   * 8 consumer warps each own a row at a time; lanes split the row into
//     block parts, compute the per-block integer dot with dp4a (exact), and
//     the f32 terms are folded strictly in block order (lane t folds token
//     t), which is the reference scalar tier's rounding sequence
//     (kernels32.c:462, kernels256.c:494,625,735): the output is bit-exact
//     with the CPU oracle.
//
// One launch may cover up to 4 weight matrices that share the same input
// (e.g. a GDN layer's qkv / gate / alpha / beta projections).
#pragma once
#include "common.cuh"

#define Q35_TRY_RC(x)          \
    do {                       \
        int _r = (x);          \
        if (_r) return _r;     \
    } while (0)

namespace q35 {

constexpr int GV_WARPS = 4;                      // consumer warps
constexpr int GV_THREADS = (GV_WARPS + 1) * 32;  // + one producer warp
constexpr int GV_MAX_SEG = 4;
constexpr int GV_MAX_NT = 16;                    // tokens per pass
constexpr int GV_FOLD_FLOATS = 640;              // per-warp fold scratch (R * NT * (BPP + 4) <= 640)

enum { GV_STORE = 0, GV_ADD = 1 };

struct GemvSeg {
    const uint8_t *w;
    float *out;
    long long rows;
    int ttype;
    int row_bytes;
    long long out_ld;   // floats between tokens in `out`
    int mode;           // GV_STORE or GV_ADD (residual add)
    int rows_per_tile;
    long long tile_begin;
};

struct GemvArgs {
    GemvSeg seg[GV_MAX_SEG];
    int nseg;
    long long total_tiles;
    const uint8_t *xq;   // API-layout activation: Q8_0 (34 B/32) or Q8_K (292 B/256)
    long long act_row_bytes;
    int ntok;
    int cols;
    int family;          // 32 or 256
    int stage_bytes;     // bytes of one stage buffer (multiple of 16)
    int nstage;
    int act_stride;      // bytes per token of the shared activation layout
};

// shared activation layout per token: qs int8[cols] | dsc f32[cols/32] | bsum i32[cols/16]
__host__ __device__ inline int gemv_act_stride(int cols, int family) {
    int s = cols + (cols / 32) * 4 + (family == 256 ? (cols / 16) * 4 : 0);
    return (s + 15) & ~15;
}

struct ActView {
    const uint8_t *base;
    int stride, cols;
    int il = 0;  // Q8_0 blocks staged in the IQ4_NL interleaved order (gemv_lpr.cuh)
    Q35_DEV const int8_t *qs(int t) const { return reinterpret_cast<const int8_t *>(base + t * stride); }
    Q35_DEV float dsc(int t, int b) const {
        return reinterpret_cast<const float *>(base + t * stride + cols)[b];
    }
    Q35_DEV int bsum(int t, int g) const {
        return reinterpret_cast<const int *>(base + t * stride + cols + (cols / 32) * 4)[g];
    }
    // 4 consecutive words (16 elements) starting at element e (e % 16 == 0)
    Q35_DEV uint4 q16(int t, int e) const { return *reinterpret_cast<const uint4 *>(base + t * stride + e); }
};

Q35_DEV int dot4x4(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint4 y, int acc) {
    acc = __dp4a((int)a0, (int)y.x, acc);
    acc = __dp4a((int)a1, (int)y.y, acc);
    acc = __dp4a((int)a2, (int)y.z, acc);
    acc = __dp4a((int)a3, (int)y.w, acc);
    return acc;
}

// ---- per-type block parts --------------------------------------------------
// Each returns per-token integer sums for its part; the caller reduces the
// parts of one block (integer, exact) and forms the f32 term.

template <int NT>
Q35_DEV void part_q8_0(const uint8_t *wb, const ActView &A, int ntok, int b, int (&is)[NT]) {
    uint32_t q[8];
    lds_words_a2<8>(wb + 2, q);
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if (t < ntok) {
            const uint4 y0 = A.q16(t, b * 32), y1 = A.q16(t, b * 32 + 16);
            int s = dot4x4(q[0], q[1], q[2], q[3], y0, 0);
            is[t] = dot4x4(q[4], q[5], q[6], q[7], y1, s);
        }
    }
}

template <int NT>
Q35_DEV void part_iq4_nl(const uint8_t *wb, const ActView &A, int ntok, int b, int (&is)[NT]) {
    uint32_t q[4], lo[4], hi[4];
    lds_words_a2<4>(wb + 2, q);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        lo[i] = iq4_lookup4(q[i] & 0x0F0F0F0Fu);
        hi[i] = iq4_lookup4((q[i] >> 4) & 0x0F0F0F0Fu);
    }
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if (t < ntok) {
            const uint4 y0 = A.q16(t, b * 32), y1 = A.q16(t, b * 32 + 16);
            int s = dot4x4(lo[0], lo[1], lo[2], lo[3], y0, 0);
            is[t] = dot4x4(hi[0], hi[1], hi[2], hi[3], y1, s);
        }
    }
}

// IQ4_XS sub-block b (32 elements) of the 256-element block at wb: the
// IQ4_NL lookup on its 16 bytes of nibbles, Q8_K activation elements 32b..
template <int NT>
Q35_DEV void part_iq4_xs(const uint8_t *wb, const ActView &A, int ntok, int b, int (&is)[NT]) {
    uint32_t q[4], lo[4], hi[4];
    lds_words_a2<4>(wb + 8 + 16 * (b & 7), q);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        lo[i] = iq4_lookup4(q[i] & 0x0F0F0F0Fu);
        hi[i] = iq4_lookup4((q[i] >> 4) & 0x0F0F0F0Fu);
    }
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if (t < ntok) {
            const uint4 y0 = A.q16(t, b * 32), y1 = A.q16(t, b * 32 + 16);
            int s = dot4x4(lo[0], lo[1], lo[2], lo[3], y0, 0);
            is[t] = dot4x4(hi[0], hi[1], hi[2], hi[3], y1, s);
        }
    }
}

// f32 term of IQ4_XS sub-block ib (iq_kernels.c:975-990):
// d4d8 = d * dy, d1 = d4d8 * (ls - 32), sumf += d1 * (float)isum
Q35_DEV float iq4xs_term(const uint8_t *wb, int ib, float dy, int is) {
    const float d4d8 = __fmul_rn(f16_to_f32(ld_u16(wb)), dy);
    const int ls = iq4xs_ls(wb[4 + (ib >> 1)], ld_u16(wb + 2), ib);
    return __fmul_rn(__fmul_rn(d4d8, __int2float_rn(ls - 32)), __int2float_rn(is));
}

// spread the 4 bits of x (bits 0..3) to bit 4 of bytes 0..3
Q35_DEV uint32_t bits4_to_b4(uint32_t x) {
    return ((x & 1u) | ((x & 2u) << 7) | ((x & 4u) << 14) | ((x & 8u) << 21)) << 4;
}

// Q4_0 / Q4_1 / Q5_0 / Q5_1 block (GGUF layout): the 32 quantized values as
// signed bytes -- lo[i] = elements 4i..4i+3, hi[i] = elements 16+4i.. --
// centred (q - 8 / q - 16) for the symmetric types, raw q for the affine ones
// (kernels32.c:297-340, 546-652)
Q35_DEV void legacy_bytes(int tt, uint32_t qh, const uint32_t (&q)[4], uint32_t (&lo)[4], uint32_t (&hi)[4]) {
    const bool five = legacy_five(tt), affine = legacy_affine(tt);
    const uint32_t bias = five ? 0x10101010u : 0x08080808u;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        lo[i] = q[i] & 0x0F0F0F0Fu;
        hi[i] = (q[i] >> 4) & 0x0F0F0F0Fu;
        if (five) {
            lo[i] |= bits4_to_b4((qh >> (4 * i)) & 0xFu);
            hi[i] |= bits4_to_b4((qh >> (16 + 4 * i)) & 0xFu);
        }
        if (!affine) {
            lo[i] = __vsub4(lo[i], bias);
            hi[i] = __vsub4(hi[i], bias);
        }
    }
}

// is: sum of q * y; ms (affine types): sum of the 32 activation values
template <int NT>
Q35_DEV void part_legacy(int tt, const uint8_t *wb, const ActView &A, int ntok, int b, int (&is)[NT],
                         int (&ms)[NT]) {
    uint32_t q[4], lo[4], hi[4], h[1] = {0u};
    lds_words_a2<4>(wb + legacy_qs_off(tt), q);
    if (legacy_five(tt)) lds_words_a2<1>(wb + legacy_qh_off(tt), h);
    legacy_bytes(tt, h[0], q, lo, hi);
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if (t < ntok) {
            const uint4 y0 = A.q16(t, b * 32), y1 = A.q16(t, b * 32 + 16);
            int s = dot4x4(lo[0], lo[1], lo[2], lo[3], y0, 0);
            is[t] = dot4x4(hi[0], hi[1], hi[2], hi[3], y1, s);
            if (legacy_affine(tt)) {
                constexpr uint32_t one = 0x01010101u;
                ms[t] = dot4x4(one, one, one, one, y1, dot4x4(one, one, one, one, y0, 0));
            }
        }
    }
}

// f32 term of one legacy block (kernels32.c:313, 338): dx*dy*sumi, plus
// mx*dy*sumy for the affine types, added as one term
Q35_DEV float legacy_term(int tt, const uint8_t *wb, float dy, int is, int ms) {
    const float t0 = __fmul_rn(__fmul_rn(f16_to_f32(ld_u16(wb)), dy), __int2float_rn(is));
    if (!legacy_affine(tt)) return t0;
    return __fadd_rn(t0, __fmul_rn(__fmul_rn(f16_to_f32(ld_u16(wb + 2)), dy), __int2float_rn(ms)));
}

// Q4_K / Q5_K: part c covers elements [64c, 64c+64) = sub-blocks 2c, 2c+1
template <int NT, bool Q5>
Q35_DEV void part_q45_k(const uint8_t *wb, const ActView &A, int ntok, int b, int c, int (&is)[NT],
                        int (&ms)[NT]) {
    int sc0, m0, sc1, m1;
    kq_scale_min(2 * c, wb + 4, sc0, m0);
    kq_scale_min(2 * c + 1, wb + 4, sc1, m1);
    uint32_t ql[8], lo[8], hi[8];
    lds_words_a2<8>(wb + (Q5 ? 48 : 16) + 32 * c, ql);
    if (Q5) {
        uint32_t qh[8];
        lds_words_a2<8>(wb + 16, qh);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            lo[i] = (ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> (2 * c)) & 0x01010101u) << 4);
            hi[i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * c + 1)) & 0x01010101u) << 4);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            lo[i] = ql[i] & 0x0F0F0F0Fu;
            hi[i] = (ql[i] >> 4) & 0x0F0F0F0Fu;
        }
    }
    const int e0 = b * 256 + 64 * c;
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if (t < ntok) {
            int dl = dot4x4(lo[0], lo[1], lo[2], lo[3], A.q16(t, e0), 0);
            dl = dot4x4(lo[4], lo[5], lo[6], lo[7], A.q16(t, e0 + 16), dl);
            int dh = dot4x4(hi[0], hi[1], hi[2], hi[3], A.q16(t, e0 + 32), 0);
            dh = dot4x4(hi[4], hi[5], hi[6], hi[7], A.q16(t, e0 + 48), dh);
            is[t] = sc0 * dl + sc1 * dh;
            const int g = b * 16 + 4 * c;
            ms[t] = m0 * (A.bsum(t, g) + A.bsum(t, g + 1)) + m1 * (A.bsum(t, g + 2) + A.bsum(t, g + 3));
        }
    }
}

// Q6_K: part p -> half h = p>>1 (128 elements), l-range [16*(p&1), +16)
template <int NT>
Q35_DEV void part_q6_k(const uint8_t *wb, const ActView &A, int ntok, int b, int p, int (&is)[NT]) {
    const int h = p >> 1, hf = p & 1;
    uint32_t qa[4], qb[4], qh[4];
    lds_words_a2<4>(wb + h * 64 + 16 * hf, qa);
    lds_words_a2<4>(wb + h * 64 + 32 + 16 * hf, qb);
    lds_words_a2<4>(wb + 128 + h * 32 + 16 * hf, qh);
    const int8_t *sc = reinterpret_cast<const int8_t *>(wb + 192) + h * 8 + hf;
    const int s1 = sc[0], s2 = sc[2], s3 = sc[4], s4 = sc[6];
    uint32_t v1[4], v2[4], v3[4], v4[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        v1[i] = __vsub4((qa[i] & 0x0F0F0F0Fu) | ((qh[i] & 0x03030303u) << 4), 0x20202020u);
        v2[i] = __vsub4((qb[i] & 0x0F0F0F0Fu) | (((qh[i] >> 2) & 0x03030303u) << 4), 0x20202020u);
        v3[i] = __vsub4(((qa[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 4) & 0x03030303u) << 4), 0x20202020u);
        v4[i] = __vsub4(((qb[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 6) & 0x03030303u) << 4), 0x20202020u);
    }
    const int e0 = b * 256 + h * 128 + 16 * hf;
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if (t < ntok) {
            const int d1 = dot4x4(v1[0], v1[1], v1[2], v1[3], A.q16(t, e0), 0);
            const int d2 = dot4x4(v2[0], v2[1], v2[2], v2[3], A.q16(t, e0 + 32), 0);
            const int d3 = dot4x4(v3[0], v3[1], v3[2], v3[3], A.q16(t, e0 + 64), 0);
            const int d4 = dot4x4(v4[0], v4[1], v4[2], v4[3], A.q16(t, e0 + 96), 0);
            is[t] = s1 * d1 + s2 * d2 + s3 * d3 + s4 * d4;
        }
    }
}

// R rows per warp, LR = 32/R lanes per row.  Lane (g, q) = (lane / LR,
// lane % LR) works on row g: with LPB lanes per block it takes block part
// q % LPB of block cb + q / LPB, for BPP = LR / LPB blocks per pass.  Lane
// (g, t) with t < ntok then folds token t's terms of that pass in block
// order into its running sum -- the reference scalar tier's rounding
// sequence -- so R rows (and NT tokens) fold concurrently on different lanes.
template <int NT, int LPB, int R>
Q35_DEV void gemv_rows(int tt, const uint8_t *rowp0, int row_bytes, int nvalid, const ActView &A, int ntok, int nb,
                       float *fold, float *out_r0, long long out_ld, int mode, int lane) {
    constexpr int LR = 32 / R;
    constexpr int BPP = LR / LPB;
    constexpr int FL = BPP + 4;
    static_assert(NT <= LR, "one folding lane per (row, token)");
    const int bsz = geom_of(tt).bytes;
    const int g = lane / LR, q = lane % LR;
    const int j = q / LPB, p = q % LPB;
    const bool row_ok = g < nvalid;
    const uint8_t *rowp = rowp0 + (size_t)(row_ok ? g : 0) * row_bytes;
    float *fg = fold + g * NT * FL;
    float acc = 0.0f;
    for (int cb = 0; cb < nb; cb += BPP) {
        const int b = cb + j;
        const bool act = row_ok && b < nb;
        // IQ4_XS: b counts 32-element sub-blocks, wb is their 256-element block
        const uint8_t *wb = rowp + (size_t)(act ? (tt == TT_IQ4_XS ? b >> 3 : b) : 0) * bsz;
        int is[NT], ms[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) is[t] = 0, ms[t] = 0;
        if (act) {
            if (LPB == 1) {
                if (tt == TT_Q8_0)
                    part_q8_0<NT>(wb, A, ntok, b, is);
                else if (tt == TT_IQ4_NL)
                    part_iq4_nl<NT>(wb, A, ntok, b, is);
                else if (tt == TT_IQ4_XS)
                    part_iq4_xs<NT>(wb, A, ntok, b, is);
                else
                    part_legacy<NT>(tt, wb, A, ntok, b, is, ms);
            } else {
                if (tt == TT_Q4_K)
                    part_q45_k<NT, false>(wb, A, ntok, b, p, is, ms);
                else if (tt == TT_Q5_K)
                    part_q45_k<NT, true>(wb, A, ntok, b, p, is, ms);
                else
                    part_q6_k<NT>(wb, A, ntok, b, p, is);
            }
        }
        if (LPB > 1) {
#pragma unroll
            for (int t = 0; t < NT; t++) {
                is[t] += __shfl_xor_sync(0xffffffffu, is[t], 1);
                is[t] += __shfl_xor_sync(0xffffffffu, is[t], 2);
                ms[t] += __shfl_xor_sync(0xffffffffu, ms[t], 1);
                ms[t] += __shfl_xor_sync(0xffffffffu, ms[t], 2);
            }
        }
        if (act && p == 0) {
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < ntok) {
                    float term;
                    if (tt == TT_Q8_0 || tt == TT_IQ4_NL) {
                        // sumf += dx * dy * (float)sumi
                        term = __fmul_rn(__fmul_rn(f16_to_f32(ld_u16(wb)), A.dsc(t, b)), __int2float_rn(is[t]));
                    } else if (legacy_type(tt)) {
                        term = legacy_term(tt, wb, A.dsc(t, b), is[t], ms[t]);
                    } else if (tt == TT_IQ4_XS) {
                        term = iq4xs_term(wb, b & 7, A.dsc(t, b >> 3), is[t]);
                    } else if (tt == TT_Q6_K || tt == TT_Q6_K_P) {
                        // sumf += d_w * dy * (float)isum
                        term = __fmul_rn(__fmul_rn(f16_to_f32(ld_u16(wb + 208)), A.dsc(t, b)), __int2float_rn(is[t]));
                    } else {
                        // d = dy*d_w; dmin = dy*dmin_w; sumf += d*isum - dmin*sumi
                        const float dy = A.dsc(t, b);
                        const float d = __fmul_rn(dy, f16_to_f32(ld_u16(wb)));
                        const float dm = __fmul_rn(dy, f16_to_f32(ld_u16(wb + 2)));
                        term = __fsub_rn(__fmul_rn(d, __int2float_rn(is[t])), __fmul_rn(dm, __int2float_rn(ms[t])));
                    }
                    fg[t * FL + j] = term;
                }
            }
        }
        __syncwarp();
        if (row_ok && q < ntok) {
            const float *f = fg + q * FL;
            if (BPP >= 4 && nb - cb >= BPP) {
                float4 v[BPP / 4 > 0 ? BPP / 4 : 1];
#pragma unroll
                for (int i = 0; i < BPP / 4; i++) v[i] = reinterpret_cast<const float4 *>(f)[i];
#pragma unroll
                for (int i = 0; i < BPP / 4; i++) {
                    acc = __fadd_rn(acc, v[i].x);
                    acc = __fadd_rn(acc, v[i].y);
                    acc = __fadd_rn(acc, v[i].z);
                    acc = __fadd_rn(acc, v[i].w);
                }
            } else {
                const int n = min(BPP, nb - cb);
                for (int i = 0; i < n; i++) acc = __fadd_rn(acc, f[i]);
            }
        }
        __syncwarp();
    }
    if (row_ok && q < ntok) {
        float *o = out_r0 + g + (long long)q * out_ld;
        *o = mode == GV_ADD ? __fadd_rn(*o, acc) : acc;
    }
}

Q35_DEV int gemv_find_seg(const GemvArgs &a, long long tile) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < GV_MAX_SEG; i++)
        if (i < a.nseg && tile >= a.seg[i].tile_begin) s = i;
    return s;
}

template <int NT, int R>
__global__ void __launch_bounds__(GV_THREADS) k_gemv(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + a.nstage;
    float *foldbase = reinterpret_cast<float *>(smem + 256);
    uint8_t *act = smem + 256 + GV_WARPS * GV_FOLD_FLOATS * 4;
    act = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(act) + 127) & ~uintptr_t(127));
    uint8_t *stages = act + (size_t)a.ntok * a.act_stride;
    stages = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(stages) + 127) & ~uintptr_t(127));
    const int stage_ld = a.stage_bytes + 32;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.nstage; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GV_WARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == GV_WARPS) {
        // ---------------- producer: stream weight tiles ----------------
        if (lane != 0) return;
        long long it = 0;
        for (long long tile = blockIdx.x; tile < a.total_tiles; tile += gridDim.x, it++) {
            const int s = (int)(it % a.nstage);
            if (it >= a.nstage && !mbar_wait(&empty[s], (uint32_t)(((it / a.nstage) - 1) & 1), 101)) return;
            const GemvSeg &sg = a.seg[gemv_find_seg(a, tile)];
            const long long lt = tile - sg.tile_begin;
            const long long r0 = lt * sg.rows_per_tile;
            const long long nr = min((long long)sg.rows_per_tile, sg.rows - r0);
            const uintptr_t wbase = reinterpret_cast<uintptr_t>(sg.w);
            const uintptr_t wend = wbase + (uintptr_t)sg.rows * sg.row_bytes;
            const uintptr_t start = wbase + (uintptr_t)r0 * sg.row_bytes;
            const uintptr_t end = start + (uintptr_t)nr * sg.row_bytes;
            const uintptr_t g0 = start & ~uintptr_t(15);
            uintptr_t lo = (wbase + 15) & ~uintptr_t(15);
            lo = lo > g0 ? lo : g0;
            uintptr_t hi = (end + 15) & ~uintptr_t(15);
            const uintptr_t hcap = wend & ~uintptr_t(15);
            hi = hi < hcap ? hi : hcap;
            uint8_t *buf = stages + (size_t)s * stage_ld;
            // bytes outside the 16-byte-aligned interior of the matrix: plain loads
            for (uintptr_t p = start; p < end && p < lo; p++) buf[p - g0] = *reinterpret_cast<const uint8_t *>(p);
            for (uintptr_t p = (hi > start ? hi : start); p < end; p++)
                buf[p - g0] = *reinterpret_cast<const uint8_t *>(p);
            if (hi > lo) {
                mbar_arrive_expect_tx(&full[s], (uint32_t)(hi - lo));
                bulk_g2s(buf + (lo - g0), reinterpret_cast<const void *>(lo), (uint32_t)(hi - lo), &full[s]);
            } else {
                mbar_arrive(&full[s]);
            }
        }
        // drain: do not exit while copies into this CTA's shared memory are in flight
        const long long n = it;
        for (long long k = (n > a.nstage ? n - a.nstage : 0); k < n; k++)
            if (!mbar_wait(&full[k % a.nstage], (uint32_t)((k / a.nstage) & 1), 102)) return;
        return;
    }

    // ---------------- consumers ----------------
    // The producer streams weights (never written during a step) without
    // waiting; the activation and the outputs belong to earlier kernels.
    pdl_wait();
    // 1. activation -> shared aligned layout
    const int ctid = threadIdx.x;
    const int cthreads = GV_WARPS * 32;
    if (a.family == 32) {
        const int nb = a.cols / 32;
        for (int idx = ctid; idx < a.ntok * nb; idx += cthreads) {
            const int t = idx / nb, b = idx - t * nb;
            const uint8_t *src = a.xq + (size_t)t * a.act_row_bytes + (size_t)b * 34;
            uint8_t *dst = act + (size_t)t * a.act_stride;
            reinterpret_cast<float *>(dst + a.cols)[b] = f16_to_f32(ld_u16(src));
            uint32_t *q = reinterpret_cast<uint32_t *>(dst + b * 32);
#pragma unroll
            for (int i = 0; i < 8; i++)
                q[i] = (uint32_t)ld_u16(src + 2 + 4 * i) | ((uint32_t)ld_u16(src + 4 + 4 * i) << 16);
        }
    } else {
        const int nb = a.cols / 256;
        for (int idx = ctid; idx < a.ntok * nb * 17; idx += cthreads) {
            const int part = idx % 17, tb = idx / 17, t = tb / nb, b = tb - t * nb;
            const uint8_t *src = a.xq + (size_t)t * a.act_row_bytes + (size_t)b * 292;
            uint8_t *dst = act + (size_t)t * a.act_stride;
            if (part < 16) {
                const uint32_t *s4 = reinterpret_cast<const uint32_t *>(src + 4 + part * 16);
                uint32_t *d4 = reinterpret_cast<uint32_t *>(dst + b * 256 + part * 16);
#pragma unroll
                for (int i = 0; i < 4; i++) d4[i] = s4[i];
            } else {
                reinterpret_cast<float *>(dst + a.cols)[b] = *reinterpret_cast<const float *>(src);
                int *bs = reinterpret_cast<int *>(dst + a.cols + (a.cols / 32) * 4) + b * 16;
                const int16_t *sb = reinterpret_cast<const int16_t *>(src + 260);
#pragma unroll
                for (int g = 0; g < 16; g++) bs[g] = sb[g];
            }
        }
    }
    named_bar_sync(1, cthreads);

    ActView A{act, a.act_stride, a.cols};
    float *fold = foldbase + warp * GV_FOLD_FLOATS;
    long long it = 0;
    for (long long tile = blockIdx.x; tile < a.total_tiles; tile += gridDim.x, it++) {
        const int s = (int)(it % a.nstage);
        if (!mbar_wait(&full[s], (uint32_t)((it / a.nstage) & 1), 103)) return;
        const GemvSeg &sg = a.seg[gemv_find_seg(a, tile)];
        const long long lt = tile - sg.tile_begin;
        const long long r0 = lt * sg.rows_per_tile;
        const int nr = (int)min((long long)sg.rows_per_tile, sg.rows - r0);
        const uintptr_t start = reinterpret_cast<uintptr_t>(sg.w) + (uintptr_t)r0 * sg.row_bytes;
        const uint8_t *buf = stages + (size_t)s * stage_ld + (start & 15);
        const int nb = a.cols / term_elems(sg.ttype);  // f32 terms per row
        const bool lpb1 = term_elems(sg.ttype) == 32;
        for (int rg = warp * R; rg < nr; rg += GV_WARPS * R) {
            const int nv = min(R, nr - rg);
            if (lpb1)
                gemv_rows<NT, 1, R>(sg.ttype, buf + (size_t)rg * sg.row_bytes, sg.row_bytes, nv, A, a.ntok, nb, fold,
                                    sg.out + r0 + rg, sg.out_ld, sg.mode, lane);
            else
                gemv_rows<NT, 4, R>(sg.ttype, buf + (size_t)rg * sg.row_bytes, sg.row_bytes, nv, A, a.ntok, nb, fold,
                                    sg.out + r0 + rg, sg.out_ld, sg.mode, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct GemvSegDesc {
    const void *w;
    float *out;
    long long rows;
    int ttype;
    long long out_ld;
    int mode;
};

int gemv_sm_count();

inline size_t gemv_smem_bytes(int ntok, int act_stride, int stage_bytes, int nstage) {
    size_t s = 256 + (size_t)GV_WARPS * GV_FOLD_FLOATS * 4 + 128;
    s += (size_t)ntok * act_stride + 128;
    s += (size_t)nstage * (stage_bytes + 32);
    return s;
}

// Set the dynamic shared-memory ceiling of every instantiation once, outside
// any stream capture (attribute calls are not stream work, but doing them
// up front keeps a captured step free of host-side configuration).
template <int NT, int R>
inline cudaError_t gemv_set_smem() {
    return cudaFuncSetAttribute(k_gemv<NT, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}
inline int gemv_prepare() {
    static int done = 0;
    if (done) return 0;
    const cudaError_t es[] = {gemv_set_smem<1, 1>(), gemv_set_smem<1, 2>(), gemv_set_smem<1, 4>(),
                              gemv_set_smem<2, 1>(), gemv_set_smem<2, 2>(), gemv_set_smem<2, 4>(),
                              gemv_set_smem<4, 1>(), gemv_set_smem<4, 2>(), gemv_set_smem<4, 4>(),
                              gemv_set_smem<8, 1>(), gemv_set_smem<8, 2>(), gemv_set_smem<8, 4>(),
                              gemv_set_smem<16, 1>(), gemv_set_smem<16, 2>()};
    for (cudaError_t e : es)
        if (e != cudaSuccess) return (int)e;
    done = 1;
    return 0;
}

template <int NT, int R>
inline int gemv_launch_nt(GemvArgs &a, cudaStream_t st) {
    const size_t smem = gemv_smem_bytes(a.ntok, a.act_stride, a.stage_bytes, a.nstage);
    if (smem > 227 * 1024) return (int)cudaErrorInvalidValue;
    Q35_TRY_RC(gemv_prepare());
    // resident CTAs per SM from shared memory (228 KB per SM, 1 KB reserved
    // per CTA) and registers (<= 96 x 160 threads): at most 3
    int occ = (int)((228 * 1024) / (smem + 1024));
    occ = occ < 1 ? 1 : (occ > 3 ? 3 : occ);
    long long grid = (long long)gemv_sm_count() * occ;
    if (grid > a.total_tiles) grid = a.total_tiles;
    if (grid < 1) grid = 1;
    return launch_k(k_gemv<NT, R>, dim3((unsigned)grid), dim3(GV_THREADS), smem, st, a);
}

template <int NT>
inline int gemv_launch_r(GemvArgs &a, int R, cudaStream_t st) {
    if (NT <= 8 && R >= 4) return gemv_launch_nt<NT, (NT <= 8 ? 4 : 2)>(a, st);
    if (R >= 2) return gemv_launch_nt<NT, 2>(a, st);
    return gemv_launch_nt<NT, 1>(a, st);
}

// Launch y = W x for up to GV_MAX_SEG matrices sharing one activation with
// the block-splitting kernel (any alignment, every type).
// `xq` is the API-layout quantized activation (tokens rows of act_row_bytes).
inline int gemv_launch_split(const GemvSegDesc *segs, int nseg, const void *xq, int cols, int ntok, cudaStream_t st,
                             long long xq_ld = 0) {
    if (nseg < 1 || nseg > GV_MAX_SEG || cols <= 0 || ntok <= 0) return (int)cudaErrorInvalidValue;
    const int fam = geom_of(segs[0].ttype).family;
    if (!fam) return (int)cudaErrorInvalidValue;
    for (int i = 0; i < nseg; i++) {
        const Geom g = geom_of(segs[i].ttype);
        if (g.family != fam || cols % g.elems != 0 || cols % 256 != 0 && g.elems == 256) return (int)cudaErrorInvalidValue;
        if ((reinterpret_cast<uintptr_t>(segs[i].w) & 1u) != 0) return (int)cudaErrorMisalignedAddress;
    }
    if (fam == 256 && (reinterpret_cast<uintptr_t>(xq) & 3u) != 0) return (int)cudaErrorMisalignedAddress;
    const long long act_row_bytes =
        xq_ld > 0 ? xq_ld : (fam == 32 ? (long long)(cols / 32) * 34 : (long long)(cols / 256) * 292);
    if (fam == 256 && (act_row_bytes & 3)) return (int)cudaErrorMisalignedAddress;
    const int nsm = gemv_sm_count();
    int max_rb = 0;
    long long total_rows = 0;
    for (int i = 0; i < nseg; i++) {
        const Geom g = geom_of(segs[i].ttype);
        const int rb = cols / g.elems * g.bytes;
        max_rb = rb > max_rb ? rb : max_rb;
        total_rows += segs[i].rows;
    }
    // rows per warp: several short rows per warp amortise the ordered fold
    const int R = max_rb <= 1152 ? 4 : (max_rb <= 2304 ? 2 : 1);
    // a stage holds at least one round (every consumer warp busy on R rows)
    int stage = GV_WARPS * R * max_rb + 32;
    if (stage < 16384) stage = 16384;
    stage = (stage + 15) & ~15;
    // tokens per pass: the largest group whose shared activation copy plus a
    // 3-stage weight ring fits the CTA's shared memory
    int group = GV_MAX_NT;
    while (group > 1 && gemv_smem_bytes(group, gemv_act_stride(cols, fam), stage, 3) > 220 * 1024) group >>= 1;
    for (int t0 = 0; t0 < ntok; t0 += group) {
        const int nt = ntok - t0 < group ? ntok - t0 : group;
        GemvArgs a{};
        a.nseg = nseg;
        a.xq = reinterpret_cast<const uint8_t *>(xq) + (size_t)t0 * act_row_bytes;
        a.act_row_bytes = act_row_bytes;
        a.ntok = nt;
        a.cols = cols;
        a.family = fam;
        a.act_stride = gemv_act_stride(cols, fam);
        a.stage_bytes = stage;
        a.nstage = 4;
        while (a.nstage > 2 && gemv_smem_bytes(nt, a.act_stride, stage, a.nstage) > 220 * 1024) a.nstage--;
        long long tiles = 0;
        for (int i = 0; i < nseg; i++) {
            const Geom g = geom_of(segs[i].ttype);
            GemvSeg &s = a.seg[i];
            s.w = reinterpret_cast<const uint8_t *>(segs[i].w);
            s.rows = segs[i].rows;
            s.ttype = segs[i].ttype;
            s.row_bytes = cols / g.elems * g.bytes;
            s.out = segs[i].out + (size_t)t0 * segs[i].out_ld;
            s.out_ld = segs[i].out_ld;
            s.mode = segs[i].mode;
            int rpt = (stage - 16) / s.row_bytes;
            // at least ~2 tiles per SM when the matrix is small
            const long long want = (total_rows + 2LL * nsm - 1) / (2LL * nsm);
            if (want < rpt) rpt = (int)(((want > 0 ? want : 1) + R - 1) / R * R) < rpt ? (int)(((want > 0 ? want : 1) + R - 1) / R * R) : rpt;
            if (rpt < 1) rpt = 1;
            s.rows_per_tile = rpt;
            s.tile_begin = tiles;
            tiles += (s.rows + rpt - 1) / rpt;
        }
        a.total_tiles = tiles;
        if (tiles == 0) continue;
        int rc;
        if (nt == 1)
            rc = gemv_launch_r<1>(a, R, st);
        else if (nt == 2)
            rc = gemv_launch_r<2>(a, R, st);
        else if (nt <= 4)
            rc = gemv_launch_r<4>(a, R, st);
        else if (nt <= 8)
            rc = gemv_launch_r<8>(a, R, st);
        else
            rc = gemv_launch_r<16>(a, R, st);
        if (rc) return rc;
    }
    return 0;
}

}  // namespace q35
