// gemv_lpr.cuh -- decode GEMV with one lane per weight row (sm_100a).
//
// A lane owns one row and walks its blocks in order, so the f32 fold
// `sumf += term_b` runs in the reference scalar tier's order
// (kernels32.c:462, kernels256.c:494,625) without any cross-lane exchange:
// no fold scratch, no shuffles, no per-pass warp syncs.  Per 32-weight block a
// lane spends ~20 instructions at one token.
//
// Data movement: a warp owns 32 consecutive rows (a "warp tile") and streams
// them in 256-column chunks: one 2D TMA load (cp.async.bulk.tensor, a box of
// 32 rows x one chunk, completing on the warp's mbarrier) per stage of a
// per-warp ring.  At 256 columns a row's chunk is 272 (Q8_0), 144 (IQ4_NL,
// Q4_K) or 176 (Q5_K) bytes -- an odd multiple of 16 -- so the 128-bit shared
// loads of 32 lanes (32 rows at the same column) hit distinct bank groups.
// The warp refills a slot right after it has consumed it; nothing else
// touches the ring, so only "full" barriers exist.  Weight loads are issued
// before the programmatic-launch wait, so they overlap the previous kernel's
// tail.  (Per-row copies of a few hundred bytes were issue-bound in the TMA
// unit at ~3.3 TB/s; one box per stage removes that.)
//
// Eligible: Q8_0 / IQ4_NL / Q4_K / Q5_K rows whose byte length and base are
// multiples of 16 (cols % 256 == 0).  Anything else uses k_gemv.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include "gemv.cuh"

namespace q35 {

constexpr int LPR_MAX_CW = 16;   // warps per CTA (passes of 1-2 tokens; wider passes: 8)
// warps per CTA a pass of NT tokens may use: the NT = 4 / 8 kernels need
// more than the 128 registers a 512-thread block leaves each thread
constexpr int lpr_cw_max(int nt) { return nt <= 2 ? LPR_MAX_CW : LPR_MAX_CW / 2; }
constexpr int LPR_MAX_NS = 16;   // ring stages per warp
constexpr int LPR_MAX_NT = 8;    // tokens per pass
// dynamic shared memory ceiling: the 227 KB opt-in limit less room for the
// kernel's static shared variables (the CTA-wide serial sum's ~4.3 KB)
constexpr size_t LPR_SMEM_MAX = 222 * 1024;
// per-CTA reserve when several CTAs share an SM's 228 KB: static shared
// variables plus the 1 KB the system keeps per CTA
constexpr size_t LPR_CTA_RESERVE = 5 * 1024;

struct LprSeg {
    const uint8_t *w;
    float *out;
    long long rows;
    long long out_ld;
    long long tile_begin;   // first warp tile of this matrix
    int ttype;
    int row_bytes;
    int chunk_bytes;        // bytes of one row's column chunk
    int mode;
};

struct LprArgs {
    CUtensorMap tmap[GV_MAX_SEG];  // per matrix: u64 elements, box = 32 rows x one chunk
    LprSeg seg[GV_MAX_SEG];
    int nseg;
    long long total_tiles;  // warp tiles (32 rows) over all matrices
    const uint8_t *xq;
    long long act_row_bytes;
    int ntok, cols, family, act_stride;
    int chunk_cols, nchunk; // columns per chunk, chunks per row
    int ns, rs;             // ring stages per warp, shared row stride (bytes)
    int kw;                 // warps splitting one warp tile's columns (1: no split)
    int tst;                // floats between lanes' term rows (odd), when kw > 1
    int t_off;              // byte offset of the term buffers, when kw > 1
    int act_off;            // byte offset of the activation in shared memory
    int ring_off;           // byte offset of warp 0's ring
    // prologue: build the quantized activation in shared memory from f32
    // rows instead of reading `xq` (LPR_PRO_NORM: rmsnorm(px) * pw;
    // LPR_PRO_SWIGLU: silu(px) * pu)
    int prologue;
    const float *px, *pu, *pw;
    long long px_ld;
    float eps;
    int x_off;              // byte offset of the staged f32 rows (norm)
    int il;                 // every matrix IQ4_NL / every one IQ4_XS: the activation is staged interleaved
    // pair mode (the MLP's gate / up projections): seg[0] = gate, seg[1] =
    // up, same rows; tile 2t is gate tile t and tile 2t+1 up tile t, taken
    // by row groups 2p and 2p+1 of one CTA.  The epilogue forms
    // h = silu(gate) * up per row (engine.zig:2027-2036) and writes it as
    // Q8_0 blocks into `hq` (32 rows = one block of the down projection's
    // input; hq_ld bytes between tokens) or, when hq is null, as f32 rows
    // into `hf` (hf_ld floats between tokens).
    int pair;
    int p_off;              // byte offset of the pair exchange buffers
    uint8_t *hq;
    long long hq_ld;
    float *hf;
    long long hf_ld;
};

enum { LPR_PRO_NONE = 0, LPR_PRO_NORM = 1, LPR_PRO_SWIGLU = 2, LPR_PRO_ROWS = 3 };

// The activation quantizers (quant_q8_0_warp / quant_q8_K_warp), writing the
// GEMV's shared layout directly: int8 plane, f32 scale per block (for Q8_0
// the f16-rounded scale the API layout would carry), int32 16-element sums.
// The same Q8_0 quantizer with 4 threads per 32-element block (x: the
// block's f32 values in shared memory; thread q of the quad takes elements
// 8q .. 8q+7): the block max by two shuffles (max is exact in any order),
// then every element takes the warp version's operations.
Q35_DEV void lpr_quant_q8_0_quad(const float *x, uint8_t *at, int cols, int b, int q, bool store,
                                 float scale_x = 0.0f, const float *w = nullptr) {
    float v[8];
    const float4 *x4 = reinterpret_cast<const float4 *>(x + 8 * q);
    const float4 t0 = x4[0], t1 = x4[1];
    v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
    v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
    if (w) {  // rmsnorm fused: v = (x * scale) * w (elementwise.zig:43-57)
        const float4 *w4 = reinterpret_cast<const float4 *>(w + 8 * q);
        const float4 u0 = w4[0], u1 = w4[1];
        const float wv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = __fmul_rn(__fmul_rn(v[k], scale_x), wv[k]);
    }
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) amax = fmaxf(amax, fabsf(v[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = amax > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    if (store && q == 0) reinterpret_cast<float *>(at + cols)[b] = f16_to_f32(f32_to_f16_bits(scale, 0x0380u));
    uint32_t word[2] = {0u, 0u};
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float xx = __fmul_rn(v[k], inv);
        int qv = __float2int_rz(__fadd_rn(xx, xx >= 0.0f ? 0.5f : -0.5f));
        qv = qv > 127 ? 127 : (qv < -128 ? -128 : qv);
        word[k >> 2] |= (uint32_t)(qv & 0xFF) << (8 * (k & 3));
    }
    if (store) *reinterpret_cast<uint2 *>(at + b * 32 + 8 * q) = make_uint2(word[0], word[1]);
}

Q35_DEV void lpr_quant_q8_K(const float (&v)[8], uint8_t *at, int cols, int b, int lane) {
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) a = fmaxf(a, fabsf(v[i]));
    const float amax = warp_max(a);
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = amax > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    if (lane == 0) reinterpret_cast<float *>(at + cols)[b] = scale;
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
    uint32_t *qs = reinterpret_cast<uint32_t *>(at + b * 256 + lane * 8);
    qs[0] = w0;
    qs[1] = w1;
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if ((lane & 1) == 0) reinterpret_cast<int *>(at + cols + (cols / 32) * 4)[b * 16 + (lane >> 1)] = s;
}

Q35_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2D tiled TMA load of one box into shared memory, completing on `bar`
Q35_DEV void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// The same load with an L2 eviction-priority hint.  Decode weights are
// streamed once per step and come back only after the whole model (0.8 to 15
// GB) has passed through the 126 MB L2, so they are marked evict-first: the
// data that IS reused from step to step (GDN state at small batch, KV rows,
// activations, kernel code) keeps its lines.
Q35_DEV uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
Q35_DEV void tma_load_2d_hint(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

Q35_DEV float f16_lo(uint32_t w) { return f16_to_f32((uint16_t)(w & 0xFFFFu)); }
Q35_DEV float f16_hi(uint32_t w) { return f16_to_f32((uint16_t)(w >> 16)); }

// Eight IQ4_NL values from one word of packed nibbles: lo = codebook of the
// four low nibbles (elements j..j+3), hi = of the four high nibbles
// (elements j+16..j+19).  Byte permutes over the codebook split in halves;
// bit 3 of each index then picks the half.
// iq4_word_il: the values in nibble order, v0 = [lo b0, hi b0, lo b1, hi b1]
// and v1 = [lo b2, hi b2, lo b3, hi b3] (elements j, j+16, j+1, j+17 and
// j+2, j+18, j+3, j+19), which an activation staged in the same interleaved
// order (lpr_interleave_act) dots without re-ordering.
Q35_DEV void iq4_word_il(uint32_t q, uint32_t &v0, uint32_t &v1) {
    const uint32_t s = q & 0x77777777u, s1 = s >> 16;
    const uint32_t l0 = __byte_perm(kIq4T0, kIq4T1, s), h0 = __byte_perm(kIq4T2, kIq4T3, s);
    const uint32_t l1 = __byte_perm(kIq4T0, kIq4T1, s1), h1 = __byte_perm(kIq4T2, kIq4T3, s1);
    // nibble n of q -> value n: choose the upper table half where bit 3 is
    // set; one mask serves both halves (a permute reads 16 selector bits)
    const uint32_t m = ((q >> 1) & 0x44444444u) | 0x32103210u;
    v0 = __byte_perm(l0, h0, m);
    v1 = __byte_perm(l1, h1, m >> 16);
}
Q35_DEV void iq4_word(uint32_t q, uint32_t &lo, uint32_t &hi) {
    uint32_t v0, v1;
    iq4_word_il(q, v0, v1);
    lo = __byte_perm(v0, v1, 0x6420u);
    hi = __byte_perm(v0, v1, 0x7531u);
}

// One 32-element Q8_0 activation block (8 words) re-ordered in place so
// word 2i + h holds elements 4i+2h, 16+4i+2h, 4i+2h+1, 17+4i+2h: the order
// iq4_word_il leaves the weights in.  Integer dots are exact in any order.
Q35_DEV void lpr_interleave_act(uint32_t *w) {
    uint32_t x[8];
#pragma unroll
    for (int i = 0; i < 8; i++) x[i] = w[i];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        w[2 * i] = __byte_perm(x[i], x[i + 4], 0x5140u);
        w[2 * i + 1] = __byte_perm(x[i], x[i + 4], 0x7362u);
    }
}

// byte k of the 12 K-quant scale bytes held in words S[0..2]
Q35_DEV int kq_byte(const uint32_t *S, int k) { return (int)((S[k >> 2] >> ((k & 3) * 8)) & 0xFFu); }
Q35_DEV void kq_scale_min_w(int j, const uint32_t *S, int &sc, int &m) {
    if (j < 4) {
        sc = kq_byte(S, j) & 63;
        m = kq_byte(S, j + 4) & 63;
    } else {
        sc = (kq_byte(S, j + 4) & 0xF) | ((kq_byte(S, j - 4) >> 6) << 4);
        m = (kq_byte(S, j + 4) >> 4) | ((kq_byte(S, j) >> 6) << 4);
    }
}

// ---- one lane, one row, one column chunk ---------------------------------
// rp: the row's chunk in shared memory (16-byte aligned); gb0: global block
// index of the chunk's first block.  Each block's f32 term goes to a sink:
// FoldSink adds it to the lane's running sums (the whole row is this
// lane's), TermSink stores it for the ordered fold after a K split.
template <int NT>
struct FoldSink {
    float (&acc)[NT];
    Q35_DEV void put(int t, int, float v) { acc[t] = __fadd_rn(acc[t], v); }
};
struct TermSink {
    float *tl;     // this lane's term row (token 0)
    int tok_ld;    // floats between tokens
    Q35_DEV void put(int t, int b, float v) { tl[t * tok_ld + b] = v; }
};

template <int NT, class Sink>
Q35_DEV void lpr_q8_0(const uint8_t *rp, const ActView &A, int ntok, int gb0, int nblk, Sink &sk) {
    for (int g = 0; g < nblk; g += 8) {  // 8 blocks = 272 bytes = 17 x 16
        uint32_t W[68];
        const uint4 *s = reinterpret_cast<const uint4 *>(rp + g * 34);
#pragma unroll
        for (int i = 0; i < 17; i++) {
            const uint4 v = s[i];
            W[4 * i] = v.x;
            W[4 * i + 1] = v.y;
            W[4 * i + 2] = v.z;
            W[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int o = 34 * k, w0 = o >> 2;
            uint32_t q[8];
            float dx;
            if ((o & 3) == 0) {  // d in the low half of W[w0], qs start 2 bytes in
                dx = f16_lo(W[w0]);
#pragma unroll
                for (int i = 0; i < 8; i++) q[i] = __funnelshift_r(W[w0 + i], W[w0 + i + 1], 16);
            } else {             // d in the high half, qs word-aligned
                dx = f16_hi(W[w0]);
#pragma unroll
                for (int i = 0; i < 8; i++) q[i] = W[w0 + 1 + i];
            }
            const int b = gb0 + g + k;
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < ntok) {
                    const int s0 = dot4x4(q[0], q[1], q[2], q[3], A.q16(t, b * 32), 0);
                    const int si = s0 + dot4x4(q[4], q[5], q[6], q[7], A.q16(t, b * 32 + 16), 0);
                    // sumf += dx * dy * (float)sumi
                    sk.put(t, b, __fmul_rn(__fmul_rn(dx, A.dsc(t, b)), __int2float_rn(si)));
                }
            }
        }
    }
}

// IL: the activation is staged interleaved (lpr_interleave_act)
template <int NT, bool IL, class Sink>
Q35_DEV void lpr_iq4_nl(const uint8_t *rp, const ActView &A, int ntok, int gb0, int nblk, Sink &sk) {
    for (int g = 0; g < nblk; g += 8) {  // 8 blocks = 144 bytes = 9 x 16
        uint32_t W[36];
        const uint4 *s = reinterpret_cast<const uint4 *>(rp + g * 18);
#pragma unroll
        for (int i = 0; i < 9; i++) {
            const uint4 v = s[i];
            W[4 * i] = v.x;
            W[4 * i + 1] = v.y;
            W[4 * i + 2] = v.z;
            W[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int o = 18 * k, w0 = o >> 2;
            uint32_t q[4];
            float dx;
            if ((o & 3) == 0) {
                dx = f16_lo(W[w0]);
#pragma unroll
                for (int i = 0; i < 4; i++) q[i] = __funnelshift_r(W[w0 + i], W[w0 + i + 1], 16);
            } else {
                dx = f16_hi(W[w0]);
#pragma unroll
                for (int i = 0; i < 4; i++) q[i] = W[w0 + 1 + i];
            }
            uint32_t lo[4], hi[4];  // IL: v0 / v1 of each word
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (IL)
                    iq4_word_il(q[i], lo[i], hi[i]);
                else
                    iq4_word(q[i], lo[i], hi[i]);
            }
            const int b = gb0 + g + k;
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < ntok) {
                    int si;
                    if (IL) {
                        const int s0 = dot4x4(lo[0], hi[0], lo[1], hi[1], A.q16(t, b * 32), 0);
                        si = s0 + dot4x4(lo[2], hi[2], lo[3], hi[3], A.q16(t, b * 32 + 16), 0);
                    } else {
                        const int s0 = dot4x4(lo[0], lo[1], lo[2], lo[3], A.q16(t, b * 32), 0);
                        si = s0 + dot4x4(hi[0], hi[1], hi[2], hi[3], A.q16(t, b * 32 + 16), 0);
                    }
                    sk.put(t, b, __fmul_rn(__fmul_rn(dx, A.dsc(t, b)), __int2float_rn(si)));
                }
            }
        }
    }
}

// IQ4_XS: two 136-byte blocks per 272-byte step (chunks of 512 columns).
// Eight f32 terms per block, one per 32-element sub-block, in sub-block
// order: d4d8 = d * dy, term = (d4d8 * (ls - 32)) * isum
// (iq_kernels.c:967-1000).  IL: the Q8_K plane is staged interleaved.
template <int NT, bool IL, class Sink>
Q35_DEV void lpr_iq4_xs(const uint8_t *rp, const ActView &A, int ntok, int gb0, int nblk, Sink &sk) {
    for (int g = 0; g < nblk; g += 2) {
        uint32_t W[68];
        const uint4 *s = reinterpret_cast<const uint4 *>(rp + g * 136);
#pragma unroll
        for (int i = 0; i < 17; i++) {
            const uint4 v = s[i];
            W[4 * i] = v.x;
            W[4 * i + 1] = v.y;
            W[4 * i + 2] = v.z;
            W[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int w0 = 34 * k;  // 136 bytes = 34 words: both blocks word-aligned
            const int b = gb0 + g + k;
            const float d = f16_lo(W[w0]);
            const int sh = (int)(W[w0] >> 16);
            const uint32_t sl = W[w0 + 1];
            float d4d8[NT];
#pragma unroll
            for (int t = 0; t < NT; t++) d4d8[t] = t < ntok ? __fmul_rn(d, A.dsc(t, b)) : 0.0f;
#pragma unroll
            for (int ib = 0; ib < 8; ib++) {
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    if (IL)
                        iq4_word_il(W[w0 + 2 + 4 * ib + i], lo[i], hi[i]);
                    else
                        iq4_word(W[w0 + 2 + 4 * ib + i], lo[i], hi[i]);
                }
                const float dls = __int2float_rn(iq4xs_ls((int)((sl >> (8 * (ib >> 1))) & 0xFFu), sh, ib) - 32);
                const int e0 = b * 256 + ib * 32;
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    if (t < ntok) {
                        int si;
                        if (IL) {
                            const int s0 = dot4x4(lo[0], hi[0], lo[1], hi[1], A.q16(t, e0), 0);
                            si = s0 + dot4x4(lo[2], hi[2], lo[3], hi[3], A.q16(t, e0 + 16), 0);
                        } else {
                            const int s0 = dot4x4(lo[0], lo[1], lo[2], lo[3], A.q16(t, e0), 0);
                            si = s0 + dot4x4(hi[0], hi[1], hi[2], hi[3], A.q16(t, e0 + 16), 0);
                        }
                        sk.put(t, b * 8 + ib, __fmul_rn(__fmul_rn(d4d8[t], dls), __int2float_rn(si)));
                    }
                }
            }
        }
    }
}

// u32 at an even byte offset o of a register copy of 16-byte-aligned words
template <int N>
Q35_DEV uint32_t w32_at(const uint32_t (&W)[N], int o) {
    return (o & 3) == 0 ? W[o >> 2] : __funnelshift_r(W[o >> 2], W[(o >> 2) + 1], 16);
}
template <int N>
Q35_DEV float f16_at_w(const uint32_t (&W)[N], int o) {
    return (o & 3) == 0 ? f16_lo(W[o >> 2]) : f16_hi(W[o >> 2]);
}

// Q4_0 / Q4_1 / Q5_0 / Q5_1 (18 / 20 / 22 / 24-byte blocks): 8 blocks of a
// 256-column chunk (144 / 160 / 176 / 192 bytes, 16-byte multiples) in
// registers; per block the signed bytes of legacy_bytes, dot products with
// the Q8_0 activation, the f32 term of kernels32.c (legacy_term's steps)
template <int NT, int TT, class Sink>
Q35_DEV void lpr_legacy(const uint8_t *rp, const ActView &A, int ntok, int gb0, int nblk, Sink &sk) {
    constexpr int B = TT == TT_Q4_0 ? 18 : TT == TT_Q4_1 ? 20 : TT == TT_Q5_0 ? 22 : 24;
    constexpr int NW = 2 * B;  // words of 8 blocks
    constexpr int QS = legacy_qs_off(TT), QH = legacy_qh_off(TT);
    constexpr bool AFF = legacy_affine(TT), FIVE = legacy_five(TT);
    for (int g = 0; g < nblk; g += 8) {
        uint32_t W[NW + 1];
        const uint4 *s = reinterpret_cast<const uint4 *>(rp + g * B);
#pragma unroll
        for (int i = 0; i < NW / 4; i++) {
            const uint4 v = s[i];
            W[4 * i] = v.x;
            W[4 * i + 1] = v.y;
            W[4 * i + 2] = v.z;
            W[4 * i + 3] = v.w;
        }
        W[NW] = 0u;  // read by the funnel shift of the last block's last word, never used
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int o = B * k;
            const float dx = f16_at_w(W, o);
            const float mx = AFF ? f16_at_w(W, o + 2) : 0.0f;
            uint32_t q[4], lo[4], hi[4];
#pragma unroll
            for (int i = 0; i < 4; i++) q[i] = w32_at(W, o + QS + 4 * i);
            legacy_bytes(TT, FIVE ? w32_at(W, o + QH) : 0u, q, lo, hi);
            const int b = gb0 + g + k;
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < ntok) {
                    const uint4 y0 = A.q16(t, b * 32), y1 = A.q16(t, b * 32 + 16);
                    const int si = dot4x4(hi[0], hi[1], hi[2], hi[3], y1, dot4x4(lo[0], lo[1], lo[2], lo[3], y0, 0));
                    const float dy = A.dsc(t, b);
                    float term = __fmul_rn(__fmul_rn(dx, dy), __int2float_rn(si));
                    if (AFF) {
                        constexpr uint32_t one = 0x01010101u;
                        const int sy = dot4x4(one, one, one, one, y1, dot4x4(one, one, one, one, y0, 0));
                        term = __fadd_rn(term, __fmul_rn(__fmul_rn(mx, dy), __int2float_rn(sy)));
                    }
                    sk.put(t, b, term);
                }
            }
        }
    }
}

// Q4_K (144 B: d|dmin, 12 scale bytes, 128 qs) and Q5_K (176 B: d|dmin,
// scales, 32 qh, 128 qs); both 16-byte multiples, so every block of the
// chunk starts 16-byte aligned.
template <int NT, bool Q5, class Sink>
Q35_DEV void lpr_q45_k(const uint8_t *rp, const ActView &A, int ntok, int gb0, int nblk, Sink &sk) {
    constexpr int NW = Q5 ? 44 : 36;
    for (int k = 0; k < nblk; k++) {
        uint32_t W[NW];
        const uint4 *s = reinterpret_cast<const uint4 *>(rp + k * NW * 4);
#pragma unroll
        for (int i = 0; i < NW / 4; i++) {
            const uint4 v = s[i];
            W[4 * i] = v.x;
            W[4 * i + 1] = v.y;
            W[4 * i + 2] = v.z;
            W[4 * i + 3] = v.w;
        }
        const int b = gb0 + k;
        int is[NT], ms[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) is[t] = 0, ms[t] = 0;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            int sc0, m0, sc1, m1;
            kq_scale_min_w(2 * c, W + 1, sc0, m0);
            kq_scale_min_w(2 * c + 1, W + 1, sc1, m1);
            uint32_t lo[8], hi[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t ql = W[(Q5 ? 12 : 4) + 8 * c + i];
                lo[i] = ql & 0x0F0F0F0Fu;
                hi[i] = (ql >> 4) & 0x0F0F0F0Fu;
                if (Q5) {
                    const uint32_t qh = W[4 + i];
                    lo[i] |= ((qh >> (2 * c)) & 0x01010101u) << 4;
                    hi[i] |= ((qh >> (2 * c + 1)) & 0x01010101u) << 4;
                }
            }
            const int e0 = b * 256 + 64 * c;
            const int gq = b * 16 + 4 * c;
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < ntok) {
                    const int dl = dot4x4(lo[0], lo[1], lo[2], lo[3], A.q16(t, e0), 0) +
                                   dot4x4(lo[4], lo[5], lo[6], lo[7], A.q16(t, e0 + 16), 0);
                    const int dh = dot4x4(hi[0], hi[1], hi[2], hi[3], A.q16(t, e0 + 32), 0) +
                                   dot4x4(hi[4], hi[5], hi[6], hi[7], A.q16(t, e0 + 48), 0);
                    is[t] += sc0 * dl + sc1 * dh;
                    ms[t] += m0 * (A.bsum(t, gq) + A.bsum(t, gq + 1)) + m1 * (A.bsum(t, gq + 2) + A.bsum(t, gq + 3));
                }
            }
        }
        const float dw = f16_lo(W[0]), dmw = f16_hi(W[0]);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t < ntok) {
                // d = dy*d_w; dmin = dy*dmin_w; sumf += d*isum - dmin*sumi
                const float dy = A.dsc(t, b);
                const float d = __fmul_rn(dy, dw), dm = __fmul_rn(dy, dmw);
                sk.put(t, b, __fsub_rn(__fmul_rn(d, __int2float_rn(is[t])), __fmul_rn(dm, __int2float_rn(ms[t]))));
            }
        }
    }
}

// Q6_K in the padded 224-byte layout: ql[128] @0, qh[64] @128, int8
// scales[16] @192, f16 d @208 (kernels256.c:720-738): 4 parts (2 halves x 2
// sixteen-element ranges) of 4 x 16 elements, isum = sum of scale x
// 16-element dot, sumf += (d_w*dy)*(float)isum
template <int NT, class Sink>
Q35_DEV void lpr_q6_k(const uint8_t *rp, const ActView &A, int ntok, int gb0, int nblk, Sink &sk) {
    for (int k = 0; k < nblk; k++) {
        uint32_t W[56];
        const uint4 *s = reinterpret_cast<const uint4 *>(rp + k * 224);
#pragma unroll
        for (int i = 0; i < 14; i++) {
            const uint4 v = s[i];
            W[4 * i] = v.x;
            W[4 * i + 1] = v.y;
            W[4 * i + 2] = v.z;
            W[4 * i + 3] = v.w;
        }
        const int b = gb0 + k;
        int is[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) is[t] = 0;
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int h = p >> 1, hf = p & 1;
            int sc[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int byte = h * 8 + hf + 2 * u;  // scales[h*8 + hf + 2u]
                sc[u] = (int)(int8_t)((W[48 + (byte >> 2)] >> ((byte & 3) * 8)) & 0xFFu);
            }
            uint32_t v1[4], v2[4], v3[4], v4[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t qa = W[(h * 64 + 16 * hf) / 4 + i];
                const uint32_t qb = W[(h * 64 + 32 + 16 * hf) / 4 + i];
                const uint32_t qh = W[(128 + h * 32 + 16 * hf) / 4 + i];
                v1[i] = __vsub4((qa & 0x0F0F0F0Fu) | ((qh & 0x03030303u) << 4), 0x20202020u);
                v2[i] = __vsub4((qb & 0x0F0F0F0Fu) | (((qh >> 2) & 0x03030303u) << 4), 0x20202020u);
                v3[i] = __vsub4(((qa >> 4) & 0x0F0F0F0Fu) | (((qh >> 4) & 0x03030303u) << 4), 0x20202020u);
                v4[i] = __vsub4(((qb >> 4) & 0x0F0F0F0Fu) | (((qh >> 6) & 0x03030303u) << 4), 0x20202020u);
            }
            const int e0 = b * 256 + h * 128 + 16 * hf;
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < ntok) {
                    const int d1 = dot4x4(v1[0], v1[1], v1[2], v1[3], A.q16(t, e0), 0);
                    const int d2 = dot4x4(v2[0], v2[1], v2[2], v2[3], A.q16(t, e0 + 32), 0);
                    const int d3 = dot4x4(v3[0], v3[1], v3[2], v3[3], A.q16(t, e0 + 64), 0);
                    const int d4 = dot4x4(v4[0], v4[1], v4[2], v4[3], A.q16(t, e0 + 96), 0);
                    is[t] += sc[0] * d1 + sc[1] * d2 + sc[2] * d3 + sc[3] * d4;
                }
            }
        }
        const float dw = f16_lo(W[52]);
#pragma unroll
        for (int t = 0; t < NT; t++)
            if (t < ntok) sk.put(t, b, __fmul_rn(__fmul_rn(dw, A.dsc(t, b)), __int2float_rn(is[t])));
    }
}

Q35_DEV int lpr_find_seg(const LprArgs &a, long long tile) {
    if (a.pair) return (int)(tile & 1);
    int s = 0;
#pragma unroll
    for (int i = 1; i < GV_MAX_SEG; i++)
        if (i < a.nseg && tile >= a.seg[i].tile_begin) s = i;
    return s;
}
// first row of `tile` within its matrix
Q35_DEV long long lpr_tile_row0(const LprArgs &a, const LprSeg &sg, long long tile) {
    return a.pair ? (tile >> 1) * 32 : (tile - sg.tile_begin) * 32;
}

template <int NT, class Sink>
Q35_DEV void lpr_chunk(int tt, const uint8_t *rp, const ActView &A, int ntok, int c, int chunk_cols, Sink &sk) {
    switch (tt) {
    case TT_Q8_0: lpr_q8_0<NT>(rp, A, ntok, c * (chunk_cols / 32), chunk_cols / 32, sk); break;
    case TT_IQ4_NL:
        if (A.il)
            lpr_iq4_nl<NT, true>(rp, A, ntok, c * (chunk_cols / 32), chunk_cols / 32, sk);
        else
            lpr_iq4_nl<NT, false>(rp, A, ntok, c * (chunk_cols / 32), chunk_cols / 32, sk);
        break;
    case TT_Q4_0: lpr_legacy<NT, TT_Q4_0>(rp, A, ntok, c * (chunk_cols / 32), chunk_cols / 32, sk); break;
    case TT_Q4_1: lpr_legacy<NT, TT_Q4_1>(rp, A, ntok, c * (chunk_cols / 32), chunk_cols / 32, sk); break;
    case TT_Q5_0: lpr_legacy<NT, TT_Q5_0>(rp, A, ntok, c * (chunk_cols / 32), chunk_cols / 32, sk); break;
    case TT_Q5_1: lpr_legacy<NT, TT_Q5_1>(rp, A, ntok, c * (chunk_cols / 32), chunk_cols / 32, sk); break;
    case TT_Q4_K: lpr_q45_k<NT, false>(rp, A, ntok, c * (chunk_cols / 256), chunk_cols / 256, sk); break;
    case TT_IQ4_XS:
        if (A.il)
            lpr_iq4_xs<NT, true>(rp, A, ntok, c * (chunk_cols / 256), chunk_cols / 256, sk);
        else
            lpr_iq4_xs<NT, false>(rp, A, ntok, c * (chunk_cols / 256), chunk_cols / 256, sk);
        break;
    case TT_Q6_K_P: lpr_q6_k<NT>(rp, A, ntok, c * (chunk_cols / 256), chunk_cols / 256, sk); break;
    default: lpr_q45_k<NT, true>(rp, A, ntok, c * (chunk_cols / 256), chunk_cols / 256, sk); break;
    }
}

// CTA = rw row groups x kw column warps.  A row group owns a warp tile (32
// rows) at a time; its kw warps take contiguous column-chunk ranges of it.
// kw == 1: the lane folds its row in registers.  kw > 1: lanes store their
// block terms, and after a named barrier warp 0 of the group folds each row's
// terms in block order (the same rounding sequence).
template <int NT>
__global__ void __launch_bounds__(lpr_cw_max(NT) * 32) k_gemv_lpr(const __grid_constant__ LprArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int cw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kw = a.kw, rg = warp / kw, kq = warp - rg * kw, rw = cw / kw;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem) + warp * LPR_MAX_NS;
    uint8_t *act = smem + a.act_off;
    uint8_t *ring = smem + a.ring_off + (size_t)warp * a.ns * 32 * a.rs;
    float *terms = reinterpret_cast<float *>(smem + a.t_off) + (size_t)rg * NT * 32 * a.tst;
    pdl_trigger();
    if (lane == 0) {
        for (int s = 0; s < a.ns; s++) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    const long long tstride = (long long)gridDim.x * rw;
    const long long t0 = (long long)blockIdx.x * rw + rg;
    const long long my_tiles = t0 < a.total_tiles ? (a.total_tiles - 1 - t0) / tstride + 1 : 0;
    const int c_lo = kq * a.nchunk / kw, c_hi = (kq + 1) * a.nchunk / kw, nck = c_hi - c_lo;
    const long long nst = my_tiles * nck;  // stages this warp consumes
    const uint64_t wpol = l2_policy_evict_first();

    // stage i of this warp -> (matrix, first row, chunk); lane `lane` copies its row
    // The producer walks the stages in order with running counters (tile
    // index, chunk, ring slot): no 64-bit division on the issue path.
    long long p_tile = t0;
    int p_c = 0, p_slot = 0;
    auto issue = [&]() {
        const long long tile = p_tile;
        const int c = c_lo + p_c;
        const int slot = p_slot;
        if (++p_c == nck) {
            p_c = 0;
            p_tile += tstride;
        }
        if (++p_slot == a.ns) p_slot = 0;
        const int si = lpr_find_seg(a, tile);
        const LprSeg &sg = a.seg[si];
        const long long r0 = lpr_tile_row0(a, sg, tile);
        if (lane == 0) {
            // the box is always 32 full rows (rows past the end are zero-filled)
            mbar_arrive_expect_tx(&bar[slot], (uint32_t)(32 * sg.chunk_bytes));
            tma_load_2d_hint(ring + (size_t)slot * 32 * a.rs, &a.tmap[si], c * (sg.chunk_bytes / 8), (int)r0,
                             &bar[slot], wpol);
        }
    };
    long long issued = nst < a.ns ? nst : a.ns;
    for (long long i = 0; i < issued; i++) issue();
    // the norm weight is constant: staged before the dependency wait
    if (a.prologue == LPR_PRO_NORM) {
        float4 *wd = reinterpret_cast<float4 *>(smem + a.x_off) + (size_t)a.ntok * (a.cols / 4);
        for (int j = threadIdx.x; j < a.cols / 4; j += blockDim.x) wd[j] = reinterpret_cast<const float4 *>(a.pw)[j];
    }

    // the activation belongs to the previous kernel
    pdl_wait();
    if (a.prologue != LPR_PRO_NONE) {
        // Build the f32 input rows in shared memory first, every global load
        // independent of the others (coalesced float4), then quantize from
        // shared memory; the per-block quantize steps are warp-synchronous
        // and would otherwise wait out one memory round trip each.
        __shared__ float s_scale[LPR_MAX_NT];
        float *xs = reinterpret_cast<float *>(smem + a.x_off);  // [ntok][cols]
        float *ws = xs + (size_t)a.ntok * a.cols;                 // norm weight [cols]
        const int c4 = a.cols / 4;
        float4 *xd = reinterpret_cast<float4 *>(xs);
        if (a.prologue == LPR_PRO_NORM) {
            // rmsnorm (engine.zig:1507, elementwise.zig:43-57): the sum of
            // squares in the CPU's serial order, one thread per token
            for (int idx = threadIdx.x; idx < a.ntok * c4; idx += blockDim.x) {
                const int t = idx / c4, j = idx - t * c4;
                xd[idx] = reinterpret_cast<const float4 *>(a.px + (long long)t * a.px_ld)[j];
            }
            __syncthreads();
            if (a.ntok == 1 && cw >= 2) {
                // one row: the whole CTA runs the chain (segments in parallel)
                const float ss = cta_spec_sumsq(xs, a.cols);
                if (threadIdx.x == 0)
                    s_scale[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.cols), a.eps)));
            } else if ((int)threadIdx.x < a.ntok) {
                const float ss = serial_sumsq(xs + (size_t)threadIdx.x * a.cols, a.cols);
                s_scale[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.cols), a.eps)));
            }
        } else if (a.prologue == LPR_PRO_ROWS) {
            // f32 rows as they are (a producer already applied the activation)
            for (int idx = threadIdx.x; idx < a.ntok * c4; idx += blockDim.x) {
                const int t = idx / c4, j = idx - t * c4;
                xd[idx] = reinterpret_cast<const float4 *>(a.px + (long long)t * a.px_ld)[j];
            }
        } else {
            // silu(gate) * up (engine.zig:2027-2036)
            for (int idx = threadIdx.x; idx < a.ntok * c4; idx += blockDim.x) {
                const int t = idx / c4, j = idx - t * c4;
                const float4 g = reinterpret_cast<const float4 *>(a.px + (long long)t * a.px_ld)[j];
                const float4 u = reinterpret_cast<const float4 *>(a.pu + (long long)t * a.px_ld)[j];
                xd[idx] = make_float4(__fmul_rn(silu_f(g.x), u.x), __fmul_rn(silu_f(g.y), u.y),
                                      __fmul_rn(silu_f(g.z), u.z), __fmul_rn(silu_f(g.w), u.w));
            }
        }
        __syncthreads();
        if (a.family == 32) {
            const int nb = a.cols / 32;
            const bool nrm = a.prologue == LPR_PRO_NORM;
            // quads of threads per block; every quad of a warp takes part in
            // the shuffles, so the loop runs whole-warp rounds
            const int nq = a.ntok * nb * 4;
            for (int base = warp * 32; base < nq; base += blockDim.x) {
                const int qi = base + lane;
                const int bi = qi >> 2, q = qi & 3;
                const bool live = bi < a.ntok * nb;
                const int bs = live ? bi : 0;  // lanes past the end redo block 0 without storing
                const int t = bs / nb, b = bs - t * nb;
                lpr_quant_q8_0_quad(xs + (size_t)t * a.cols + b * 32, act + (size_t)t * a.act_stride, a.cols, b, q,
                                    live, nrm ? s_scale[t] : 0.0f, nrm ? ws + b * 32 : nullptr);
            }
        } else {
            const int nb = a.cols / 256;
            for (int bi = warp; bi < a.ntok * nb; bi += cw) {
                const int t = bi / nb, b = bi - t * nb;
                float v[8];
                const float4 *src = reinterpret_cast<const float4 *>(xs + (size_t)t * a.cols + b * 256 + lane * 8);
                const float4 v0 = src[0], v1 = src[1];
                v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
                v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
                if (a.prologue == LPR_PRO_NORM) {
#pragma unroll
                    for (int k = 0; k < 8; k++) v[k] = __fmul_rn(__fmul_rn(v[k], s_scale[t]), ws[b * 256 + lane * 8 + k]);
                }
                lpr_quant_q8_K(v, act + (size_t)t * a.act_stride, a.cols, b, lane);
            }
        }
    } else if (a.family == 32) {
        const int nb = a.cols / 32;
        for (int idx = threadIdx.x; idx < a.ntok * nb; idx += blockDim.x) {
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
        for (int idx = threadIdx.x; idx < a.ntok * nb * 17; idx += blockDim.x) {
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
    __syncthreads();
    if (a.il) {
        const int nb = a.cols / 32;
        for (int idx = threadIdx.x; idx < a.ntok * nb; idx += blockDim.x) {
            const int t = idx / nb, b = idx - t * nb;
            lpr_interleave_act(reinterpret_cast<uint32_t *>(act + (size_t)t * a.act_stride + b * 32));
        }
        __syncthreads();
    }

    const ActView A{act, a.act_stride, a.cols, a.il};
    const int nb = a.cols / term_elems(a.seg[0].ttype);  // f32 terms per row
    bool failed = false;
    long long waited = 0;
    long long i = 0;
    int slot = 0;        // ring slot of stage i, and the parity of its fill
    uint32_t par = 0;
    for (long long ti = 0; ti < my_tiles; ti++) {
        const long long tile = t0 + ti * tstride;
        const LprSeg &sg = a.seg[lpr_find_seg(a, tile)];
        const long long r0 = lpr_tile_row0(a, sg, tile);
        const int nv = (int)min(32LL, sg.rows - r0);
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.0f;
        for (int c = c_lo; c < c_hi; c++, i++) {
            if (!failed) {
                if (mbar_wait(&bar[slot], par, 111))
                    waited = i + 1;
                else
                    failed = true;  // keep walking the loop: the named barriers below need every warp
            }
            if (!failed && lane < nv) {
                const uint8_t *rp = ring + (size_t)slot * 32 * a.rs + (size_t)lane * sg.chunk_bytes;
                if (kw == 1) {
                    FoldSink<NT> sk{acc};
                    lpr_chunk<NT>(sg.ttype, rp, A, a.ntok, c, a.chunk_cols, sk);
                } else {
                    TermSink sk{terms + (size_t)lane * a.tst, 32 * a.tst};
                    lpr_chunk<NT>(sg.ttype, rp, A, a.ntok, c, a.chunk_cols, sk);
                }
            }
            // every lane is done reading this slot before the bulk engine refills it
            __syncwarp();
            fence_proxy_async_smem();
            if (!failed && issued < nst && issued == i + a.ns) {
                issue();  // stage i + ns, into the slot just consumed
                issued++;
            }
            if (++slot == a.ns) {
                slot = 0;
                par ^= 1u;
            }
        }
        if (kw > 1) {
            named_bar_sync(1 + rg, kw * 32);  // the group's terms for this tile are stored
            if (kq == 0 && !failed && lane < nv) {
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    if (t < a.ntok) {
                        const float *tl = terms + ((size_t)t * 32 + lane) * a.tst;
                        float s = 0.0f;
#pragma unroll 8
                        for (int b = 0; b < nb; b++) s = __fadd_rn(s, tl[b]);
                        acc[t] = s;
                    }
                }
            }
            named_bar_sync(1 + rg, kw * 32);  // folded before the next tile's terms land
        }
        if (a.pair) {
            // gate / up epilogue: the up group hands its sums to the gate
            // group of the same pair through shared memory
            if (kq == 0) {
                const int pr = rg >> 1;
                float *xb = reinterpret_cast<float *>(smem + a.p_off) + (size_t)pr * NT * 32;
                if (rg & 1) {
#pragma unroll
                    for (int t = 0; t < NT; t++) xb[t * 32 + lane] = (!failed && lane < nv) ? acc[t] : 0.0f;
                }
                named_bar_sync(8 + pr, 64);
                if (!(rg & 1)) {
                    const long long blk = tile >> 1;  // = r0 / 32
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        if (t < a.ntok) {
                            const float h = (!failed && lane < nv) ? __fmul_rn(silu_f(acc[t]), xb[t * 32 + lane]) : 0.0f;
                            if (a.hq)
                                quant_q8_0_warp(h, a.hq + (long long)t * a.hq_ld + blk * 34, lane);
                            else if (lane < nv)
                                a.hf[(long long)t * a.hf_ld + r0 + lane] = h;
                        }
                    }
                }
                named_bar_sync(8 + pr, 64);  // the buffer is read before the next tile's sums land
            }
        } else if (kq == 0 && !failed && lane < nv) {
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < a.ntok) {
                    float *o = sg.out + r0 + lane + (long long)t * sg.out_ld;
                    *o = sg.mode == GV_ADD ? __fadd_rn(*o, acc[t]) : acc[t];
                }
            }
        }
    }
    if (failed) {
        // give the copies still in flight into this warp's ring a bounded chance to land
        for (long long k = waited + 1; k < issued; k++)
            if (!mbar_wait(&bar[k % a.ns], (uint32_t)((k / a.ns) & 1), 112)) break;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int NT>
inline cudaError_t gemv_lpr_set_smem() {
    return cudaFuncSetAttribute(k_gemv_lpr<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LPR_SMEM_MAX);
}
inline int gemv_lpr_prepare() {
    static int done = 0;
    if (done) return 0;
    const cudaError_t es[] = {gemv_lpr_set_smem<1>(), gemv_lpr_set_smem<2>(), gemv_lpr_set_smem<4>(),
                              gemv_lpr_set_smem<8>()};
    for (cudaError_t e : es)
        if (e != cudaSuccess) return (int)e;
    done = 1;
    return 0;
}

inline bool lpr_type_ok(int tt) {
    return tt == TT_Q8_0 || tt == TT_IQ4_NL || tt == TT_Q4_K || tt == TT_Q5_K || tt == TT_Q6_K_P || tt == TT_IQ4_XS ||
           legacy_type(tt);
}

// f32 rows the launch quantizes itself (see LprArgs::prologue)
struct LprPrologue {
    int kind;              // LPR_PRO_NORM, LPR_PRO_SWIGLU or LPR_PRO_ROWS
    const float *x, *u, *w;
    long long ld;          // floats between tokens of x (and u)
    float eps;
};
constexpr size_t LPR_PRO_STAGE_MAX = 64 * 1024;  // f32 rows a fused prologue stages in shared memory

// pair mode destination (see LprArgs::pair): Q8_0 blocks, or f32 rows
struct LprPair {
    uint8_t *hq;
    long long hq_ld;
    float *hf;
    long long hf_ld;
};

// Try the lane-per-row kernel.  Returns -1 (nothing launched) when the
// matrices or the shape are not eligible, else the launch status.
#ifndef LPR_TALL_OCC
#define LPR_TALL_OCC 3          // CTAs per SM for tall matrices (4 row groups each)
#endif
#ifndef LPR_TALL_OCC_SMALL
#define LPR_TALL_OCC_SMALL 4    // the same for 144-byte row chunks at 1-2 tokens
#endif
constexpr int LPR_CHUNK_COLS = 256;  // columns per streamed chunk (row chunks are odd multiples of 16 B)

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
inline PFN_cuTensorMapEncodeTiled_v12000 lpr_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// the weight matrix as [rows][row_bytes / 8] u64 elements; box = 32 rows x
// one chunk.  Base and row length are multiples of 16 bytes (checked by the
// caller), as the tensor-map rules require.
inline bool lpr_encode(CUtensorMap *m, const void *w, int row_bytes, long long rows, int chunk_bytes) {
    const auto fn = lpr_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(chunk_bytes / 8), 32u};
    const cuuint32_t estr[2] = {1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
#ifndef LPR_WARPS_PER_SM
// warps per SM aimed at for short matrices (columns split): the register-
// limited capacity (65536 registers / (32 lanes x ~128 registers)), so the
// whole split still runs in one wave
#define LPR_WARPS_PER_SM 16
#endif

inline int lpr_tmpl_nt(int nt) { return nt == 1 ? 1 : (nt == 2 ? 2 : (nt <= 4 ? 4 : 8)); }

inline int gemv_lpr_launch(const GemvSegDesc *segs, int nseg, const void *xq, int cols, int ntok, cudaStream_t st,
                           long long xq_ld, const LprPrologue *pro = nullptr, const LprPair *pair = nullptr) {
    if (nseg < 1 || nseg > GV_MAX_SEG || cols <= 0 || ntok <= 0 || cols % 256 != 0) return -1;
    if (pair) {
        // gate / up of one MLP: same rows and type, activation built in the
        // kernel (the epilogue's Q8_0 output may be the buffer a caller would
        // otherwise pass as xq)
        if (nseg != 2 || !pro || segs[0].rows != segs[1].rows || segs[0].ttype != segs[1].ttype) return -1;
        if (pair->hq ? (pair->hq_ld <= 0) : (!pair->hf || pair->hf_ld < segs[0].rows)) return -1;
        if (pair->hq && segs[0].rows % 32) return -1;
    }
    if (pro) {
        if (pro->kind != LPR_PRO_NORM && pro->kind != LPR_PRO_SWIGLU && pro->kind != LPR_PRO_ROWS) return -1;
        // 8 tokens or more: the tensor-core path (MMQ_MIN_TOK), after a separate prologue kernel
        if (ntok >= 8) return -1;
        if ((reinterpret_cast<uintptr_t>(pro->x) & 15u) || (pro->ld & 3)) return -1;
    }
    const int fam = geom_of(segs[0].ttype).family;
    // IQ4_XS blocks are 136 bytes: two per chunk keep the chunk a 16-byte
    // multiple (the TMA box rule); its eight terms per block need every
    // matrix of the launch to be IQ4_XS
    bool xs = false;
    for (int i = 0; i < nseg; i++) xs = xs || segs[i].ttype == TT_IQ4_XS;
    for (int i = 0; i < nseg && xs; i++)
        if (segs[i].ttype != TT_IQ4_XS) return -1;
    const int chunk_cols = xs ? 2 * LPR_CHUNK_COLS : LPR_CHUNK_COLS;
    if (cols % chunk_cols) return -1;
    int rs = 0;
    long long T = 0;
    for (int i = 0; i < nseg; i++) {
        const Geom g = geom_of(segs[i].ttype);
        if (!lpr_type_ok(segs[i].ttype) || g.family != fam) return -1;
        const int rb = cols / g.elems * g.bytes;
        if (rb % 16 != 0 || (reinterpret_cast<uintptr_t>(segs[i].w) & 15u) != 0) return -1;
        const int cb = chunk_cols / g.elems * g.bytes;  // 272 / 144 / 144 / 176
        rs = cb > rs ? cb : rs;
        T += (segs[i].rows + 31) / 32;
    }
    if (!pro && fam == 256 && (reinterpret_cast<uintptr_t>(xq) & 3u) != 0) return -1;
    const long long act_row_bytes =
        xq_ld > 0 ? xq_ld : (fam == 32 ? (long long)(cols / 32) * 34 : (long long)(cols / 256) * 292);
    if (!pro && fam == 256 && (act_row_bytes & 3)) return -1;
    if (T == 0) return 0;
    Q35_TRY_RC(gemv_lpr_prepare());
    const int nsm = gemv_sm_count();
    const int nchunk = cols / chunk_cols;
    const int nb = cols / term_elems(segs[0].ttype);  // f32 terms per row
    const int tst = nb % 2 == 0 ? nb + 1 : nb;
    const int act_stride = gemv_act_stride(cols, fam);

    // launch geometry: tall matrices keep a whole row per lane (kw = 1, four
    // row groups per CTA); short ones split each warp tile's columns over kw
    // warps so that ~LPR_WARPS_PER_SM warps per SM stream the matrix
    int kw = 1, rw = 4, occ = LPR_TALL_OCC;
    long long ctas;
    if (T >= (long long)nsm * LPR_TALL_OCC * 4) {
        ctas = (T + 3) / 4;
        // 144-byte chunks (IQ4_NL, Q4_0, Q4_K): the decode is instruction-
        // bound (the integer ALU pipe, not DRAM, is the busiest unit), so a
        // fourth CTA per SM (the registers allow it; the ring still gets two
        // stages) adds warps to issue from
        if (rs <= 144 && ntok <= 2) occ = LPR_TALL_OCC_SMALL;
    } else {
        rw = pair ? 2 : 1;  // pair mode: a CTA takes a gate tile and the matching up tile
        // the widest column split (any count of warps, at most one chunk
        // range per warp) whose CTAs still fit in one wave at the register-
        // limited LPR_WARPS_PER_SM warps per SM
        const long long tiles_ctas = (T + rw - 1) / rw;
        const int nt_pass = ntok < LPR_MAX_NT ? ntok : LPR_MAX_NT;
        const int warps_sm = nt_pass <= 2 ? LPR_WARPS_PER_SM : LPR_WARPS_PER_SM * 3 / 4;  // wider: ~169 registers
        for (int k = 2; rw * k <= lpr_cw_max(nt_pass) && k <= nchunk; k++) {
            const int per_sm = warps_sm / (rw * k);
            if (per_sm < 1 || tiles_ctas > (long long)nsm * per_sm) break;
            kw = k;
        }
        ctas = (T + rw - 1) / rw;
        occ = (int)((ctas + nsm - 1) / nsm);
    }
    occ = occ < 1 ? 1 : (occ > 8 ? 8 : occ);
    int cw = rw * kw;
    size_t budget = occ == 1 ? LPR_SMEM_MAX : (size_t)(228 * 1024) / occ - LPR_CTA_RESERVE;
    // prologue staging: the f32 rows (+ the norm weight) of one pass
    auto xbytes = [&](int nt) -> size_t {
        if (!pro) return 0;
        const size_t b = (size_t)(nt + (pro->kind == LPR_PRO_NORM ? 1 : 0)) * cols * 4;
        return (b + 127) & ~size_t(127);
    };
    auto tbytes = [&](int nt) { return kw > 1 ? (size_t)rw * lpr_tmpl_nt(nt) * 32 * tst * 4 : 0; };
    auto pbytes = [&](int nt) { return pair ? (size_t)(rw / 2) * lpr_tmpl_nt(nt) * 32 * 4 : 0; };
    auto base_of = [&](int nt) {  // barriers | activation | staged rows | terms | pair buffers
        return (size_t)(LPR_MAX_CW * LPR_MAX_NS * 8) + (((size_t)nt * act_stride + 127) & ~size_t(127)) + xbytes(nt) +
               ((tbytes(nt) + 127) & ~size_t(127)) + ((pbytes(nt) + 127) & ~size_t(127));
    };
    // tokens per pass: at most LPR_MAX_NT, with room for a 2-stage ring
    // tokens per pass: as many as the kernel takes (each pass streams the
    // weights again), giving up CTAs per SM, then ring depth, before tokens
    int group = ntok < LPR_MAX_NT ? lpr_tmpl_nt(ntok) : LPR_MAX_NT;
    if (pro && xbytes(group) > LPR_PRO_STAGE_MAX) return -1;  // a fused prologue stages a whole pass
    auto need = [&](int g, int nsmin) { return base_of(g) + (size_t)cw * nsmin * 32 * rs; };
    auto budget_of = [](int o) { return o == 1 ? LPR_SMEM_MAX : (size_t)(228 * 1024) / o - LPR_CTA_RESERVE; };
    // CTAs per SM come down only when the minimum ring no longer fits.  Short
    // matrices need one stage per warp: keeping every warp tile in the first
    // wave matters more at decode (weights prefetched before the dependency
    // wait, compute latency-bound) than a deeper ring.  A tall matrix streams
    // many chunks per warp and keeps at least two stages in flight.
    const bool tall = kw == 1 && rw == 4;
    const int nsmin = tall ? 2 : 1;
    // a short matrix first narrows its column split (fewer warps, smaller
    // rings) until the CTAs of one wave fit, then gives up CTAs per SM
    while (!tall && kw > 1 && need(group, 1) > budget) {
        kw >>= 1;
        cw = rw * kw;
    }
    while (occ > 1 && need(group, nsmin) > budget) budget = budget_of(--occ);
    while (group > 1 && need(group, 1) > budget) group >>= 1;
    if (need(group, 1) > budget) return -1;
    const long long grid = ctas < (long long)nsm * occ ? ctas : (long long)nsm * occ;
    for (int t0 = 0; t0 < ntok; t0 += group) {
        const int nt = ntok - t0 < group ? ntok - t0 : group;
        LprArgs a{};
        a.nseg = nseg;
        a.xq = reinterpret_cast<const uint8_t *>(xq) + (size_t)t0 * act_row_bytes;
        a.act_row_bytes = act_row_bytes;
        a.ntok = nt;
        a.cols = cols;
        a.family = fam;
        a.act_stride = act_stride;
        a.chunk_cols = chunk_cols;
        a.nchunk = nchunk;
        a.rs = rs;
        a.kw = kw;
        a.tst = tst;
        a.act_off = LPR_MAX_CW * LPR_MAX_NS * 8;
        a.x_off = (int)(a.act_off + (((size_t)nt * act_stride + 127) & ~size_t(127)));
        a.t_off = (int)(a.x_off + xbytes(nt));
        a.p_off = (int)(a.t_off + ((tbytes(nt) + 127) & ~size_t(127)));
        a.ring_off = (int)base_of(nt);
        if (pair) {
            a.pair = 1;
            a.hq = pair->hq ? pair->hq + (size_t)t0 * pair->hq_ld : nullptr;
            a.hq_ld = pair->hq_ld;
            a.hf = pair->hf ? pair->hf + (size_t)t0 * pair->hf_ld : nullptr;
            a.hf_ld = pair->hf_ld;
        }
        if (pro) {
            a.prologue = pro->kind;
            a.px = pro->x + (size_t)t0 * pro->ld;
            a.pu = pro->u ? pro->u + (size_t)t0 * pro->ld : nullptr;
            a.pw = pro->w;
            a.px_ld = pro->ld;
            a.eps = pro->eps;
        }
        long long tiles = 0;
        // every matrix IQ4_NL (Q8_0 plane) or every one IQ4_XS (Q8_K plane)
        a.il = 1;
        for (int i = 0; i < nseg; i++)
            if (segs[i].ttype != segs[0].ttype || (segs[i].ttype != TT_IQ4_NL && segs[i].ttype != TT_IQ4_XS)) a.il = 0;
        for (int i = 0; i < nseg; i++) {
            const Geom g = geom_of(segs[i].ttype);
            LprSeg &s = a.seg[i];
            s.w = reinterpret_cast<const uint8_t *>(segs[i].w);
            s.rows = segs[i].rows;
            s.ttype = segs[i].ttype;
            s.row_bytes = cols / g.elems * g.bytes;
            s.chunk_bytes = chunk_cols / g.elems * g.bytes;
            s.out = segs[i].out ? segs[i].out + (size_t)t0 * segs[i].out_ld : nullptr;
            s.out_ld = segs[i].out_ld;
            s.mode = segs[i].mode;
            s.tile_begin = tiles;
            tiles += (s.rows + 31) / 32;
            if (!lpr_encode(&a.tmap[i], s.w, s.row_bytes, s.rows, s.chunk_bytes)) return t0 == 0 ? -1 : 1;
        }
        a.total_tiles = tiles;
        const size_t base = base_of(nt);
        long long ns = base < budget ? (long long)((budget - base) / ((size_t)cw * 32 * rs)) : 0;
        // no more stages than the busiest warp consumes
        const long long per_warp = ((tiles + grid * rw - 1) / (grid * rw)) * ((nchunk + kw - 1) / kw);
        if (ns > per_warp) ns = per_warp;
        if (ns > LPR_MAX_NS) ns = LPR_MAX_NS;
        if (ns < 1) ns = 1;
        a.ns = (int)ns;
        const size_t smem = base + (size_t)cw * ns * 32 * rs;
        if (smem > LPR_SMEM_MAX) return (int)cudaErrorInvalidValue;
        int rc;
        const dim3 gd((unsigned)grid), bd((unsigned)(cw * 32));
        if (nt == 1)
            rc = launch_k(k_gemv_lpr<1>, gd, bd, smem, st, a);
        else if (nt == 2)
            rc = launch_k(k_gemv_lpr<2>, gd, bd, smem, st, a);
        else if (nt <= 4)
            rc = launch_k(k_gemv_lpr<4>, gd, bd, smem, st, a);
        else
            rc = launch_k(k_gemv_lpr<8>, gd, bd, smem, st, a);
        if (rc) return rc;
    }
    return 0;
}

// y = W x for up to GV_MAX_SEG matrices sharing one activation: the tensor-
// core MMQ for >= 16 tokens of Q8_0 / IQ4_NL, the lane-per-row kernel where
// the matrices allow it, else the block-splitting kernel.  Validation
// (types, families, alignment) is the latter's.
inline int mmq_launch(const GemvSegDesc *segs, int nseg, const void *xq, int cols, int ntok, cudaStream_t st,
                      long long xq_ld, float *terms, size_t terms_bytes);

// terms / terms_bytes: optional scratch that lets the K-quant MMQ split K
// over CTAs when one matrix has too few row tiles to fill the GPU
inline int gemv_launch(const GemvSegDesc *segs, int nseg, const void *xq, int cols, int ntok, cudaStream_t st,
                       long long xq_ld = 0, float *terms = nullptr, size_t terms_bytes = 0) {
    int rc = mmq_launch(segs, nseg, xq, cols, ntok, st, xq_ld, terms, terms_bytes);
    if (rc != -1) return rc;
    rc = gemv_lpr_launch(segs, nseg, xq, cols, ntok, st, xq_ld);
    if (rc != -1) return rc;
    return gemv_launch_split(segs, nseg, xq, cols, ntok, st, xq_ld);
}

}  // namespace q35
