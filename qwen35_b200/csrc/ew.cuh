// ew.cuh -- elementwise, normalisation, conv, gamma, RoPE and argmax kernels.
//
// Per-element arithmetic follows src/elementwise.zig operation for operation
// (silu = x/(1+exp(-x)), rmsnorm = x*scale*w, conv = ((p0+p1)+p2)+p3, ...).
// exp / log1p / pow / sin / cos are evaluated in double and rounded once, so
// they agree with the host C library's f32 functions except in rare
// double-rounding cases.  Row reductions (sum of squares, softmax sum) use a
// fixed tree, not the CPU's serial order: those outputs differ from the CPU
// by a few ulp, as the reference's own device kernels do.
#pragma once
#include "common.cuh"

namespace q35 {

#define Q35_GRID_STRIDE(i, n) \
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (n); i += (long long)gridDim.x * blockDim.x)

inline unsigned ew_grid(long long n, int threads = 256) {
    long long g = (n + threads - 1) / threads;
    if (g > 148 * 16) g = 148 * 16;
    return (unsigned)(g < 1 ? 1 : g);
}

__global__ void k_scale_vec(float *x, float s, long long n) {
    Q35_GRID_STRIDE(i, n) x[i] = __fmul_rn(x[i], s);
}
__global__ void k_scale_vec_strided(float *x, int offset, float s, int n, int tokens, int stride) {
    Q35_GRID_STRIDE(i, (long long)n * tokens) {
        const long long t = i / n, j = i - t * n;
        float *p = x + offset + t * stride + j;
        *p = __fmul_rn(*p, s);
    }
}
__global__ void k_add_resid(float *d, const float *s, long long n) {
    Q35_GRID_STRIDE(i, n) d[i] = __fadd_rn(d[i], s[i]);
}
__global__ void k_copy(float *d, const float *s, long long n) {
    Q35_GRID_STRIDE(i, n) d[i] = s[i];
}
__global__ void k_zero(float *d, long long n) {
    Q35_GRID_STRIDE(i, n) d[i] = 0.0f;
}
__global__ void k_set_int1(int *d, int v) { *d = v; }
__global__ void k_deinterleave_qg(float *q, float *g, const float *src, int heads, int hd, int tokens) {
    const long long per = (long long)heads * hd;
    Q35_GRID_STRIDE(i, per * tokens) {
        const long long t = i / per, r = i - t * per, h = r / hd, j = r - h * hd;
        const float *s = src + t * 2 * per + h * 2 * hd;
        q[i] = s[j];
        g[i] = s[hd + j];
    }
}
__global__ void k_silu(float *x, long long n) {
    Q35_GRID_STRIDE(i, n) x[i] = silu_f(x[i]);
}
__global__ void k_mul_silu(float *o, const float *g, long long n) {
    Q35_GRID_STRIDE(i, n) o[i] = __fmul_rn(o[i], silu_f(g[i]));
}
__global__ void k_mul_sigmoid(float *o, const float *g, long long n) {
    Q35_GRID_STRIDE(i, n) o[i] = __fmul_rn(o[i], sigmoid_f(g[i]));
}
__global__ void k_swiglu(float *g, const float *u, long long n) {
    Q35_GRID_STRIDE(i, n) g[i] = __fmul_rn(silu_f(g[i]), u[i]);
}

// ---- row norms: one block per row ----------------------------------------
// rmsnorm: scale = 1/sqrt(ss/n + eps); out = x*scale*w  (elementwise.zig:43-57)
template <int NT>
__global__ void __launch_bounds__(NT) k_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    const float *xr = x + (long long)blockIdx.x * n;
    float *orow = out + (long long)blockIdx.x * n;
    extern __shared__ __align__(16) float xs[];  // n floats
    for (int i = threadIdx.x; i < n; i += NT) xs[i] = xr[i];
    __syncthreads();
    const float ss = cta_spec_sumsq(xs, n);  // the serial order's result, segments in parallel
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += NT) orow[i] = __fmul_rn(__fmul_rn(xs[i], scale), w[i]);
}

// l2norm: inv = 1/sqrt(ss + eps); x *= inv  (elementwise.zig:104-110)
// Row r of token t lives at x + offset + t*row_stride + r*n.
template <int NT>
__global__ void __launch_bounds__(NT) k_l2norm(float *x, int offset, int rows, int n, float eps, int row_stride,
                                               float post_scale, int apply_scale) {
    const int r = blockIdx.x % rows, t = blockIdx.x / rows;
    float *xr = x + offset + (long long)t * row_stride + (long long)r * n;
    extern __shared__ __align__(16) float xs[];  // n floats
    const float ss = cta_serial_sumsq(xr, n, xs);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, eps)));
    for (int i = threadIdx.x; i < n; i += NT) {
        float v = __fmul_rn(xs[i], inv);
        if (apply_scale) v = __fmul_rn(v, post_scale);
        xr[i] = v;
    }
}

// softmax over one vector (elementwise.zig:93-102)
__global__ void __launch_bounds__(1024) k_softmax(float *x, int n) {
    __shared__ float red[32];
    float m = -3.40282347e38f;
    for (int i = threadIdx.x; i < n; i += 1024) m = fmaxf(m, x[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < 32; i++) m = fmaxf(m, red[i]);
    __syncthreads();
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += 1024) {
        const float e = exp_f(__fsub_rn(x[i], m));
        x[i] = e;
        s = __fadd_rn(s, e);
    }
    s = block_sum<32>(s, red);
    for (int i = threadIdx.x; i < n; i += 1024) x[i] = __fdiv_rn(x[i], s);
}

// ---- causal conv k=4 + silu (elementwise.zig:322-342) --------------------
// One thread per channel walks `tokens` rows in order (the history is the
// cross-token dependency), writing the conv output; silu follows in place.
__global__ void k_conv_rows(float *conv, float *y, const float *w, int n, int tokens, int y_stride) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float h0 = conv[i * 3], h1 = conv[i * 3 + 1], h2 = conv[i * 3 + 2];
    const float w0 = w[i * 4], w1 = w[i * 4 + 1], w2 = w[i * 4 + 2], w3 = w[i * 4 + 3];
    for (int t = 0; t < tokens; t++) {
        float *yp = y + (long long)t * y_stride + i;
        const float cur = *yp;
        const float s = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(h0, w0), __fmul_rn(h1, w1)), __fmul_rn(h2, w2)),
                                  __fmul_rn(cur, w3));
        *yp = silu_f(s);
        h0 = h1;
        h1 = h2;
        h2 = cur;
    }
    conv[i * 3] = h0;
    conv[i * 3 + 1] = h1;
    conv[i * 3 + 2] = h2;
}

// ---- beta = sigmoid(b) in place; gamma = exp(ssm_a*softplus(a+dt)) -------
// (elementwise.zig:378-384)
__global__ void k_gdn_gamma(const float *a, float *b, const float *ssm_a, const float *dt, float *gamma, int nv,
                            int tokens, int a_stride, int b_stride, int g_stride) {
    Q35_GRID_STRIDE(i, (long long)nv * tokens) {
        const int t = (int)(i / nv), h = (int)(i - (long long)t * nv);
        float *bp = b + (long long)t * b_stride + h;
        *bp = sigmoid_f(*bp);
        const float g = __fmul_rn(ssm_a[h], softplus_f(__fadd_rn(a[(long long)t * a_stride + h], dt[h])));
        gamma[(long long)t * g_stride + h] = exp_f(g);
    }
}

// ---- RoPE on dims 0..63 of each head, pairs (j, j+32) --------------------
// theta = (f32)pos * base^(-(2j)/64) (elementwise.zig:306-318)
Q35_DEV void rope_cs(int pos, float base, int j, float &c, float &s) {
    const float ex = __fdiv_rn(-(float)(2 * j), 64.0f);
    const float p = (float)pow((double)base, (double)ex);
    const float th = __fmul_rn((float)pos, p);
    c = (float)cos((double)th);
    s = (float)sin((double)th);
}
// The rotation of pair j at `pos` from the engine's table when there is one
// (values computed on the host with the C library's f32 powf / cosf / sinf,
// the functions the reference's CPU engine calls, so they are the CPU's
// bits), else evaluated here in double precision (within an ulp of them)
Q35_DEV void rope_lookup(const float2 *tab, int pos, float base, int j, float &c, float &s) {
    if (tab) {
        const float2 v = tab[(long long)pos * 32 + j];
        c = v.x;
        s = v.y;
    } else {
        rope_cs(pos, base, j, c, s);
    }
}
Q35_DEV void rope_apply(float *hp, int j, float c, float s) {
    const float a = hp[j], b = hp[j + 32];
    hp[j] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    hp[j + 32] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}
// rows x heads heads; row r at pos0 + r (pos0 from `dyn` when non-null)
__global__ void k_rope64(float *x, int rows, int heads, int hd, int pos0, float base, const int *dyn) {
    const int j = threadIdx.x & 31;
    const long long rh = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (rh >= (long long)rows * heads) return;
    int p0 = pos0;
    float bs = base;
    if (dyn) {
        p0 = dyn[0];
        bs = __int_as_float(dyn[1]);
    }
    const int r = (int)(rh / heads);
    float c, s;
    rope_cs(p0 + r, bs, j, c, s);
    rope_apply(x + rh * hd, j, c, s);
}
__global__ void k_rope_setenv(int *d, int pos, float base) {
    d[0] = pos;
    d[1] = __float_as_int(base);
}

// ---- argmax: first index of the strict maximum (elementwise.zig:395-405) -
// one block per row of `n` values
__global__ void __launch_bounds__(1024) k_argmax(const float *x, long long row_stride, int n, int *out) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *xr = x + (long long)blockIdx.x * row_stride;
    float bv = -INFINITY;
    int bi = n;
    for (int i = threadIdx.x; i < n; i += 1024) {
        const float v = xr[i];
        if (v > bv) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 32; w++)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        out[blockIdx.x] = bi >= n ? 0 : bi;
    }
}

// The same first-index-of-max over AM_SPLIT CTAs per row: each CTA takes a
// contiguous slice (float4 loads), writes its (max, index) partial, and the
// CTA that arrives last on the row's counter combines the partials with the
// same rule (larger value, then lower index) and resets the counter for the
// next use.  Partials and counters are engine-owned device memory; counters
// start at zero.
constexpr int AM_SPLIT = 32;
__global__ void __launch_bounds__(256) k_argmax_split(const float *x, long long row_stride, int n, int *out,
                                                      float *pv, int *pi, unsigned *cnt) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[8];
    __shared__ int si[8];
    __shared__ int s_last;
    const int row = blockIdx.y, part = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (long long)row * row_stride;
    const int per = ((n + AM_SPLIT - 1) / AM_SPLIT + 3) & ~3;
    const int i0 = min(n, part * per), i1 = min(n, i0 + per);
    float bv = -INFINITY;
    int bi = n;
    const bool vec = (reinterpret_cast<uintptr_t>(xr) & 15u) == 0;
    for (int i = i0 + 4 * tid; i < i1; i += 4 * 256) {
        if (vec && i + 4 <= i1) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + i);
            if (v.x > bv) { bv = v.x; bi = i; }
            if (v.y > bv) { bv = v.y; bi = i + 1; }
            if (v.z > bv) { bv = v.z; bi = i + 2; }
            if (v.w > bv) { bv = v.w; bi = i + 3; }
        } else {
            for (int k = i; k < min(i + 4, i1); k++)
                if (xr[k] > bv) { bv = xr[k]; bi = k; }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((tid & 31) == 0) { sv[tid >> 5] = bv; si[tid >> 5] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < 8; w++)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        pv[row * AM_SPLIT + part] = bv;
        pi[row * AM_SPLIT + part] = bi;
        __threadfence();
        s_last = atomicAdd(&cnt[row], 1u) == AM_SPLIT - 1;
    }
    __syncthreads();
    if (s_last && tid < 32) {
        __threadfence();
        float v = __ldcg(&pv[row * AM_SPLIT + tid]);
        int ix = __ldcg(&pi[row * AM_SPLIT + tid]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
            if (ov > v || (ov == v && oi < ix)) { v = ov; ix = oi; }
        }
        if (tid == 0) {
            out[row] = ix >= n ? 0 : ix;
            cnt[row] = 0u;
        }
    }
}

// Unquantized weights (f32, f16, bf16) x f32 activation, in the order of the
// reference's CUDA kernels (mmvq.cu:339-367, dotq.cuh:202-218): one f32 chain
// per (row, token), acc = fmaf(w[c], x[c], acc) for c = 0, 1, ..., cols - 1,
// the weights widened exactly (bf16: bits << 16; f16: the half's value).  A
// warp owns 32 rows: each 32-column chunk arrives as 32 coalesced row reads
// (lane = column) while the previous chunk, transposed through shared
// memory, feeds lane r's chain for row r; the activation chunk is one
// coalesced read broadcast by shuffles.
enum { MV_F32 = 0, MV_F16 = 1, MV_BF16 = 2 };
template <int KIND>
__global__ void __launch_bounds__(128) k_matvec_seq(const void *__restrict__ w, const float *__restrict__ x,
                                                    float *__restrict__ out, int rows, int cols) {
    __shared__ float tw[4][32][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = blockIdx.y;
    const long long r0 = ((long long)blockIdx.x * 4 + warp) * 32;
    if (r0 >= rows) return;
    const int nr = (int)min(32LL, (long long)rows - r0);
    const float *xr = x + (long long)t * cols;
    float(*T)[33] = tw[warp];
    auto ld = [&](int rr, int c) -> float {
        if (rr >= nr || c >= cols) return 0.0f;
        const long long off = (r0 + rr) * cols + c;
        if (KIND == MV_F32) return static_cast<const float *>(w)[off];
        const uint16_t h = static_cast<const uint16_t *>(w)[off];
        return KIND == MV_BF16 ? __uint_as_float((uint32_t)h << 16) : __half2float(__ushort_as_half(h));
    };
    float cur[32], nxt[32];
#pragma unroll
    for (int rr = 0; rr < 32; rr++) cur[rr] = ld(rr, lane);
    float acc = 0.0f;
    for (int c0 = 0; c0 < cols; c0 += 32) {
        const bool more = c0 + 32 < cols;
#pragma unroll
        for (int rr = 0; rr < 32; rr++) nxt[rr] = more ? ld(rr, c0 + 32 + lane) : 0.0f;
#pragma unroll
        for (int rr = 0; rr < 32; rr++) T[rr][lane] = cur[rr];
        const float xv = c0 + lane < cols ? xr[c0 + lane] : 0.0f;
        __syncwarp();
        const int nc = min(32, cols - c0);
        for (int c = 0; c < nc; c++) acc = __fmaf_rn(T[lane][c], __shfl_sync(0xffffffffu, xv, c), acc);
        __syncwarp();
#pragma unroll
        for (int rr = 0; rr < 32; rr++) cur[rr] = nxt[rr];
    }
    if (lane < nr) out[(long long)t * rows + r0 + lane] = acc;
}

}  // namespace q35
