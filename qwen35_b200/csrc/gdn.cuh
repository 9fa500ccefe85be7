// gdn.cuh -- gated delta-net state update, sm_100a.
//
// One CTA per (value head, sequence); thread j owns state column j and keeps
// all kd = 128 entries of it in registers for the whole call, so the 64 KB
// per-head f32 state is read from HBM once and written once per call no
// matter how many tokens are stepped (a prefill chunk steps them in order
// inside the kernel).
//
// Per token, per column j (src/elementwise.zig:221-278, gdnFused):
//   pass 1: acc = sum_i S[i][j]*k[i] (i ascending); km = acc*gamma
//           delta = (v[j] - km)*beta
//   pass 2: S[i][j] = S[i][j]*gamma + k[i]*delta; out[j] += S[i][j]*q[i]
// Every product and sum is one IEEE operation in the CPU's order, so the
// state, km, delta and out are bit-exact with the CPU oracle.
// Value head h reads k/q head h % nk (src/backend_cpu.zig:1006).
#pragma once
#include "common.cuh"

namespace q35 {

constexpr int GDN_KD = 128;

struct GdnArgs {
    float *state;
    long long state_head;   // floats between heads' [kd, vd] blocks
    long long state_slot;   // floats between sequences' states
    const int *slots;       // per-sequence slot index (nullptr: slot = sequence index)
    const float *k, *v, *q;
    long long k_tok, v_tok, q_tok;   // floats between tokens
    long long k_head, v_head, q_head;  // floats between heads
    float *km, *delta, *out;         // km/delta may be null
    long long km_tok, delta_tok, out_tok;
    long long km_head, delta_head, out_head;
    const float *gamma, *beta;       // null: use the immediates
    long long g_tok, b_tok;
    float gamma_imm, beta_imm;
    int heads, nk, rows;             // rows: tokens stepped in order per sequence
    const int *active;               // optional per-sequence flag: 0 = skip
};

__global__ void __launch_bounds__(GDN_KD) k_gdn_step(const __grid_constant__ GdnArgs a) {
    __shared__ float sk[GDN_KD], sq[GDN_KD];
    const int h = blockIdx.x, seq = blockIdx.y, j = threadIdx.x;
    if (a.active && !a.active[seq]) return;
    const long long slot = a.slots ? a.slots[seq] : seq;
    float *S = a.state + slot * a.state_slot + h * a.state_head;
    const int kh = h % a.nk;
    float col[GDN_KD];
#pragma unroll
    for (int i = 0; i < GDN_KD; i++) col[i] = S[(long long)i * GDN_KD + j];

    for (int r = 0; r < a.rows; r++) {
        const long long tok = (long long)seq * a.rows + r;
        __syncthreads();
        sk[j] = a.k[tok * a.k_tok + kh * a.k_head + j];
        sq[j] = a.q[tok * a.q_tok + kh * a.q_head + j];
        __syncthreads();
        const float g = a.gamma ? a.gamma[tok * a.g_tok + h] : a.gamma_imm;
        const float be = a.beta ? a.beta[tok * a.b_tok + h] : a.beta_imm;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < GDN_KD; i++) acc = __fadd_rn(acc, __fmul_rn(col[i], sk[i]));
        const float km = __fmul_rn(acc, g);
        const float vj = a.v[tok * a.v_tok + h * a.v_head + j];
        const float d = __fmul_rn(__fsub_rn(vj, km), be);
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < GDN_KD; i++) {
            const float nv = __fadd_rn(__fmul_rn(col[i], g), __fmul_rn(sk[i], d));
            col[i] = nv;
            o = __fadd_rn(o, __fmul_rn(nv, sq[i]));
        }
        a.out[tok * a.out_tok + h * a.out_head + j] = o;
        if (a.km) a.km[tok * a.km_tok + h * a.km_head + j] = km;
        if (a.delta) a.delta[tok * a.delta_tok + h * a.delta_head + j] = d;
    }
#pragma unroll
    for (int i = 0; i < GDN_KD; i++) S[(long long)i * GDN_KD + j] = col[i];
}

inline int gdn_launch(const GdnArgs &a, int nseq, cudaStream_t st) {
    if (a.heads <= 0 || nseq <= 0 || a.rows <= 0) return 0;
    if (a.nk <= 0) return (int)cudaErrorInvalidValue;
    dim3 grid((unsigned)a.heads, (unsigned)nseq);
    k_gdn_step<<<grid, GDN_KD, 0, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace q35

namespace q35 {

// ---------------------------------------------------------------------------
// Fused GDN layer core for the batched decode step: one CTA per (value head,
// sequence), 128 threads, everything between the input projections and the
// output projection of a GDN layer (src/engine.zig:1505-1667):
//   causal conv k=4 + silu on this head's q / k / v channels
//   l2norm(q) * 1/sqrt(kd), l2norm(k)            (norm sums in serial order)
//   beta = sigmoid(b), gamma = exp(ssm_a * softplus(a + dt_bias))
//   delta-rule state update (column j per thread, state in registers)
//   gated RMSNorm(out, ssm_norm) * silu(z), quantized for ssm_out
// The conv history is double-buffered by position parity: every CTA reads the
// history of position p and the owner of a channel writes position p+1's, so
// value heads that share a k head (nv > nk) never race on it.
// ---------------------------------------------------------------------------
struct GdnCoreArgs {
    const float *qkv;   // raw projections, [n][conv_dim]
    long long qkv_ld;
    const float *z;     // gate projection, [n][nv*vd]
    long long z_ld;
    const float *ab;    // [n][2 nv]: alpha (a) then beta (b)
    long long ab_ld;
    const float *conv_w;  // [conv_dim][4]
    float *hist;          // per slot: 2 x [conv_dim][3]
    long long hist_slot;
    const float *ssm_a, *dt_bias, *ssm_norm;
    float *state;
    long long state_slot;
    const int *slots, *pos;
    const int *run_end;   // null: token b is its own run; else run r = tokens [run_end[r-1], run_end[r])
    int nv, nk;
    float eps, qscale;
    int fam;              // activation family of ssm_out (32: quantize here)
    uint8_t *xq;
    long long xq_ld;
    float *gout;          // f32 gated output when fam != 32
    long long gout_ld;
};

__global__ void __launch_bounds__(GDN_KD) k_gdn_core(const __grid_constant__ GdnCoreArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ __align__(16) float sq[GDN_KD], sk[GDN_KD], so[GDN_KD];
    __shared__ float s_scal[4];
    const int h = blockIdx.x, r = blockIdx.y, j = threadIdx.x;
    const int kd = GDN_KD, kq = a.nk * kd, conv_dim = 2 * kq + a.nv * kd;
    const int kh = h % a.nk;
    // the run: consecutive positions of one sequence, stepped in order
    const int i0 = a.run_end ? (r == 0 ? 0 : a.run_end[r - 1]) : r;
    const int i1 = a.run_end ? a.run_end[r] : r + 1;
    const long long slot = a.slots[i0];
    const int p0 = a.pos[i0];
    // history: read the buffer of the run's first position's parity, write
    // the other one -- CTAs of value heads sharing a k head read the q / k
    // history at their start, so nothing may write that buffer during the
    // kernel.  A run of even length ends on its first parity: k_gdn_hist_settle
    // moves the result there afterwards.
    const float *hin = a.hist + slot * a.hist_slot + (long long)(p0 & 1) * conv_dim * 3;
    float *hout = a.hist + slot * a.hist_slot + (long long)((p0 & 1) ^ 1) * conv_dim * 3;

    // loads that do not depend on the token, issued up front so their
    // latencies overlap: the 64 KB state block (one bulk copy into shared
    // memory), conv taps and history, the norm
    float *S = a.state + slot * a.state_slot + (long long)h * kd * kd;
    extern __shared__ __align__(128) float s_state[];  // [kd][kd]
    __shared__ __align__(8) uint64_t s_bar;
    if (j == 0) {
        mbar_init(&s_bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&s_bar, (uint32_t)(kd * kd * 4));
        bulk_g2s(s_state, S, (uint32_t)(kd * kd * 4), &s_bar);
    }
    const int chq = kh * kd + j, chk = kq + kh * kd + j, chv = 2 * kq + h * kd + j;
    // conv history and taps of this thread's q / k / v channels, kept in
    // shared memory (the state column already takes the registers)
    __shared__ float s_h[3][3][GDN_KD], s_w[3][4][GDN_KD];
    const int chs[3] = {chq, chk, chv};
#pragma unroll
    for (int c = 0; c < 3; c++) {
#pragma unroll
        for (int i = 0; i < 3; i++) s_h[c][i][j] = hin[(long long)chs[c] * 3 + i];
#pragma unroll
        for (int i = 0; i < 4; i++) s_w[c][i][j] = a.conv_w[(long long)chs[c] * 4 + i];
    }
    const float nwj = a.ssm_norm[j];
    const float ssm_a = a.ssm_a[h], dtb = a.dt_bias[h];
    __shared__ int s_ok;
    if (j == 0) s_ok = mbar_wait(&s_bar, 0u, 140) ? 1 : 0;
    __syncthreads();  // thread 0 saw the copy land (or gave up); all threads learn which
    if (!s_ok) {
        // the copy did not land in time: let it finish (bounded) before the
        // shared memory is released, write nothing
        if (j == 0) mbar_wait(&s_bar, 0u, 141);
        return;
    }
    float col[GDN_KD];
#pragma unroll
    for (int i = 0; i < GDN_KD; i++) col[i] = s_state[i * GDN_KD + j];

    // causal conv k=4 + silu: y = w0*h0 + w1*h1 + w2*h2 + w3*x, left to right;
    // then the history shifts in x
    auto conv = [&](int c, float cur) {
        const float s = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(s_h[c][0][j], s_w[c][0][j]),
                                                      __fmul_rn(s_h[c][1][j], s_w[c][1][j])),
                                            __fmul_rn(s_h[c][2][j], s_w[c][2][j])),
                                  __fmul_rn(cur, s_w[c][3][j]));
        s_h[c][0][j] = s_h[c][1][j];
        s_h[c][1][j] = s_h[c][2][j];
        s_h[c][2][j] = cur;
        return silu_f(s);
    };
    for (int b = i0; b < i1; b++) {
        const float *raw = a.qkv + (long long)b * a.qkv_ld;
        const float cq = raw[chq], ck = raw[chk], cv = raw[chv];
        const float zj = a.z[(long long)b * a.z_ld + (long long)h * kd + j];
        const float *ar = a.ab + (long long)b * a.ab_ld;
        const float a_raw = ar[h], b_raw = ar[a.nv + h];
        sq[j] = conv(0, cq);
        sk[j] = conv(1, ck);
        const float vj = conv(2, cv);
        __syncthreads();
        if (j == 0) s_scal[0] = serial_sumsq(sq, kd);
        if (j == 32) s_scal[1] = serial_sumsq(sk, kd);
        if (j == 64) {
            s_scal[2] = sigmoid_f(b_raw);
            s_scal[3] = exp_f(__fmul_rn(ssm_a, softplus_f(__fadd_rn(a_raw, dtb))));
        }
        __syncthreads();
        const float iq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s_scal[0], 1e-6f)));
        const float ik = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s_scal[1], 1e-6f)));
        const float qj = __fmul_rn(__fmul_rn(sq[j], iq), a.qscale);
        const float kj = __fmul_rn(sk[j], ik);
        const float be = s_scal[2], g = s_scal[3];
        __syncthreads();
        sq[j] = qj;
        sk[j] = kj;
        __syncthreads();
        // pass 1: acc = sum_i S[i][j] k[i] (i ascending), products ahead of the adds
        float acc = 0.0f;
        const float4 *sk4 = reinterpret_cast<const float4 *>(sk), *sq4 = reinterpret_cast<const float4 *>(sq);
#pragma unroll
        for (int i4 = 0; i4 < GDN_KD / 4; i4++) {
            const float4 kv = sk4[i4];
            const float p0 = __fmul_rn(col[4 * i4], kv.x), p1 = __fmul_rn(col[4 * i4 + 1], kv.y);
            const float p2 = __fmul_rn(col[4 * i4 + 2], kv.z), p3 = __fmul_rn(col[4 * i4 + 3], kv.w);
            acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, p0), p1), p2), p3);
        }
        const float km = __fmul_rn(acc, g);
        const float d = __fmul_rn(__fsub_rn(vj, km), be);
        // pass 2: S[i][j] = S[i][j]*g + k[i]*d; out += S[i][j]*q[i]
        float o = 0.0f;
#pragma unroll
        for (int i4 = 0; i4 < GDN_KD / 4; i4++) {
            const float4 kv = sk4[i4], qv = sq4[i4];
            const float kk[4] = {kv.x, kv.y, kv.z, kv.w}, qq[4] = {qv.x, qv.y, qv.z, qv.w};
            float pr[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = 4 * i4 + u;
                const float nvv = __fadd_rn(__fmul_rn(col[i], g), __fmul_rn(kk[u], d));
                col[i] = nvv;
                pr[u] = __fmul_rn(nvv, qq[u]);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) o = __fadd_rn(o, pr[u]);
        }
        so[j] = o;
        __syncthreads();
        if (j == 0) s_scal[0] = serial_sumsq(so, kd);
        __syncthreads();
        const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s_scal[0], (float)kd), a.eps)));
        float y = __fmul_rn(__fmul_rn(o, sc), nwj);
        y = __fmul_rn(y, silu_f(zj));
        if (a.fam == 32) {
            const int w = j >> 5;
            quant_q8_0_warp(y, a.xq + (long long)b * a.xq_ld + (long long)(h * (kd / 32) + w) * 34, j & 31);
        } else {
            a.gout[(long long)b * a.gout_ld + (long long)h * kd + j] = y;
        }
        __syncthreads();  // s_scal / sq / sk / so reused by the next token
    }
#pragma unroll
    for (int i = 0; i < GDN_KD; i++) S[(long long)i * GDN_KD + j] = col[i];
    // the history after the run, for the position after it; the owner of a
    // k head's q / k channels writes those
    auto store = [&](int c) {
        float *ho = hout + (long long)chs[c] * 3;
        ho[0] = s_h[c][0][j];
        ho[1] = s_h[c][1][j];
        ho[2] = s_h[c][2][j];
    };
    if (h < a.nk) {
        store(0);
        store(1);
    }
    store(2);
}

// k_gdn_core stages the 64 KB state block in dynamic shared memory
inline int gdn_prepare() {
    static int done = 0;
    if (done) return 0;
    const cudaError_t e =
        cudaFuncSetAttribute(k_gdn_core, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_KD * GDN_KD * 4);
    if (e != cudaSuccess) return (int)e;
    done = 1;
    return 0;
}

// after k_gdn_core over runs: a run of even length wrote its final conv
// history to the buffer of the other parity; move it to the parity of the
// position after the run (its first position's), where the next step reads it
__global__ void k_gdn_hist_settle(float *hist, long long hist_slot, int conv_dim, const int *slots, const int *pos,
                                  const int *run_end) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.y;
    const int i0 = r == 0 ? 0 : run_end[r - 1], i1 = run_end[r];
    if ((i1 - i0) & 1) return;
    const int p0 = pos[i0];
    float *base = hist + (long long)slots[i0] * hist_slot;
    const float *src = base + (long long)((p0 & 1) ^ 1) * conv_dim * 3;
    float *dst = base + (long long)(p0 & 1) * conv_dim * 3;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < conv_dim * 3; i += gridDim.x * blockDim.x) dst[i] = src[i];
}

}  // namespace q35
