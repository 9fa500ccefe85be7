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

// asynchronous global -> shared copies (LDGSTS): 16 bytes through L2 only,
// 4 bytes through L1; a thread's own copies are visible to it after the wait
Q35_DEV void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
Q35_DEV void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
Q35_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
Q35_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

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
    int gamma_log;                   // WY kernels: gamma holds floored log decays (not decays)
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
    int wy_min;           // > 0: runs of at least wy_min tokens take the WY form (k_gdn_core skips them)
};

__global__ void __launch_bounds__(GDN_KD) k_gdn_core(const __grid_constant__ GdnCoreArgs a) {
    pdl_trigger();
    // Before the dependency wait: everything this kernel reads that the
    // step's earlier kernels do not write -- the batch descriptor (uploaded
    // before the step), the state block and conv history (written by this
    // layer's previous step, which finished before the step's first,
    // ordinarily launched kernel began), conv taps and norm weights.  The
    // projections (qkv, z, alpha / beta) are read after the wait.
    __shared__ __align__(16) float sq[GDN_KD], sk[GDN_KD], so[GDN_KD];
    __shared__ float s_scal[4];
    const int h = blockIdx.x, r = blockIdx.y, j = threadIdx.x;
    const int kd = GDN_KD, kq = a.nk * kd, conv_dim = 2 * kq + a.nv * kd;
    const int kh = h % a.nk;
    // the run: consecutive positions of one sequence, stepped in order
    const int i0 = a.run_end ? (r == 0 ? 0 : a.run_end[r - 1]) : r;
    const int i1 = a.run_end ? a.run_end[r] : r + 1;
    if (a.wy_min > 0 && i1 - i0 >= a.wy_min) return;  // a WY run
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
    pdl_wait();
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
    // the next token's inputs are copied (cp.async, no registers held) while
    // this one is stepped: a run's tokens would otherwise each wait a full L2
    // round trip first.  Thread j copies and reads only its own slots.
    __shared__ float s_in[2][4][GDN_KD], s_gab[2][2];
    auto fetch = [&](int b) {
        const int pb = b & 1;
        const float *raw = a.qkv + (long long)b * a.qkv_ld;
        cp_async4(&s_in[pb][0][j], raw + chq);
        cp_async4(&s_in[pb][1][j], raw + chk);
        cp_async4(&s_in[pb][2][j], raw + chv);
        cp_async4(&s_in[pb][3][j], a.z + (long long)b * a.z_ld + (long long)h * kd + j);
        if (j == 64) {
            const float *ar = a.ab + (long long)b * a.ab_ld;
            cp_async4(&s_gab[pb][0], ar + h);
            cp_async4(&s_gab[pb][1], ar + a.nv + h);
        }
        cp_async_commit();
    };
    fetch(i0);
    for (int b = i0; b < i1; b++) {
        if (b + 1 < i1) {
            fetch(b + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        const int pb = b & 1;
        const float cq = s_in[pb][0][j], ck = s_in[pb][1][j], cv = s_in[pb][2][j], zj = s_in[pb][3][j];
        const float a_raw = j == 64 ? s_gab[pb][0] : 0.0f, b_raw = j == 64 ? s_gab[pb][1] : 0.0f;
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
    // the state block goes back the way it came: into shared memory (row i,
    // column j: conflict-free), then one bulk copy to global memory
#pragma unroll
    for (int i = 0; i < GDN_KD; i++) s_state[i * GDN_KD + j] = col[i];
    fence_proxy_async();
    __syncthreads();
    if (j == 0) bulk_s2g(S, s_state, (uint32_t)(kd * kd * 4));
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
    if (j == 0) bulk_s2g_wait_read();  // shared memory stays live until the copy has read it
}

// ---------------------------------------------------------------------------
// Chunked (WY) form of the same recurrence (the reference's q35_gdn_step_wy,
// gdn.cu:452-631): per chunk of WY_C tokens, with cumulative log decay
// L_t = sum_{s<=t} log g_s and decay(t, s) = exp(L_t - L_s),
//   km_t    = exp(L_t) S0^T k_t + sum_{s<t} decay(t,s) (k_t.k_s) delta_s
//   delta_t = beta_t (v_t - km_t)
//   o_t     = exp(L_t) S0^T q_t + sum_{s<=t} decay(t,s) (q_t.k_s) delta_s
//   S       = exp(L_C) S0 + sum_s decay(C,s) k_s delta_s^T
// which unrolls  S_t = g_t S_{t-1} + k_t delta_t^T,
// km_t = g_t S_{t-1}^T k_t, o_t = S_t^T q_t  exactly; the sums are
// re-associated (f32, fused multiply-adds), so this form agrees with the
// per-token kernels to f32 rounding, not bitwise.
// k_gdn_wy_rows: CTA per value head, thread j owns state column j (128 registers);
// the chunk's q / k / v rows sit in shared memory with a 132-float pitch
// (an odd multiple of 16 bytes: float4 row reads by 8 lanes of different
// rows hit 8 distinct bank quads).
// ---------------------------------------------------------------------------
constexpr int WY_C = 32;
constexpr int WY_LD = GDN_KD + 4;
// chunk buffers of wy_bufs (Qs..Ws, Am, Mm, the per-token vectors) and log g
constexpr size_t WY_ROWS_SMEM =
    (size_t)5 * WY_C * WY_LD * 4 + (size_t)2 * WY_C * (WY_C + 1) * 4 + (size_t)8 * WY_C * 4;
constexpr float WY_LOG_MIN = -88.0f;  // log decay floor: exp() of it is ~0, sums stay finite

struct WyBufs {
    float *Qs, *Ks, *Vs;  // [C][WY_LD] chunk rows (q scaled and normalised, k normalised)
    float *Us, *Ws;       // [C][WY_LD] S0^T k_t, S0^T q_t; Us then holds o_t
    float *Am, *Mm;       // [C][C+1] decay(t,s) k_t.k_s (s < t), decay(t,s) q_t.k_s (s <= t)
    float *Lc;            // [C] cumulative log decay
    float *eL, *eE;       // [C] exp(L_t), exp(L_end - L_t)
    float *bet;           // [C]
};

__device__ __forceinline__ WyBufs wy_bufs(float *base) {
    WyBufs m;
    m.Qs = base;
    m.Ks = m.Qs + WY_C * WY_LD;
    m.Vs = m.Ks + WY_C * WY_LD;
    m.Us = m.Vs + WY_C * WY_LD;
    m.Ws = m.Us + WY_C * WY_LD;
    m.Am = m.Ws + WY_C * WY_LD;
    m.Mm = m.Am + WY_C * (WY_C + 1);
    m.Lc = m.Mm + WY_C * (WY_C + 1);
    m.eL = m.Lc + WY_C;
    m.eE = m.eL + WY_C;
    m.bet = m.eE + WY_C;
    return m;
}

// cumulative log decay of the chunk from per-token log decays lg[0..nc)
// (thread 127; the caller synchronises before and after)
__device__ __forceinline__ void wy_cumulate(const WyBufs &m, const float *lg, int nc, int j) {
    if (j == GDN_KD - 1) {
        float L = 0.0f;
        for (int t = 0; t < nc; t++) {
            L = __fadd_rn(L, lg[t]);
            m.Lc[t] = L;
        }
    }
}

// One chunk for state column j (col).  On entry Qs / Ks / Vs, Lc and bet
// hold the chunk's nc tokens and every thread has passed a barrier since
// they were written.  On exit Us[t][j] = o_t, col is the state after the
// chunk, and sink(t, km_t, delta_t) has seen every token; the caller
// synchronises before the buffers are reused.
template <class Sink>
__device__ __forceinline__ void wy_chunk(float (&col)[GDN_KD], const WyBufs &m, int nc, int j, Sink sink) {
    const int warp = j >> 5, lane = j & 31;
    if (j < nc) {
        m.eL[j] = expf(m.Lc[j]);
        m.eE[j] = expf(m.Lc[nc - 1] - m.Lc[j]);
    }
    // U = S0^T k_t, W = S0^T q_t (column j); four partial sums per dot
    // (i mod 4) keep eight independent FMA chains in flight
    for (int t = 0; t < nc; t++) {
        const float4 *k4 = reinterpret_cast<const float4 *>(m.Ks + t * WY_LD);
        const float4 *q4 = reinterpret_cast<const float4 *>(m.Qs + t * WY_LD);
        float u0 = 0.0f, u1 = 0.0f, u2 = 0.0f, u3 = 0.0f, w0 = 0.0f, w1 = 0.0f, w2 = 0.0f, w3 = 0.0f;
#pragma unroll
        for (int i4 = 0; i4 < GDN_KD / 4; i4++) {
            const float4 kv = k4[i4], qv = q4[i4];
            u0 = __fmaf_rn(col[4 * i4], kv.x, u0);
            u1 = __fmaf_rn(col[4 * i4 + 1], kv.y, u1);
            u2 = __fmaf_rn(col[4 * i4 + 2], kv.z, u2);
            u3 = __fmaf_rn(col[4 * i4 + 3], kv.w, u3);
            w0 = __fmaf_rn(col[4 * i4], qv.x, w0);
            w1 = __fmaf_rn(col[4 * i4 + 1], qv.y, w1);
            w2 = __fmaf_rn(col[4 * i4 + 2], qv.z, w2);
            w3 = __fmaf_rn(col[4 * i4 + 3], qv.w, w3);
        }
        m.Us[t * WY_LD + j] = (u0 + u1) + (u2 + u3);
        m.Ws[t * WY_LD + j] = (w0 + w1) + (w2 + w3);
    }
    // A and M: lane = s, warp w takes t = w, w + 4, ...
    {
        const int s = lane;
        const float4 *ks4 = reinterpret_cast<const float4 *>(m.Ks + s * WY_LD);
        for (int t = warp; t < nc; t += 4) {
            const float4 *kt4 = reinterpret_cast<const float4 *>(m.Ks + t * WY_LD);
            const float4 *qt4 = reinterpret_cast<const float4 *>(m.Qs + t * WY_LD);
            float kk = 0.0f, qk = 0.0f;
            if (s <= t) {
                float k0 = 0.0f, k1 = 0.0f, k2 = 0.0f, k3 = 0.0f, q0 = 0.0f, q1 = 0.0f, q2 = 0.0f, q3 = 0.0f;
#pragma unroll 8
                for (int i4 = 0; i4 < GDN_KD / 4; i4++) {
                    const float4 x = ks4[i4], y = kt4[i4], z = qt4[i4];
                    k0 = __fmaf_rn(y.x, x.x, k0);
                    k1 = __fmaf_rn(y.y, x.y, k1);
                    k2 = __fmaf_rn(y.z, x.z, k2);
                    k3 = __fmaf_rn(y.w, x.w, k3);
                    q0 = __fmaf_rn(z.x, x.x, q0);
                    q1 = __fmaf_rn(z.y, x.y, q1);
                    q2 = __fmaf_rn(z.z, x.z, q2);
                    q3 = __fmaf_rn(z.w, x.w, q3);
                }
                kk = (k0 + k1) + (k2 + k3);
                qk = (q0 + q1) + (q2 + q3);
            }
            const float dec = s <= t ? expf(m.Lc[t] - m.Lc[s]) : 0.0f;
            m.Am[t * (WY_C + 1) + s] = s < t ? dec * kk : 0.0f;
            m.Mm[t * (WY_C + 1) + s] = s <= t ? dec * qk : 0.0f;
        }
    }
    __syncthreads();
    // forward substitution for km / delta of column j, then the outputs
    float dl[WY_C];
#pragma unroll
    for (int t = 0; t < WY_C; t++) {
        dl[t] = 0.0f;
        if (t < nc) {
            float km = m.eL[t] * m.Us[t * WY_LD + j];
#pragma unroll
            for (int s = 0; s < t; s++) km = __fmaf_rn(m.Am[t * (WY_C + 1) + s], dl[s], km);
            dl[t] = m.bet[t] * (m.Vs[t * WY_LD + j] - km);
            sink(t, km, dl[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < WY_C; t++) {
        if (t < nc) {
            float o = m.eL[t] * m.Ws[t * WY_LD + j];
#pragma unroll
            for (int s = 0; s <= t; s++) o = __fmaf_rn(m.Mm[t * (WY_C + 1) + s], dl[s], o);
            m.Us[t * WY_LD + j] = o;  // U no longer needed: o_t
        }
    }
    // state: exp(L_end) S0 + sum_t decay(end, t) k_t delta_t^T, t ascending
    const float gend = m.eL[nc - 1];
#pragma unroll
    for (int i = 0; i < GDN_KD; i++) col[i] = gend * col[i];
#pragma unroll
    for (int t = 0; t < WY_C; t++) {
        if (t < nc) {
            const float e = m.eE[t] * dl[t];
            const float4 *k4 = reinterpret_cast<const float4 *>(m.Ks + t * WY_LD);
#pragma unroll
            for (int i4 = 0; i4 < GDN_KD / 4; i4++) {
                const float4 kv = k4[i4];
                col[4 * i4] = __fmaf_rn(kv.x, e, col[4 * i4]);
                col[4 * i4 + 1] = __fmaf_rn(kv.y, e, col[4 * i4 + 1]);
                col[4 * i4 + 2] = __fmaf_rn(kv.z, e, col[4 * i4 + 2]);
                col[4 * i4 + 3] = __fmaf_rn(kv.w, e, col[4 * i4 + 3]);
            }
        }
    }
}

struct WyNoSink {
    __device__ void operator()(int, float, float) const {}
};

// The engine's GDN layer core over prefill runs in the WY form, as three
// steps around the operator's chunked recurrence (wy_tc_launch: the tensor-
// core Gram pass and the column-split kernel, one launch pair per run):
//   k_gdn_wy_prep  CTA per (token, head): causal conv k=4 + silu, the q / k
//                  l2 norms (serial sums), the floored log decay and beta --
//                  every per-token operation of k_gdn_core in its order, run
//                  for all tokens at once (a token's conv window is its
//                  run's previous three inputs, or the slot's history)
//   recurrence     per run, on the slot's state (q35::wy_tc_launch)
//   k_gdn_wy_post  CTA per (token, head): gated RMSNorm (serial sum) x
//                  silu(z), quantized for ssm_out as k_gdn_core does
// The conv history after a run is written by the CTAs of the run's last
// token into the other parity buffer, as k_gdn_core's (k_gdn_hist_settle
// follows either).
// shortest run the engine steps in the WY form: a shorter one costs
// k_gdn_core less than the per-run launches of the chunked recurrence
constexpr int WY_MIN_RUN = 16;

// the run holding token b: the first r with run_end[r] > b
__device__ __forceinline__ int run_of(const int *run_end, int nrun, int b) {
    int lo = 0, hi = nrun - 1;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (run_end[mid] > b)
            hi = mid;
        else
            lo = mid + 1;
    }
    return lo;
}

struct WyPrepOut {
    float *q, *k;     // [n][nk * kd]: l2-normalised (q also scaled)
    float *v;         // [n][nv * kd]: conv + silu
    float *lg, *beta; // [n][nv]: floored log decay, beta
    int nrun;
};

__global__ void __launch_bounds__(GDN_KD) k_gdn_wy_prep(const __grid_constant__ GdnCoreArgs a,
                                                        const __grid_constant__ WyPrepOut o) {
    pdl_trigger();
    __shared__ float sq[GDN_KD], sk[GDN_KD];
    __shared__ float s_sc[2];
    const int b = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
    const int kd = GDN_KD, kq = a.nk * kd, vdim = a.nv * kd, conv_dim = 2 * kq + vdim;
    const int lo = run_of(a.run_end, o.nrun, b);
    const int i0 = lo == 0 ? 0 : a.run_end[lo - 1], i1 = a.run_end[lo];
    if (i1 - i0 < a.wy_min) return;  // a short run: k_gdn_core's
    const long long slot = a.slots[i0];
    const int p0 = a.pos[i0], u = b - i0;
    const float *hin = a.hist + slot * a.hist_slot + (long long)(p0 & 1) * conv_dim * 3;
    float *hout = a.hist + slot * a.hist_slot + (long long)((p0 & 1) ^ 1) * conv_dim * 3;
    const bool qk = h < a.nk;  // this CTA also owns k head h's q / k channels
    const int chq = h * kd + j, chk = kq + h * kd + j, chv = 2 * kq + h * kd + j;
    // history and taps (not written by this step's kernels) before the wait
    float hv[3][3], wv[3][4];
    const int chs[3] = {chq, chk, chv};
#pragma unroll
    for (int c = 0; c < 3; c++) {
        if (c < 2 && !qk) continue;
#pragma unroll
        for (int i = 0; i < 3; i++) hv[c][i] = hin[(long long)chs[c] * 3 + i];
#pragma unroll
        for (int i = 0; i < 4; i++) wv[c][i] = a.conv_w[(long long)chs[c] * 4 + i];
    }
    const float ssm_a = a.ssm_a[h], dtb = a.dt_bias[h];
    pdl_wait();
    // input at run offset m of channel c: the projection, or the history
    // before the run's first token
    auto input = [&](int c, int m) {
        return m >= 0 ? a.qkv[(long long)(i0 + m) * a.qkv_ld + chs[c]] : hv[c][3 + m];
    };
    // k_gdn_core's conv: w0*x[u-3] + w1*x[u-2] + w2*x[u-1] + w3*x[u], left to right
    auto conv = [&](int c) {
        const float x0 = input(c, u - 3), x1 = input(c, u - 2), x2 = input(c, u - 1), x3 = input(c, u);
        if (b == i1 - 1) {  // the history after the run
            float *ho = hout + (long long)chs[c] * 3;
            ho[0] = x1;
            ho[1] = x2;
            ho[2] = x3;
        }
        const float s = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(x0, wv[c][0]), __fmul_rn(x1, wv[c][1])),
                                            __fmul_rn(x2, wv[c][2])),
                                  __fmul_rn(x3, wv[c][3]));
        return silu_f(s);
    };
    o.v[(long long)b * vdim + h * kd + j] = conv(2);
    if (j == 64) {
        const float *ar = a.ab + (long long)b * a.ab_ld;
        o.lg[(long long)b * a.nv + h] = fmaxf(__fmul_rn(ssm_a, softplus_f(__fadd_rn(ar[h], dtb))), WY_LOG_MIN);
        o.beta[(long long)b * a.nv + h] = sigmoid_f(ar[a.nv + h]);
    }
    if (qk) {  // uniform over the CTA
        const float yq = conv(0), yk = conv(1);
        sq[j] = yq;
        sk[j] = yk;
        __syncthreads();
        if (j == 0) s_sc[0] = serial_sumsq(sq, kd);
        if (j == 32) s_sc[1] = serial_sumsq(sk, kd);
        __syncthreads();
        const float iq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s_sc[0], 1e-6f)));
        const float ik = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s_sc[1], 1e-6f)));
        o.q[(long long)b * kq + h * kd + j] = __fmul_rn(__fmul_rn(yq, iq), a.qscale);
        o.k[(long long)b * kq + h * kd + j] = __fmul_rn(yk, ik);
    }
}

// gated RMSNorm of the recurrence output y ([n][nv * kd]) x silu(z),
// quantized per token (or f32 when ssm_out takes another family)
__global__ void __launch_bounds__(GDN_KD) k_gdn_wy_post(const __grid_constant__ GdnCoreArgs a, const float *y,
                                                        int nrun) {
    pdl_trigger();
    __shared__ float so[GDN_KD];
    __shared__ float s_sc;
    const int b = blockIdx.x, h = blockIdx.y, j = threadIdx.x, warp = j >> 5, lane = j & 31;
    {
        const int r = run_of(a.run_end, nrun, b);
        if (a.run_end[r] - (r ? a.run_end[r - 1] : 0) < a.wy_min) return;  // a short run: k_gdn_core's
    }
    const int kd = GDN_KD, vdim = a.nv * kd;
    const float nwj = a.ssm_norm[j];
    pdl_wait();
    const float ov = y[(long long)b * vdim + h * kd + j];
    so[j] = ov;
    __syncthreads();
    if (j == 0) s_sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(serial_sumsq(so, kd), (float)kd), a.eps)));
    __syncthreads();
    float r = __fmul_rn(__fmul_rn(ov, s_sc), nwj);
    r = __fmul_rn(r, silu_f(a.z[(long long)b * a.z_ld + (long long)h * kd + j]));
    if (a.fam == 32)
        quant_q8_0_warp(r, a.xq + (long long)b * a.xq_ld + (long long)(h * (kd / 32) + warp) * 34, lane);
    else
        a.gout[(long long)b * a.gout_ld + (long long)h * kd + j] = r;
}

// The operator form (q35_launch_gdn_step_wy, api.h:290-308): q / k already
// normalised, gamma / beta given per token; writes out, km, delta and the
// state like the per-token k_gdn_step over `rows` tokens of one sequence.
// CTA per value head; the state column streams from HBM straight into
// registers (no shared copy: the chunk buffers need the room).
__global__ void __launch_bounds__(GDN_KD) k_gdn_wy_rows(const __grid_constant__ GdnArgs a) {
    extern __shared__ __align__(128) float smr[];
    const WyBufs m = wy_bufs(smr);
    float *lg = m.bet + WY_C;
    const int h = blockIdx.x, j = threadIdx.x;
    const int kh = h % a.nk;
    float *S = a.state + h * a.state_head;
    float col[GDN_KD];
#pragma unroll
    for (int i = 0; i < GDN_KD; i++) col[i] = S[(long long)i * GDN_KD + j];
    for (int t0 = 0; t0 < a.rows; t0 += WY_C) {
        const int nc = min(WY_C, a.rows - t0);
        for (int t = 0; t < nc; t++) {
            const long long tok = t0 + t;
            m.Qs[t * WY_LD + j] = a.q[tok * a.q_tok + kh * a.q_head + j];
            m.Ks[t * WY_LD + j] = a.k[tok * a.k_tok + kh * a.k_head + j];
            m.Vs[t * WY_LD + j] = a.v[tok * a.v_tok + h * a.v_head + j];
        }
        if (j < nc) {
            const long long tok = t0 + j;
            lg[j] = a.gamma_log ? a.gamma[tok * a.g_tok + h]
                                : fmaxf(logf(a.gamma ? a.gamma[tok * a.g_tok + h] : a.gamma_imm), WY_LOG_MIN);
            m.bet[j] = a.beta ? a.beta[tok * a.b_tok + h] : a.beta_imm;
        }
        __syncthreads();
        wy_cumulate(m, lg, nc, j);
        __syncthreads();
        auto sink = [&](int t, float km, float d) {
            const long long tok = t0 + t;
            if (a.km) a.km[tok * a.km_tok + h * a.km_head + j] = km;
            if (a.delta) a.delta[tok * a.delta_tok + h * a.delta_head + j] = d;
        };
        wy_chunk(col, m, nc, j, sink);
        for (int t = 0; t < nc; t++) a.out[(t0 + t) * a.out_tok + h * a.out_head + j] = m.Us[t * WY_LD + j];
        __syncthreads();  // chunk buffers reused
    }
#pragma unroll
    for (int i = 0; i < GDN_KD; i++) S[(long long)i * GDN_KD + j] = col[i];
}


inline int gdn_wy_rows_launch(const GdnArgs &a, cudaStream_t st) {
    if (a.heads <= 0 || a.rows <= 0) return 0;
    if (a.nk <= 0) return (int)cudaErrorInvalidValue;
    k_gdn_wy_rows<<<(unsigned)a.heads, GDN_KD, WY_ROWS_SMEM, st>>>(a);
    return (int)cudaGetLastError();
}

// The API's WY prefill with each head's state columns split over
// GDN_KD / CB CTAs (CB columns each).  The delta rule updates every value
// column on its own (km_j, delta_j and column j of S involve only column j),
// so the split needs no exchange; each CTA recomputes the chunk's shared
// quantities (cumulative decay, A, M) and runs the per-column steps for its
// columns with the threads spread over (token, column) and (state row,
// column) pairs.  A and M come from the tensor-core pass's Gram matrices (G,
// staged with the chunk) or, with G null, from wy_chunk's own dots; with G
// null every dot and chain runs in wy_chunk's order and the results equal
// k_gdn_wy_rows' bit for bit.  Two 256-thread CTAs fit on an SM, so a 16-head sequence
// runs on 256 CTAs of 8 columns, a 32-head one on 256 CTAs of 16.
constexpr int WY_AP = WY_C + 4;                // pitch of A^T (floats)
constexpr int WY_GC = 2 * WY_C * WY_C;         // floats of G per (chunk, k head): K K^T, then Q K^T
constexpr int WY_SP = GDN_KD + 4;              // pitch of the state columns (floats)
template <int CB>
constexpr size_t wy_cols_smem() {
    return (size_t)2 * 2 * WY_C * WY_LD * 4          // Qs, Ks (two buffers)
           + (size_t)2 * WY_GC * 4                   // G (two buffers)
           + (size_t)2 * WY_C * (CB + 1) * 4         // Vc (two buffers)
           + (size_t)3 * WY_C * (CB + 1) * 4         // Uc (then km), Wc, Dc
           + (size_t)WY_C * (CB + 1) * 4             // Ec: eE[t] * delta
           + (size_t)CB * WY_SP * 4                  // state columns, column-major
           + (size_t)WY_C * WY_AP * 4                // At: A transposed
           + (size_t)WY_C * (WY_C + 1) * 4           // Mm
           + (size_t)4 * WY_C * 4                    // Lc, eL, eE, bet
           + (size_t)2 * 2 * WY_C * 4;               // gamma, beta (two buffers)
}

// G: null, or the tensor-core pass's Gram matrices per (chunk, k head)
// ([2][WY_C][WY_C]: K K^T, then Q K^T; wy_tc.cuh), used for A and M
constexpr int WY_NT = 256;  // threads per CTA of the column-split kernel
template <int CB>
__global__ void __launch_bounds__(WY_NT, 2) k_gdn_wy_cols(const __grid_constant__ GdnArgs a, const float *__restrict__ G) {
    constexpr int NT = WY_NT, NW = NT / 32;
    constexpr int CLD = CB + 1;       // pitch of the per-column tiles (floats)
    constexpr int NCB = GDN_KD / CB;  // CTAs per head
    constexpr int NTG = NT / CB;      // token groups of the (token, column) loops
    constexpr int TPT = WY_C / NTG;   // tokens per thread in them
    constexpr int P = NT / CB;        // lanes per column in the forward substitution
    constexpr int NSLOT = WY_C / P;   // tokens each of those lanes owns
    constexpr int RPT = GDN_KD / NTG; // state rows per thread
    constexpr int RG = RPT % 8 == 0 ? 8 : 4;  // state rows per pass
    static_assert(P <= 32 && 32 % P == 0 && NSLOT >= 1 && RPT % 4 == 0 && (TPT == 1 || TPT % 2 == 0),
                  "column split");
    extern __shared__ __align__(128) float smc[];
    float *Qb = smc, *Kb = Qb + 2 * WY_C * WY_LD;     // [2][C][LD]
    float *Gs = Kb + 2 * WY_C * WY_LD;                // [2][2][C][C]
    float *Vb = Gs + 2 * WY_GC;                       // [2][C][CLD]
    float *Uc = Vb + 2 * WY_C * CLD, *Wc = Uc + WY_C * CLD, *Dc = Wc + WY_C * CLD;
    float *Ec = Dc + WY_C * CLD, *St = Ec + WY_C * CLD;  // St[column][row]
    float *At = St + CB * WY_SP, *Mm = At + WY_C * WY_AP;
    static_assert((2 * 2 * WY_C * WY_LD + 2 * WY_GC + 6 * WY_C * CLD) % 4 == 0, "St 16-byte aligned");
    float *Lc = Mm + WY_C * (WY_C + 1), *eL = Lc + WY_C, *eE = eL + WY_C, *bet = eE + WY_C;
    float *Gb = bet + WY_C, *Bb = Gb + 2 * WY_C;      // [2][C] gamma, beta
    const int h = blockIdx.x / NCB, cb = blockIdx.x - h * NCB, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int kh = h % a.nk, c0 = cb * CB;
    const int jj = tid & (CB - 1), tg = tid / CB;     // (token group, column) of the pair loops
    float *S = a.state + h * a.state_head;
    // the chunk starting at token t0 into buffer b: every copy in flight at once
    auto stage = [&](int t0, int b) {
        const int nc = min(WY_C, a.rows - t0);
        if (nc > 0) {
            float *qd = Qb + b * WY_C * WY_LD, *kd = Kb + b * WY_C * WY_LD, *vd = Vb + b * WY_C * CLD;
            for (int idx = tid; idx < nc * (GDN_KD / 4); idx += NT) {
                const int t = idx / (GDN_KD / 4), c = idx - t * (GDN_KD / 4);
                const long long tok = t0 + t;
                cp_async16(qd + t * WY_LD + 4 * c, a.q + tok * a.q_tok + kh * a.q_head + 4 * c);
                cp_async16(kd + t * WY_LD + 4 * c, a.k + tok * a.k_tok + kh * a.k_head + 4 * c);
            }
            for (int idx = tid; idx < nc * CB; idx += NT) {
                const int t = idx / CB, c = idx - t * CB;
                cp_async4(vd + t * CLD + c, a.v + (t0 + t) * a.v_tok + h * a.v_head + c0 + c);
            }
            if (tid < nc) {
                const long long tok = t0 + tid;
                if (a.gamma) cp_async4(Gb + b * WY_C + tid, a.gamma + tok * a.g_tok + h);
                if (a.beta) cp_async4(Bb + b * WY_C + tid, a.beta + tok * a.b_tok + h);
            }
            if (G) {
                const float *gsrc = G + ((long long)(t0 / WY_C) * a.nk + kh) * WY_GC;
                for (int idx = tid; idx < WY_GC / 4; idx += NT)
                    cp_async16(Gs + b * WY_GC + 4 * idx, gsrc + 4 * idx);
            }
        }
        cp_async_commit();  // one group per chunk, empty past the end
    };
    for (int idx = tid; idx < GDN_KD * CB; idx += NT) {
        const int i = idx / CB, c = idx - i * CB;
        St[c * WY_SP + i] = S[(long long)i * GDN_KD + c0 + c];
    }
    stage(0, 0);
    for (int t0 = 0, buf = 0; t0 < a.rows; t0 += WY_C, buf ^= 1) {
        const int nc = min(WY_C, a.rows - t0);
        stage(t0 + WY_C, buf ^ 1);  // the next chunk, into the buffer the previous one left
        cp_async_wait<1>();         // this thread's copies of this chunk landed
        __syncthreads();            // everyone's
        const float *Qs = Qb + buf * WY_C * WY_LD, *Ks = Kb + buf * WY_C * WY_LD, *Vc = Vb + buf * WY_C * CLD;
        // the last warp: floored log decays (in Lc), their running sum
        // (wy_cumulate, one lane, in token order) and its exponentials; the
        // other warps start on U / W, which needs none of them
        if (warp == NW - 1) {
            if (lane < nc) {
                Lc[lane] = a.gamma_log ? Gb[buf * WY_C + lane]
                                       : fmaxf(logf(a.gamma ? Gb[buf * WY_C + lane] : a.gamma_imm), WY_LOG_MIN);
                bet[lane] = a.beta ? Bb[buf * WY_C + lane] : a.beta_imm;
            }
            __syncwarp();
            if (lane == 0) {
                float lv[WY_C];
#pragma unroll
                for (int t = 0; t < WY_C; t++) lv[t] = Lc[t];
                float L = 0.0f;
#pragma unroll
                for (int t = 0; t < WY_C; t++)
                    if (t < nc) {
                        L = __fadd_rn(L, lv[t]);
                        Lc[t] = L;
                    }
            }
            __syncwarp();
            if (lane < nc) {
                eL[lane] = expf(Lc[lane]);
                eE[lane] = expf(Lc[nc - 1] - Lc[lane]);
            }
        }
        // U = S0^T k_t, W = S0^T q_t for (token, column) pairs, two tokens
        // (t, t + NTG) at a time where a thread has several, so each state
        // load serves both; wy_chunk's four partial sums per dot
        auto uw = [&](int t, int t2, bool two) {
            const float4 *k4 = reinterpret_cast<const float4 *>(Ks + t * WY_LD);
            const float4 *q4 = reinterpret_cast<const float4 *>(Qs + t * WY_LD);
            const float4 *k4b = reinterpret_cast<const float4 *>(Ks + t2 * WY_LD);
            const float4 *q4b = reinterpret_cast<const float4 *>(Qs + t2 * WY_LD);
            const float4 *st4 = reinterpret_cast<const float4 *>(St + jj * WY_SP);
            float u0 = 0.0f, u1 = 0.0f, u2 = 0.0f, u3 = 0.0f, w0 = 0.0f, w1 = 0.0f, w2 = 0.0f, w3 = 0.0f;
            float x0 = 0.0f, x1 = 0.0f, x2 = 0.0f, x3 = 0.0f, y0 = 0.0f, y1 = 0.0f, y2 = 0.0f, y3 = 0.0f;
#pragma unroll 4
            for (int i4 = 0; i4 < GDN_KD / 4; i4++) {
                const float4 kv = k4[i4], qv = q4[i4];
                const float4 sv = st4[i4];
                const float s0 = sv.x, s1 = sv.y, s2 = sv.z, s3 = sv.w;
                u0 = __fmaf_rn(s0, kv.x, u0);
                u1 = __fmaf_rn(s1, kv.y, u1);
                u2 = __fmaf_rn(s2, kv.z, u2);
                u3 = __fmaf_rn(s3, kv.w, u3);
                w0 = __fmaf_rn(s0, qv.x, w0);
                w1 = __fmaf_rn(s1, qv.y, w1);
                w2 = __fmaf_rn(s2, qv.z, w2);
                w3 = __fmaf_rn(s3, qv.w, w3);
                if (two) {
                    const float4 kb = k4b[i4], qb = q4b[i4];
                    x0 = __fmaf_rn(s0, kb.x, x0);
                    x1 = __fmaf_rn(s1, kb.y, x1);
                    x2 = __fmaf_rn(s2, kb.z, x2);
                    x3 = __fmaf_rn(s3, kb.w, x3);
                    y0 = __fmaf_rn(s0, qb.x, y0);
                    y1 = __fmaf_rn(s1, qb.y, y1);
                    y2 = __fmaf_rn(s2, qb.z, y2);
                    y3 = __fmaf_rn(s3, qb.w, y3);
                }
            }
            Uc[t * CLD + jj] = (u0 + u1) + (u2 + u3);
            Wc[t * CLD + jj] = (w0 + w1) + (w2 + w3);
            if (two && t2 < nc) {
                Uc[t2 * CLD + jj] = (x0 + x1) + (x2 + x3);
                Wc[t2 * CLD + jj] = (y0 + y1) + (y2 + y3);
            }
        };
        if constexpr (TPT == 1) {
            if (tg < nc) uw(tg, tg, false);
        } else {
            // t2 < WY_C: in the buffer (stale past nc, not stored)
            for (int t = tg; t < nc; t += 2 * NTG) uw(t, t + NTG, true);
        }
        __syncthreads();
        // A and M: the Gram matrices with this head's decays, or wy_chunk's
        // own computation (lane = s, warp w takes t = w, w + NW, ...)
        if (G) {
            const float *gk = Gs + buf * WY_GC, *gq = gk + WY_C * WY_C;
            // every load first (shared stores would otherwise pin them)
            constexpr int NE = WY_C * WY_C / NT;
            float lt[NE], ls[NE], vk[NE], vq[NE];
#pragma unroll
            for (int k = 0; k < NE; k++) {
                const int idx = tid + k * NT, t = idx / WY_C, s2 = idx - t * WY_C;
                lt[k] = Lc[t];
                ls[k] = Lc[s2];
                vk[k] = gk[idx];
                vq[k] = gq[idx];
            }
#pragma unroll
            for (int k = 0; k < NE; k++) {
                const int idx = tid + k * NT, t = idx / WY_C, s2 = idx - t * WY_C;
                if (t < nc) {
                    const float dec = s2 <= t ? expf(lt[k] - ls[k]) : 0.0f;
                    At[s2 * WY_AP + t] = s2 < t ? dec * vk[k] : 0.0f;
                    Mm[t * (WY_C + 1) + s2] = s2 <= t ? dec * vq[k] : 0.0f;
                }
            }
        } else {
            const int sidx = lane;
            const float4 *ks4 = reinterpret_cast<const float4 *>(Ks + sidx * WY_LD);
            for (int t = warp; t < nc; t += NW) {
                const float4 *kt4 = reinterpret_cast<const float4 *>(Ks + t * WY_LD);
                const float4 *qt4 = reinterpret_cast<const float4 *>(Qs + t * WY_LD);
                float kk = 0.0f, qk = 0.0f;
                if (sidx <= t) {
                    float k0 = 0.0f, k1 = 0.0f, k2 = 0.0f, k3 = 0.0f, q0 = 0.0f, q1 = 0.0f, q2 = 0.0f, q3 = 0.0f;
#pragma unroll 8
                    for (int i4 = 0; i4 < GDN_KD / 4; i4++) {
                        const float4 x = ks4[i4], y = kt4[i4], z = qt4[i4];
                        k0 = __fmaf_rn(y.x, x.x, k0);
                        k1 = __fmaf_rn(y.y, x.y, k1);
                        k2 = __fmaf_rn(y.z, x.z, k2);
                        k3 = __fmaf_rn(y.w, x.w, k3);
                        q0 = __fmaf_rn(z.x, x.x, q0);
                        q1 = __fmaf_rn(z.y, x.y, q1);
                        q2 = __fmaf_rn(z.z, x.z, q2);
                        q3 = __fmaf_rn(z.w, x.w, q3);
                    }
                    kk = (k0 + k1) + (k2 + k3);
                    qk = (q0 + q1) + (q2 + q3);
                }
                const float dec = sidx <= t ? expf(Lc[t] - Lc[sidx]) : 0.0f;
                At[sidx * WY_AP + t] = sidx < t ? dec * kk : 0.0f;
                Mm[t * (WY_C + 1) + sidx] = sidx <= t ? dec * qk : 0.0f;
            }
        }
        __syncthreads();
        // forward substitution for km / delta: P lanes per column, lane r
        // owning tokens r, r + P, ...; right looking, so once delta_s is
        // known (from its owner, by shuffle) it enters every later km_t at
        // once; each km_t still sums eL_t U_t, then A_t0 delta_0,
        // A_t1 delta_1, ... in wy_chunk's order.  The loop holds everything
        // in registers (no shared stores between the loads of A); km and
        // delta of the owned tokens go to Uc and Dc after it.
        {
            const int c = tid / P, r = tid % P;
            float kmv[NSLOT], vv[NSLOT], bb[NSLOT], dv[NSLOT];
#pragma unroll
            for (int j = 0; j < NSLOT; j++) {
                const int t = r + j * P;
                kmv[j] = eL[t] * Uc[t * CLD + c];
                vv[j] = Vc[t * CLD + c];
                bb[j] = bet[t];
                dv[j] = 0.0f;
            }
#pragma unroll
            for (int s2 = 0; s2 < WY_C; s2++) {
                constexpr int PM = P - 1;
                const int js = s2 / P;
                const float mine = bb[js] * (vv[js] - kmv[js]);
                const float d = __shfl_sync(0xffffffffu, mine, (lane & ~PM) | (s2 & PM));
                if (r == (s2 & PM)) dv[js] = d;
#pragma unroll
                for (int j = js; j < NSLOT; j++)
                    if (r + j * P > s2) kmv[j] = __fmaf_rn(At[s2 * WY_AP + r + j * P], d, kmv[j]);
            }
#pragma unroll
            for (int j = 0; j < NSLOT; j++) {
                const int t = r + j * P;
                Dc[t * CLD + c] = dv[j];
                Ec[t * CLD + c] = eE[t] * dv[j];
                Uc[t * CLD + c] = kmv[j];
            }
        }
        __syncthreads();
        // outputs for (token, column) pairs; where a thread has several
        // tokens, t and its mirror in the group's span go together so every
        // thread's chains have equal length; km and delta leave with them
        auto emit = [&](int t) {
            if (t < nc) {
                float o = eL[t] * Wc[t * CLD + jj];
                for (int s2 = 0; s2 <= t; s2++) o = __fmaf_rn(Mm[t * (WY_C + 1) + s2], Dc[s2 * CLD + jj], o);
                const long long tok = t0 + t;
                a.out[tok * a.out_tok + h * a.out_head + c0 + jj] = o;
                if (a.km) a.km[tok * a.km_tok + h * a.km_head + c0 + jj] = Uc[t * CLD + jj];
                if (a.delta) a.delta[tok * a.delta_tok + h * a.delta_head + c0 + jj] = Dc[t * CLD + jj];
            }
        };
        if constexpr (TPT == 1) {
            emit(tg);
        } else {
            for (int base = 0; base < WY_C; base += 2 * NTG) {
                emit(base + tg);
                emit(base + 2 * NTG - 1 - tg);
            }
        }
        // state for (row, column) pairs: exp(L_end) S0 + sum_t decay(end, t) k_t delta_t,
        // RG consecutive rows per pass so RG chains are in flight and the
        // k rows load as 16-byte vectors
        const float gend = eL[nc - 1];
#pragma unroll 1
        for (int i0 = tg * RPT; i0 < tg * RPT + RPT; i0 += RG) {
            float x[RG];
#pragma unroll
            for (int m4 = 0; m4 < RG; m4 += 4) {
                const float4 sv = *reinterpret_cast<const float4 *>(St + jj * WY_SP + i0 + m4);
                x[m4] = gend * sv.x;
                x[m4 + 1] = gend * sv.y;
                x[m4 + 2] = gend * sv.z;
                x[m4 + 3] = gend * sv.w;
            }
            for (int t = 0; t < nc; t++) {
                const float e = Ec[t * CLD + jj];
#pragma unroll
                for (int m4 = 0; m4 < RG; m4 += 4) {
                    const float4 kv = *reinterpret_cast<const float4 *>(Ks + t * WY_LD + i0 + m4);
                    x[m4] = __fmaf_rn(kv.x, e, x[m4]);
                    x[m4 + 1] = __fmaf_rn(kv.y, e, x[m4 + 1]);
                    x[m4 + 2] = __fmaf_rn(kv.z, e, x[m4 + 2]);
                    x[m4 + 3] = __fmaf_rn(kv.w, e, x[m4 + 3]);
                }
            }
#pragma unroll
            for (int m4 = 0; m4 < RG; m4 += 4)
                *reinterpret_cast<float4 *>(St + jj * WY_SP + i0 + m4) = make_float4(x[m4], x[m4 + 1], x[m4 + 2], x[m4 + 3]);
        }
        __syncthreads();  // chunk buffers and the state columns are reused
    }
    cp_async_wait<0>();
    for (int idx = tid; idx < GDN_KD * CB; idx += NT) {
        const int i = idx / CB, c = idx - i * CB;
        S[(long long)i * GDN_KD + c0 + c] = St[c * WY_SP + i];
    }
}

// 8 columns per CTA while the heads' CTAs stay within two per SM, else 16
inline int gdn_wy_cols_launch(const GdnArgs &a, cudaStream_t st, const float *G = nullptr) {
    if (a.heads <= 0 || a.rows <= 0) return 0;
    if (a.nk <= 0) return (int)cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (a.heads * (GDN_KD / 8) <= 2 * sms)
        k_gdn_wy_cols<8><<<(unsigned)(a.heads * (GDN_KD / 8)), WY_NT, wy_cols_smem<8>(), st>>>(a, G);
    else
        k_gdn_wy_cols<16><<<(unsigned)(a.heads * (GDN_KD / 16)), WY_NT, wy_cols_smem<16>(), st>>>(a, G);
    return (int)cudaGetLastError();
}

// k_gdn_core stages the 64 KB state block in dynamic shared memory
inline int gdn_prepare() {
    static int done = 0;
    if (done) return 0;
    cudaError_t e = cudaFuncSetAttribute(k_gdn_core, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_KD * GDN_KD * 4);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gdn_wy_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WY_ROWS_SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gdn_wy_cols<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wy_cols_smem<8>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gdn_wy_cols<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)wy_cols_smem<16>());
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
