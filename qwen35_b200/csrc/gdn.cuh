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
