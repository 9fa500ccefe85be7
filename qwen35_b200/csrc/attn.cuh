// attn.cuh -- GQA decode attention over per-sequence f32 KV slots, sm_100a.
//
// Split-KV ("flash decoding"): CTA (sequence, kv head, split) streams a
// contiguous range of positions once, serving all gqa query heads of that kv
// head from the same K/V bytes (coalesced 1 KB rows), with an online softmax
// per warp; a second kernel merges the splits and applies the sigmoid gate.
// With one split the first kernel finishes the output itself.
//
// Semantics (src/elementwise.zig:349-372): score_t = (q . k_t) * scale over
// t in [0, len), softmax, out = sum_t p_t v_t, then out *= sigmoid(gate);
// kv head = q head / gqa (SPEC B13).  The rescaled online form re-associates
// the sums, so outputs agree with the CPU to ~1e-6 relative, not bitwise.
#pragma once
#include "common.cuh"

namespace q35 {

constexpr int ATT_HD = 256;
constexpr int ATT_WARPS = 4;
constexpr int ATT_MAXG = 8;

struct AttnArgs {
    const float *q, *gate;
    long long q_tok;          // floats between tokens in q / gate
    const float *kc, *vc;
    long long kv_slot;        // floats between slots (sequences) in the cache
    int kv_dim;
    const int *slots;         // per-sequence slot (null: sequence index)
    const int *lens;          // per-sequence context length (null: see below)
    const int *last_pos;      // device scalar: len = *last_pos + 1 (null: len_imm)
    int len_imm;
    float *out;
    long long out_tok;
    float *part_acc, *part_ml;  // split partials (nsplit > 1)
    int nsplit, split_len;
    int heads, kv_heads;
    float scale;
    const int *active;
};

template <int G>
__global__ void __launch_bounds__(ATT_WARPS * 32) k_attn_split(const __grid_constant__ AttnArgs a) {
    __shared__ float s_m[ATT_WARPS][G], s_l[ATT_WARPS][G];
    __shared__ float s_acc[ATT_WARPS][G][ATT_HD];
    const int kvh = blockIdx.x, seq = blockIdx.y, sp = blockIdx.z;
    if (a.active && !a.active[seq]) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long slot = a.slots ? a.slots[seq] : seq;
    const int len = a.lens ? a.lens[seq] : (a.last_pos ? a.last_pos[0] + 1 : a.len_imm);
    const int p0 = sp * a.split_len;
    const int p1 = min(len, p0 + a.split_len);
    const float *K = a.kc + slot * a.kv_slot + kvh * ATT_HD + lane * 8;
    const float *V = a.vc + slot * a.kv_slot + kvh * ATT_HD + lane * 8;

    float qv[G][8], acc[G][8], m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float *qp = a.q + (long long)seq * a.q_tok + (long long)(kvh * G + g) * ATT_HD + lane * 8;
        const float4 x0 = reinterpret_cast<const float4 *>(qp)[0], x1 = reinterpret_cast<const float4 *>(qp)[1];
        qv[g][0] = x0.x; qv[g][1] = x0.y; qv[g][2] = x0.z; qv[g][3] = x0.w;
        qv[g][4] = x1.x; qv[g][5] = x1.y; qv[g][6] = x1.z; qv[g][7] = x1.w;
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) acc[g][i] = 0.0f;
    }
    for (int t = p0 + warp; t < p1; t += ATT_WARPS) {
        const float4 *kp = reinterpret_cast<const float4 *>(K + (long long)t * a.kv_dim);
        const float4 k0 = kp[0], k1 = kp[1];
        const float4 *vp = reinterpret_cast<const float4 *>(V + (long long)t * a.kv_dim);
        const float4 v0 = vp[0], v1 = vp[1];
        const float kk[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
        const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int g = 0; g < G; g++) {
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) s = __fadd_rn(s, __fmul_rn(qv[g][i], kk[i]));
            s = __fmul_rn(warp_sum(s), a.scale);
            const float mn = fmaxf(m[g], s);
            const float c = exp_f(__fsub_rn(m[g], mn));
            const float e = exp_f(__fsub_rn(s, mn));
            l[g] = __fadd_rn(__fmul_rn(l[g], c), e);
#pragma unroll
            for (int i = 0; i < 8; i++) acc[g][i] = __fadd_rn(__fmul_rn(acc[g][i], c), __fmul_rn(e, vv[i]));
            m[g] = mn;
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        if (lane == 0) {
            s_m[warp][g] = m[g];
            s_l[warp][g] = l[g];
        }
#pragma unroll
        for (int i = 0; i < 8; i++) s_acc[warp][g][lane * 8 + i] = acc[g][i];
    }
    __syncthreads();
    // merge the warps: thread handles dims j and j+128 for every head
    for (int idx = threadIdx.x; idx < G * ATT_HD; idx += ATT_WARPS * 32) {
        const int g = idx / ATT_HD, j = idx - g * ATT_HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; w++) M = fmaxf(M, s_m[w][g]);
        float L = 0.0f, A = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < ATT_WARPS; w++) {
                if (s_m[w][g] == -INFINITY) continue;
                const float c = exp_f(__fsub_rn(s_m[w][g], M));
                L = __fadd_rn(L, __fmul_rn(s_l[w][g], c));
                A = __fadd_rn(A, __fmul_rn(s_acc[w][g][j], c));
            }
        }
        const int h = kvh * G + g;
        if (a.nsplit == 1) {
            const float o = __fdiv_rn(A, L);
            const long long off = (long long)seq * a.q_tok + (long long)h * ATT_HD + j;
            a.out[(long long)seq * a.out_tok + (long long)h * ATT_HD + j] = __fmul_rn(o, sigmoid_f(a.gate[off]));
        } else {
            const long long pi = ((long long)seq * a.heads + h) * a.nsplit + sp;
            a.part_acc[pi * ATT_HD + j] = A;
            if (j == 0) {
                a.part_ml[pi * 2] = M;
                a.part_ml[pi * 2 + 1] = L;
            }
        }
    }
}

__global__ void __launch_bounds__(ATT_HD) k_attn_merge(const __grid_constant__ AttnArgs a) {
    const int h = blockIdx.x, seq = blockIdx.y, j = threadIdx.x;
    if (a.active && !a.active[seq]) return;
    const long long pb = ((long long)seq * a.heads + h) * a.nsplit;
    const int len = a.lens ? a.lens[seq] : (a.last_pos ? a.last_pos[0] + 1 : a.len_imm);
    const int ns = min(a.nsplit, (len + a.split_len - 1) / a.split_len);
    float M = -INFINITY;
    for (int s = 0; s < ns; s++) M = fmaxf(M, a.part_ml[(pb + s) * 2]);
    float L = 0.0f, A = 0.0f;
    for (int s = 0; s < ns; s++) {
        const float ms = a.part_ml[(pb + s) * 2];
        if (ms == -INFINITY) continue;
        const float c = exp_f(__fsub_rn(ms, M));
        L = __fadd_rn(L, __fmul_rn(a.part_ml[(pb + s) * 2 + 1], c));
        A = __fadd_rn(A, __fmul_rn(a.part_acc[(pb + s) * ATT_HD + j], c));
    }
    const float o = __fdiv_rn(A, L);
    const long long off = (long long)seq * a.q_tok + (long long)h * ATT_HD + j;
    a.out[(long long)seq * a.out_tok + (long long)h * ATT_HD + j] = __fmul_rn(o, sigmoid_f(a.gate[off]));
}

inline int attn_launch(AttnArgs a, int nseq, int max_len, cudaStream_t st) {
    if (nseq <= 0) return 0;
    if (a.kv_heads <= 0 || a.heads % a.kv_heads != 0) return (int)cudaErrorInvalidValue;
    const int G = a.heads / a.kv_heads;
    if (G > ATT_MAXG || max_len <= 0) return (int)cudaErrorInvalidValue;
    if (a.nsplit < 1) a.nsplit = 1;
    if (a.nsplit > 1 && (!a.part_acc || !a.part_ml)) a.nsplit = 1;
    if (a.nsplit == 1) a.split_len = max_len;
    if (a.split_len < 1) a.split_len = 1;
    dim3 grid((unsigned)a.kv_heads, (unsigned)nseq, (unsigned)a.nsplit);
    switch (G) {
    case 1: k_attn_split<1><<<grid, ATT_WARPS * 32, 0, st>>>(a); break;
    case 2: k_attn_split<2><<<grid, ATT_WARPS * 32, 0, st>>>(a); break;
    case 3: k_attn_split<3><<<grid, ATT_WARPS * 32, 0, st>>>(a); break;
    case 4: k_attn_split<4><<<grid, ATT_WARPS * 32, 0, st>>>(a); break;
    case 6: k_attn_split<6><<<grid, ATT_WARPS * 32, 0, st>>>(a); break;
    case 8: k_attn_split<8><<<grid, ATT_WARPS * 32, 0, st>>>(a); break;
    default: return (int)cudaErrorInvalidValue;
    }
    int rc = (int)cudaGetLastError();
    if (rc || a.nsplit == 1) return rc;
    k_attn_merge<<<dim3((unsigned)a.heads, (unsigned)nseq), ATT_HD, 0, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace q35
