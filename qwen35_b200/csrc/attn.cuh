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
constexpr int ATT_SPLIT = 32 * ATT_WARPS;  // positions per split CTA in the engine

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

// CTA (kv head, sequence, split): up to 32 * ATT_WARPS positions.  Warp w
// takes positions p0 + 32 w + lane: each lane computes its position's scores
// for the gqa heads with a serial dot over the 256 dims (the CPU's order, so a
// score is bit-exact given q and k), then the warp forms max / exp / sum, and
// P.V runs lane-per-dim over the warp's positions (V rows read coalesced).
// The ATT_WARPS partials are merged in shared memory.
template <int G>
__global__ void __launch_bounds__(ATT_WARPS * 32) k_attn_split(const __grid_constant__ AttnArgs a) {
    __shared__ __align__(16) float s_q[G][ATT_HD];
    __shared__ float s_m[ATT_WARPS][G], s_l[ATT_WARPS][G];
    __shared__ __align__(16) float s_acc[ATT_WARPS][G][ATT_HD];
    const int kvh = blockIdx.x, seq = blockIdx.y, sp = blockIdx.z;
    if (a.active && !a.active[seq]) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long slot = a.slots ? a.slots[seq] : seq;
    const int len = a.lens ? a.lens[seq] : (a.last_pos ? a.last_pos[0] + 1 : a.len_imm);
    const int p0 = sp * a.split_len;
    const int p1 = min(len, p0 + a.split_len);
    for (int i = threadIdx.x; i < G * ATT_HD; i += ATT_WARPS * 32) {
        const int g = i / ATT_HD, j = i - g * ATT_HD;
        s_q[g][j] = a.q[(long long)seq * a.q_tok + (long long)(kvh * G + g) * ATT_HD + j];
    }
    __syncthreads();
    const float *Kb = a.kc + slot * a.kv_slot + kvh * ATT_HD;
    const float *Vb = a.vc + slot * a.kv_slot + kvh * ATT_HD;
    float m[G], l[G], acc[G][8];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) acc[g][i] = 0.0f;
    }
    for (int base = p0 + 32 * warp; base < p1; base += 32 * ATT_WARPS) {
        const int t = base + lane;
        const bool live = t < p1;
        float s[G];
#pragma unroll
        for (int g = 0; g < G; g++) s[g] = 0.0f;
        if (live) {
            const float4 *kr = reinterpret_cast<const float4 *>(Kb + (long long)t * a.kv_dim);
#pragma unroll 4
            for (int c = 0; c < ATT_HD / 4; c++) {
                const float4 kv = kr[c];
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const float4 qv = reinterpret_cast<const float4 *>(s_q[g])[c];
                    s[g] = __fadd_rn(s[g], __fmul_rn(qv.x, kv.x));
                    s[g] = __fadd_rn(s[g], __fmul_rn(qv.y, kv.y));
                    s[g] = __fadd_rn(s[g], __fmul_rn(qv.z, kv.z));
                    s[g] = __fadd_rn(s[g], __fmul_rn(qv.w, kv.w));
                }
            }
        }
        const int nlive = min(32, p1 - base);
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float sc = live ? __fmul_rn(s[g], a.scale) : -INFINITY;
            const float mw = fmaxf(warp_max(sc), m[g]);
            const float p = live ? expf(__fsub_rn(sc, mw)) : 0.0f;
            const float c = expf(__fsub_rn(m[g], mw));  // 0 on the first chunk (m = -inf)
            l[g] = __fadd_rn(__fmul_rn(l[g], c), warp_sum(p));
#pragma unroll
            for (int i = 0; i < 8; i++) acc[g][i] = __fmul_rn(acc[g][i], c);
            m[g] = mw;
            for (int u = 0; u < nlive; u++) {
                const float pu = __shfl_sync(0xffffffffu, p, u);
                const float4 *vr = reinterpret_cast<const float4 *>(Vb + (long long)(base + u) * a.kv_dim + lane * 8);
                const float4 v0 = vr[0], v1 = vr[1];
                acc[g][0] = __fadd_rn(acc[g][0], __fmul_rn(pu, v0.x));
                acc[g][1] = __fadd_rn(acc[g][1], __fmul_rn(pu, v0.y));
                acc[g][2] = __fadd_rn(acc[g][2], __fmul_rn(pu, v0.z));
                acc[g][3] = __fadd_rn(acc[g][3], __fmul_rn(pu, v0.w));
                acc[g][4] = __fadd_rn(acc[g][4], __fmul_rn(pu, v1.x));
                acc[g][5] = __fadd_rn(acc[g][5], __fmul_rn(pu, v1.y));
                acc[g][6] = __fadd_rn(acc[g][6], __fmul_rn(pu, v1.z));
                acc[g][7] = __fadd_rn(acc[g][7], __fmul_rn(pu, v1.w));
            }
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
                const float c = expf(__fsub_rn(s_m[w][g], M));
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
        const float c = expf(__fsub_rn(ms, M));
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
