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

namespace q35 {

// ---------------------------------------------------------------------------
// Decode attention in the CPU's exact operation order (src/elementwise.zig:
// 349-372): score_t = (sum_j q_j k_tj) * scale with j ascending; softmax as
// max, e_t = exp(score_t - max), serial sum over t, e_t / sum; out_j =
// sum_t p_t v_tj with t ascending; out_j *= sigmoid(gate_j).
// Kernel 1 (scores): CTA (kv head, sequence, 32-position chunk), one warp;
// the chunk's K rows are copied to shared memory with cp.async (every copy
// in flight at once), then a lane per position computes the gqa heads'
// serial dots from there.
// Kernel 2 (softmax): CTA (q head, sequence), probabilities in place.
// Kernel 3 (P.V): CTA (kv head, sequence, 64-dim chunk), the group's q heads
// together so V streams once per kv head; thread (head, dim) walks t in
// order over a 4-deep cp.async ring of V tiles.
// Parallelism comes from heads and dims, not positions, so no split
// re-associates a sum.
// ---------------------------------------------------------------------------
constexpr int ATTX_CHUNK = 32;             // positions per score CTA
constexpr int ATTX_KLD = ATT_HD + 4;       // shared K row stride (floats): 1040 B, an odd multiple of 16
constexpr int ATTX_DIMS = 64;


struct AttnXArgs {
    const float *q, *gate;
    long long q_tok;
    const float *kc, *vc;
    long long kv_slot;
    int kv_dim;
    const int *slots, *lens;
    const int *last_pos;
    int len_imm;
    int len_step;        // no lens / last_pos: token t attends to len_imm + len_step * t positions
    float *scores;       // [n][heads][max_len]
    int max_len;
    float *out;          // gated attention output
    long long out_tok;
    int heads, kv_heads;
    float scale;
    int fam;             // 32: also quantize the output (Q8_0 blocks) into xq
    uint8_t *xq;
    long long xq_ld;
};

Q35_DEV int attx_len(const AttnXArgs &a, int seq) {
    return a.lens ? a.lens[seq] : (a.last_pos ? a.last_pos[0] + 1 : a.len_imm + a.len_step * seq);
}

template <int G>
__global__ void __launch_bounds__(ATTX_CHUNK) k_attx_scores(const __grid_constant__ AttnXArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ __align__(16) float s_q[G][ATT_HD];
    __shared__ __align__(16) float s_k[ATTX_CHUNK][ATTX_KLD];
    const int kvh = blockIdx.x, seq = blockIdx.y, p0 = blockIdx.z * ATTX_CHUNK, lane = threadIdx.x;
    const int len = attx_len(a, seq);
    if (p0 >= len) return;
    const int np = min(ATTX_CHUNK, len - p0);
    const long long slot = a.slots ? a.slots[seq] : seq;
    const float *kb = a.kc + slot * a.kv_slot + (long long)p0 * a.kv_dim + kvh * ATT_HD;
    for (int idx = lane; idx < np * (ATT_HD / 4); idx += ATTX_CHUNK) {
        const int r = idx / (ATT_HD / 4), c = idx - r * (ATT_HD / 4);
        cp_async16(&s_k[r][c * 4], kb + (long long)r * a.kv_dim + c * 4);
    }
    cp_async_commit();
    for (int i = lane; i < G * ATT_HD; i += ATTX_CHUNK) {
        const int g = i / ATT_HD, j = i - g * ATT_HD;
        s_q[g][j] = a.q[(long long)seq * a.q_tok + (long long)(kvh * G + g) * ATT_HD + j];
    }
    cp_async_wait<0>();
    __syncthreads();
    if (lane >= np) return;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; g++) s[g] = 0.0f;
    const float4 *kr = reinterpret_cast<const float4 *>(s_k[lane]);
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
#pragma unroll
    for (int g = 0; g < G; g++)
        a.scores[((long long)seq * a.heads + kvh * G + g) * a.max_len + p0 + lane] = __fmul_rn(s[g], a.scale);
}

// Softmax of one (sequence, head) row of scores, in place: the max (any
// order gives the same value), exp(s - max), the sum in position order (one
// thread, from shared memory), then p = e / sum -- the CPU's operations
// (src/elementwise.zig:349-372).  Dynamic shared memory: len floats.
constexpr int ATTX_SMT = 256;
__global__ void __launch_bounds__(ATTX_SMT) k_attx_softmax(const __grid_constant__ AttnXArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float s_e[];
    __shared__ float s_red[ATTX_SMT / 32], s_sum;
    const int h = blockIdx.x, seq = blockIdx.y, j = threadIdx.x;
    const int len = attx_len(a, seq);
    float *sc = a.scores + ((long long)seq * a.heads + h) * a.max_len;
    float m = -3.40282347e38f;
    for (int t = j; t < len; t += ATTX_SMT) {
        const float v = sc[t];
        s_e[t] = v;
        m = fmaxf(m, v);
    }
    m = warp_max(m);
    if ((j & 31) == 0) s_red[j >> 5] = m;
    __syncthreads();
    m = s_red[0];
#pragma unroll
    for (int w = 1; w < ATTX_SMT / 32; w++) m = fmaxf(m, s_red[w]);
    for (int t = j; t < len; t += ATTX_SMT) s_e[t] = exp_f(__fsub_rn(s_e[t], m));
    __syncthreads();
    if (j == 0) {
        // serial sum; the loads of the next 32 run ahead of the add chain
        float sum = 0.0f;
        int t = 0;
        for (; t + 32 <= len; t += 32) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = s_e[t + i];
#pragma unroll
            for (int i = 0; i < 32; i++) sum = __fadd_rn(sum, v[i]);
        }
        for (; t < len; t++) sum = __fadd_rn(sum, s_e[t]);
        s_sum = sum;
    }
    __syncthreads();
    const float sum = s_sum;
    for (int t = j; t < len; t += ATTX_SMT) sc[t] = __fdiv_rn(s_e[t], sum);
}

// P.V: CTA per (kv head, sequence, 64-dim chunk) with G x 64 threads, thread
// = (q head g of the group, dim j); the V tiles (64 positions x 64 dims) and
// the G probability rows stream through a 4-deep cp.async ring shared by the
// group's q heads, so V is read once per kv head.  acc += p[t] * v[t] in
// position order, then the gate (sigmoid) and, for a Q8_0 consumer, the
// quantized output block.
constexpr int ATTX_PT = 64;   // positions per tile
constexpr int ATTX_NST = 4;   // tiles in flight
inline size_t attx_pv_smem(int G) { return (size_t)ATTX_NST * ATTX_PT * (ATTX_DIMS + G) * 4; }

__global__ void __launch_bounds__(8 * ATTX_DIMS) k_attx_pv(const __grid_constant__ AttnXArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float s_dyn[];
    const int G = a.heads / a.kv_heads;
    float *s_v = s_dyn;                                    // [NST][PT][DIMS]
    float *s_p = s_dyn + ATTX_NST * ATTX_PT * ATTX_DIMS;   // [NST][G][PT]
    const int kvh = blockIdx.x, seq = blockIdx.y, dc = blockIdx.z;
    const int tid = threadIdx.x, nthr = G * ATTX_DIMS, g = tid / ATTX_DIMS, j = tid - g * ATTX_DIMS;
    const int h = kvh * G + g;
    const int len = attx_len(a, seq);
    const long long slot = a.slots ? a.slots[seq] : seq;
    const float *vb = a.vc + slot * a.kv_slot + kvh * ATT_HD + dc * ATTX_DIMS;
    const float *pb = a.scores + ((long long)seq * a.heads + (long long)kvh * G) * a.max_len;
    const int ntile = (len + ATTX_PT - 1) / ATTX_PT;
    auto load_tile = [&](int k) {
        if (k < ntile) {
            const int t0 = k * ATTX_PT, nt = min(ATTX_PT, len - t0);
            float *dv = s_v + (k % ATTX_NST) * ATTX_PT * ATTX_DIMS;
            float *dp = s_p + (k % ATTX_NST) * G * ATTX_PT;
            for (int idx = tid; idx < nt * (ATTX_DIMS / 4); idx += nthr) {
                const int r = idx / (ATTX_DIMS / 4), c = idx - r * (ATTX_DIMS / 4);
                cp_async16(dv + r * ATTX_DIMS + c * 4, vb + (long long)(t0 + r) * a.kv_dim + c * 4);
            }
            for (int idx = tid; idx < G * nt; idx += nthr) {
                const int gg = idx / nt, r = idx - gg * nt;
                cp_async4(dp + gg * ATTX_PT + r, pb + (long long)gg * a.max_len + t0 + r);
            }
        }
        cp_async_commit();  // one group per tile index, empty past the end
    };
#pragma unroll
    for (int k = 0; k < ATTX_NST - 1; k++) load_tile(k);
    float acc = 0.0f;
    for (int k = 0; k < ntile; k++) {
        cp_async_wait<ATTX_NST - 2>();  // this thread's copies of tile k landed
        __syncthreads();                // everyone's; and tile k-1's buffer is no longer read
        load_tile(k + ATTX_NST - 1);
        const float *v = s_v + (k % ATTX_NST) * ATTX_PT * ATTX_DIMS + j;
        const float *p = s_p + (k % ATTX_NST) * G * ATTX_PT + g * ATTX_PT;
        const int nt = min(ATTX_PT, len - k * ATTX_PT);
#pragma unroll 8
        for (int r = 0; r < nt; r++) acc = __fadd_rn(acc, __fmul_rn(p[r], v[r * ATTX_DIMS]));
    }
    const int dim = dc * ATTX_DIMS + j;
    const float gt = a.gate[(long long)seq * a.q_tok + (long long)h * ATT_HD + dim];
    const float o = __fmul_rn(acc, sigmoid_f(gt));
    a.out[(long long)seq * a.out_tok + (long long)h * ATT_HD + dim] = o;
    if (a.fam == 32) {
        const int blk = (h * ATT_HD + dc * ATTX_DIMS) / 32 + (j >> 5);
        quant_q8_0_warp(o, a.xq + (long long)seq * a.xq_ld + (long long)blk * 34, j & 31);
    }
}

// dynamic shared-memory ceilings: the softmax stages max_len floats, the
// P.V ring needs attx_pv_smem(8) (a high-water mark; the engine calls this
// before any capture)
inline int attx_prepare(int max_len) {
    static size_t configured = 0;
    const size_t smem = std::max((size_t)max_len * 4, attx_pv_smem(8));
    if (smem <= configured) return 0;
    if ((size_t)max_len * 4 > 227 * 1024 - 1024) return (int)cudaErrorInvalidValue;
    int rc = (int)cudaFuncSetAttribute(k_attx_softmax, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)std::max((size_t)max_len * 4, (size_t)48 * 1024));
    if (!rc) rc = (int)cudaFuncSetAttribute(k_attx_pv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attx_pv_smem(8));
    if (rc) return rc;
    configured = smem;
    return 0;
}

inline int attx_launch(const AttnXArgs &a, int nseq, int max_len, cudaStream_t st) {
    if (nseq <= 0) return 0;
    if (a.kv_heads <= 0 || a.heads % a.kv_heads) return (int)cudaErrorInvalidValue;
    const int G = a.heads / a.kv_heads;
    if (max_len <= 0 || max_len > a.max_len) return (int)cudaErrorInvalidValue;
    const dim3 g1((unsigned)a.kv_heads, (unsigned)nseq, (unsigned)((max_len + ATTX_CHUNK - 1) / ATTX_CHUNK));
    int rc = 0;
    switch (G) {
    case 1: rc = launch_k(k_attx_scores<1>, g1, dim3(ATTX_CHUNK), 0, st, a); break;
    case 2: rc = launch_k(k_attx_scores<2>, g1, dim3(ATTX_CHUNK), 0, st, a); break;
    case 3: rc = launch_k(k_attx_scores<3>, g1, dim3(ATTX_CHUNK), 0, st, a); break;
    case 4: rc = launch_k(k_attx_scores<4>, g1, dim3(ATTX_CHUNK), 0, st, a); break;
    case 6: rc = launch_k(k_attx_scores<6>, g1, dim3(ATTX_CHUNK), 0, st, a); break;
    case 8: rc = launch_k(k_attx_scores<8>, g1, dim3(ATTX_CHUNK), 0, st, a); break;
    default: return (int)cudaErrorInvalidValue;
    }
    if (rc) return rc;
    Q35_TRY_RC(attx_prepare(max_len));
    rc = launch_k(k_attx_softmax, dim3((unsigned)a.heads, (unsigned)nseq), dim3(ATTX_SMT), (size_t)max_len * 4, st, a);
    if (rc) return rc;
    return launch_k(k_attx_pv, dim3((unsigned)a.kv_heads, (unsigned)nseq, ATT_HD / ATTX_DIMS), dim3(G * ATTX_DIMS),
                    attx_pv_smem(G), st, a);
}


// ---------------------------------------------------------------------------
// Prefill-shaped causal attention: the same three steps for a run of
// consecutive positions of ONE sequence (a prompt chunk), with the run's
// tokens tiled ATTP_QT at a time so that each K chunk and each V tile is
// loaded once per tile instead of once per token.  Token i of the run attends
// to lens[i] positions.  Every per-element operation and its order is the
// token-by-token kernels' (serial dots over dims, serial softmax sum, serial
// P.V over positions), so the results are identical bit for bit.
//   k_attp_scores: CTA (kv head, token tile, 32-position chunk), thread
//     (token of the tile, position of the chunk), the group's G dots;
//   k_attx_softmax: unchanged (a row per (head, token));
//   k_attp_pv: CTA (kv head, token tile, 64-dim chunk), thread (token, dim)
//     with the G heads' sums, V and probability tiles through a cp.async ring.
// ---------------------------------------------------------------------------
constexpr int ATTP_QT = 8;    // tokens per tile
constexpr int ATTP_NST = 3;   // P.V tiles in flight

inline size_t attp_scores_smem(int G) { return (size_t)(ATTX_CHUNK * ATTX_KLD + ATTP_QT * G * ATT_HD) * 4; }
inline size_t attp_pv_smem(int G) { return (size_t)ATTP_NST * ATTX_PT * (ATTX_DIMS + ATTP_QT * G) * 4; }

Q35_DEV int attp_len(const AttnXArgs &a, int t) { return attx_len(a, t); }

template <int G>
__global__ void __launch_bounds__(ATTX_CHUNK * ATTP_QT) k_attp_scores(const __grid_constant__ AttnXArgs a, int ntok) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float s_ps[];
    float *s_k = s_ps;                                // [CHUNK][KLD]
    float *s_q = s_ps + ATTX_CHUNK * ATTX_KLD;        // [QT][G][HD]
    const int kvh = blockIdx.x, t0 = blockIdx.y * ATTP_QT, p0 = blockIdx.z * ATTX_CHUNK;
    const int tid = threadIdx.x, ti = tid / ATTX_CHUNK, lane = tid - ti * ATTX_CHUNK;
    const int nt = min(ATTP_QT, ntok - t0);
    const int len_max = attp_len(a, t0 + nt - 1);  // positions ascend along the run
    if (p0 >= len_max) return;
    const int np = min(ATTX_CHUNK, len_max - p0);
    const long long slot = a.slots ? a.slots[t0] : 0;
    const float *kb = a.kc + slot * a.kv_slot + (long long)p0 * a.kv_dim + kvh * ATT_HD;
    for (int idx = tid; idx < np * (ATT_HD / 4); idx += blockDim.x) {
        const int r = idx / (ATT_HD / 4), c = idx - r * (ATT_HD / 4);
        cp_async16(&s_k[r * ATTX_KLD + c * 4], kb + (long long)r * a.kv_dim + c * 4);
    }
    cp_async_commit();
    for (int idx = tid; idx < nt * G * (ATT_HD / 4); idx += blockDim.x) {
        const int i = idx / (G * ATT_HD / 4), rem = idx - i * (G * ATT_HD / 4);
        const int g = rem / (ATT_HD / 4), c = rem - g * (ATT_HD / 4);
        reinterpret_cast<float4 *>(s_q + (i * G + g) * ATT_HD)[c] =
            reinterpret_cast<const float4 *>(a.q + (long long)(t0 + i) * a.q_tok + (long long)(kvh * G + g) * ATT_HD)[c];
    }
    cp_async_wait<0>();
    __syncthreads();
    if (ti >= nt || p0 + lane >= attp_len(a, t0 + ti)) return;
    float sc[G];
#pragma unroll
    for (int g = 0; g < G; g++) sc[g] = 0.0f;
    const float4 *kr = reinterpret_cast<const float4 *>(s_k + lane * ATTX_KLD);
    const float *qt = s_q + ti * G * ATT_HD;
#pragma unroll 4
    for (int c = 0; c < ATT_HD / 4; c++) {
        const float4 kv = kr[c];
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float4 qv = reinterpret_cast<const float4 *>(qt + g * ATT_HD)[c];
            sc[g] = __fadd_rn(sc[g], __fmul_rn(qv.x, kv.x));
            sc[g] = __fadd_rn(sc[g], __fmul_rn(qv.y, kv.y));
            sc[g] = __fadd_rn(sc[g], __fmul_rn(qv.z, kv.z));
            sc[g] = __fadd_rn(sc[g], __fmul_rn(qv.w, kv.w));
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++)
        a.scores[((long long)(t0 + ti) * a.heads + kvh * G + g) * a.max_len + p0 + lane] = __fmul_rn(sc[g], a.scale);
}

template <int G>
__global__ void __launch_bounds__(ATTP_QT * ATTX_DIMS) k_attp_pv(const __grid_constant__ AttnXArgs a, int ntok) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float s_pv[];
    constexpr int PW = ATTP_QT * G;                              // probability rows per tile
    float *s_v = s_pv;                                           // [NST][PT][DIMS]
    float *s_p = s_pv + ATTP_NST * ATTX_PT * ATTX_DIMS;          // [NST][QT*G][PT]
    const int kvh = blockIdx.x, t0 = blockIdx.y * ATTP_QT, dc = blockIdx.z;
    const int tid = threadIdx.x, ti = tid / ATTX_DIMS, j = tid - ti * ATTX_DIMS;
    const int nt = min(ATTP_QT, ntok - t0);
    const int len_max = attp_len(a, t0 + nt - 1);
    const int my_len = ti < nt ? attp_len(a, t0 + ti) : 0;
    const long long slot = a.slots ? a.slots[t0] : 0;
    const float *vb = a.vc + slot * a.kv_slot + kvh * ATT_HD + dc * ATTX_DIMS;
    const int ntile = (len_max + ATTX_PT - 1) / ATTX_PT;
    auto load_tile = [&](int k) {
        if (k < ntile) {
            const int q0 = k * ATTX_PT, np = min(ATTX_PT, len_max - q0);
            float *dv = s_v + (k % ATTP_NST) * ATTX_PT * ATTX_DIMS;
            float *dp = s_p + (k % ATTP_NST) * PW * ATTX_PT;
            for (int idx = tid; idx < np * (ATTX_DIMS / 4); idx += blockDim.x) {
                const int r = idx / (ATTX_DIMS / 4), c = idx - r * (ATTX_DIMS / 4);
                cp_async16(dv + r * ATTX_DIMS + c * 4, vb + (long long)(q0 + r) * a.kv_dim + c * 4);
            }
            // probability rows: only positions a token attends to were written
            for (int idx = tid; idx < nt * G * np; idx += blockDim.x) {
                const int row = idx / np, r = idx - row * np;
                const int i = row / G, g = row - i * G;
                if (q0 + r < attp_len(a, t0 + i))
                    cp_async4(dp + row * ATTX_PT + r,
                              a.scores + ((long long)(t0 + i) * a.heads + kvh * G + g) * a.max_len + q0 + r);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int k = 0; k < ATTP_NST - 1; k++) load_tile(k);
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; g++) acc[g] = 0.0f;
    for (int k = 0; k < ntile; k++) {
        cp_async_wait<ATTP_NST - 2>();
        __syncthreads();
        load_tile(k + ATTP_NST - 1);
        const float *v = s_v + (k % ATTP_NST) * ATTX_PT * ATTX_DIMS + j;
        const float *p = s_p + (k % ATTP_NST) * PW * ATTX_PT + ti * G * ATTX_PT;
        const int nr = max(0, min(ATTX_PT, my_len - k * ATTX_PT));
        for (int r = 0; r < nr; r++) {
            const float vv = v[r * ATTX_DIMS];
#pragma unroll
            for (int g = 0; g < G; g++) acc[g] = __fadd_rn(acc[g], __fmul_rn(p[g * ATTX_PT + r], vv));
        }
    }
    if (ti >= nt) return;
    const long long tok = t0 + ti;
#pragma unroll
    for (int g = 0; g < G; g++) {
        const int h = kvh * G + g, dim = dc * ATTX_DIMS + j;
        const float gt = a.gate[tok * a.q_tok + (long long)h * ATT_HD + dim];
        const float o = __fmul_rn(acc[g], sigmoid_f(gt));
        a.out[tok * a.out_tok + (long long)h * ATT_HD + dim] = o;
        if (a.fam == 32) {
            const int blk = (h * ATT_HD + dc * ATTX_DIMS) / 32 + (j >> 5);
            quant_q8_0_warp(o, a.xq + tok * a.xq_ld + (long long)blk * 34, j & 31);
        }
    }
}

template <int G>
inline int attp_launch_g(const AttnXArgs &a, int ntok, int max_len, cudaStream_t st) {
    static bool ready = false;
    if (!ready) {
        int rc = (int)cudaFuncSetAttribute(k_attp_scores<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)attp_scores_smem(G));
        if (!rc) rc = (int)cudaFuncSetAttribute(k_attp_pv<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)attp_pv_smem(G));
        if (rc) return rc;
        ready = true;
    }
    const unsigned tiles = (unsigned)((ntok + ATTP_QT - 1) / ATTP_QT);
    Q35_TRY_RC(launch_k(k_attp_scores<G>, dim3((unsigned)a.kv_heads, tiles, (unsigned)((max_len + ATTX_CHUNK - 1) / ATTX_CHUNK)),
                        dim3(ATTX_CHUNK * ATTP_QT), attp_scores_smem(G), st, a, ntok));
    Q35_TRY_RC(attx_prepare(max_len));
    Q35_TRY_RC(launch_k(k_attx_softmax, dim3((unsigned)a.heads, (unsigned)ntok), dim3(ATTX_SMT), (size_t)max_len * 4, st,
                        a));
    return launch_k(k_attp_pv<G>, dim3((unsigned)a.kv_heads, tiles, ATT_HD / ATTX_DIMS), dim3(ATTP_QT * ATTX_DIMS),
                    attp_pv_smem(G), st, a, ntok);
}

// a run of ntok tokens of one sequence (a.slots[0..ntok) all the same slot,
// or none: slot 0; lengths ascending: a.lens, or len_imm + len_step * t);
// max_len bounds the lengths.  -1: this group size is not served
inline int attp_launch(const AttnXArgs &a, int ntok, int max_len, cudaStream_t st) {
    if (ntok <= 0) return 0;
    if (a.kv_heads <= 0 || a.heads % a.kv_heads) return (int)cudaErrorInvalidValue;
    if (max_len <= 0 || max_len > a.max_len) return (int)cudaErrorInvalidValue;
    switch (a.heads / a.kv_heads) {
    case 1: return attp_launch_g<1>(a, ntok, max_len, st);
    case 2: return attp_launch_g<2>(a, ntok, max_len, st);
    case 4: return attp_launch_g<4>(a, ntok, max_len, st);
    case 6: return attp_launch_g<6>(a, ntok, max_len, st);
    case 8: return attp_launch_g<8>(a, ntok, max_len, st);
    default: return -1;
    }
}

// ---------------------------------------------------------------------------
// Fused decode attention for short contexts: prelude + scores + softmax +
// P.V in ONE launch.  A cluster of ATTF_CS CTAs owns one (kv head, sequence);
// the CTAs exchange through distributed shared memory:
//   A. prelude: CTA g < G normalises / rotates q head g (RMSNorm with the
//      serial sum, RoPE of dims 0..63); CTA kp = G % ATTF_CS does the kv
//      head's k (norm, RoPE) and appends k and v to the cache at pos
//      (engine.zig:1975-2010, the CPU operations of k_attn_prelude);
//   B. scores: positions in 32-position chunks, chunk c on CTA c % ATTF_CS;
//      thread (g, t) forms q_g . k_t over the 256 dims in order, times the
//      scale (elementwise.zig:349-356);
//   C. softmax: every CTA gathers the whole score rows of its G heads and
//      takes max, exp(s - max), the serial sum in position order and the
//      division (elementwise.zig:357-366);
//   D. P.V: CTA r owns dims 32r .. 32r+31 of the G heads: acc += p_t * v_t
//      in position order (elementwise.zig:367-372), then the sigmoid gate
//      and, for a Q8_0 consumer, the quantized block (one warp = one block).
// Same operations in the same order as the separate kernels, so the results
// are identical; what goes away is three launches and the score round trips.
// ---------------------------------------------------------------------------
constexpr int ATTF_CS = 8;        // CTAs per cluster (dims 32 x 8 = 256)
constexpr int ATTF_THREADS = 256;
constexpr int ATTF_MAX_LEN = 1024;
constexpr int ATTF_VT = 64;       // V rows per staged tile
constexpr int ATTF_VST = 3;       // V tiles in flight

struct AttfArgs {
    const float *qg;      // [n][heads][q_h | gate_h] (2 * q_dim per token)
    const float *kb, *vb; // [n][kv_dim]: this step's k and v projections
    const float *qw, *kw; // q / k RMSNorm weights (256)
    float eps, base, scale;
    const int *pos, *slots;
    float *kc, *vc;       // KV pools of this layer: [slot][max_seq][kv_dim]
    long long kv_slot;
    int heads, kv_heads;
    float *out;           // gated attention output, [n][q_dim]
    int fam;              // 32: also quantize the output into xq
    uint8_t *xq;
    long long xq_ld;
    const float2 *rope;   // (cos, sin) per (position, pair), or null: evaluated here
};

inline size_t attf_smem(int G) {
    // q rows | own head (k or q) | v row | K chunk | own scores | all scores | V ring
    return (size_t)(G * ATT_HD + 2 * ATT_HD + ATT_HD + ATTX_CHUNK * ATTX_KLD + 2 * G * ATTF_MAX_LEN +
                    ATTF_VST * ATTF_VT * 32) * 4;
}

Q35_DEV float *attf_remote(float *p, int rank) {
    uint32_t a = smem_u32(p), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return reinterpret_cast<float *>((uintptr_t)r);  // a shared::cluster address, read with attf_ld
}
Q35_DEV float attf_ld(const float *p) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"((uint32_t)(uintptr_t)p) : "memory");
    return v;
}
Q35_DEV void attf_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
Q35_DEV int attf_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return (int)r;
}

// RMSNorm (serial sum of squares) then RoPE on dims 0..63 of one 256-float
// head vector in shared memory, by the whole CTA (as k_attn_prelude); the
// rotation's cos / sin (threads 0..31) are computed by the caller
Q35_DEV void attf_norm_rope(float *y, const float *wn, float eps, float rc, float rs, float *s_ss) {
    const int j = threadIdx.x;
    const float x = y[j];
    __syncthreads();
    if (j == 0) *s_ss = serial_sumsq(y, ATT_HD);
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(*s_ss, (float)ATT_HD), eps)));
    y[j] = __fmul_rn(__fmul_rn(x, scale), wn[j]);
    __syncthreads();
    if (j < 32) {
        const float a = y[j], b = y[j + 32];
        y[j] = __fsub_rn(__fmul_rn(a, rc), __fmul_rn(b, rs));
        y[j + 32] = __fadd_rn(__fmul_rn(a, rs), __fmul_rn(b, rc));
    }
    __syncthreads();
}

__global__ void __launch_bounds__(ATTF_THREADS) k_attn_fused(const __grid_constant__ AttfArgs a) {
    pdl_trigger();
    extern __shared__ __align__(16) float s_f[];
    __shared__ float s_ss, s_red[ATTF_THREADS / 32];
    const int G = a.heads / a.kv_heads;
    const int r = attf_rank(), kvh = blockIdx.y, seq = blockIdx.z, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    float *s_q = s_f;                              // [G][256]  all q rows (gathered)
    float *s_own = s_q + G * ATT_HD;               // [2][256]  this CTA's q row / k row
    float *s_vrow = s_own + 2 * ATT_HD;            // [256]     this step's v row
    float *s_k = s_vrow + ATT_HD;                  // [32][ATTX_KLD]
    float *s_sc = s_k + ATTX_CHUNK * ATTX_KLD;     // [G][MAX_LEN] own scores
    float *s_p = s_sc + G * ATTF_MAX_LEN;          // [G][MAX_LEN] gathered rows -> probabilities
    float *s_v = s_p + G * ATTF_MAX_LEN;           // [VST][VT][32]
    // Before the dependency wait: the batch descriptor (uploaded before the
    // step) and the rotation for this position (pow / cos / sin, the slow
    // part of the prelude)
    const int p = a.pos[seq], len = p + 1;
    const long long slot = a.slots[seq];
    float rc = 1.0f, rs = 0.0f;
    if (tid < 32) rope_lookup(a.rope, p, a.base, tid, rc, rs);
    pdl_wait();
    const int q_dim = a.heads * ATT_HD, kv_dim = a.kv_heads * ATT_HD;
    const int kp = G % ATTF_CS;  // the CTA doing the k head
    float *kdst = a.kc + slot * a.kv_slot + (long long)p * kv_dim + kvh * ATT_HD;
    float *vdst = a.vc + slot * a.kv_slot + (long long)p * kv_dim + kvh * ATT_HD;

    // ---- A: prelude ----
    if (r < G) {
        const int h = kvh * G + r;
        s_own[tid] = a.qg[(long long)seq * 2 * q_dim + (long long)h * 2 * ATT_HD + tid];
        attf_norm_rope(s_own, a.qw, a.eps, rc, rs, &s_ss);
    }
    if (r == kp) {
        float *yk = s_own + ATT_HD;
        yk[tid] = a.kb[(long long)seq * kv_dim + kvh * ATT_HD + tid];
        const float v = a.vb[(long long)seq * kv_dim + kvh * ATT_HD + tid];
        s_vrow[tid] = v;
        attf_norm_rope(yk, a.kw, a.eps, rc, rs, &s_ss);
        // the cache rows for later steps; this kernel reads position p's k and
        // v from this CTA's shared memory instead
        kdst[tid] = yk[tid];
        vdst[tid] = v;
    }
    attf_cluster_sync();

    // ---- B: scores of this CTA's position chunks ----
    for (int i = tid; i < G * ATT_HD; i += ATTF_THREADS) {
        const int g = i / ATT_HD, d = i - g * ATT_HD;
        s_q[i] = attf_ld(attf_remote(s_own + d, g));
    }
    const float *kbase = a.kc + slot * a.kv_slot + kvh * ATT_HD;
    for (int c = r; c * ATTX_CHUNK < len; c += ATTF_CS) {
        const int p0 = c * ATTX_CHUNK, np = min(ATTX_CHUNK, len - p0);
        const int ncache = min(np, p - p0);  // rows from the cache; row p (if in the chunk) from the k CTA
        __syncthreads();  // s_k free (previous chunk done), s_q complete
        for (int idx = tid; idx < ncache * (ATT_HD / 4); idx += ATTF_THREADS) {
            const int rr = idx / (ATT_HD / 4), cc = idx - rr * (ATT_HD / 4);
            cp_async16(&s_k[rr * ATTX_KLD + cc * 4], kbase + (long long)(p0 + rr) * kv_dim + cc * 4);
        }
        cp_async_commit();
        if (ncache < np) s_k[(p - p0) * ATTX_KLD + tid] = attf_ld(attf_remote(s_own + ATT_HD + tid, kp));
        cp_async_wait<0>();
        __syncthreads();
        for (int w = warp; w < G; w += ATTF_THREADS / 32) {
            if (lane < np) {
                const float4 *kr = reinterpret_cast<const float4 *>(s_k + lane * ATTX_KLD);
                const float4 *qr = reinterpret_cast<const float4 *>(s_q + w * ATT_HD);
                float sacc = 0.0f;
#pragma unroll 8
                for (int d4 = 0; d4 < ATT_HD / 4; d4++) {
                    const float4 kv = kr[d4], qv = qr[d4];
                    sacc = __fadd_rn(sacc, __fmul_rn(qv.x, kv.x));
                    sacc = __fadd_rn(sacc, __fmul_rn(qv.y, kv.y));
                    sacc = __fadd_rn(sacc, __fmul_rn(qv.z, kv.z));
                    sacc = __fadd_rn(sacc, __fmul_rn(qv.w, kv.w));
                }
                s_sc[w * ATTF_MAX_LEN + p0 + lane] = __fmul_rn(sacc, a.scale);
            }
        }
    }
    // position p's v row, this CTA's 32 dims (before the barrier below, the
    // last point at which the k CTA's shared memory may be read)
    float *s_vp = s_vrow;  // reused: [32]
    const float vp_own = tid < 32 ? attf_ld(attf_remote(s_vrow + r * 32 + tid, kp)) : 0.0f;
    attf_cluster_sync();

    // ---- C: whole score rows, softmax ----
    for (int i = tid; i < G * len; i += ATTF_THREADS) {
        const int g = i / len, t = i - g * len;
        const int owner = (t / ATTX_CHUNK) % ATTF_CS;
        s_p[g * ATTF_MAX_LEN + t] = attf_ld(attf_remote(s_sc + g * ATTF_MAX_LEN + t, owner));
    }
    attf_cluster_sync();  // no remote reads after this point: CTAs may finish independently
    if (tid < 32) s_vp[tid] = vp_own;
    // all heads at once: warp w serves head w % G (positions strided over the
    // head's warps); max in any order, then exp(s - max)
    const int hg = warp % G, hq = warp / G, hn = (ATTF_THREADS / 32 - hg + G - 1) / G;
    {
        float *row = s_p + hg * ATTF_MAX_LEN;
        float m = -3.40282347e38f;
        for (int t = hq * 32 + lane; t < len; t += hn * 32) m = fmaxf(m, row[t]);
        m = warp_max(m);
        if (lane == 0) s_red[warp] = m;
        __syncthreads();
        m = s_red[hg];
        for (int w = hg + G; w < ATTF_THREADS / 32; w += G) m = fmaxf(m, s_red[w]);
        for (int t = hq * 32 + lane; t < len; t += hn * 32) row[t] = exp_f(__fsub_rn(row[t], m));
    }
    __syncthreads();
    if (lane == 0 && warp < G) {  // one thread per head: the serial sum, loads running ahead of the adds
        const float *row = s_p + warp * ATTF_MAX_LEN;
        float sum = 0.0f;
        int t = 0;
        for (; t + 32 <= len; t += 32) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = row[t + i];
#pragma unroll
            for (int i = 0; i < 32; i++) sum = __fadd_rn(sum, v[i]);
        }
        for (; t < len; t++) sum = __fadd_rn(sum, row[t]);
        s_red[warp] = sum;
    }
    __syncthreads();
    for (int i = tid; i < G * len; i += ATTF_THREADS) {
        const int g = i / len, t = i - g * len;
        s_p[g * ATTF_MAX_LEN + t] = __fdiv_rn(s_p[g * ATTF_MAX_LEN + t], s_red[g]);
    }

    // ---- D: P.V for dims 32r .. 32r+31 ----
    const float *vbase = a.vc + slot * a.kv_slot + kvh * ATT_HD + r * 32;
    const int ntile = (len + ATTF_VT - 1) / ATTF_VT;
    auto load_tile = [&](int k) {
        if (k < ntile) {
            const int t0 = k * ATTF_VT, nt = min(ATTF_VT, p - t0);  // row p comes from s_vp
            float *dv = s_v + (k % ATTF_VST) * ATTF_VT * 32;
            for (int idx = tid; idx < nt * 8; idx += ATTF_THREADS) {
                const int rr = idx >> 3, cc = idx & 7;
                cp_async16(dv + rr * 32 + cc * 4, vbase + (long long)(t0 + rr) * kv_dim + cc * 4);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int k = 0; k < ATTF_VST - 1; k++) load_tile(k);
    const int g = warp, dl = lane;  // thread = (head g of the group, dim 32r + dl)
    float acc = 0.0f;
    for (int k = 0; k < ntile; k++) {
        cp_async_wait<ATTF_VST - 2>();
        __syncthreads();  // tile k landed everywhere; tile k-1's buffer is free (and s_p, s_vp are final)
        load_tile(k + ATTF_VST - 1);
        if (g < G) {
            const float *v = s_v + (k % ATTF_VST) * ATTF_VT * 32 + dl;
            const float *pr = s_p + g * ATTF_MAX_LEN + k * ATTF_VT;
            const int t0 = k * ATTF_VT, nt = min(ATTF_VT, len - t0);
            const int nc = min(nt, p - t0);  // cached rows of this tile
#pragma unroll 8
            for (int t = 0; t < nc; t++) acc = __fadd_rn(acc, __fmul_rn(pr[t], v[t * 32]));
            if (nc < nt) acc = __fadd_rn(acc, __fmul_rn(pr[nc], s_vp[dl]));  // position p, the last
        }
    }
    cp_async_wait<0>();
    if (g < G) {
        const int h = kvh * G + g, dim = r * 32 + dl;
        const float gt = a.qg[(long long)seq * 2 * q_dim + (long long)h * 2 * ATT_HD + ATT_HD + dim];
        const float o = __fmul_rn(acc, sigmoid_f(gt));
        a.out[(long long)seq * q_dim + (long long)h * ATT_HD + dim] = o;
        if (a.fam == 32) quant_q8_0_warp(o, a.xq + (long long)seq * a.xq_ld + (long long)(h * 8 + r) * 34, lane);
    }
}

inline int attf_prepare() {
    static int done = 0;
    if (done) return 0;
    const int rc = (int)cudaFuncSetAttribute(k_attn_fused, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)attf_smem(8));
    if (!rc) done = 1;
    return rc;
}

// Returns -1 (nothing launched) when the fused kernel does not apply: heads
// of 256 only, G <= 8, contexts up to ATTF_MAX_LEN positions, batches that
// fit in one wave of clusters.
inline int attf_launch(const AttfArgs &a, int nseq, int max_len, cudaStream_t st) {
    if (nseq <= 0) return 0;
    if (a.kv_heads <= 0 || a.heads % a.kv_heads) return -1;
    const int G = a.heads / a.kv_heads;
    if (G > 8 || max_len > ATTF_MAX_LEN) return -1;
    // one wave (two clusters' CTAs per SM): beyond that the split kernels,
    // which parallelise over positions without a cluster, are faster
    if ((long long)nseq * a.kv_heads * ATTF_CS > 2LL * gemv_sm_count()) return -1;
    Q35_TRY_RC(attf_prepare());
    launch_count()++;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ATTF_CS, (unsigned)a.kv_heads, (unsigned)nseq);
    cfg.blockDim = dim3(ATTF_THREADS);
    cfg.dynamicSmemBytes = attf_smem(G);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ATTF_CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return (int)cudaLaunchKernelEx(&cfg, k_attn_fused, a);
}

}  // namespace q35
