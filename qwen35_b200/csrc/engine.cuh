// engine.cuh -- batched decode step of the Qwen3.5 hybrid model on B200.
//
// The op order per layer is src/engine.zig's forwardGdn (:1505-1672),
// forwardFull (:1949-2023) and forwardMlp (:2027-2036); the model head is
// forwardLogits (:1242-1312) with greedy argmax.  What is new here (the
// reference is a single-sequence engine) is the batch: one step advances n
// independent sequences by one token each, every sequence owning a slot in
// the KV / GDN-state pools, with per-sequence positions read from device
// memory so the whole step is one CUDA graph that replays for any positions.
//
// Kernels per layer (n tokens): fused rmsnorm+quantize -> one multi-matrix
// GEMV launch -> layer core (conv/gamma/l2norm + GDN state step, or q/k norm
// + RoPE + KV append + split-KV attention) -> fused norm/gate+quantize ->
// GEMV with the residual add in its epilogue -> MLP (norm+quantize, gate|up
// GEMV, swiglu+quantize, down GEMV + residual).
#pragma once
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "tp.cuh"

namespace q35 {

// ---------------------------------------------------------------------------
// fused producers of quantized activations (warp per quant block)
// ---------------------------------------------------------------------------
__host__ __device__ inline long long act_row_bytes(int cols, int fam) {
    return fam == 32 ? (long long)(cols / 32) * 34 : (long long)(cols / 256) * 292;
}

// quantize a row whose element i is produced by `f(i)`; called by whole CTA
template <class F>
Q35_DEV void quantize_row_cta(F f, int cols, int fam, uint8_t *dst) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (fam == 32) {
        for (int b = warp; b < cols / 32; b += nw) quant_q8_0_warp(f(b * 32 + lane), dst + (size_t)b * 34, lane);
    } else {
        for (int b = warp; b < cols / 256; b += nw) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = f(b * 256 + lane * 8 + i);
            quant_q8_K_warp(v, dst + (size_t)b * 292, lane);
        }
    }
}

// rmsnorm(x_row, w) -> quantized activation (CTA per token)
__global__ void __launch_bounds__(256) k_rmsnorm_quant(const float *x, const float *w, int cols, float eps, int fam,
                                                       uint8_t *xq, long long xq_ld, const int *active) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    if (active && !active[t]) return;
    const float *xr = x + (long long)t * cols;
    extern __shared__ __align__(16) float xs[];  // cols floats
    for (int i = threadIdx.x; i < cols; i += blockDim.x) xs[i] = xr[i];
    __syncthreads();
    const float ss = cta_spec_sumsq(xs, cols);  // the serial order's sum, segments in parallel
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), eps)));
    quantize_row_cta([&](int i) { return __fmul_rn(__fmul_rn(xs[i], scale), w[i]); }, cols, fam,
                     xq + (long long)t * xq_ld);
}

// silu(g)*u -> quantized activation; grid (blocks, tokens), warp per block
__global__ void __launch_bounds__(256) k_swiglu_quant(const float *g, const float *u, int cols, int fam, uint8_t *xq,
                                                      long long xq_ld) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    const float *gr = g + (long long)t * cols, *ur = u + (long long)t * cols;
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
    uint8_t *dst = xq + (long long)t * xq_ld;
    if (fam == 32) {
        if (b >= cols / 32) return;
        const int i = b * 32 + lane;
        quant_q8_0_warp(__fmul_rn(silu_f(gr[i]), ur[i]), dst + (size_t)b * 34, lane);
    } else {
        if (b >= cols / 256) return;
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int i = b * 256 + lane * 8 + k;
            v[k] = __fmul_rn(silu_f(gr[i]), ur[i]);
        }
        quant_q8_K_warp(v, dst + (size_t)b * 292, lane);
    }
}

// plain f32 rows -> quantized activation; grid (blocks, tokens)
__global__ void __launch_bounds__(256) k_quant_rows(const float *x, long long x_ld, int cols, int fam, uint8_t *xq,
                                                    long long xq_ld) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    const float *xr = x + (long long)t * x_ld;
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
    uint8_t *dst = xq + (long long)t * xq_ld;
    if (fam == 32) {
        if (b >= cols / 32) return;
        quant_q8_0_warp(xr[b * 32 + lane], dst + (size_t)b * 34, lane);
    } else {
        if (b >= cols / 256) return;
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = xr[b * 256 + lane * 8 + k];
        quant_q8_K_warp(v, dst + (size_t)b * 292, lane);
    }
}

// ---------------------------------------------------------------------------
// attention prelude: q/gate split, q/k RMSNorm, RoPE at pos[t], KV append
// CTA (head index, token): heads q heads then kv_heads kv heads; hd = 256
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_attn_prelude(const float *qg, const float *kb, const float *vb, float *q,
                                                      float *gate, const float *qw, const float *kw, int heads,
                                                      int kv_heads, float eps, float base, const int *pos,
                                                      const int *slots, float *kpool, float *vpool, long long kv_slot,
                                                      const float2 *rope) {
    pdl_trigger();
    pdl_wait();
    __shared__ float y[256];
    const int hi = blockIdx.x, t = blockIdx.y, j = threadIdx.x;
    const int hd = 256, q_dim = heads * hd, kv_dim = kv_heads * hd;
    float x;
    const float *wn;
    if (hi < heads) {
        const float *src = qg + (long long)t * 2 * q_dim + (long long)hi * 2 * hd;
        x = src[j];
        gate[(long long)t * q_dim + hi * hd + j] = src[hd + j];
        wn = qw;
    } else {
        x = kb[(long long)t * kv_dim + (hi - heads) * hd + j];
        wn = kw;
    }
    y[j] = x;
    __syncthreads();
    __shared__ float sss;
    if (j == 0) sss = serial_sumsq(y, hd);
    __syncthreads();
    const float ss = sss;
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), eps)));
    y[j] = __fmul_rn(__fmul_rn(x, scale), wn[j]);
    __syncthreads();
    const int p = pos[t];
    if (j < 32) {
        float c, s;
        rope_lookup(rope, p, base, j, c, s);
        const float a = y[j], b = y[j + 32];
        y[j] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        y[j + 32] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    __syncthreads();
    if (hi < heads) {
        q[(long long)t * q_dim + hi * hd + j] = y[j];
    } else {
        const int kh = hi - heads;
        const long long base_off = (long long)slots[t] * kv_slot + (long long)p * kv_dim + kh * hd + j;
        kpool[base_off] = y[j];
        vpool[base_off] = vb[(long long)t * kv_dim + kh * hd + j];
    }
}

// lengths from positions; positions outside [0, max_seq) and slots outside
// [0, n_slots) are clamped in place (error 161 / 162 recorded), so the step's
// KV, state and RoPE indexing stays inside the pools whatever the inputs
__global__ void k_pos_to_len(int *pos, int *slots, int *len, int n, int max_seq, int n_slots) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        int p = pos[i];
        if (p < 0 || p >= max_seq) {
            set_error(161);
            p = p < 0 ? 0 : max_seq - 1;
            pos[i] = p;
        }
        const int s = slots[i];
        if (s < 0 || s >= n_slots) {
            set_error(162);
            slots[i] = 0;
        }
        len[i] = p + 1;
    }
}

__global__ void k_copy_rows(float *dst, const float *src, long long n) {
    pdl_trigger();
    pdl_wait();
    Q35_GRID_STRIDE(i, n) dst[i] = src[i];
}

__global__ void k_zero_bytes(uint8_t *p, long long n) {
    Q35_GRID_STRIDE(i, n) p[i] = 0;
}

// ---------------------------------------------------------------------------
// engine
// ---------------------------------------------------------------------------
struct Lin {
    const uint8_t *w = nullptr;
    int tt = -1;
    long long rows = 0, cols = 0;
};
struct LayerW {
    const float *attn_norm = nullptr, *post_norm = nullptr;
    Lin qkv, gate, alpha, beta, ssm_out;
    const float *conv1d = nullptr, *dt_bias = nullptr, *ssm_a = nullptr, *ssm_norm = nullptr;
    Lin q, k, v, o;
    const float *q_norm = nullptr, *k_norm = nullptr;
    Lin ffn_gate, ffn_up, ffn_down;
};

}  // namespace q35

struct q35b_engine {
    q35b_config c;
    int n_slots = 0, max_seq = 0, max_batch = 0;
    q35::Lin token_embd, output;
    const float *output_norm = nullptr;
    std::vector<q35::LayerW> L;
    std::vector<int> gdn_idx, full_idx;  // per layer: index into its pool (-1 if other kind)
    bool finalized = false, probe = false;
    int device = 0;
    // pools
    float *conv_pool = nullptr, *state_pool = nullptr, *kpool = nullptr, *vpool = nullptr;
    long long conv_slot = 0, state_slot = 0, kv_slot = 0;
    // per-step buffers
    int *d_in = nullptr;  // tokens | slots | pos | run_end (4 * max_batch)
    int *h_io = nullptr;
    float2 *rope_tab = nullptr;  // RoPE (cos, sin) per (position, pair): [max_seq][32]  // pinned host staging: tokens | slots | pos (as d_in), then next (max_batch)
    int *d_len = nullptr, *d_next = nullptr;
    float *x = nullptr, *qkv = nullptr, *z = nullptr, *ab = nullptr, *gam = nullptr, *gout = nullptr;
    float *q = nullptr, *gate = nullptr, *kb = nullptr, *vb = nullptr, *mh = nullptr, *mh1 = nullptr;
    float *logits = nullptr, *scores = nullptr, *probe_buf = nullptr;
    float *xh = nullptr;  // last row of each run, gathered for the model head
    bool gdn_wy = false;  // prefill runs through the chunked (WY) GDN form
    // WY scratch (allocated at the first WY forward): conv'd / normalised
    // q | k | v, log decays | betas, the recurrence output, Gram blocks
    float *wy_q = nullptr, *wy_k = nullptr, *wy_v = nullptr, *wy_lg = nullptr, *wy_beta = nullptr, *wy_o = nullptr;
    float *wy_g = nullptr;
    size_t wy_g_bytes = 0;
    // the current forward's runs as the host passed them (prefill forwards)
    std::vector<int> h_run_end, h_run_slot;
    bool sampling = false;  // next tokens drawn by the device sampler (per-slot parameters) instead of argmax
    int *samp = nullptr;    // per-slot sampler control blocks [n_slots][SC_INTS]
    // tensor parallelism (1 rank: off)
    int tp_n = 1, tp_rank = 0;
    long long vocab_local = 0, vocab_off = 0;  // this rank's lm_head rows
    ncclComm_t comm = nullptr;
    float *part = nullptr;                     // row-parallel partial sums [n][hidden]
    // the peer all-reduce (k_tp_allreduce_add): its own partial-sum buffer
    // (never handed to NCCL, whose graph-captured collectives may register
    // `part` with the driver), flag words and epoch state, every rank's
    // buffers as mapped here, the mappings opened, and the mode
    float *ppart = nullptr;
    int *ar_flags = nullptr, *ar_state = nullptr;
    q35::TpPeers peers{};
    bool peers_open = false, ar_peer = false;
    std::vector<void *> ipc_open;
    unsigned long long ar_limit_ns = 5000000000ull;
    int *am_pair = nullptr, *am_all = nullptr; // (max, index) per run: local / every rank
    float *am_v = nullptr;                     // split argmax partials [max_batch][AM_SPLIT]
    float *mmq_terms = nullptr;                // split-K terms of the K-quant MMQ (row-parallel projections)
    size_t mmq_terms_bytes = 0;
    int *am_i = nullptr;
    unsigned *am_cnt = nullptr;                // per row arrival counters (kept at zero between uses)
    uint8_t *xq = nullptr;
    long long xq_ld = 0;
    std::map<long long, cudaGraphExec_t> graphs;
    std::vector<void *> allocs;
    long long launches = 0;
};

namespace q35 {

inline int eng_alloc(q35b_engine *e, void **p, size_t bytes) {
    cudaError_t r = cudaMalloc(p, bytes ? bytes : 16);
    if (r != cudaSuccess) return (int)r;
    e->allocs.push_back(*p);
    return 0;
}

inline bool is_full_layer(const q35b_config &c, int li) {
    return c.full_attention_interval > 0 && li % c.full_attention_interval == c.full_attention_interval - 1;
}

#define Q35_TRY(x)                 \
    do {                           \
        int _rc = (x);             \
        if (_rc) return _rc;       \
    } while (0)

// one GEMV launch over up to 4 matrices of the same family sharing `xq`
inline int eng_gemv(q35b_engine *e, int n, std::initializer_list<GemvSegDesc> segs, const uint8_t *xq, int cols,
                    cudaStream_t st) {
    return gemv_launch(segs.begin(), (int)segs.size(), xq, cols, n, st, e->xq_ld, e->mmq_terms, e->mmq_terms_bytes);
}

inline int family_of(const Lin &l) { return geom_of(l.tt).family; }
inline long long weight_row_bytes(int tt, long long cols) {
    const Geom g = geom_of(tt);
    return g.elems ? cols / g.elems * g.bytes : 0;
}

inline int eng_rmsnorm_quant(q35b_engine *e, int n, const float *w, int fam, cudaStream_t st,
                             const float *src = nullptr) {
    return launch_k(k_rmsnorm_quant, dim3(n), dim3(256), (size_t)e->c.hidden * 4, st, src ? src : (const float *)e->x, w,
                    e->c.hidden, e->c.rms_eps, fam,
                    e->xq, e->xq_ld, (const int *)nullptr);
}

// rmsnorm(x) * w -> quantize -> GEMV: one launch where the lane-per-row GEMV
// takes the matrices (it builds the activation itself), else two
inline int eng_norm_gemv(q35b_engine *e, int n, const float *w, std::initializer_list<GemvSegDesc> segs,
                         cudaStream_t st, const float *src = nullptr) {
    const float *x = src ? src : e->x;
    const LprPrologue pro{LPR_PRO_NORM, x, nullptr, w, (long long)e->c.hidden, e->c.rms_eps};
    const int rc = gemv_lpr_launch(segs.begin(), (int)segs.size(), nullptr, e->c.hidden, n, st, e->xq_ld, &pro);
    if (rc != -1) return rc;
    Q35_TRY(eng_rmsnorm_quant(e, n, w, geom_of(segs.begin()->ttype).family, st, x));
    return eng_gemv(e, n, segs, e->xq, e->c.hidden, st);
}

// Row-parallel projections (attn_output, ssm_out, ffn_down) add into the
// residual stream.  Under tensor parallelism they write partial sums, which
// are all-reduced over the ranks and then added.
inline GemvSegDesc eng_rowpar_seg(q35b_engine *e, const Lin &w) {
    if (e->tp_n > 1) return {w.w, e->ar_peer ? e->ppart : e->part, w.rows, w.tt, (long long)e->c.hidden, GV_STORE};
    return {w.w, e->x, w.rows, w.tt, (long long)e->c.hidden, GV_ADD};
}
inline int eng_rowpar_finish(q35b_engine *e, int n, cudaStream_t st) {
    if (e->tp_n <= 1) return 0;
    if (e->ar_peer) {
        const TpArArgs a{e->peers, e->ar_state, e->tp_rank, e->tp_n, e->c.hidden, n, e->ar_limit_ns};
        return tp_ar_launch(a, st);
    }
    const long long cnt = (long long)n * e->c.hidden;
    const NcclApi &api = nccl_api();
    if (api.all_reduce(e->part, e->part, (size_t)cnt, ncclFloat32, ncclSum, e->comm, st) != ncclSuccess)
        return (int)cudaErrorUnknown;
    return launch_k(k_add_rows, dim3((unsigned)std::min<long long>((cnt + 255) / 256, 1024)), dim3(256), 0, st, e->x,
                    (const float *)e->part, cnt);
}

inline int eng_layer_gdn(q35b_engine *e, int li, int n, int nrun, cudaStream_t st) {
    const q35b_config &c = e->c;
    const LayerW &W = e->L[li];
    const int nv = c.gdn_n_heads, nk = c.gdn_num_k_heads, kd = c.gdn_head_dim;
    const int kq = nk * kd, vdim = nv * kd, conv_dim = 2 * kq + vdim;
    const int fam = family_of(W.qkv);
    Q35_TRY(eng_norm_gemv(e, n, W.attn_norm,
                          {{W.qkv.w, e->qkv, W.qkv.rows, W.qkv.tt, conv_dim, GV_STORE},
                           {W.gate.w, e->z, W.gate.rows, W.gate.tt, vdim, GV_STORE},
                           {W.alpha.w, e->ab, W.alpha.rows, W.alpha.tt, 2 * nv, GV_STORE},
                           {W.beta.w, e->ab + nv, W.beta.rows, W.beta.tt, 2 * nv, GV_STORE}},
                          st));
    const int gi = e->gdn_idx[li];
    const int fo = family_of(W.ssm_out);
    GdnCoreArgs g{};
    g.qkv = e->qkv;
    g.qkv_ld = conv_dim;
    g.z = e->z;
    g.z_ld = vdim;
    g.ab = e->ab;
    g.ab_ld = 2 * nv;
    g.conv_w = W.conv1d;
    g.hist = e->conv_pool + gi * (long long)e->n_slots * e->conv_slot;
    g.hist_slot = e->conv_slot;
    g.ssm_a = W.ssm_a;
    g.dt_bias = W.dt_bias;
    g.ssm_norm = W.ssm_norm;
    g.state = e->state_pool + gi * (long long)e->n_slots * e->state_slot;
    g.state_slot = e->state_slot;
    g.slots = e->d_in + e->max_batch;
    g.pos = e->d_in + 2 * e->max_batch;
    g.run_end = nrun < n ? e->d_in + 3 * e->max_batch : nullptr;
    g.nv = nv;
    g.nk = nk;
    g.eps = c.rms_eps;
    g.qscale = 1.0f / sqrtf((float)kd);
    g.fam = fo;
    g.xq = e->xq;
    g.xq_ld = e->xq_ld;
    g.gout = e->gout;
    g.gout_ld = vdim;
    if (g.run_end && e->gdn_wy) {
        // WY form for runs of WY_MIN_RUN tokens or more: per-token prologue,
        // the chunked recurrence per run on its slot's state, per-token
        // epilogue; shorter runs (decode tokens in a mixed forward, prompt
        // tails) stay with k_gdn_core, which skips the others
        g.wy_min = WY_MIN_RUN;
        bool any_short = false, any_long = false;
        for (int r = 0; r < nrun; r++) {
            const int len = e->h_run_end[r] - (r ? e->h_run_end[r - 1] : 0);
            (len >= WY_MIN_RUN ? any_long : any_short) = true;
        }
        if (any_short)
            Q35_TRY(launch_k(k_gdn_core, dim3(nv, nrun), dim3(GDN_KD), (size_t)GDN_KD * GDN_KD * 4, st, g));
        if (any_long) {
            WyPrepOut o{e->wy_q, e->wy_k, e->wy_v, e->wy_lg, e->wy_beta, nrun};
            Q35_TRY(launch_k(k_gdn_wy_prep, dim3(n, nv), dim3(GDN_KD), 0, st, g, o));
            for (int r = 0; r < nrun; r++) {
                const int i0 = r ? e->h_run_end[r - 1] : 0, i1 = e->h_run_end[r];
                if (i1 - i0 < WY_MIN_RUN) continue;
                GdnArgs w{};
                w.state = g.state + (long long)e->h_run_slot[r] * e->state_slot;
                w.state_head = (long long)kd * kd;
                w.q = e->wy_q + (long long)i0 * kq;
                w.k = e->wy_k + (long long)i0 * kq;
                w.v = e->wy_v + (long long)i0 * vdim;
                w.q_tok = w.k_tok = kq;
                w.v_tok = vdim;
                w.q_head = w.k_head = w.v_head = kd;
                w.out = e->wy_o + (long long)i0 * vdim;
                w.out_tok = vdim;
                w.out_head = kd;
                w.gamma = e->wy_lg + (long long)i0 * nv;
                w.g_tok = nv;
                w.gamma_log = 1;
                w.beta = e->wy_beta + (long long)i0 * nv;
                w.b_tok = nv;
                w.heads = nv;
                w.nk = nk;
                w.rows = i1 - i0;
                Q35_TRY(wy_tc_launch(w, st, e->wy_g, e->wy_g_bytes));
            }
            Q35_TRY(launch_k(k_gdn_wy_post, dim3(n, nv), dim3(GDN_KD), 0, st, g, (const float *)e->wy_o, nrun));
        }
    } else {
        Q35_TRY(launch_k(k_gdn_core, dim3(nv, nrun), dim3(GDN_KD), (size_t)GDN_KD * GDN_KD * 4, st, g));
    }
    if (g.run_end)
        Q35_TRY(launch_k(k_gdn_hist_settle, dim3((unsigned)((conv_dim * 3 + 255) / 256), (unsigned)nrun), dim3(256), 0,
                         st, g.hist, g.hist_slot, conv_dim, g.slots, g.pos, g.run_end));
    if (fo != 32) {
        Q35_TRY(launch_k(k_quant_rows, dim3((vdim / 256 + 7) / 8, n), dim3(256), 0, st, (const float *)e->gout,
                         (long long)vdim, vdim, fo, e->xq, e->xq_ld));
    }
    Q35_TRY(eng_gemv(e, n, {eng_rowpar_seg(e, W.ssm_out)}, e->xq, vdim, st));
    return eng_rowpar_finish(e, n, st);
}

// context bucket a captured step is built for: the score / P.V grids cover
// max_len positions (power of two multiple of 128, capped at the slot size)
inline int eng_len_bucket(int max_len, int max_seq) {
    int b = 128;
    while (b < max_len) b <<= 1;
    return b < max_seq ? b : max_seq;
}

inline int eng_layer_full(q35b_engine *e, int li, int n, int nrun, int max_len, cudaStream_t st) {
    const q35b_config &c = e->c;
    const LayerW &W = e->L[li];
    const int heads = c.n_heads, kvh = c.n_kv_heads, hd = c.head_dim;
    const int q_dim = heads * hd, kv_dim = kvh * hd;
    Q35_TRY(eng_norm_gemv(e, n, W.attn_norm,
                          {{W.q.w, e->qkv, W.q.rows, W.q.tt, 2 * q_dim, GV_STORE},
                           {W.k.w, e->kb, W.k.rows, W.k.tt, kv_dim, GV_STORE},
                           {W.v.w, e->vb, W.v.rows, W.v.tt, kv_dim, GV_STORE}},
                          st));
    const int fi = e->full_idx[li];
    float *kp = e->kpool + fi * (long long)e->n_slots * e->kv_slot;
    float *vp = e->vpool + fi * (long long)e->n_slots * e->kv_slot;
    const int *slots = e->d_in + e->max_batch, *pos = e->d_in + 2 * e->max_batch;
    const int fo = family_of(W.o);
    if (nrun == n && hd == ATT_HD) {
        // decode (every token a sequence of its own): prelude, scores,
        // softmax and P.V in one clustered launch at short contexts
        AttfArgs f{};
        f.qg = e->qkv;
        f.kb = e->kb;
        f.vb = e->vb;
        f.qw = W.q_norm;
        f.kw = W.k_norm;
        f.eps = c.rms_eps;
        f.base = c.rope_freq_base;
        f.scale = 1.0f / sqrtf((float)hd);
        f.pos = pos;
        f.slots = slots;
        f.kc = kp;
        f.vc = vp;
        f.kv_slot = e->kv_slot;
        f.heads = heads;
        f.kv_heads = kvh;
        f.out = e->gout;
        f.fam = fo;
        f.xq = e->xq;
        f.xq_ld = e->xq_ld;
        f.rope = e->rope_tab;
        const int rc = attf_launch(f, n, max_len, st);
        if (rc == 0) {
            if (fo != 32) {
                Q35_TRY(launch_k(k_quant_rows, dim3((q_dim / 256 + 7) / 8, n), dim3(256), 0, st,
                                 (const float *)e->gout, (long long)q_dim, q_dim, fo, e->xq, e->xq_ld));
            }
            Q35_TRY(eng_gemv(e, n, {eng_rowpar_seg(e, W.o)}, e->xq, q_dim, st));
            return eng_rowpar_finish(e, n, st);
        }
        if (rc != -1) return rc;
    }
    Q35_TRY(launch_k(k_attn_prelude, dim3(heads + kvh, n), dim3(256), 0, st, (const float *)e->qkv,
                     (const float *)e->kb, (const float *)e->vb, e->q, e->gate, W.q_norm, W.k_norm, heads, kvh,
                     c.rms_eps, c.rope_freq_base, pos, slots, kp, vp, e->kv_slot, (const float2 *)e->rope_tab));
    AttnXArgs a{};
    a.q = e->q;
    a.gate = e->gate;
    a.q_tok = q_dim;
    a.kc = kp;
    a.vc = vp;
    a.kv_slot = e->kv_slot;
    a.kv_dim = kv_dim;
    a.slots = slots;
    a.lens = e->d_len;
    a.scores = e->scores;
    a.max_len = e->max_seq;
    a.out = e->gout;
    a.out_tok = q_dim;
    a.heads = heads;
    a.kv_heads = kvh;
    a.scale = 1.0f / sqrtf((float)hd);
    a.fam = fo;
    a.xq = e->xq;
    a.xq_ld = e->xq_ld;
    // one run of several tokens (a prompt chunk of one sequence): the
    // prefill-shaped kernels; otherwise (decode tokens, or several runs in one
    // forward) a row per token
    int arc = nrun == 1 && n > 1 ? attp_launch(a, n, max_len, st) : -1;
    if (arc == -1) arc = attx_launch(a, n, max_len, st);
    Q35_TRY(arc);
    if (fo != 32) {
        Q35_TRY(launch_k(k_quant_rows, dim3((q_dim / 256 + 7) / 8, n), dim3(256), 0, st, (const float *)e->gout,
                         (long long)q_dim, q_dim, fo, e->xq, e->xq_ld));
    }
    Q35_TRY(eng_gemv(e, n, {eng_rowpar_seg(e, W.o)}, e->xq, q_dim, st));
    return eng_rowpar_finish(e, n, st);
}

inline int eng_mlp(q35b_engine *e, int li, int n, cudaStream_t st) {
    const q35b_config &c = e->c;
    const LayerW &W = e->L[li];
    const int fd = family_of(W.ffn_down);
    {
        // decode: rmsnorm -> gate / up GEMV whose epilogue forms
        // silu(gate) * up once per row -- as Q8_0 blocks the down projection
        // reads directly, or as f32 rows it quantizes (Q8_K family)
        const LprPrologue pro{LPR_PRO_NORM, e->x, nullptr, W.post_norm, (long long)c.hidden, c.rms_eps};
        const LprPair pr{fd == 32 ? e->xq : nullptr, e->xq_ld, fd == 32 ? nullptr : e->mh, (long long)c.n_ff};
        const GemvSegDesc gu[2] = {{W.ffn_gate.w, nullptr, W.ffn_gate.rows, W.ffn_gate.tt, c.n_ff, GV_STORE},
                                   {W.ffn_up.w, nullptr, W.ffn_up.rows, W.ffn_up.tt, c.n_ff, GV_STORE}};
        const int rc = gemv_lpr_launch(gu, 2, nullptr, c.hidden, n, st, e->xq_ld, &pro, &pr);
        if (rc == 0) {
            const GemvSegDesc down = eng_rowpar_seg(e, W.ffn_down);
            if (fd == 32) {
                Q35_TRY(eng_gemv(e, n, {down}, e->xq, c.n_ff, st));
            } else {
                const LprPrologue rows{LPR_PRO_ROWS, e->mh, nullptr, nullptr, (long long)c.n_ff, 0.0f};
                const int r2 = gemv_lpr_launch(&down, 1, nullptr, c.n_ff, n, st, e->xq_ld, &rows);
                if (r2 == -1) {
                    Q35_TRY(launch_k(k_quant_rows, dim3((c.n_ff / 256 + 7) / 8, n), dim3(256), 0, st,
                                     (const float *)e->mh, (long long)c.n_ff, c.n_ff, fd, e->xq, e->xq_ld));
                    Q35_TRY(eng_gemv(e, n, {down}, e->xq, c.n_ff, st));
                } else if (r2) {
                    return r2;
                }
            }
            return eng_rowpar_finish(e, n, st);
        }
        if (rc != -1) return rc;
    }
    Q35_TRY(eng_norm_gemv(e, n, W.post_norm,
                          {{W.ffn_gate.w, e->mh, W.ffn_gate.rows, W.ffn_gate.tt, c.n_ff, GV_STORE},
                           {W.ffn_up.w, e->mh1, W.ffn_up.rows, W.ffn_up.tt, c.n_ff, GV_STORE}},
                          st));
    const GemvSegDesc down = eng_rowpar_seg(e, W.ffn_down);
    const LprPrologue pro{LPR_PRO_SWIGLU, e->mh, e->mh1, nullptr, (long long)c.n_ff, 0.0f};
    const int rc = gemv_lpr_launch(&down, 1, nullptr, c.n_ff, n, st, e->xq_ld, &pro);
    if (rc == -1) {
        Q35_TRY(launch_k(k_swiglu_quant, dim3((c.n_ff / (fd == 32 ? 32 : 256) + 7) / 8, n), dim3(256), 0, st,
                         (const float *)e->mh, (const float *)e->mh1, c.n_ff, fd, e->xq, e->xq_ld));
        Q35_TRY(eng_gemv(e, n, {down}, e->xq, c.n_ff, st));
    } else if (rc) {
        return rc;
    }
    return eng_rowpar_finish(e, n, st);
}

// the whole step body (graph-capturable: every per-step value is in device memory)
struct PdlScope {
    bool prev;
    PdlScope() : prev(pdl_enabled()) { pdl_enabled() = true; }
    ~PdlScope() { pdl_enabled() = prev; }
};

// gather the last row of each run (x[run_end[r] - 1]) into xh[r]
__global__ void k_gather_run_rows(const float *x, const int *run_end, float *xh, int cols) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.y;
    const float *src = x + (long long)(run_end[r] - 1) * cols;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x)
        xh[(long long)r * cols + i] = src[i];
}

// n tokens in nrun runs (nrun == n: every token its own run, the decode
// step; nrun < n: runs of consecutive positions of one sequence each, the
// boundaries in d_in[3 max_batch ..]); logits / next token for the last
// token of each run
inline int eng_step_body(q35b_engine *e, int n, int nrun, int max_len, cudaStream_t st) {
    const PdlScope pdl_scope;
    const q35b_config &c = e->c;
    const long long l0 = launch_count();
    const int *tok = e->d_in;
    // The step's first kernel is an ordinary launch: it starts only after
    // everything earlier on the stream (the previous step included) is done,
    // so the kernels of this step may read per-layer state the previous step
    // wrote (GDN state, conv history) before their own dependency wait.
    pdl_enabled() = false;
    const int rc_embed = launch_k(k_embed_rows, dim3((c.hidden + 255) / 256, n), dim3(256), 0, st, e->token_embd.tt,
                                  e->token_embd.w, (size_t)weight_row_bytes(e->token_embd.tt, c.hidden), tok, e->x,
                                  c.hidden, (long long)e->token_embd.rows);
    pdl_enabled() = true;
    Q35_TRY(rc_embed);
    Q35_TRY(launch_k(k_pos_to_len, dim3((n + 127) / 128), dim3(128), 0, st, e->d_in + 2 * e->max_batch,
                     e->d_in + e->max_batch, e->d_len, n, e->max_seq, e->n_slots));
    for (int li = 0; li < c.n_layers; li++) {
        if (is_full_layer(c, li))
            Q35_TRY(eng_layer_full(e, li, n, nrun, max_len, st));
        else
            Q35_TRY(eng_layer_gdn(e, li, n, nrun, st));
        Q35_TRY(eng_mlp(e, li, n, st));
        if (e->probe) {
            Q35_TRY(launch_k(k_copy_rows, dim3(ew_grid((long long)n * c.hidden)), dim3(256), 0, st,
                             e->probe_buf + (long long)li * e->max_batch * c.hidden, (const float *)e->x,
                             (long long)n * c.hidden));
        }
    }
    const Lin &H = e->output.w ? e->output : e->token_embd;
    const long long vl = e->tp_n > 1 ? e->vocab_local : c.vocab;  // lm_head rows on this rank
    if (nrun < n) {
        Q35_TRY(launch_k(k_gather_run_rows, dim3((unsigned)((c.hidden + 255) / 256), (unsigned)nrun), dim3(256), 0,
                         st, (const float *)e->x, (const int *)(e->d_in + 3 * e->max_batch), e->xh, c.hidden));
        Q35_TRY(eng_norm_gemv(e, nrun, e->output_norm, {{H.w, e->logits, H.rows, H.tt, vl, GV_STORE}}, st, e->xh));
    } else {
        Q35_TRY(eng_norm_gemv(e, n, e->output_norm, {{H.w, e->logits, H.rows, H.tt, vl, GV_STORE}}, st));
    }
    int rc;
    if (e->sampling) {
        if (e->tp_n > 1) return (int)cudaErrorNotSupported;
        const SmpArgs sa{e->logits, (long long)c.vocab, c.vocab, nrun, e->samp, SC_INTS, e->d_in + e->max_batch,
                         nrun < n ? (const int *)(e->d_in + 3 * e->max_batch) : nullptr, e->d_next, 1};
        rc = sample_launch(sa, st);
    } else if (e->tp_n > 1) {
        Q35_TRY(launch_k(k_argmax_pair, dim3(nrun), dim3(1024), 0, st, (const float *)e->logits, vl, (int)vl,
                         (int)e->vocab_off, e->am_pair));
        if (nccl_api().all_gather(e->am_pair, e->am_all, (size_t)2 * nrun, ncclInt32, e->comm, st) != ncclSuccess)
            return (int)cudaErrorUnknown;
        rc = launch_k(k_argmax_combine, dim3((unsigned)((nrun + 127) / 128)), dim3(128), 0, st,
                      (const int *)e->am_all, nrun, e->tp_n, e->d_next);
    } else {
        rc = launch_k(k_argmax_split, dim3(AM_SPLIT, nrun), dim3(256), 0, st, (const float *)e->logits,
                      (long long)c.vocab, c.vocab, e->d_next, e->am_v, e->am_i, e->am_cnt);
    }
    e->launches = launch_count() - l0;
    return rc;
}

}  // namespace q35
