// engine_api.cuh -- q35b_engine_* / q35b_serve: the batched engine's C ABI.
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <deque>

#include "engine.cuh"

using namespace q35;

namespace {

int set_lin(Lin &l, int tt, const void *d, long long rows, long long cols) {
    if (!geom_of(tt).elems || !d || rows <= 0 || cols <= 0 || cols % geom_of(tt).elems) return (int)cudaErrorInvalidValue;
    l.w = reinterpret_cast<const uint8_t *>(d);
    l.tt = tt;
    l.rows = rows;
    l.cols = cols;
    return 0;
}

bool lin_ok(const Lin &l, long long rows, long long cols) { return l.w && l.rows == rows && l.cols == cols; }

long long graph_key(int n, int len_bucket) { return (long long)n * (1LL << 32) + len_bucket; }

// the WY prefill's scratch for max_batch tokens: allocated when the WY form
// is switched on for a finalized engine, or at finalize, so that no forward
// allocates (a forward may run inside the caller's stream capture)
int eng_wy_scratch(q35b_engine *e) {
    if (e->wy_g) return 0;  // the last of them: all allocated
    const q35b_config &c = e->c;
    const size_t B = (size_t)e->max_batch, kq = (size_t)c.gdn_num_k_heads * GDN_KD,
                 vd = (size_t)c.gdn_n_heads * GDN_KD;
    float **dst[6] = {&e->wy_q, &e->wy_k, &e->wy_v, &e->wy_o, &e->wy_lg, &e->wy_beta};
    const size_t len[6] = {B * kq, B * kq, B * vd, B * vd, B * c.gdn_n_heads, B * c.gdn_n_heads};
    for (int i = 0; i < 6; i++) {
        void *p = nullptr;
        Q35_TRY(eng_alloc(e, &p, 4 * len[i]));
        *dst[i] = static_cast<float *>(p);
    }
    void *p = nullptr;
    const size_t gb = wy_gram_bytes(e->max_batch, c.gdn_num_k_heads);
    Q35_TRY(eng_alloc(e, &p, gb));
    e->wy_g = static_cast<float *>(p);
    e->wy_g_bytes = gb;
    return 0;
}

}  // namespace

extern "C" {

int q35b_engine_create(const q35b_config *cfg, int n_slots, int max_seq, int max_batch, q35b_engine **out) {
    if (!cfg || !out || n_slots <= 0 || max_seq <= 0 || max_batch <= 0) return (int)cudaErrorInvalidValue;
    if (cfg->gdn_head_dim != GDN_KD || cfg->head_dim != ATT_HD || cfg->conv_kernel != 4)
        return (int)cudaErrorInvalidValue;
    if (cfg->n_heads % cfg->n_kv_heads || cfg->n_heads / cfg->n_kv_heads > ATT_MAXG) return (int)cudaErrorInvalidValue;
    if (cfg->gdn_num_k_heads <= 0 || cfg->gdn_n_heads % cfg->gdn_num_k_heads || cfg->gdn_n_heads > 64)
        return (int)cudaErrorInvalidValue;
    q35b_engine *e = new q35b_engine();
    e->c = *cfg;
    e->n_slots = n_slots;
    e->max_seq = max_seq;
    e->max_batch = max_batch;
    e->L.resize(cfg->n_layers);
    cudaGetDevice(&e->device);
    *out = e;
    return 0;
}

int q35b_engine_destroy(q35b_engine *e) {
    if (!e) return 0;
    // graphs holding collectives go before the communicator
    for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
    for (void *p : e->ipc_open) cudaIpcCloseMemHandle(p);
    e->ipc_open.clear();
    if (e->comm) nccl_api().comm_destroy(e->comm);
    for (void *p : e->allocs) cudaFree(p);
    if (e->h_io) cudaFreeHost(e->h_io);
    delete e;
    return 0;
}

int q35b_engine_set_prefill_wy(q35b_engine *e, int on) {
    if (!e) return (int)cudaErrorInvalidValue;
    e->gdn_wy = on != 0;
    if (e->gdn_wy && e->finalized) return eng_wy_scratch(e);
    return 0;
}

int q35b_engine_set_sampling(q35b_engine *e, int on) {
    if (!e) return (int)cudaErrorInvalidValue;
    if (on && e->tp_n > 1) return (int)cudaErrorNotSupported;
    if (on && e->c.vocab > SMP_MAX_N) return (int)cudaErrorInvalidValue;
    if (e->sampling != (on != 0)) {
        for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
        e->graphs.clear();
    }
    e->sampling = on != 0;
    return 0;
}

int q35b_engine_set_sampler(q35b_engine *e, int slot, float temperature, int top_k, float top_p,
                            unsigned long long seed) {
    if (!e || !e->finalized || slot < 0 || slot >= e->n_slots || top_k < 0) return (int)cudaErrorInvalidValue;
    if (seed == 0) seed = 0x9E3779B97F4A7C15ULL;  // src/sampler.zig:47
    int blk[SC_INTS] = {};
    blk[SC_VOCAB] = e->c.vocab;
    memcpy(&blk[SC_TEMP], &temperature, 4);
    blk[SC_TOPK] = top_k;
    memcpy(&blk[SC_TOPP], &top_p, 4);
    blk[SC_RNG_LO] = (int)(uint32_t)(seed & 0xFFFFFFFFu);
    blk[SC_RNG_HI] = (int)(uint32_t)(seed >> 32);
    return (int)cudaMemcpy(e->samp + (long long)slot * SC_INTS, blk, sizeof(blk), cudaMemcpyHostToDevice);
}

int q35b_tp_unique_id(void *out, int bytes) {
    const NcclApi &api = nccl_api();
    if (!api.ok) return (int)cudaErrorSharedObjectInitFailed;
    if (!out || bytes < (int)sizeof(ncclUniqueId)) return (int)cudaErrorInvalidValue;
    ncclUniqueId id;
    if (api.get_unique_id(&id) != ncclSuccess) return (int)cudaErrorUnknown;
    memcpy(out, &id, sizeof(id));
    return 0;
}

int q35b_engine_set_tp(q35b_engine *e, int nranks, int rank, long long vocab_local, long long vocab_offset,
                       const void *unique_id) {
    if (!e || e->finalized || nranks < 2 || rank < 0 || rank >= nranks || !unique_id || vocab_local <= 0 ||
        vocab_offset < 0 || vocab_offset + vocab_local > e->c.vocab || e->comm)
        return (int)cudaErrorInvalidValue;
    const NcclApi &api = nccl_api();
    if (!api.ok) return (int)cudaErrorSharedObjectInitFailed;
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof(id));
    ncclComm_t comm = nullptr;
    if (api.comm_init_rank(&comm, nranks, id, rank) != ncclSuccess) return (int)cudaErrorUnknown;
    e->comm = comm;
    e->tp_n = nranks;
    e->tp_rank = rank;
    e->vocab_local = vocab_local;
    e->vocab_off = vocab_offset;
    return 0;
}

// ---- peer all-reduce (tp.cuh k_tp_allreduce_add) ----
constexpr int TP_HANDLES = 3;  // partial sums, residual, flag words

int q35b_engine_ipc_handles(q35b_engine *e, void *out, int bytes) {
    if (!e || !e->finalized || e->tp_n < 2 || !out || bytes < TP_HANDLES * (int)sizeof(cudaIpcMemHandle_t))
        return (int)cudaErrorInvalidValue;
    cudaIpcMemHandle_t h[TP_HANDLES];
    const void *ptrs[TP_HANDLES] = {e->ppart, e->x, e->ar_flags};
    for (int i = 0; i < TP_HANDLES; i++) {
        const cudaError_t r = cudaIpcGetMemHandle(&h[i], const_cast<void *>(ptrs[i]));
        if (r != cudaSuccess) return (int)r;
    }
    memcpy(out, h, sizeof(h));
    return 0;
}

static void drop_graphs(q35b_engine *e) {
    for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
}

int q35b_engine_set_peers(q35b_engine *e, const void *all, int bytes) {
    const int hb = TP_HANDLES * (int)sizeof(cudaIpcMemHandle_t);
    if (!e || !e->finalized || e->tp_n < 2 || e->tp_n > TP_MAX || !all || bytes < e->tp_n * hb || e->peers_open)
        return (int)cudaErrorInvalidValue;
    if (e->c.hidden % (4 * e->tp_n)) return (int)cudaErrorInvalidValue;  // owned slices of whole float4s
    TpPeers pe{};
    std::vector<void *> opened;
    for (int p = 0; p < e->tp_n; p++) {
        void *ptr[TP_HANDLES] = {e->ppart, e->x, e->ar_flags};
        if (p != e->tp_rank) {
            for (int i = 0; i < TP_HANDLES; i++) {
                cudaIpcMemHandle_t h;
                memcpy(&h, static_cast<const uint8_t *>(all) + (size_t)p * hb + (size_t)i * sizeof(h), sizeof(h));
                const cudaError_t r = cudaIpcOpenMemHandle(&ptr[i], h, cudaIpcMemLazyEnablePeerAccess);
                if (r != cudaSuccess) {
                    for (void *q : opened) cudaIpcCloseMemHandle(q);
                    return (int)r;
                }
                opened.push_back(ptr[i]);
            }
        }
        pe.part[p] = static_cast<float *>(ptr[0]);
        pe.x[p] = static_cast<float *>(ptr[1]);
        pe.flags[p] = static_cast<int *>(ptr[2]);
    }
    e->peers = pe;
    e->ipc_open = opened;
    e->peers_open = true;
    e->ar_peer = true;
    drop_graphs(e);  // steps captured before hold the NCCL form
    return 0;
}

int q35b_engine_set_allreduce(q35b_engine *e, int peer) {
    if (!e || (peer && !e->peers_open)) return (int)cudaErrorInvalidValue;
    if (e->ar_peer != (peer != 0)) drop_graphs(e);
    e->ar_peer = peer != 0;
    return 0;
}

// the bounded waits of k_tp_allreduce_add on one GPU: a two-rank exchange
// whose second rank never runs (its flags are local words nothing sets);
// the kernel gives up after limit_ns per wait and records error 150
int q35b_tp_selftest_timeout(unsigned long long limit_ns, void *stream) {
    if (limit_ns == 0 || limit_ns > 2000000000ull) return (int)cudaErrorInvalidValue;
    void *buf = nullptr;
    const size_t fl = 4 * TP_FLAG_WORDS;
    cudaError_t r = cudaMalloc(&buf, 4 * 4 * 8 + 2 * fl + 8);
    if (r != cudaSuccess) return (int)r;
    r = cudaMemset(buf, 0, 4 * 4 * 8 + 2 * fl + 8);
    float *f = static_cast<float *>(buf);
    int *fl0 = reinterpret_cast<int *>(f + 32), *fl1 = fl0 + TP_FLAG_WORDS, *state = fl1 + TP_FLAG_WORDS;
    TpArArgs a{};
    a.pe.part[0] = f;
    a.pe.part[1] = f + 8;
    a.pe.x[0] = f + 16;
    a.pe.x[1] = f + 24;
    a.pe.flags[0] = fl0;
    a.pe.flags[1] = fl1;
    a.state = state;
    a.rank = 0;
    a.nranks = 2;
    a.hidden = 8;
    a.n = 1;
    a.limit_ns = limit_ns;
    if (r == cudaSuccess) r = (cudaError_t)tp_ar_launch(a, S(stream));
    if (r == cudaSuccess) r = cudaStreamSynchronize(S(stream));
    cudaFree(buf);
    return (int)r;
}

int q35b_engine_set_tensor(q35b_engine *e, const char *name, int tt, const void *d, long long rows, long long cols) {
    if (!e || !name || e->finalized) return (int)cudaErrorInvalidValue;
    if (!strcmp(name, "token_embd.weight")) return set_lin(e->token_embd, tt, d, rows, cols);
    if (!strcmp(name, "output.weight")) return set_lin(e->output, tt, d, rows, cols);
    if (!strcmp(name, "output_norm.weight")) {
        if (tt != TT_F32 || cols != e->c.hidden) return (int)cudaErrorInvalidValue;
        e->output_norm = reinterpret_cast<const float *>(d);
        return 0;
    }
    int li = -1, off = 0;
    if (sscanf(name, "blk.%d.%n", &li, &off) != 1 || li < 0 || li >= e->c.n_layers) return (int)cudaErrorInvalidValue;
    const char *t = name + off;
    LayerW &W = e->L[li];
    struct F { const char *n; const float **p; };
    const F f32s[] = {{"attn_norm.weight", &W.attn_norm},   {"post_attention_norm.weight", &W.post_norm},
                      {"ssm_conv1d.weight", &W.conv1d},     {"ssm_dt.bias", &W.dt_bias},
                      {"ssm_a", &W.ssm_a},                  {"ssm_norm.weight", &W.ssm_norm},
                      {"attn_q_norm.weight", &W.q_norm},    {"attn_k_norm.weight", &W.k_norm}};
    for (const F &x : f32s)
        if (!strcmp(t, x.n)) {
            if (tt != TT_F32 || !d) return (int)cudaErrorInvalidValue;
            *x.p = reinterpret_cast<const float *>(d);
            return 0;
        }
    struct Q { const char *n; Lin *l; };
    const Q lins[] = {{"attn_qkv.weight", &W.qkv},   {"attn_gate.weight", &W.gate}, {"ssm_alpha.weight", &W.alpha},
                      {"ssm_beta.weight", &W.beta},  {"ssm_out.weight", &W.ssm_out}, {"attn_q.weight", &W.q},
                      {"attn_k.weight", &W.k},       {"attn_v.weight", &W.v},        {"attn_output.weight", &W.o},
                      {"ffn_gate.weight", &W.ffn_gate}, {"ffn_up.weight", &W.ffn_up}, {"ffn_down.weight", &W.ffn_down}};
    for (const Q &x : lins)
        if (!strcmp(t, x.n)) return set_lin(*x.l, tt, d, rows, cols);
    return (int)cudaErrorInvalidValue;
}

// Q6_K (210 B) -> padded Q6_K (224 B): 105 halfwords of a block, then zeros

int q35b_engine_finalize(q35b_engine *e) {
    if (!e || e->finalized) return (int)cudaErrorInvalidValue;
    const q35b_config &c = e->c;
    const long long h = c.hidden, nv = c.gdn_n_heads, nk = c.gdn_num_k_heads, kd = c.gdn_head_dim;
    const long long kq = nk * kd, vdim = nv * kd, conv_dim = 2 * kq + vdim;
    const long long q_dim = (long long)c.n_heads * c.head_dim, kv_dim = (long long)c.n_kv_heads * c.head_dim;
    if (!lin_ok(e->token_embd, c.vocab, h) || !e->output_norm) return (int)cudaErrorInvalidValue;
    if (e->output.w && !lin_ok(e->output, e->tp_n > 1 ? e->vocab_local : (long long)c.vocab, h))
        return (int)cudaErrorInvalidValue;
    if (e->tp_n > 1 && !e->output.w) return (int)cudaErrorInvalidValue;  // a rank's lm_head is its own shard
    int ngdn = 0, nfull = 0;
    for (int li = 0; li < c.n_layers; li++) {
        const LayerW &W = e->L[li];
        if (!W.attn_norm || !W.post_norm || !lin_ok(W.ffn_gate, c.n_ff, h) || !lin_ok(W.ffn_up, c.n_ff, h) ||
            !lin_ok(W.ffn_down, h, c.n_ff))
            return (int)cudaErrorInvalidValue;
        if (family_of(W.ffn_gate) != family_of(W.ffn_up)) return (int)cudaErrorInvalidValue;
        if (is_full_layer(c, li)) {
            if (!lin_ok(W.q, 2 * q_dim, h) || !lin_ok(W.k, kv_dim, h) || !lin_ok(W.v, kv_dim, h) ||
                !lin_ok(W.o, h, q_dim) || !W.q_norm || !W.k_norm)
                return (int)cudaErrorInvalidValue;
            if (family_of(W.q) != family_of(W.k) || family_of(W.q) != family_of(W.v)) return (int)cudaErrorInvalidValue;
            e->full_idx.push_back(nfull++);
            e->gdn_idx.push_back(-1);
        } else {
            if (!lin_ok(W.qkv, conv_dim, h) || !lin_ok(W.gate, vdim, h) || !lin_ok(W.alpha, nv, h) ||
                !lin_ok(W.beta, nv, h) || !lin_ok(W.ssm_out, h, vdim) || !W.conv1d || !W.dt_bias || !W.ssm_a ||
                !W.ssm_norm)
                return (int)cudaErrorInvalidValue;
            const int f = family_of(W.qkv);
            if (family_of(W.gate) != f || family_of(W.alpha) != f || family_of(W.beta) != f)
                return (int)cudaErrorInvalidValue;
            e->gdn_idx.push_back(ngdn++);
            e->full_idx.push_back(-1);
        }
    }
    const long long B = e->max_batch, S = e->n_slots;
    e->conv_slot = conv_dim * 3 * 2;  // history double-buffered by position parity
    e->state_slot = nv * kd * kd;
    e->kv_slot = (long long)e->max_seq * kv_dim;
    void *p;
#define ALLOC(field, bytes)                                  \
    do {                                                     \
        Q35_TRY(eng_alloc(e, &p, (size_t)(bytes)));          \
        e->field = reinterpret_cast<decltype(e->field)>(p);  \
    } while (0)
    ALLOC(conv_pool, 4 * ngdn * S * e->conv_slot);
    ALLOC(state_pool, 4 * ngdn * S * e->state_slot);
    ALLOC(kpool, 4 * nfull * S * e->kv_slot);
    ALLOC(vpool, 4 * nfull * S * e->kv_slot);
    ALLOC(d_in, 4 * 4 * B);
    if (e->tp_n > 1) {
        ALLOC(part, 4 * B * h);
        ALLOC(am_pair, 4 * 2 * B);
        ALLOC(am_all, 4 * 2 * B * e->tp_n);
        ALLOC(ppart, 4 * B * h);
        ALLOC(ar_flags, 4 * TP_FLAG_WORDS);
        ALLOC(ar_state, 4 * 2);
        Q35_TRY((int)cudaMemset(e->ar_flags, 0, 4 * TP_FLAG_WORDS));
        Q35_TRY((int)cudaMemset(e->ar_state, 0, 4 * 2));
    }
    ALLOC(am_v, 4 * B * AM_SPLIT);
    ALLOC(am_i, 4 * B * AM_SPLIT);
    ALLOC(am_cnt, 4 * B);
    {
        // split-K terms of the K-quant MMQ: the row-parallel projections have
        // few row tiles (hidden / 128), so at batch >= 16 their K is split
        // over CTAs (up to MMQ_SPLIT_MAX_TOK tokens); nblk x tokens x rows
        // floats for the largest of them
        const size_t Bs = (size_t)std::min<long long>(B, MMQ_SPLIT_MAX_TOK);
        size_t tb = 0;
        for (const LayerW &W : e->L)
            for (const Lin *l : {&W.o, &W.ssm_out, &W.ffn_down})
                if (l->w && geom_of(l->tt).family == 256)
                    tb = std::max(tb, (size_t)(l->cols / 256) * Bs * (size_t)l->rows * 4);
        if (tb) {
            ALLOC(mmq_terms, tb);
            e->mmq_terms_bytes = tb;
        }
    }
    ALLOC(xh, 4 * B * h);
    ALLOC(samp, 4 * SC_INTS * S);  // zeroed below: every slot greedy until set_sampler
    ALLOC(d_len, 4 * B);
    ALLOC(d_next, 4 * B);
    ALLOC(x, 4 * B * h);
    ALLOC(qkv, 4 * B * std::max(conv_dim, 2 * q_dim));
    ALLOC(z, 4 * B * std::max(vdim, q_dim));
    ALLOC(ab, 4 * B * 2 * nv);
    ALLOC(gam, 4 * B * nv);
    ALLOC(gout, 4 * B * std::max(vdim, q_dim));
    ALLOC(q, 4 * B * q_dim);
    ALLOC(gate, 4 * B * q_dim);
    ALLOC(kb, 4 * B * kv_dim);
    ALLOC(vb, 4 * B * kv_dim);
    ALLOC(mh, 4 * B * c.n_ff);
    ALLOC(mh1, 4 * B * c.n_ff);
    ALLOC(logits, 4 * B * (long long)c.vocab);
    ALLOC(scores, 4 * B * c.n_heads * (long long)e->max_seq);
    ALLOC(probe_buf, 4 * (long long)c.n_layers * B * h);
    long long maxcols = std::max(std::max(h, (long long)c.n_ff), std::max(vdim, q_dim));
    e->xq_ld = ((maxcols / 32 * 34 + maxcols / 256 * 292) + 15) & ~15LL;
    ALLOC(xq, e->xq_ld * B + 64);
    ALLOC(rope_tab, (size_t)e->max_seq * 32 * sizeof(float2));
    {
        // RoPE rotations per (position, pair j): theta = pos * base^(-2j/64)
        // and its cos / sin in f32 through the C library, the expression and
        // functions of the reference's CPU engine (elementwise.zig:306-318),
        // so the device rotates with the CPU's exact values
        std::vector<float2> rt((size_t)e->max_seq * 32);
        for (int p = 0; p < e->max_seq; p++)
            for (int j = 0; j < 32; j++) {
                const float th = (float)p * powf(c.rope_freq_base, -(float)(2 * j) / 64.0f);
                rt[(size_t)p * 32 + j] = make_float2(cosf(th), sinf(th));
            }
        Q35_TRY((int)cudaMemcpy(e->rope_tab, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice));
    }
#undef ALLOC
    Q35_TRY((int)cudaMemset(e->conv_pool, 0, 4 * ngdn * S * e->conv_slot));
    Q35_TRY((int)cudaMemset(e->state_pool, 0, 4 * ngdn * S * e->state_slot));
    // KV pools start as finite zeros (positions past a slot's length are never
    // read; a caller that steps at a position it never filled reads zeros)
    Q35_TRY((int)cudaMemset(e->kpool, 0, 4 * nfull * S * e->kv_slot));
    Q35_TRY((int)cudaMemset(e->vpool, 0, 4 * nfull * S * e->kv_slot));
    Q35_TRY((int)cudaMemset(e->d_in, 0, 4 * 4 * B));
    Q35_TRY((int)cudaHostAlloc((void **)&e->h_io, 4 * 4 * B, cudaHostAllocDefault));
    Q35_TRY((int)cudaMemset(e->am_cnt, 0, 4 * B));
    Q35_TRY((int)cudaMemset(e->samp, 0, 4 * SC_INTS * S));
    // load-time repack: Q6_K projections to 224-byte blocks (16-byte rows for
    // the TMA-streamed GEMV); the caller's buffers stay untouched
    auto repack = [&](Lin &l) -> int {
        if (l.tt != TT_Q6_K || !l.w) return 0;
        const long long nblk = l.rows * (l.cols / 256);
        void *dst;
        Q35_TRY(eng_alloc(e, &dst, (size_t)nblk * 224));
        const long long nthreads = nblk * 112;
        k_repack_q6k<<<(unsigned)((nthreads + 255) / 256), 256>>>(l.w, static_cast<uint8_t *>(dst), nblk);
        Q35_TRY((int)cudaGetLastError());
        l.w = static_cast<const uint8_t *>(dst);
        l.tt = TT_Q6_K_P;
        return 0;
    };
    Q35_TRY(repack(e->output));
    for (LayerW &W : e->L)
        for (Lin *l : {&W.qkv, &W.gate, &W.alpha, &W.beta, &W.ssm_out, &W.q, &W.k, &W.v, &W.o, &W.ffn_gate, &W.ffn_up,
                       &W.ffn_down})
            Q35_TRY(repack(*l));
    Q35_TRY(gemv_prepare());
    Q35_TRY(gemv_lpr_prepare());
    Q35_TRY(gdn_prepare());
    Q35_TRY(attx_prepare(e->max_seq));
    if (e->gdn_wy) Q35_TRY(eng_wy_scratch(e));
    Q35_TRY((int)cudaDeviceSynchronize());
    e->finalized = true;
    return 0;
}

__global__ void k_reset_slot(float *conv_pool, long long conv_total, long long conv_slot, float *state_pool,
                             long long state_total, long long state_slot, int n_layers_pool, int slot) {
    // conv: n_gdn layers x [slot] x conv_slot ; state likewise
    const long long nc = (long long)n_layers_pool * conv_slot, ns = (long long)n_layers_pool * state_slot;
    Q35_GRID_STRIDE(i, nc + ns) {
        if (i < nc) {
            const long long l = i / conv_slot, j = i - l * conv_slot;
            conv_pool[l * conv_total + slot * conv_slot + j] = 0.0f;
        } else {
            const long long k = i - nc, l = k / state_slot, j = k - l * state_slot;
            state_pool[l * state_total + slot * state_slot + j] = 0.0f;
        }
    }
}

int q35b_engine_reset_slot(q35b_engine *e, int slot, void *stream) {
    if (!e || !e->finalized || slot < 0 || slot >= e->n_slots) return (int)cudaErrorInvalidValue;
    int ngdn = 0;
    for (int v : e->gdn_idx) ngdn += v >= 0;
    if (ngdn == 0) return 0;
    const long long tot = (long long)ngdn * (e->conv_slot + e->state_slot);
    k_reset_slot<<<ew_grid(tot), 256, 0, S(stream)>>>(e->conv_pool, (long long)e->n_slots * e->conv_slot, e->conv_slot,
                                                      e->state_pool, (long long)e->n_slots * e->state_slot,
                                                      e->state_slot, ngdn, slot);
    return (int)cudaGetLastError();
}

int q35b_engine_set_probe(q35b_engine *e, int on) {
    if (!e) return (int)cudaErrorInvalidValue;
    e->probe = on != 0;
    for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
    return 0;
}

const float *q35b_engine_layer_out(q35b_engine *e, int li) {
    if (!e || !e->finalized || !e->probe || li < 0 || li >= e->c.n_layers) return nullptr;
    return e->probe_buf + (long long)li * e->max_batch * e->c.hidden;
}

long long q35b_engine_launches_per_step(q35b_engine *e) { return e ? e->launches : 0; }

// Launch the step for `n` sequences whose inputs are already in e->d_in.
static int engine_run(q35b_engine *e, int n, int max_len, int use_graph, cudaStream_t st) {
    const int bucket = eng_len_bucket(max_len, e->max_seq);
    if (!use_graph) return eng_step_body(e, n, n, bucket, st);
    const long long key = graph_key(n, bucket);
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaStream_t cs;
        Q35_TRY((int)cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
        cudaGraph_t g = nullptr;
        int rc = (int)cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
        if (!rc) {
            const int brc = eng_step_body(e, n, n, bucket, cs);
            rc = (int)cudaStreamEndCapture(cs, &g);
            if (brc) rc = brc;
        }
        cudaGraphExec_t ge = nullptr;
        if (!rc) rc = (int)cudaGraphInstantiate(&ge, g, 0);
        if (g) cudaGraphDestroy(g);
        cudaStreamDestroy(cs);
        if (rc) return rc;
        it = e->graphs.emplace(key, ge).first;
    }
    return (int)cudaGraphLaunch(it->second, st);
}

__global__ void k_max_pos(const int *pos, int n, int *out) {
    int m = 0;
    for (int i = 0; i < n; i++) m = max(m, pos[i]);
    *out = m;
}

int q35b_engine_step(q35b_engine *e, int n, const int *d_tokens, const int *d_slots, const int *d_pos, int *d_next,
                     float *d_logits, int use_graph, void *stream) {
    if (!e || !e->finalized || n <= 0 || n > e->max_batch) return (int)cudaErrorInvalidValue;
    cudaStream_t st = S(stream);
    const size_t b = (size_t)n * 4;
    // inputs the graph reads live at fixed addresses inside the engine
    if (d_tokens != e->d_in) Q35_TRY((int)cudaMemcpyAsync(e->d_in, d_tokens, b, cudaMemcpyDeviceToDevice, st));
    if (d_slots != e->d_in + e->max_batch)
        Q35_TRY((int)cudaMemcpyAsync(e->d_in + e->max_batch, d_slots, b, cudaMemcpyDeviceToDevice, st));
    if (d_pos != e->d_in + 2 * e->max_batch)
        Q35_TRY((int)cudaMemcpyAsync(e->d_in + 2 * e->max_batch, d_pos, b, cudaMemcpyDeviceToDevice, st));
    // the split count must cover the longest context; without a host copy of
    // the positions it covers the whole slot
    Q35_TRY(engine_run(e, n, e->max_seq, use_graph, st));
    if (d_next && d_next != e->d_next)
        Q35_TRY((int)cudaMemcpyAsync(d_next, e->d_next, b, cudaMemcpyDeviceToDevice, st));
    if (d_logits)
        Q35_TRY((int)cudaMemcpyAsync(d_logits, e->logits, (size_t)n * e->c.vocab * 4, cudaMemcpyDeviceToDevice, st));
    return 0;
}

int q35b_engine_step_host(q35b_engine *e, int n, const int *tokens, const int *slots, const int *pos, int *next,
                          void *stream) {
    if (!e || !e->finalized || n <= 0 || n > e->max_batch) return (int)cudaErrorInvalidValue;
    cudaStream_t st = S(stream);
    const size_t b = (size_t)n * 4;
    int max_len = 1;
    for (int i = 0; i < n; i++) {
        if (pos[i] < 0 || pos[i] >= e->max_seq || slots[i] < 0 || slots[i] >= e->n_slots)
            return (int)cudaErrorInvalidValue;
        max_len = std::max(max_len, pos[i] + 1);
    }
    // the inputs go through pinned staging laid out like d_in: one
    // asynchronous copy in, one out (pageable copies would each be staged
    // and synchronous); the staging is reused only after this call's sync
    const long long B = e->max_batch;
    int *hi = e->h_io, *hn = e->h_io + 3 * B;
    std::memcpy(hi, tokens, b);
    std::memcpy(hi + B, slots, b);
    std::memcpy(hi + 2 * B, pos, b);
    const size_t span = (size_t)(2 * B + n) * 4;  // tokens .. pos[n-1]
    Q35_TRY((int)cudaMemcpyAsync(e->d_in, hi, span, cudaMemcpyHostToDevice, st));
    Q35_TRY(engine_run(e, n, max_len, 1, st));
    Q35_TRY((int)cudaMemcpyAsync(hn, e->d_next, b, cudaMemcpyDeviceToHost, st));
    Q35_TRY((int)cudaStreamSynchronize(st));
    std::memcpy(next, hn, b);
    return 0;
}

int q35b_engine_device_inputs(q35b_engine *e, int **d_tokens, int **d_slots, int **d_pos, int **d_next) {
    if (!e || !e->finalized) return (int)cudaErrorInvalidValue;
    if (d_tokens) *d_tokens = e->d_in;
    if (d_slots) *d_slots = e->d_in + e->max_batch;
    if (d_pos) *d_pos = e->d_in + 2 * e->max_batch;
    if (d_next) *d_next = e->d_next;
    return 0;
}

__global__ void k_advance(int *tok, int *pos, const int *next, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        tok[i] = next[i];
        pos[i] += 1;
    }
}

int q35b_engine_step_dev(q35b_engine *e, int n, int max_len, int use_graph, void *stream) {
    if (!e || !e->finalized || n <= 0 || n > e->max_batch || max_len <= 0 || max_len > e->max_seq)
        return (int)cudaErrorInvalidValue;
    return engine_run(e, n, max_len, use_graph, S(stream));
}

int q35b_engine_advance(q35b_engine *e, int n, void *stream) {
    if (!e || !e->finalized || n <= 0 || n > e->max_batch) return (int)cudaErrorInvalidValue;
    k_advance<<<(n + 127) / 128, 128, 0, S(stream)>>>(e->d_in, e->d_in + 2 * e->max_batch, e->d_next, n);
    return (int)cudaGetLastError();
}

// One forward over n tokens in nrun runs (host arrays); see include/q35.h.
int q35b_engine_forward(q35b_engine *e, int n, const int *tokens, const int *slots, const int *pos, int nrun,
                        const int *run_end, int *next, void *stream) {
    if (!e || !e->finalized || n <= 0 || n > e->max_batch || nrun <= 0 || nrun > n || !run_end)
        return (int)cudaErrorInvalidValue;
    if (run_end[nrun - 1] != n) return (int)cudaErrorInvalidValue;
    int max_len = 1, b0 = 0;
    std::vector<char> seen(e->n_slots, 0);
    for (int r = 0; r < nrun; r++) {
        const int b1 = run_end[r];
        if (b1 <= b0) return (int)cudaErrorInvalidValue;
        const int sl = slots[b0];
        if (sl < 0 || sl >= e->n_slots || seen[sl]) return (int)cudaErrorInvalidValue;  // one run per slot
        seen[sl] = 1;
        for (int i = b0; i < b1; i++) {
            if (slots[i] != sl || pos[i] < 0 || pos[i] >= e->max_seq) return (int)cudaErrorInvalidValue;
            if (i > b0 && pos[i] != pos[i - 1] + 1) return (int)cudaErrorInvalidValue;
            max_len = std::max(max_len, pos[i] + 1);
        }
        b0 = b1;
    }
    cudaStream_t st = S(stream);
    const size_t b = (size_t)n * 4;
    Q35_TRY((int)cudaMemcpyAsync(e->d_in, tokens, b, cudaMemcpyHostToDevice, st));
    Q35_TRY((int)cudaMemcpyAsync(e->d_in + e->max_batch, slots, b, cudaMemcpyHostToDevice, st));
    Q35_TRY((int)cudaMemcpyAsync(e->d_in + 2 * e->max_batch, pos, b, cudaMemcpyHostToDevice, st));
    if (nrun == n) {
        Q35_TRY(engine_run(e, n, max_len, 1, st));
    } else {
        // runs longer than one token (prefill): launched directly, the
        // launch cost spread over the run's tokens
        Q35_TRY((int)cudaMemcpyAsync(e->d_in + 3 * e->max_batch, run_end, (size_t)nrun * 4, cudaMemcpyHostToDevice,
                                     st));
        if (e->gdn_wy) {
            if (!e->wy_g) return (int)cudaErrorInvalidValue;  // allocated when switched on
            e->h_run_end.assign(run_end, run_end + nrun);
            e->h_run_slot.resize(nrun);
            for (int r = 0; r < nrun; r++) e->h_run_slot[r] = slots[r ? run_end[r - 1] : 0];
        }
        Q35_TRY(eng_step_body(e, n, nrun, eng_len_bucket(max_len, e->max_seq), st));
    }
    Q35_TRY((int)cudaMemcpyAsync(next, e->d_next, (size_t)nrun * 4, cudaMemcpyDeviceToHost, st));
    return (int)cudaStreamSynchronize(st);
}

int q35b_engine_prefill(q35b_engine *e, int slot, const int *tokens, int ntok, int pos0, int *next, void *stream) {
    if (!e || !e->finalized || ntok <= 0 || pos0 < 0 || pos0 + ntok > e->max_seq) return (int)cudaErrorInvalidValue;
    std::vector<int> sl(e->max_batch, slot), ps(e->max_batch);
    for (int t0 = 0; t0 < ntok; t0 += e->max_batch) {
        const int k = std::min(e->max_batch, ntok - t0);
        for (int i = 0; i < k; i++) ps[i] = pos0 + t0 + i;
        const int run_end = k;
        Q35_TRY(q35b_engine_forward(e, k, tokens + t0, sl.data(), ps.data(), 1, &run_end, next, stream));
    }
    return 0;
}

int q35b_serve(q35b_engine *e, int nseq, const int *prompts, const long long *prompt_off, const int *prompt_len,
               const int *n_gen, int *out, const long long *out_off, int max_batch, long long *steps, void *stream) {
    if (!e || !e->finalized || nseq < 0 || max_batch <= 0) return (int)cudaErrorInvalidValue;
    const int max_seqs = std::min(max_batch, std::min(e->max_batch, e->n_slots));
    const int budget = e->max_batch;  // tokens per forward
    struct Act { int seq, slot, pos, gen, last; };
    std::deque<int> waiting;
    for (int i = 0; i < nseq; i++) {
        if (prompt_len[i] <= 0 || n_gen[i] <= 0) continue;
        if (prompt_len[i] + n_gen[i] - 1 > e->max_seq) return (int)cudaErrorInvalidValue;
        waiting.push_back(i);
    }
    std::vector<int> free_slots;
    for (int s = e->n_slots - 1; s >= 0; s--) free_slots.push_back(s);
    std::vector<Act> act;
    std::vector<int> tok, slot, pos, run_end, run_act, next;
    long long nstep = 0;
    cudaStream_t st = S(stream);
    while (!waiting.empty() || !act.empty()) {
        while ((int)act.size() < max_seqs && !waiting.empty() && !free_slots.empty()) {
            const int s = free_slots.back();
            free_slots.pop_back();
            Q35_TRY(q35b_engine_reset_slot(e, s, st));
            act.push_back({waiting.front(), s, 0, 0, -1});
            waiting.pop_front();
        }
        // decoding sequences first (one token each), then prompt chunks in
        // the remaining token budget
        tok.clear();
        slot.clear();
        pos.clear();
        run_end.clear();
        run_act.clear();
        for (int pass = 0; pass < 2; pass++) {
            for (int i = 0; i < (int)act.size(); i++) {
                const Act &a = act[i];
                const int plen = prompt_len[a.seq];
                const bool decoding = a.pos >= plen;
                if (decoding != (pass == 0)) continue;
                const int room = budget - (int)tok.size();
                if (room <= 0) break;
                const int k = decoding ? 1 : std::min(plen - a.pos, room);
                for (int q = 0; q < k; q++) {
                    tok.push_back(decoding ? a.last : prompts[prompt_off[a.seq] + a.pos + q]);
                    slot.push_back(a.slot);
                    pos.push_back(a.pos + q);
                }
                run_end.push_back((int)tok.size());
                run_act.push_back(i);
            }
        }
        const int nrun = (int)run_end.size();
        next.resize(nrun);
        Q35_TRY(q35b_engine_forward(e, (int)tok.size(), tok.data(), slot.data(), pos.data(), nrun, run_end.data(),
                                    next.data(), st));
        nstep++;
        for (int r = 0; r < nrun; r++) {
            Act &a = act[run_act[r]];
            const int k = run_end[r] - (r ? run_end[r - 1] : 0);
            a.pos += k;
            if (a.pos >= prompt_len[a.seq]) {  // the run reached the last prompt token or decoded
                out[out_off[a.seq] + a.gen] = next[r];
                a.gen++;
                a.last = next[r];
            }
        }
        std::vector<Act> keep;
        for (const Act &a : act) {
            if (a.gen >= n_gen[a.seq])
                free_slots.push_back(a.slot);
            else
                keep.push_back(a);
        }
        act.swap(keep);
    }
    if (steps) *steps = nstep;
    return 0;
}

}  // extern "C"
