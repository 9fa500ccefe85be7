/*
 * q35_oracle_engine.c -- CPU restatement of the reference engine's decode
 * step (src/engine.zig forwardLogits/forwardGdn/forwardFull/forwardMlp) and
 * of its row-parallel matvec pool (src/pool.zig:468-533).  TEST
 * INFRASTRUCTURE ONLY (see q35_oracle.h).
 *
 * Built twice by oracle/Makefile:
 *   - oracle/_build/liboracle.so : dot kernels = this restatement's scalar
 *     tier (q35o_vec_dot).  Used by the parity tests.
 *   - oracle/_ref/libq35ref.so   : dot kernels and activation quantizers =
 *     the reference's own x86 C kernels (the .c files of src/kernels/x86, compiled from
 *     the reference tree, default ISA dispatch).  Used as the CPU baseline.
 *
 * Prefill is the serial per-token path (engine.zig:2110-2112, the
 * `nbatch == 0` branch), which gives every prompt token decode semantics.
 */
#include "q35_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#ifdef Q35O_REF_KERNELS
/* the reference's public C kernel API (src/kernels/x86/kernels32.h,
 * kernels256.c public dispatch) */
float q8_0_q8_0(int n, const void *vx, const void *vy);
float iq4_nl_q8_0(int n, const void *vx, const void *vy);
float q4_0_q8_0(int n, const void *vx, const void *vy);
float q4_1_q8_0(int n, const void *vx, const void *vy);
float q5_0_q8_0(int n, const void *vx, const void *vy);
float q5_1_q8_0(int n, const void *vx, const void *vy);
float q4_k_q8_k(int n, const void *vx, const void *vy);
float q5_k_q8_k(int n, const void *vx, const void *vy);
float q6_k_q8_k(int n, const void *vx, const void *vy);
float iq4_xs_q8_k(int n, const void *vx, const void *vy);  /* iq_kernels.c:1004 */
void quantize_q8_0(int n, const float *x, uint8_t *out);
void quantize_q8_K(int n, const float *x, uint8_t *out);

static float row_dot(int tt, int n, const uint8_t *w, const uint8_t *xq)
{
    switch (tt) {
    case Q35O_TT_Q8_0: return q8_0_q8_0(n, w, xq);
    case Q35O_TT_IQ4_NL: return iq4_nl_q8_0(n, w, xq);
    case Q35O_TT_Q4_0: return q4_0_q8_0(n, w, xq);
    case Q35O_TT_Q4_1: return q4_1_q8_0(n, w, xq);
    case Q35O_TT_Q5_0: return q5_0_q8_0(n, w, xq);
    case Q35O_TT_Q5_1: return q5_1_q8_0(n, w, xq);
    case Q35O_TT_Q4_K: return q4_k_q8_k(n, w, xq);
    case Q35O_TT_Q5_K: return q5_k_q8_k(n, w, xq);
    case Q35O_TT_Q6_K: return q6_k_q8_k(n, w, xq);
    case Q35O_TT_IQ4_XS: return iq4_xs_q8_k(n, w, xq);
    default: return q35o_vec_dot(tt, n, w, xq);
    }
}
static void quant_act(int tt, int n, const float *x, uint8_t *out)
{
    if (q35o_act_block_elems(tt) == 32)
        quantize_q8_0(n, x, out);
    else
        quantize_q8_K(n, x, out);
}
const char *q35o_kernel_tier(void) { return "reference-x86"; }
#else
static float row_dot(int tt, int n, const uint8_t *w, const uint8_t *xq)
{
    return q35o_vec_dot(tt, n, w, xq);
}
static void quant_act(int tt, int n, const float *x, uint8_t *out)
{
    q35o_quantize_act(tt, n, x, out);
}
const char *q35o_kernel_tier(void) { return "oracle-scalar"; }
#endif

/* ====================================================================== */
/* row-parallel pool (src/pool.zig:468-533): chunk = clamp(rows/(4n),16,256),
 * rows claimed by fetch-add, the calling thread participates, rows < 256
 * run serially.                                                           */
/* ====================================================================== */

typedef struct {
    int tt, cols;
    const uint8_t *w;
    size_t row_bytes;
    const uint8_t *xq;
    float *out;
} mv_task;

typedef struct pool {
    int n;
    pthread_t *th;
    pthread_mutex_t mu;
    pthread_cond_t cv_go, cv_done;
    long gen;
    int stop;
    mv_task task;
    int rows, chunk;
    atomic_int next;
    atomic_int busy;
} pool;

static void run_rows(const mv_task *t, int lo, int hi)
{
    for (int r = lo; r < hi; r++) t->out[r] = row_dot(t->tt, t->cols, t->w + (size_t)r * t->row_bytes, t->xq);
}

static void pool_drain(pool *p)
{
    for (;;) {
        const int lo = atomic_fetch_add(&p->next, p->chunk);
        if (lo >= p->rows) break;
        const int hi = lo + p->chunk < p->rows ? lo + p->chunk : p->rows;
        run_rows(&p->task, lo, hi);
    }
}

static void *pool_worker(void *arg)
{
    pool *p = (pool *)arg;
    long seen = 0;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        while (p->gen == seen && !p->stop) pthread_cond_wait(&p->cv_go, &p->mu);
        if (p->stop) {
            pthread_mutex_unlock(&p->mu);
            return NULL;
        }
        seen = p->gen;
        pthread_mutex_unlock(&p->mu);
        pool_drain(p);
        if (atomic_fetch_sub(&p->busy, 1) == 1) {
            pthread_mutex_lock(&p->mu);
            pthread_cond_signal(&p->cv_done);
            pthread_mutex_unlock(&p->mu);
        }
    }
}

static pool *pool_create(int n)
{
    if (n <= 1) return NULL;
    pool *p = (pool *)calloc(1, sizeof(pool));
    p->n = n;
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->cv_go, NULL);
    pthread_cond_init(&p->cv_done, NULL);
    p->th = (pthread_t *)calloc((size_t)n - 1, sizeof(pthread_t));
    for (int i = 0; i < n - 1; i++) pthread_create(&p->th[i], NULL, pool_worker, p);
    return p;
}

static void pool_destroy(pool *p)
{
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    p->stop = 1;
    pthread_cond_broadcast(&p->cv_go);
    pthread_mutex_unlock(&p->mu);
    for (int i = 0; i < p->n - 1; i++) pthread_join(p->th[i], NULL);
    free(p->th);
    free(p);
}

static void pool_matvec(pool *p, const mv_task *t, int rows)
{
    if (!p || rows < 256) {
        run_rows(t, 0, rows);
        return;
    }
    int chunk = rows / (4 * p->n);
    if (chunk < 16) chunk = 16;
    if (chunk > 256) chunk = 256;
    pthread_mutex_lock(&p->mu);
    p->task = *t;
    p->rows = rows;
    p->chunk = chunk;
    atomic_store(&p->next, 0);
    atomic_store(&p->busy, p->n - 1);
    p->gen++;
    pthread_cond_broadcast(&p->cv_go);
    pthread_mutex_unlock(&p->mu);
    pool_drain(p);
    pthread_mutex_lock(&p->mu);
    while (atomic_load(&p->busy) > 0) pthread_cond_wait(&p->cv_done, &p->mu);
    pthread_mutex_unlock(&p->mu);
}

/* ====================================================================== */
/* model                                                                   */
/* ====================================================================== */

typedef struct {
    int tt, rows, cols;
    const uint8_t *data;
} lin_t;

typedef struct {
    const float *attn_norm, *post_attention_norm;
    lin_t attn_qkv, attn_gate, ssm_alpha, ssm_beta, ssm_out;
    const float *ssm_conv1d, *ssm_dt_bias, *ssm_a, *ssm_norm;
    lin_t attn_q, attn_k, attn_v, attn_output;
    const float *attn_q_norm, *attn_k_norm;
    lin_t ffn_gate, ffn_up, ffn_down;
} layer_t;

struct q35o_model {
    q35o_config c;
    int max_seq;
    pool *pool;
    lin_t token_embd, output;
    const float *output_norm;
    layer_t *L;
    float **kc, **vc;
    int *kv_len;
    float **conv, **state;
    float *x, *x1, *x2, *qkv, *z, *ab, *gout, *q, *k, *v, *att, *mh, *mh1;
    float *logits, *delta, *km, *gamma, *lout;
    uint8_t *xq;
};

static int is_full(const q35o_config *c, int li)
{
    return c->full_attention_interval > 0 &&
           li % c->full_attention_interval == c->full_attention_interval - 1;
}

static void *zalloc(size_t n) { return calloc(n ? n : 1, 1); }

q35o_model *q35o_model_create(const q35o_config *cfg, int max_seq, int threads)
{
    q35o_model *m = (q35o_model *)zalloc(sizeof(*m));
    m->c = *cfg;
    m->max_seq = max_seq;
    m->pool = pool_create(threads);
    const q35o_config *c = cfg;
    const int nl = c->n_layers;
    m->L = (layer_t *)zalloc(sizeof(layer_t) * nl);
    m->kc = (float **)zalloc(sizeof(float *) * nl);
    m->vc = (float **)zalloc(sizeof(float *) * nl);
    m->kv_len = (int *)zalloc(sizeof(int) * nl);
    m->conv = (float **)zalloc(sizeof(float *) * nl);
    m->state = (float **)zalloc(sizeof(float *) * nl);
    const size_t kv_dim = (size_t)c->n_kv_heads * c->head_dim;
    const size_t kd = c->gdn_head_dim;
    const size_t conv_dim = 2 * (size_t)c->gdn_num_k_heads * kd + (size_t)c->gdn_n_heads * kd;
    for (int li = 0; li < nl; li++) {
        if (is_full(c, li)) {
            m->kc[li] = (float *)zalloc(sizeof(float) * max_seq * kv_dim);
            m->vc[li] = (float *)zalloc(sizeof(float) * max_seq * kv_dim);
        } else {
            m->conv[li] = (float *)zalloc(sizeof(float) * conv_dim * (c->conv_kernel - 1));
            m->state[li] = (float *)zalloc(sizeof(float) * c->gdn_n_heads * kd * kd);
        }
    }
    const size_t q_dim = (size_t)c->n_heads * c->head_dim;
    const size_t vdim = (size_t)c->gdn_n_heads * kd;
    size_t wide = conv_dim > 2 * q_dim ? conv_dim : 2 * q_dim;
    size_t zw = vdim > q_dim ? vdim : q_dim;
    m->x = (float *)zalloc(4 * c->hidden);
    m->x1 = (float *)zalloc(4 * c->hidden);
    m->x2 = (float *)zalloc(4 * c->hidden);
    m->qkv = (float *)zalloc(4 * wide);
    m->z = (float *)zalloc(4 * zw);
    m->gout = (float *)zalloc(4 * zw);
    m->ab = (float *)zalloc(4 * 2 * c->gdn_n_heads);
    m->q = (float *)zalloc(4 * q_dim);
    m->k = (float *)zalloc(4 * kv_dim);
    m->v = (float *)zalloc(4 * kv_dim);
    m->att = (float *)zalloc(4 * (size_t)max_seq);
    m->mh = (float *)zalloc(4 * c->n_ff);
    m->mh1 = (float *)zalloc(4 * c->n_ff);
    m->logits = (float *)zalloc(4 * (size_t)c->vocab);
    m->delta = (float *)zalloc(4 * vdim);
    m->km = (float *)zalloc(4 * vdim);
    m->gamma = (float *)zalloc(4 * c->gdn_n_heads);
    m->lout = (float *)zalloc(4 * (size_t)c->hidden * nl);
    size_t maxc = c->hidden;
    if ((size_t)c->n_ff > maxc) maxc = c->n_ff;
    if (vdim > maxc) maxc = vdim;
    if (q_dim > maxc) maxc = q_dim;
    m->xq = (uint8_t *)zalloc(maxc / 32 * 34 + maxc / 256 * 292 + 64);
    return m;
}

void q35o_model_set_threads(q35o_model *m, int threads)
{
    pool_destroy(m->pool);
    m->pool = pool_create(threads);
}

void q35o_model_destroy(q35o_model *m)
{
    if (!m) return;
    for (int li = 0; li < m->c.n_layers; li++) {
        free(m->kc[li]);
        free(m->vc[li]);
        free(m->conv[li]);
        free(m->state[li]);
    }
    free(m->kc); free(m->vc); free(m->kv_len); free(m->conv); free(m->state); free(m->L);
    free(m->x); free(m->x1); free(m->x2); free(m->qkv); free(m->z); free(m->gout); free(m->ab);
    free(m->q); free(m->k); free(m->v); free(m->att); free(m->mh); free(m->mh1); free(m->logits);
    free(m->delta); free(m->km); free(m->gamma); free(m->lout); free(m->xq);
    pool_destroy(m->pool);
    free(m);
}

static int set_lin(lin_t *l, int tt, const void *d, int rows, int cols)
{
    if (!q35o_act_block_elems(tt)) return -1;
    l->tt = tt;
    l->rows = rows;
    l->cols = cols;
    l->data = (const uint8_t *)d;
    return 0;
}

int q35o_model_set_tensor(q35o_model *m, const char *name, int tt, const void *d, int rows, int cols)
{
    (void)rows;
    if (!strcmp(name, "token_embd.weight")) return set_lin(&m->token_embd, tt, d, rows, cols);
    if (!strcmp(name, "output.weight")) return set_lin(&m->output, tt, d, rows, cols);
    if (!strcmp(name, "output_norm.weight")) { m->output_norm = (const float *)d; return 0; }
    int li = -1, off = 0;
    if (sscanf(name, "blk.%d.%n", &li, &off) != 1 || li < 0 || li >= m->c.n_layers) return -1;
    const char *t = name + off;
    layer_t *L = &m->L[li];
#define F32(nm, fld) if (!strcmp(t, nm)) { if (tt != Q35O_TT_F32) return -1; L->fld = (const float *)d; return 0; }
#define LIN(nm, fld) if (!strcmp(t, nm)) return set_lin(&L->fld, tt, d, rows, cols);
    F32("attn_norm.weight", attn_norm)
    F32("post_attention_norm.weight", post_attention_norm)
    F32("ssm_conv1d.weight", ssm_conv1d)
    F32("ssm_dt.bias", ssm_dt_bias)
    F32("ssm_a", ssm_a)
    F32("ssm_norm.weight", ssm_norm)
    F32("attn_q_norm.weight", attn_q_norm)
    F32("attn_k_norm.weight", attn_k_norm)
    LIN("attn_qkv.weight", attn_qkv)
    LIN("attn_gate.weight", attn_gate)
    LIN("ssm_alpha.weight", ssm_alpha)
    LIN("ssm_beta.weight", ssm_beta)
    LIN("ssm_out.weight", ssm_out)
    LIN("attn_q.weight", attn_q)
    LIN("attn_k.weight", attn_k)
    LIN("attn_v.weight", attn_v)
    LIN("attn_output.weight", attn_output)
    LIN("ffn_gate.weight", ffn_gate)
    LIN("ffn_up.weight", ffn_up)
    LIN("ffn_down.weight", ffn_down)
#undef F32
#undef LIN
    return -1;
}

int q35o_model_check(q35o_model *m)
{
    if (!m->token_embd.data || !m->output_norm) return -1;
    for (int li = 0; li < m->c.n_layers; li++) {
        const layer_t *L = &m->L[li];
        if (!L->attn_norm || !L->post_attention_norm || !L->ffn_gate.data || !L->ffn_up.data || !L->ffn_down.data)
            return -1;
        if (is_full(&m->c, li)) {
            if (!L->attn_q.data || !L->attn_k.data || !L->attn_v.data || !L->attn_output.data ||
                !L->attn_q_norm || !L->attn_k_norm)
                return -1;
        } else {
            if (!L->attn_qkv.data || !L->attn_gate.data || !L->ssm_alpha.data || !L->ssm_beta.data ||
                !L->ssm_out.data || !L->ssm_conv1d || !L->ssm_dt_bias || !L->ssm_a || !L->ssm_norm)
                return -1;
        }
    }
    return 0;
}

void q35o_model_reset(q35o_model *m)
{
    const q35o_config *c = &m->c;
    const size_t kd = c->gdn_head_dim;
    const size_t conv_dim = 2 * (size_t)c->gdn_num_k_heads * kd + (size_t)c->gdn_n_heads * kd;
    for (int li = 0; li < c->n_layers; li++) {
        m->kv_len[li] = 0;
        if (m->conv[li]) memset(m->conv[li], 0, sizeof(float) * conv_dim * (c->conv_kernel - 1));
        if (m->state[li]) memset(m->state[li], 0, sizeof(float) * c->gdn_n_heads * kd * kd);
    }
}

/* out[rows] = W . x  (backend_cpu.zig:167-289: quantize x once, one row dot
 * per output row) */
static void matvec(q35o_model *m, float *out, const lin_t *w, const float *x)
{
    quant_act(w->tt, w->cols, x, m->xq);
    mv_task t = {w->tt, w->cols, w->data, q35o_row_bytes(w->tt, w->cols), m->xq, out};
    pool_matvec(m->pool, &t, w->rows);
}

static void forward_gdn(q35o_model *m, int li)
{
    const q35o_config *c = &m->c;
    const layer_t *L = &m->L[li];
    const int nv = c->gdn_n_heads, nk = c->gdn_num_k_heads, kd = c->gdn_head_dim, vd = kd;
    const int kq_dim = nk * kd, conv_dim = 2 * kq_dim + nv * vd, vdim = nv * vd;
    (void)conv_dim;
    /* engine.zig:1505-1672 */
    q35o_rmsnorm(m->x1, m->x, L->attn_norm, c->hidden, c->rms_eps);
    matvec(m, m->qkv, &L->attn_qkv, m->x1);
    matvec(m, m->z, &L->attn_gate, m->x1);
    matvec(m, m->ab, &L->ssm_alpha, m->x1);
    matvec(m, m->ab + nv, &L->ssm_beta, m->x1);
    q35o_conv_step(m->conv[li], m->qkv, L->ssm_conv1d, 2 * kq_dim + vdim);
    q35o_gdn_gamma(m->ab, m->ab + nv, L->ssm_a, L->ssm_dt_bias, m->gamma, nv);
    const float qscale = 1.0f / sqrtf((float)kd);
    if (nk != 0 && nv % nk == 0) {
        q35o_l2norm_qk_scale(m->qkv, nk, kd, kq_dim, qscale);
    } else {
        for (int h = 0; h < nv; h++) {
            const int kh = h % nk;
            q35o_l2norm(m->qkv + kh * kd, kd);
            q35o_l2norm(m->qkv + kq_dim + kh * kd, kd);
            q35o_scale_vec(m->qkv + kh * kd, kd, qscale);
        }
    }
    q35o_gdn_step_rows(m->state[li], m->qkv + kq_dim, m->qkv + 2 * kq_dim, m->qkv, m->km, m->delta,
                       m->gout, m->gamma, m->ab + nv, nv, nk, kd, vd);
    q35o_rmsnorm_rows(m->gout, m->gout, L->ssm_norm, nv, vd, c->rms_eps);
    q35o_mul_silu(m->gout, m->z, vdim);
    matvec(m, m->x2, &L->ssm_out, m->gout);
    q35o_add_resid(m->x, m->x2, c->hidden);
}

static void forward_full(q35o_model *m, int li, int pos)
{
    const q35o_config *c = &m->c;
    const layer_t *L = &m->L[li];
    const int heads = c->n_heads, kvh = c->n_kv_heads, hd = c->head_dim;
    const int kv_dim = kvh * hd, gqa = heads / kvh;
    /* engine.zig:1949-2023 */
    q35o_rmsnorm(m->x1, m->x, L->attn_norm, c->hidden, c->rms_eps);
    matvec(m, m->qkv, &L->attn_q, m->x1);
    q35o_deinterleave_qg(m->q, m->z, m->qkv, heads, hd);
    matvec(m, m->k, &L->attn_k, m->x1);
    matvec(m, m->v, &L->attn_v, m->x1);
    q35o_rmsnorm_rows(m->q, m->q, L->attn_q_norm, heads, hd, c->rms_eps);
    q35o_rmsnorm_rows(m->k, m->k, L->attn_k_norm, kvh, hd, c->rms_eps);
    q35o_rope64_rows(m->q, 1, heads, hd, pos, c->rope_freq_base);
    q35o_rope64_rows(m->k, 1, kvh, hd, pos, c->rope_freq_base);
    const int slot = m->kv_len[li];
    memcpy(m->kc[li] + (size_t)slot * kv_dim, m->k, sizeof(float) * kv_dim);
    memcpy(m->vc[li] + (size_t)slot * kv_dim, m->v, sizeof(float) * kv_dim);
    m->kv_len[li]++;
    const float scale = 1.0f / sqrtf((float)hd);
    q35o_attn_decode(m->q, m->z, m->kc[li], m->vc[li], m->att, m->gout, slot, heads, gqa, hd, kv_dim, scale);
    matvec(m, m->x2, &L->attn_output, m->gout);
    q35o_add_resid(m->x, m->x2, c->hidden);
}

static void forward_mlp(q35o_model *m, int li)
{
    const q35o_config *c = &m->c;
    const layer_t *L = &m->L[li];
    /* engine.zig:2027-2036 */
    q35o_rmsnorm(m->x1, m->x, L->post_attention_norm, c->hidden, c->rms_eps);
    matvec(m, m->mh, &L->ffn_gate, m->x1);
    matvec(m, m->mh1, &L->ffn_up, m->x1);
    q35o_swiglu(m->mh, m->mh1, c->n_ff);
    matvec(m, m->x2, &L->ffn_down, m->mh);
    q35o_add_resid(m->x, m->x2, c->hidden);
}

const float *q35o_forward(q35o_model *m, int token, int pos)
{
    const q35o_config *c = &m->c;
    /* engine.zig:1242-1312; embedding = dequantRow of the token's row */
    const lin_t *E = &m->token_embd;
    q35o_dequant_row(E->tt, E->data + (size_t)token * q35o_row_bytes(E->tt, E->cols), m->x, c->hidden);
    for (int li = 0; li < c->n_layers; li++) {
        if (is_full(c, li))
            forward_full(m, li, pos);
        else
            forward_gdn(m, li);
        forward_mlp(m, li);
        memcpy(m->lout + (size_t)li * c->hidden, m->x, sizeof(float) * c->hidden);
    }
    q35o_rmsnorm(m->x1, m->x, m->output_norm, c->hidden, c->rms_eps);
    const lin_t *W = m->output.data ? &m->output : &m->token_embd;
    matvec(m, m->logits, W, m->x1);
    return m->logits;
}

const float *q35o_last_hidden(q35o_model *m) { return m->x1; }
const float *q35o_layer_out(q35o_model *m, int li) { return m->lout + (size_t)li * m->c.hidden; }

int q35o_generate(q35o_model *m, const int *prompt, int n_prompt, int n_gen, int *out)
{
    q35o_model_reset(m);
    const float *lg = NULL;
    for (int i = 0; i < n_prompt; i++) lg = q35o_forward(m, prompt[i], i);
    int next = q35o_argmax(lg, m->c.vocab);
    int pos = n_prompt, n = 0;
    while (n < n_gen && pos < m->max_seq) {
        out[n++] = next;
        lg = q35o_forward(m, next, pos++);
        next = q35o_argmax(lg, m->c.vocab);
    }
    return n;
}

double q35o_time_decode(q35o_model *m, int first_token, int pos, int n_steps, int *out)
{
    struct timespec a, b;
    clock_gettime(CLOCK_MONOTONIC, &a);
    int tok = first_token;
    for (int i = 0; i < n_steps && pos < m->max_seq; i++) {
        const float *lg = q35o_forward(m, tok, pos++);
        tok = q35o_argmax(lg, m->c.vocab);
        if (out) out[i] = tok;
    }
    clock_gettime(CLOCK_MONOTONIC, &b);
    return (double)(b.tv_sec - a.tv_sec) + 1e-9 * (double)(b.tv_nsec - a.tv_nsec);
}
