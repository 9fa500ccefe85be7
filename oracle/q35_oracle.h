/*
 * q35_oracle.h -- CPU restatement of the reference's hot path, used ONLY as
 * the checker.
 *
 * TEST INFRASTRUCTURE.  Nothing in the product (qwen35_b200/) links, loads or
 * calls this code.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may use it.
 *
 * What it restates (file:line inside the frybox/qwen35 tree):
 *   - block formats and f16 conversion   src/kernels/x86/kernels32.c:46-101,
 *                                         src/gguf.zig:185-215
 *   - activation quantizers Q8_0 / Q8_K  src/kernels/x86/kernels32.c:1064-1090,
 *                                         src/kernels/x86/kernels256.c:865-900
 *   - Q8_0 weight quantizer              src/quant_dequant.zig:1404-1425
 *   - dequantizers                       src/quant_dequant.zig:54-76,188-250,
 *                                         347-360,1388-1402
 *   - scalar block dots                  src/kernels/x86/kernels32.c:342-365,
 *                                         447-466; kernels256.c:185-230,474-498,
 *                                         605-629,720-738
 *   - matvec dispatch                    src/backend_cpu.zig:167-289
 *   - elementwise / norms / GDN / attn   src/elementwise.zig:43-405
 *   - engine op order                    src/engine.zig:1242-1312,1505-1672,
 *                                         1949-2036
 *
 * Parity status: pinned.  tests/test_oracle.py checks the dequantizers and
 * the dot kernels against the reference's golden vectors
 * (testdata/udtest/{Q4_K,Q5_K,Q6_K,IQ4_NL,Q4_0}, copied under tests/golden/)
 * and against the reference's own x86 C kernels compiled from source into
 * oracle/_ref/.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, so no multiply-add is
 * fused and every f32 operation rounds exactly as the reference's scalar
 * path spells it).
 */
#ifndef Q35_ORACLE_H
#define Q35_ORACLE_H

#include <math.h>
#include <stdint.h>
#include <stddef.h>

/* exp and log1p.  By default the C library's f32 functions, which the
 * reference's CPU engine calls.  Built with -DQ35O_CR_EXP: correctly rounded
 * (evaluated in double, rounded once), the device kernels' arithmetic.  The
 * two differ in a last ulp now and then, and one such difference can flip an
 * int8 activation rounding downstream, after which a long decode drifts by a
 * few percent in both directions alike; the correctly rounded build is the
 * oracle for comparisons that must stay exact over many positions. */
#ifdef Q35O_CR_EXP
#define Q35O_EXPF(x) ((float)exp((double)(x)))
#define Q35O_LOG1PF(x) ((float)log1p((double)(x)))
#else
#define Q35O_EXPF(x) expf(x)
#define Q35O_LOG1PF(x) log1pf(x)
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF TensorType ids (src/gguf.zig:87-122). */
#define Q35O_TT_F32 0
#define Q35O_TT_Q4_0 2
#define Q35O_TT_Q4_1 3
#define Q35O_TT_Q5_0 6
#define Q35O_TT_Q5_1 7
#define Q35O_TT_Q8_0 8
#define Q35O_TT_Q4_K 12
#define Q35O_TT_Q5_K 13
#define Q35O_TT_Q6_K 14
#define Q35O_TT_Q8_K 15
#define Q35O_TT_IQ4_NL 20
#define Q35O_TT_IQ4_XS 23

/* ---- formats -------------------------------------------------------- */
float q35o_f16_to_f32(uint16_t h);
uint16_t q35o_f32_to_f16(float x);
/* native block geometry; returns 1 on success */
int q35o_block_geom(int ttype, int *elems, int *bytes);
/* 32 for the Q8_0 activation family, 256 for Q8_K, 0 unknown */
int q35o_act_block_elems(int ttype);
size_t q35o_row_bytes(int ttype, int cols);
size_t q35o_act_row_bytes(int ttype, int cols);

/* ---- activation quantizers (bit-exact with the reference) ----------- */
void q35o_quantize_q8_0(int n, const float *x, uint8_t *out);
void q35o_quantize_q8_K(int n, const float *x, uint8_t *out);
/* quantize x for the activation family of `ttype` */
void q35o_quantize_act(int ttype, int n, const float *x, uint8_t *out);

/* ---- weight quantizers ---------------------------------------------- */
/* Q8_0: the reference's own weight quantizer (quant_dequant.zig:1404). */
void q35o_quantize_weight_q8_0(int n, const float *x, uint8_t *out);
/* IQ4_NL / Q4_K / Q5_K / Q6_K: the reference ships none; these are this
 * project's deterministic encoders (same algorithm as the device encoders in
 * qwen35_b200/csrc/wquant.cu).  Any valid encoding is acceptable because
 * parity is defined from the packed bytes onward. */
void q35o_quantize_weight(int ttype, int n, const float *x, uint8_t *out);
/* seeded synthetic values, bit-identical to the library's q35b_synth_fill */
void q35o_synth_fill(uint64_t key, long long n, float k, float *dst);

/* ---- dequantization -------------------------------------------------- */
void q35o_dequant_row(int ttype, const uint8_t *row, float *out, int cols);

/* ---- scalar block dots (reference scalar tier, strict block order) --- */
float q35o_vec_dot(int ttype, int n, const uint8_t *w, const uint8_t *xq);
/* per-block integer dot of one native block (for bit-exact int checks) */
int32_t q35o_block_isum(int ttype, const uint8_t *wblk, const uint8_t *xblk);

/* out[t*rows + r] = W[r] . xq[t]; xq already quantized for the family */
/* unquantized weights x f32 activation, the reference CUDA order
 * (mmvq.cu:339-367, dotq.cuh:202-218): acc = fmaf(w[c], x[c], acc) per row;
 * w16: ttype 1 (f16) or 30 (bf16), widened exactly */
void q35o_matvec_f32(const float *w, const float *x, float *out, int rows, int cols, int tokens);
void q35o_matvec_w16(int ttype, const uint16_t *w, const float *x, float *out, int rows, int cols, int tokens);
void q35o_matvec_q(int ttype, const uint8_t *w, const uint8_t *xq, float *out,
                   int rows, int cols, int tokens);
/* quantize x (tokens x cols f32) then matvec */
void q35o_matvec(int ttype, const uint8_t *w, const float *x, float *out,
                 int rows, int cols, int tokens);

/* ---- elementwise (src/elementwise.zig) ------------------------------ */
void q35o_rmsnorm(float *out, const float *x, const float *w, int n, float eps);
void q35o_rmsnorm_rows(float *out, const float *x, const float *w, int rows,
                       int n, float eps);
void q35o_l2norm(float *x, int n);
void q35o_l2norm_qk_scale(float *x, int nk, int kd, int k_offset, float qscale);
void q35o_scale_vec(float *x, int n, float s);
float q35o_silu(float x);
float q35o_sigmoid(float x);
float q35o_softplus(float x);
void q35o_silu_vec(float *x, int n);
void q35o_mul_silu(float *out, const float *gate, int n);
void q35o_mul_sigmoid(float *out, const float *gate, int n);
void q35o_swiglu(float *gate, const float *up, int n);
void q35o_softmax(float *x, int n);
void q35o_add_resid(float *dst, const float *src, int n);
void q35o_rope64(float *x, int pos, float base);
void q35o_rope64_rows(float *x, int rows, int heads, int hd, int pos0, float base);
void q35o_conv_step(float *conv, float *y, const float *wconv, int n);
void q35o_gdn_gamma(const float *a_raw, float *b_raw, const float *ssm_a,
                    const float *dt_bias, float *gamma, int nv);
void q35o_gdn_fused(float *state, const float *k, const float *v,
                    const float *q, float *km, float *delta, float *out,
                    float gamma, float beta, int kd, int vd);
void q35o_gdn_step_rows(float *state, const float *k, const float *v,
                        const float *q, float *km, float *delta, float *out,
                        const float *gamma, const float *beta, int heads,
                        int nk, int kd, int vd);
void q35o_deinterleave_qg(float *q, float *gate, const float *src, int heads,
                          int hd);
void q35o_attn_decode(const float *q, const float *gate, const float *kcache,
                      const float *vcache, float *att, float *gout, int slot,
                      int heads, int gqa, int hd, int kv_dim, float scale);
int q35o_argmax(const float *x, int n);
/* Sampler.sample (src/sampler.zig:67-190): greedy at temperature <= 0,
 * else top-k / top-p thresholds and one xorshift64* draw from *state (0
 * selects the fixed default); scratch holds n floats */
int q35o_sample(const float *logits, int n, float temperature, int top_k, float top_p, uint64_t *state,
                float *scratch);
float q35o_kth_largest(float *a, int n, int rank);

/* ---- engine (src/engine.zig forwardLogits / generate) --------------- */
typedef struct q35o_config {
    int n_layers, full_attention_interval, hidden, n_heads, n_kv_heads;
    int head_dim, n_ff, vocab;
    float rms_eps, rope_freq_base;
    int gdn_n_heads, gdn_num_k_heads, gdn_head_dim, conv_kernel;
} q35o_config;

typedef struct q35o_model q35o_model;

/* `threads` <= 1 runs serially (the parity configuration) */
q35o_model *q35o_model_create(const q35o_config *cfg, int max_seq, int threads);
/* replace the row-parallel pool with one of `threads` threads (<= 1: serial) */
void q35o_model_set_threads(q35o_model *m, int threads);
void q35o_model_destroy(q35o_model *m);
/* Register a tensor by its GGUF name.  The pointer is borrowed (caller keeps
 * it alive).  1-D f32 tensors pass ttype 0 and cols = length.  Returns 0 or
 * -1 for an unknown name / bad shape. */
int q35o_model_set_tensor(q35o_model *m, const char *name, int ttype,
                          const void *data, int rows, int cols);
/* 0 when every tensor the config needs is present, else -1 */
int q35o_model_check(q35o_model *m);
void q35o_model_reset(q35o_model *m);
/* one decode step (forwardLogits): returns a pointer to vocab logits owned
 * by the model */
const float *q35o_forward(q35o_model *m, int token, int pos);
/* hidden state after the final norm of the last forward (hidden floats) */
const float *q35o_last_hidden(q35o_model *m);
/* Per-layer probe: after q35o_forward, the residual stream after layer li. */
const float *q35o_layer_out(q35o_model *m, int li);
/* greedy: prefill `n_prompt` tokens serially (decode semantics), then emit
 * n_gen tokens into out.  Returns the number written. */
int q35o_generate(q35o_model *m, const int *prompt, int n_prompt, int n_gen,
                  int *out);
/* decode-only timing helper: runs n_steps greedy steps starting at pos and
 * returns elapsed seconds (wall). */
double q35o_time_decode(q35o_model *m, int first_token, int pos, int n_steps,
                        int *out);
/* name of the dot-kernel tier this build links: "oracle-scalar" or
 * "reference-x86" */
const char *q35o_kernel_tier(void);

#ifdef __cplusplus
}
#endif
#endif
