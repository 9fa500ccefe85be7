/*
 * q35.h -- C ABI of libq35b, the B200 (sm_100a) backend for the Qwen3.5
 * engine.
 *
 * Part 1 re-exports the reference's kernel launcher interface with identical
 * names, signatures, argument meaning and error convention
 * (src/kernels/cuda/api.h of frybox/qwen35; each declaration below cites the
 * line it replaces), so the reference's CUDA host (src/backend_cuda.zig,
 * `Kernels` extern block :80-218 and `Launch` table :283-345) links against
 * this library unchanged.
 *
 * Part 2 is additive (`q35b_*`): a batched decode engine over per-sequence
 * KV / GDN slots, a continuous-batching server loop, device weight encoders
 * and error reporting.  The reference has no counterpart for these (it is a
 * single-sequence engine); they follow the same conventions.
 *
 * Conventions (api.h:1-13): every launcher returns the numeric cudaError_t
 * (0 = success); device pointers and streams are opaque `void *` / typed
 * pointers; the caller owns all memory; zero-size work returns 0 without a
 * launch; nothing aborts.  Launchers are not re-entrant across host threads
 * (per-process static caches), as in the reference.
 */
#ifndef Q35_B200_H
#define Q35_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ===================================================================== */
/* Part 1: the reference's launcher interface (api.h)                     */
/* ===================================================================== */

#define Q35_API_QK8_0 32            /* api.h:23 */
#define Q35_API_Q8_0_BLOCK_BYTES 34 /* api.h:24 */
#define Q35_API_QK_K 256            /* api.h:28 */
#define Q35_API_Q8_K_BLOCK_BYTES 292/* api.h:29 */

/* TensorType ids, equal to GGUF's (api.h:42-75). */
#define Q35_TT_F32 0
#define Q35_TT_F16 1
#define Q35_TT_Q4_0 2
#define Q35_TT_Q8_0 8
#define Q35_TT_Q4_K 12
#define Q35_TT_Q5_K 13
#define Q35_TT_Q6_K 14
#define Q35_TT_Q8_K 15
#define Q35_TT_IQ4_NL 20
#define Q35_TT_IQ4_XS 23
#define Q35_TT_BF16 30

/* device capability probe (api.h:35-37) */
int q35_gpu_cc(void);
int q35_gpu_sm_count(void);
const char *q35_gpu_name(void);

/* activation quantization (api.h:79-93; the _q8_K_mmq twin is exported by
 * the reference's mmvq.cu:1042).  Bit-exact with the reference CPU
 * quantizers.  The mmq layouts are not produced by this backend: the _mmq
 * entry points return cudaErrorNotSupported and q35_mmq_dp4a_wants() is 0,
 * so the caller never asks for them. */
int q35_launch_quantize_q8_0(const float *d_x, void *d_out, int nblocks, void *stream);
int q35_launch_quantize_q8_K(const float *d_x, void *d_out, int nblocks, void *stream);
int q35_launch_quantize_q8_1_mmq(const float *d_x, void *d_y, int nblocks_k, int nrows, void *stream);
int q35_launch_quantize_q8_K_mmq(const float *d_x, void *d_out, void *d_mmq, int nblocks, void *stream);

/* dequantization (api.h:95-105) */
int q35_launch_dequantize(int ttype, const void *d_src, float *d_dst, int nblocks, void *stream);
int q35_launch_dequantize_row(int ttype, const void *d_src_row, float *d_dst, int cols, void *stream);

/* matvec (api.h:110-124): out[t*rows + r] = W[r] . xq[t], bit-exact with the
 * reference scalar CPU tier (per-block integer dot, f32 fold in block order).
 * Types: Q8_0, IQ4_NL, Q4_0, Q4_1, Q5_0, Q5_1 (Q8_0 activation) and Q4_K,
 * Q5_K, Q6_K, IQ4_XS (Q8_K activation; IQ4_XS folds one term per 32-element
 * sub-block, iq_kernels.c:967-1000); others -> cudaErrorInvalidValue. */
int q35_launch_mul_mat_vec(const void *d_w, const void *d_xq, float *d_out, int rows, int cols, int tokens,
                           int ttype, void *stream);
int q35_launch_mul_mat_vec_q8_0(const void *d_w, const void *d_xq, float *d_out, int rows, int cols,
                                int tokens, void *stream);
/* f32 weights x f32 activation (reference mmvq.cu:994) and f16 / bf16
 * weights x f32 activation (mmvq.cu:1011): the reference's CUDA order, one
 * chain per (row, token) acc = fmaf(w[c], x[c], acc) over c = 0..cols-1, the
 * 2-byte weights widened exactly (mmvq.cu:339-367, dotq.cuh:202-218). */
int q35_launch_mul_mat_vec_f32(const float *d_w, const float *d_x, float *d_out, int rows, int cols, int tokens,
                               void *stream);
int q35_launch_mul_mat_vec_w16(const void *d_w, const float *d_x, float *d_out, int rows, int cols, int tokens,
                               int ttype, void *stream);
/* prefill tile path (mmq.cu:2232-2245 in the reference): returns -1
 * ("decline, use q35_launch_mul_mat_vec") for every shape in this build. */
int q35_launch_mul_mat_vec_tile(const void *d_w, const void *d_xq, float *d_out, int rows, int cols, int tokens,
                                int ttype, void *stream);

/* elementwise (api.h:135-154) */
int q35_launch_l2norm_qk_scale(float *d_x, int nk, int kd, int k_offset, float eps, float qscale, void *stream);
int q35_launch_scale_vec(float *d_x, float s, int n, void *stream);
int q35_launch_scale_vec_strided(float *d_x, int offset, float s, int n, int tokens, int stride, void *stream);
int q35_launch_add_resid(float *d_dst, const float *d_src, int n, void *stream);
int q35_launch_copy_range(float *d_dst, const float *d_src, int n, void *stream);
int q35_launch_deinterleave_qg(float *d_q, float *d_gate, const float *d_src, int heads, int hd, void *stream);
int q35_launch_deinterleave_qg_strided(float *d_q, float *d_gate, const float *d_src, int heads, int hd,
                                       int tokens, void *stream);
int q35_launch_zero_buf(float *d_buf, int n, void *stream);
void *q35_func_copy_range(void); /* reference elementwise.cu:157 */
int q35_launch_set_int1(int *d, int v, void *stream);

/* norms (api.h:168-176) */
int q35_launch_rmsnorm(float *d_out, const float *d_x, const float *d_w, int rows, int n, float eps, void *stream);
int q35_launch_l2norm(float *d_x, int rows, int n, float eps, void *stream);
int q35_launch_l2norm_strided(float *d_x, int row_offset, int rows, int n, float eps, int tokens, int row_stride,
                              void *stream);

/* activations / conv (api.h:185-202) */
int q35_launch_silu(float *d_x, int n, void *stream);
int q35_launch_mul_silu(float *d_out, const float *d_gate, int n, void *stream);
int q35_launch_mul_sigmoid(float *d_out, const float *d_gate, int n, void *stream);
int q35_launch_swiglu(float *d_gate, const float *d_up, int n, void *stream);
int q35_launch_softmax(float *d_x, int n, void *stream);
int q35_launch_conv_step(float *d_conv, float *d_y, const float *d_wconv, int n, void *stream);
int q35_launch_conv_step_rows(float *d_conv, float *d_y, const float *d_wconv, int n, int tokens, int y_stride,
                              void *stream);
int q35_launch_argmax(const float *d_x, int n, int *d_out, void *stream);

/* rotary embedding (api.h:217-239) */
int q35_launch_rope64(float *d_x, int heads, int hd, int pos, float base, void *stream);
int q35_launch_rope64_rows(float *d_x, int rows, int heads, int hd, int pos0, float base, void *stream);
void *q35_func_rope64(void); /* reference rope.cu:243-277 */
int q35_launch_rope64_dpos(float *d_x, int heads, int hd, const void *d_dyn, void *stream);
void *q35_func_rope64_dpos(void);
int q35_launch_rope64_rows_dpos(float *d_x, int rows, int heads, int hd, const void *d_dyn, void *stream);
void *q35_func_rope64_rows_dpos(void);
int q35_launch_rope64_setenv(int *d_dyn, int pos, float base, void *stream);

/* gated delta net (api.h:256-335): bit-exact with the CPU gdnFused.
 * q35_launch_gdn_step_wy (api.h:290-308) takes the chunk form's arguments and
 * solves the same recurrence in the WY form, 32 tokens per block, with each
 * block's K K^T and Q K^T on the tensor cores (tf32 x3 split) when the q / k
 * rows are 16-byte aligned: within 1e-4 relative L2 of the per-token kernels,
 * not bitwise.  Calls on one device share the buffer of those products, so
 * order them (one stream, or events). */
int q35_launch_gdn_step_rows(float *d_state, int state_stride, const float *d_k, int k_stride, const float *d_v,
                             int v_stride, const float *d_q, int q_stride, float *d_km, float *d_delta, float *d_out,
                             const float *d_gamma, const float *d_beta, int heads, int nk, int kd, int vd,
                             void *stream);
int q35_launch_gdn_step_rows_chunk(float *d_state, int state_stride, const float *d_k, int k_stride,
                                   const float *d_v, int v_stride, const float *d_q, int q_stride, float *d_km,
                                   int km_stride, float *d_delta, int delta_stride, float *d_out, int out_stride,
                                   const float *d_gamma, int gamma_stride, const float *d_beta, int beta_stride,
                                   int heads, int nk, int kd, int vd, int rows, void *stream);
int q35_launch_gdn_step_wy(float *d_state, int state_stride, const float *d_k, int k_stride, const float *d_v,
                           int v_stride, const float *d_q, int q_stride, float *d_km, int km_stride, float *d_delta,
                           int delta_stride, float *d_out, int out_stride, const float *d_gamma, int gamma_stride,
                           const float *d_beta, int beta_stride, int heads, int nk, int kd, int vd, int rows,
                           void *stream);
int q35_launch_gdn_step(float *d_state, const float *d_k, const float *d_v, const float *d_q, float *d_km,
                        float *d_delta, float *d_out, float gamma, float beta, int vd, void *stream);
int q35_launch_gdn_gamma(const float *d_a_raw, float *d_b_raw, const float *d_ssm_a, const float *d_dt_bias,
                         float *d_gamma, int nv, void *stream);
int q35_launch_gdn_gamma_rows(const float *d_a_raw, float *d_b_raw, const float *d_ssm_a, const float *d_dt_bias,
                              float *d_gamma, int nv, int tokens, int a_stride, int b_stride, int gamma_stride,
                              void *stream);

/* full-attention decode (api.h:337-415); hd must be 256 */
int q35_launch_attn_decode(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                           float *d_att, float *d_gout, int slot, int heads, int gqa, int hd, int kv_dim,
                           float scale, void *stream);
int q35_launch_attn_chunk(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                          float *d_gout, int slot0, int rows, int heads, int gqa, int hd, int kv_dim, float scale,
                          void *stream);
int q35_attn_chunk_max_rows(int slot0);
void *q35_func_attn_decode(void); /* reference attn.cu:393 */
void *q35_func_attn_decode_dyn(void);
void *q35_func_attn_decode_coal(void);
void *q35_func_attn_score_split(void);
int q35_launch_attn_decode_dyn(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                               float *d_att, float *d_gout, const int *d_slot, int heads, int gqa, int hd,
                               int kv_dim, float scale, void *stream);
int q35_launch_attn_decode_coal(const float *d_q, const float *d_gate, const float *d_kcache,
                                const float *d_vcache, float *d_att, float *d_gout, int slot, int heads, int gqa,
                                int hd, int kv_dim, float scale, void *stream);
void *q35_func_attn_score_split_dyn(void);
void *q35_func_attn_pv_split_dyn(void);
void *q35_func_attn_softmax_dyn(void);
void *q35_func_attn_reduce(void);
int q35_launch_attn_decode_split_dyn(const float *d_q, const float *d_gate, const float *d_kcache,
                                     const float *d_vcache, float *d_att, float *d_gout, float *d_part,
                                     const int *d_slot, int heads, int gqa, int hd, int kv_dim, float scale,
                                     int split, void *stream);
int q35_launch_attn_decode_split2(const float *d_q, const float *d_gate, const float *d_kcache,
                                  const float *d_vcache, float *d_att, float *d_gout, float *d_part, int slot,
                                  int heads, int gqa, int hd, int kv_dim, float scale, int split, void *stream);

/* device sampler (reference sample.cu:559-664, control block of 16 int32:
 * [1] temperature bits, [2] top_k, [3] top_p bits, [4..5] PRNG state in,
 * [6] token out, [7..8] PRNG state out, [9] threshold bits out, [10] flags).
 * The selection rules are src/sampler.zig's (greedy at temperature <= 0, the
 * k-th largest value as the top-k threshold with ties kept, top-p as a raised
 * threshold, one xorshift64* draw walked in index order).  n <= 262144.
 * _init allocates the two regions, as in the reference; the kernel keeps its
 * working state on chip, so the scratch region is not written. */
int q35_sample_scratch_ints(void);
int q35_sample_ctl_ints(void);
int q35_launch_sample_init(void **d_ctl, void **d_scratch);
void q35_launch_sample_deinit(void **d_ctl, void **d_scratch);
int q35_launch_sample(const float *d_logits, int n, int *d_ctl, void *d_scratch, void *stream);
/* Prefill-shaped causal attention over a chunk of one sequence: row r
 * (q, gate, out: rows x heads x hd floats) attends to cache positions
 * [0, slot0 + r] in the CPU's operation order (serial dots, max, exp, serial
 * sum, divide, serial P.V, sigmoid gate; src/elementwise.zig:349-372), i.e.
 * bit for bit the rows of a token-by-token decode, with each K / V tile
 * loaded once per 8 rows.  d_scores: caller workspace of rows x heads x
 * scores_ld floats (scores_ld >= slot0 + rows).  hd = 256; heads / gqa kv
 * heads; q, K and V 16-byte aligned.  No counterpart in the reference, whose
 * q35_launch_attn_chunk runs the rows one by one (attn.cu:107-189). */
int q35b_attn_prefill(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                      float *d_gout, float *d_scores, long long scores_ld, int slot0, int rows, int heads, int gqa,
                      int hd, int kv_dim, float scale, void *stream);

/* The sampler over `rows` logits rows (ld floats apart) in one launch; row r
 * uses the control block d_ctl + r * ctl_ld (ctl_ld >= 16).  advance = 1 also
 * writes the advanced PRNG state over the input state ([4..5]), so the next
 * call continues the stream; d_tokens (optional) receives the tokens.  No
 * counterpart in the reference, whose engine samples one row. */
int q35b_sample_rows(const float *d_logits, long long ld, int n, int rows, int *d_ctl, long long ctl_ld, int advance,
                     int *d_tokens, void *stream);

/* codebook upload (api.h:433-442).  The IQ4_NL codebook is compiled into
 * the kernels, so init is a no-op that reports success. */
int q35_launch_init_tables(void *stream);
unsigned long long q35_iq_tables_bytes(void);
int q35_iq_tables_ready(void);
void q35_launch_deinit_tables(void);

/* geometry queries (api.h:446-464) */
int q35_quant_act_block_elems(int ttype);
int q35_quant_geom(int ttype, int *block_elems, int *block_bytes);
int q35_mmq_dp4a_wants(int ttype);
int q35_mmq_act_block_bytes(void);

/* ===================================================================== */
/* Part 2: additive B200 API (no counterpart in the reference)            */
/* ===================================================================== */

/* Last bounded-wait failure recorded by a kernel (0 = none); reading clears
 * it.  A kernel that gives up on a wait records a site code and returns
 * instead of hanging. */
int q35b_get_error(int *code);

/* Failure-detection self-test: one kernel waits on an mbarrier that nothing
 * completes, with the same bounded wait every kernel of this library uses,
 * here limited to limit_ms (1..2000); it gives up, records site 150 for
 * q35b_get_error and returns.  The call returns 0 once the kernel has ended;
 * the context stays usable. */
int q35b_selftest_wait(int limit_ms, void *stream);

/* Device weight encoder: `nblocks` native blocks of `ttype` from f32.
 * Q8_0 is the reference's weight quantizer (src/quant_dequant.zig:1404);
 * IQ4_NL / Q4_K / Q5_K / Q6_K are this library's deterministic encoders. */
int q35b_quantize_weight(int ttype, const float *d_src, void *d_dst, long long nblocks, void *stream);

/* Seeded synthetic values (no counterpart in the reference; its benchmarks
 * load real checkpoints): d_dst[i] = (h0 + h1 + h2 + h3 - 131070) * k for
 * i < n, where h0..h3 are the four 16-bit fields of splitmix64's finalizer
 * applied to key * 0x9E3779B97F4A7C15 + i * 0xD1B54A32D192ED03, and the
 * product is one f32 multiply.  With k = sigma / 37837.23 the values are
 * approximately N(0, sigma^2).  A C restatement of the same integer steps
 * gives the same bits on the host, which lets a CPU run decode the same
 * weights without touching the GPU. */
int q35b_synth_fill(unsigned long long key, long long n, float k, float *d_dst, void *stream);

/* Matvec over up to 4 matrices sharing one quantized activation, with an
 * optional residual add (mode 1: out += W x).  out_ld = floats between
 * tokens.  All matrices must share the activation family of `ttype[0]`.
 * Besides the GGML codes, ttype may be Q35B_TT_Q6_K_PADDED: Q6_K blocks
 * padded from 210 to 224 bytes (zeros after byte 210), the layout the engine
 * repacks Q6_K weights to at load so that rows are 16-byte multiples for TMA
 * (the tensor-core path for 8 tokens and more requires it for Q6_K). */
#define Q35B_TT_Q6_K_PADDED 0x100E

int q35b_mul_mat_vec_multi(int nmat, const void *const *d_w, const int *ttype, const long long *rows,
                           float *const *d_out, const long long *out_ld, const int *mode, const void *d_xq,
                           int cols, int tokens, void *stream);

/* q35b_mul_mat_vec_multi with a caller-provided device workspace (no
 * reference counterpart).  With one matrix of a 256-element family (Q4_K,
 * Q5_K, padded Q6_K) at 8 tokens or more whose row tiles (128 rows each)
 * leave more than half the SMs idle, the tensor-core path splits K over CTAs
 * when work_bytes >= (cols / 256) * tokens * rows * 4: each block's f32 term
 * goes to d_work and a second kernel adds them in block order, so results
 * are identical to the unsplit call.  d_work must not be in use by another
 * call in flight; work_bytes = 0 behaves as q35b_mul_mat_vec_multi. */
int q35b_mul_mat_vec_multi_ws(int nmat, const void *const *d_w, const int *ttype, const long long *rows,
                              float *const *d_out, const long long *out_ld, const int *mode, const void *d_xq,
                              int cols, int tokens, float *d_work, long long work_bytes, void *stream);

/* Decode attention that allocates nothing (no counterpart in the reference):
 * q35_launch_attn_decode's arguments and result, computed split-KV with the
 * partials in one fixed 4.2 MB device array per device instead of a
 * caller buffer.  heads <= 64 (larger: cudaErrorInvalidValue, nothing
 * launched).  The first call on a device looks the array up (make it before
 * any stream capture).  Calls on one device share the array: calls that may
 * overlap in time race on it, so order them on one stream or with events. */
int q35b_attn_decode_noalloc(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                             float *d_gout, int slot, int heads, int gqa, int hd, int kv_dim, float scale,
                             void *stream);

/* ---- batched engine --------------------------------------------------- */
typedef struct q35b_config {
    int n_layers, full_attention_interval, hidden, n_heads, n_kv_heads;
    int head_dim, n_ff, vocab;
    float rms_eps, rope_freq_base;
    int gdn_n_heads, gdn_num_k_heads, gdn_head_dim, conv_kernel;
} q35b_config;

typedef struct q35b_engine q35b_engine;

/* Create an engine on the current device with `n_slots` sequence slots of
 * `max_seq` positions each and room for `max_batch` tokens per step. */
int q35b_engine_create(const q35b_config *cfg, int n_slots, int max_seq, int max_batch, q35b_engine **out);
int q35b_engine_destroy(q35b_engine *e);
/* Register a tensor by GGUF name (blk.N.attn_qkv.weight, token_embd.weight,
 * output.weight, output_norm.weight, ...).  `d_data` is a DEVICE pointer the
 * caller keeps alive.  1-D f32 tensors pass ttype 0 and cols = length. */
int q35b_engine_set_tensor(q35b_engine *e, const char *name, int ttype, const void *d_data, long long rows,
                           long long cols);
/* Validate the tensor set and allocate slots / scratch.  0 or an error. */
int q35b_engine_finalize(q35b_engine *e);
/* Zero the GDN state / conv history of `slot` and forget its KV. */
int q35b_engine_reset_slot(q35b_engine *e, int slot, void *stream);
/* One decode step for `n` sequences, one token each (device arrays of n
 * ints): token id, slot and position (= KV length before the step).  Writes
 * the greedy next token per sequence to d_next; d_logits (n x vocab f32) is
 * optional.  Captured into a CUDA graph per n when use_graph != 0. */
int q35b_engine_step(q35b_engine *e, int n, const int *d_tokens, const int *d_slots, const int *d_pos,
                     int *d_next, float *d_logits, int use_graph, void *stream);
/* Same step with HOST arrays: copies in, runs, copies the next tokens out,
 * synchronizes the stream. */
int q35b_engine_step_host(q35b_engine *e, int n, const int *tokens, const int *slots, const int *pos, int *next,
                          void *stream);
/* The engine's own device input/output arrays (max_batch ints each).  A
 * caller that keeps tokens/slots/positions there steps without copies:
 * q35b_engine_step_dev runs the step on them (max_len = longest context in
 * the batch, an upper bound is fine) and q35b_engine_advance feeds the
 * sampled tokens back (tokens = next, positions += 1) on the device. */
int q35b_engine_device_inputs(q35b_engine *e, int **d_tokens, int **d_slots, int **d_pos, int **d_next);
int q35b_engine_step_dev(q35b_engine *e, int n, int max_len, int use_graph, void *stream);
int q35b_engine_advance(q35b_engine *e, int n, void *stream);
/* Device pointer of the residual stream after layer `li` for the last step
 * (n x hidden f32), for per-layer parity probes; NULL when probing is off. */
int q35b_engine_set_probe(q35b_engine *e, int on);
const float *q35b_engine_layer_out(q35b_engine *e, int li);
/* Kernel launches issued by the last step (graph replays count the nodes). */
long long q35b_engine_launches_per_step(q35b_engine *e);

/* ---- continuous batching --------------------------------------------- */
/* Tensor parallelism (no counterpart in the reference: it runs one GPU).  A
 * rank's engine is created with the rank-local config (heads, kv heads, GDN
 * value / k heads and n_ff divided by nranks; hidden and vocab whole) and fed
 * its shard of every tensor (qwen35_b200/tp.py): row-parallel projections
 * then produce partial sums that are all-reduced (NCCL, loaded at run time)
 * before the residual add, and the lm_head covers rows [vocab_offset,
 * vocab_offset + vocab_local) with a global greedy argmax.  q35b_tp_unique_id
 * (one rank) makes the 128-byte NCCL id every rank passes to
 * q35b_engine_set_tp, which is called by all ranks together, before
 * finalize. */
int q35b_tp_unique_id(void *out, int bytes);
int q35b_engine_set_tp(q35b_engine *e, int nranks, int rank, long long vocab_local, long long vocab_offset,
                       const void *unique_id);
/* The peer all-reduce: the row-parallel all-reduce and the residual add as
 * one kernel over NVLink peer memory (up to 8 ranks, hidden a multiple of
 * 4 x nranks).  After finalize, q35b_engine_ipc_handles writes this rank's
 * 192 bytes of CUDA IPC handles (partial sums, residual, flag words); the
 * ranks exchange them (rank p's at offset 192 p) and each passes the whole
 * set to q35b_engine_set_peers, which maps the other ranks' buffers and
 * switches the engine to the peer form; q35b_engine_set_allreduce(e, 0 / 1)
 * then selects NCCL or the peer form (every rank the same, between steps).
 * Rank q sums the partials of hidden columns [q h/N, (q+1) h/N) in rank
 * order, so all ranks hold the same residual bits; every wait is bounded (2 s)
 * and records error 150 / 151 (q35b_get_error) instead of hanging. */
int q35b_engine_ipc_handles(q35b_engine *e, void *out, int bytes);
int q35b_engine_set_peers(q35b_engine *e, const void *all, int bytes);
int q35b_engine_set_allreduce(q35b_engine *e, int peer);
/* one GPU: runs the peer all-reduce kernel as rank 0 of two whose rank 1
 * never runs, with waits bounded at limit_ns (<= 2 s); returns the stream's
 * status, and q35b_get_error then reports 150 */
int q35b_tp_selftest_timeout(unsigned long long limit_ns, void *stream);

/* One forward over n tokens packed as nrun runs: run r is tokens
 * [run_end[r-1], run_end[r]) (run_end[-1] = 0), all of one slot at
 * consecutive positions; a decode token is a run of one, a prompt chunk a
 * longer run, and one call may mix them (continuous batching; no slot in two
 * runs).  The GDN recurrence steps each run in order; attention is causal per
 * token.  next[r] = greedy token after the last token of run r.  Host
 * arrays; n <= max_batch.  Runs of one token use the step's CUDA graph. */
int q35b_engine_forward(q35b_engine *e, int n, const int *tokens, const int *slots, const int *pos, int nrun,
                        const int *run_end, int *next, void *stream);

/* Runs of 16 tokens or more in a forward with runs longer than one token
 * (prefill, prompt chunks of q35b_serve) through the chunked WY form of the
 * GDN recurrence on the tensor-core Gram pass (on), or every run token by
 * token (off, the default); shorter runs stay per token either way.  WY
 * re-associates the recurrence's sums: it agrees with the per-token form to
 * rounding, not bitwise.  Switching it on for a finalized engine (or
 * finalizing with it on) allocates its scratch; forwards allocate nothing. */
int q35b_engine_set_prefill_wy(q35b_engine *e, int on);

/* Sampling in the engine's step (replaces the greedy argmax when on): every
 * run's next token is drawn with the parameters of its slot, whose PRNG state
 * advances on the device, so the step stays one CUDA graph.  set_sampler sets
 * a slot's parameters and restarts its stream at `seed` (0: the reference's
 * fixed default); temperature <= 0 keeps that slot greedy.  Not with tensor
 * parallelism (the logits are split over the ranks). */
int q35b_engine_set_sampling(q35b_engine *e, int on);
int q35b_engine_set_sampler(q35b_engine *e, int slot, float temperature, int top_k, float top_p,
                            unsigned long long seed);

/* Prompt prefill of one slot: ntok tokens from position pos0 as runs of up
 * to max_batch tokens (src/engine.zig:2078-2177, forwardChunk); *next = greedy token after
 * the last one. */
int q35b_engine_prefill(q35b_engine *e, int slot, const int *tokens, int ntok, int pos0, int *next, void *stream);

/* Serve `nseq` independent requests to completion with at most
 * `max_batch` in flight: each forward packs one token of every decoding
 * sequence, then chunks of waiting prompts up to the engine's max_batch
 * tokens (runs, see q35b_engine_forward), admits waiting requests into freed
 * slots, and stops a sequence after n_gen[i] generated tokens.  prompts are concatenated (prompt_off[i],
 * prompt_len[i]); generated tokens go to out + out_off[i].  Returns 0 or an
 * error; *steps receives the number of engine steps taken. */
int q35b_serve(q35b_engine *e, int nseq, const int *prompts, const long long *prompt_off, const int *prompt_len,
               const int *n_gen, int *out, const long long *out_off, int max_batch, long long *steps,
               void *stream);

#ifdef __cplusplus
}
#endif
#endif
