// api.cuh -- the reference's launcher interface (src/kernels/cuda/api.h),
// implemented on this library's sm_100a kernels.  Same names, signatures,
// argument meaning and error convention; see include/q35.h.
#pragma once
#include "common.cuh"

namespace q35 {

inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }

struct DevCaps {
    int dev = -1, cc = -1, sms = 0;
    char name[256] = {0};
};

inline DevCaps &caps() {
    static DevCaps c[16];
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 16) d = 0;
    DevCaps &x = c[d];
    if (x.dev != d) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) == cudaSuccess) {
            x.cc = p.major * 100 + p.minor;
            x.sms = p.multiProcessorCount;
            strncpy(x.name, p.name, sizeof(x.name) - 1);
        } else {
            x.cc = -1;
            x.sms = 0;
        }
        x.dev = d;
    }
    return x;
}

int gemv_sm_count() {
    const int n = caps().sms;
    return n > 0 ? n : 148;
}

}  // namespace q35

using namespace q35;

extern "C" {

// ---- caps (api.h:35-37) ----
int q35_gpu_cc(void) { return caps().cc; }
int q35_gpu_sm_count(void) { return caps().sms; }
const char *q35_gpu_name(void) { return caps().name; }

// ---- activation quantizers (api.h:79-93) ----
int q35_launch_quantize_q8_0(const float *d_x, void *d_out, int nblocks, void *stream) {
    if (nblocks <= 0) return 0;
    k_quantize_q8_0<<<(nblocks + 7) / 8, 256, 0, S(stream)>>>(d_x, (uint8_t *)d_out, nblocks);
    return (int)cudaGetLastError();
}
int q35_launch_quantize_q8_K(const float *d_x, void *d_out, int nblocks, void *stream) {
    if (nblocks <= 0) return 0;
    if ((reinterpret_cast<uintptr_t>(d_out) & 3u) || (reinterpret_cast<uintptr_t>(d_x) & 15u))
        return (int)cudaErrorMisalignedAddress;
    k_quantize_q8_K<<<(nblocks + 7) / 8, 256, 0, S(stream)>>>(d_x, (uint8_t *)d_out, nblocks);
    return (int)cudaGetLastError();
}
int q35_launch_quantize_q8_1_mmq(const float *, void *, int, int, void *) { return (int)cudaErrorNotSupported; }
int q35_launch_quantize_q8_K_mmq(const float *, void *, void *, int, void *) { return (int)cudaErrorNotSupported; }

// ---- dequantization (api.h:95-105) ----
int q35_launch_dequantize_row(int ttype, const void *d_src_row, float *d_dst, int cols, void *stream) {
    const Geom g = geom_of(ttype);
    if (!g.elems) return (int)cudaErrorInvalidValue;
    if (cols <= 0) return 0;
    if (cols % g.elems) return (int)cudaErrorInvalidValue;
    k_dequant_row<<<(cols + 255) / 256, 256, 0, S(stream)>>>(ttype, (const uint8_t *)d_src_row, d_dst, cols);
    return (int)cudaGetLastError();
}
int q35_launch_dequantize(int ttype, const void *d_src, float *d_dst, int nblocks, void *stream) {
    const Geom g = geom_of(ttype);
    if (!g.elems) return (int)cudaErrorInvalidValue;
    if (nblocks <= 0) return 0;
    return q35_launch_dequantize_row(ttype, d_src, d_dst, nblocks * g.elems, stream);
}

// ---- matvec (api.h:110-124) ----
// Raw 210-byte Q6_K rows at MMQ_MIN_TOK tokens or more go to the tensor-core
// MMQ after a repack to the 224-byte layout, in a per-device buffer kept
// between calls.  The buffer grows only outside stream capture (cudaMalloc
// there would break a capture); a captured call that finds it too small runs
// the block-splitting kernel on the raw rows instead.  Calls on one device
// share the buffer, so they must be ordered (one stream, or events), as the
// single-threaded host of the reference orders them.
struct Q6Repack {
    void *p = nullptr;
    size_t bytes = 0;
};
inline Q6Repack &q6_repack_buf(int dev) {
    static Q6Repack bufs[64];
    return bufs[dev & 63];
}
inline int q6k_raw_mmq(const void *d_w, const void *d_xq, float *d_out, int rows, int cols, int tokens,
                       cudaStream_t st) {
    if (tokens < MMQ_MIN_TOK || cols % 256 || (reinterpret_cast<uintptr_t>(d_w) & 1u)) return -1;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    Q6Repack &b = q6_repack_buf(dev);
    const long long nblk = (long long)rows * (cols / 256);
    const size_t need = (size_t)nblk * 224;
    if (b.bytes < need) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusActive;
        if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return -1;
        void *p = nullptr;
        if (cudaMalloc(&p, need) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        if (b.p) cudaFree(b.p);
        b.p = p;
        b.bytes = need;
    }
    k_repack_q6k<<<(unsigned)((nblk * 112 + 255) / 256), 256, 0, st>>>(static_cast<const uint8_t *>(d_w),
                                                                      static_cast<uint8_t *>(b.p), nblk);
    const int rc = (int)cudaGetLastError();
    if (rc) return rc;
    GemvSegDesc s{b.p, d_out, rows, TT_Q6_K_P, rows, GV_STORE};
    return mmq_launch(&s, 1, d_xq, cols, tokens, st, 0, nullptr, 0);
}

int q35_launch_mul_mat_vec(const void *d_w, const void *d_xq, float *d_out, int rows, int cols, int tokens, int ttype,
                           void *stream) {
    if (rows <= 0 || cols <= 0 || tokens <= 0) return 0;
    const Geom g = geom_of(ttype);
    if (!g.elems || cols % g.elems) return (int)cudaErrorInvalidValue;
    if (ttype == TT_Q6_K) {
        const int rc = q6k_raw_mmq(d_w, d_xq, d_out, rows, cols, tokens, S(stream));
        if (rc != -1) return rc;
    }
    GemvSegDesc s{d_w, d_out, rows, ttype, rows, GV_STORE};
    return gemv_launch(&s, 1, d_xq, cols, tokens, S(stream));
}
int q35_launch_mul_mat_vec_q8_0(const void *d_w, const void *d_xq, float *d_out, int rows, int cols, int tokens,
                                void *stream) {
    return q35_launch_mul_mat_vec(d_w, d_xq, d_out, rows, cols, tokens, TT_Q8_0, stream);
}
int q35_launch_mul_mat_vec_f32(const float *d_w, const float *d_x, float *d_out, int rows, int cols, int tokens,
                               void *stream) {
    if (rows <= 0 || cols <= 0 || tokens <= 0) return 0;
    k_matvec_seq<MV_F32><<<dim3((unsigned)((rows + 127) / 128), (unsigned)tokens), 128, 0, S(stream)>>>(
        d_w, d_x, d_out, rows, cols);
    return (int)cudaGetLastError();
}
int q35_launch_mul_mat_vec_w16(const void *d_w, const float *d_x, float *d_out, int rows, int cols, int tokens, int ttype,
                               void *stream) {
    if (rows <= 0 || cols <= 0 || tokens <= 0) return 0;
    if (ttype != TT_F16 && ttype != TT_BF16) return (int)cudaErrorInvalidValue;
    const dim3 grid((unsigned)((rows + 127) / 128), (unsigned)tokens);
    if (ttype == TT_BF16)
        k_matvec_seq<MV_BF16><<<grid, 128, 0, S(stream)>>>(d_w, d_x, d_out, rows, cols);
    else
        k_matvec_seq<MV_F16><<<grid, 128, 0, S(stream)>>>(d_w, d_x, d_out, rows, cols);
    return (int)cudaGetLastError();
}
int q35_launch_mul_mat_vec_tile(const void *, const void *, float *, int, int, int, int, void *) { return -1; }

// ---- elementwise (api.h:135-154) ----
int q35_launch_scale_vec(float *d_x, float s, int n, void *stream) {
    if (n <= 0) return 0;
    k_scale_vec<<<ew_grid(n), 256, 0, S(stream)>>>(d_x, s, n);
    return (int)cudaGetLastError();
}
int q35_launch_scale_vec_strided(float *d_x, int offset, float s, int n, int tokens, int stride, void *stream) {
    if (n <= 0 || tokens <= 0) return 0;
    k_scale_vec_strided<<<ew_grid((long long)n * tokens), 256, 0, S(stream)>>>(d_x, offset, s, n, tokens, stride);
    return (int)cudaGetLastError();
}
int q35_launch_add_resid(float *d_dst, const float *d_src, int n, void *stream) {
    if (n <= 0) return 0;
    k_add_resid<<<ew_grid(n), 256, 0, S(stream)>>>(d_dst, d_src, n);
    return (int)cudaGetLastError();
}
int q35_launch_copy_range(float *d_dst, const float *d_src, int n, void *stream) {
    if (n <= 0) return 0;
    k_copy<<<ew_grid(n), 256, 0, S(stream)>>>(d_dst, d_src, n);
    return (int)cudaGetLastError();
}
int q35_launch_deinterleave_qg_strided(float *d_q, float *d_gate, const float *d_src, int heads, int hd, int tokens,
                                       void *stream) {
    if (heads <= 0 || hd <= 0 || tokens <= 0) return 0;
    k_deinterleave_qg<<<ew_grid((long long)heads * hd * tokens), 256, 0, S(stream)>>>(d_q, d_gate, d_src, heads, hd,
                                                                                    tokens);
    return (int)cudaGetLastError();
}
int q35_launch_deinterleave_qg(float *d_q, float *d_gate, const float *d_src, int heads, int hd, void *stream) {
    return q35_launch_deinterleave_qg_strided(d_q, d_gate, d_src, heads, hd, 1, stream);
}
void *q35_func_copy_range(void) { return (void *)k_copy; }
int q35_launch_zero_buf(float *d_buf, int n, void *stream) {
    if (n <= 0) return 0;
    k_zero<<<ew_grid(n), 256, 0, S(stream)>>>(d_buf, n);
    return (int)cudaGetLastError();
}
int q35_launch_set_int1(int *d, int v, void *stream) {
    k_set_int1<<<1, 1, 0, S(stream)>>>(d, v);
    return (int)cudaGetLastError();
}

// ---- norms (api.h:135, 168-176) ----
int q35_launch_rmsnorm(float *d_out, const float *d_x, const float *d_w, int rows, int n, float eps, void *stream) {
    if (rows <= 0 || n <= 0) return 0;
    if (n > 8192) return (int)cudaErrorInvalidValue;
    k_rmsnorm<256><<<rows, 256, (size_t)n * 4, S(stream)>>>(d_out, d_x, d_w, n, eps);
    return (int)cudaGetLastError();
}
int q35_launch_l2norm_strided(float *d_x, int row_offset, int rows, int n, float eps, int tokens, int row_stride,
                              void *stream) {
    if (rows <= 0 || n <= 0 || tokens <= 0) return 0;
    if (n > 8192) return (int)cudaErrorInvalidValue;
    k_l2norm<128><<<rows * tokens, 128, (size_t)n * 4, S(stream)>>>(d_x, row_offset, rows, n, eps, row_stride, 1.0f, 0);
    return (int)cudaGetLastError();
}
int q35_launch_l2norm(float *d_x, int rows, int n, float eps, void *stream) {
    return q35_launch_l2norm_strided(d_x, 0, rows, n, eps, 1, rows * n, stream);
}
// q rows: l2norm then *= qscale (two roundings, as l2norm + scaleVec); k rows: l2norm
int q35_launch_l2norm_qk_scale(float *d_x, int nk, int kd, int k_offset, float eps, float qscale, void *stream) {
    if (nk <= 0 || kd <= 0) return 0;
    if (k_offset < nk * kd) return (int)cudaErrorInvalidValue;
    if (kd > 8192) return (int)cudaErrorInvalidValue;
    k_l2norm<128><<<nk, 128, (size_t)kd * 4, S(stream)>>>(d_x, 0, nk, kd, eps, nk * kd, qscale, 1);
    k_l2norm<128><<<nk, 128, (size_t)kd * 4, S(stream)>>>(d_x, k_offset, nk, kd, eps, nk * kd, 1.0f, 0);
    return (int)cudaGetLastError();
}

// ---- activations / conv (api.h:185-202) ----
int q35_launch_silu(float *d_x, int n, void *stream) {
    if (n <= 0) return 0;
    k_silu<<<ew_grid(n), 256, 0, S(stream)>>>(d_x, n);
    return (int)cudaGetLastError();
}
int q35_launch_mul_silu(float *d_out, const float *d_gate, int n, void *stream) {
    if (n <= 0) return 0;
    k_mul_silu<<<ew_grid(n), 256, 0, S(stream)>>>(d_out, d_gate, n);
    return (int)cudaGetLastError();
}
int q35_launch_mul_sigmoid(float *d_out, const float *d_gate, int n, void *stream) {
    if (n <= 0) return 0;
    k_mul_sigmoid<<<ew_grid(n), 256, 0, S(stream)>>>(d_out, d_gate, n);
    return (int)cudaGetLastError();
}
int q35_launch_swiglu(float *d_gate, const float *d_up, int n, void *stream) {
    if (n <= 0) return 0;
    k_swiglu<<<ew_grid(n), 256, 0, S(stream)>>>(d_gate, d_up, n);
    return (int)cudaGetLastError();
}
int q35_launch_softmax(float *d_x, int n, void *stream) {
    if (n <= 0) return 0;
    k_softmax<<<1, 1024, 0, S(stream)>>>(d_x, n);
    return (int)cudaGetLastError();
}
int q35_launch_conv_step_rows(float *d_conv, float *d_y, const float *d_wconv, int n, int tokens, int y_stride,
                              void *stream) {
    if (n <= 0 || tokens <= 0) return 0;
    k_conv_rows<<<(n + 127) / 128, 128, 0, S(stream)>>>(d_conv, d_y, d_wconv, n, tokens, y_stride);
    return (int)cudaGetLastError();
}
int q35_launch_conv_step(float *d_conv, float *d_y, const float *d_wconv, int n, void *stream) {
    return q35_launch_conv_step_rows(d_conv, d_y, d_wconv, n, 1, n, stream);
}
int q35_launch_argmax(const float *d_x, int n, int *d_out, void *stream) {
    if (n <= 0) return 0;
    k_argmax<<<1, 1024, 0, S(stream)>>>(d_x, n, n, d_out);
    return (int)cudaGetLastError();
}

// ---- RoPE (api.h:217-239) ----
int q35_launch_rope64(float *d_x, int heads, int hd, int pos, float base, void *stream) {
    if (heads <= 0) return 0;
    if (hd < 64) return (int)cudaErrorInvalidValue;
    k_rope64<<<(heads + 7) / 8, 256, 0, S(stream)>>>(d_x, 1, heads, hd, pos, base, nullptr);
    return (int)cudaGetLastError();
}
int q35_launch_rope64_rows_dpos(float *d_x, int rows, int heads, int hd, const void *d_dyn, void *stream) {
    if (heads <= 0 || rows <= 0) return 0;
    if (hd < 64 || !d_dyn) return (int)cudaErrorInvalidValue;
    k_rope64<<<(rows * heads + 7) / 8, 256, 0, S(stream)>>>(d_x, rows, heads, hd, 0, 0.0f, (const int *)d_dyn);
    return (int)cudaGetLastError();
}
int q35_launch_rope64_dpos(float *d_x, int heads, int hd, const void *d_dyn, void *stream) {
    return q35_launch_rope64_rows_dpos(d_x, 1, heads, hd, d_dyn, stream);
}
int q35_launch_rope64_rows(float *d_x, int rows, int heads, int hd, int pos0, float base, void *stream) {
    if (heads <= 0 || rows <= 0) return 0;
    if (hd < 64) return (int)cudaErrorInvalidValue;
    k_rope64<<<(rows * heads + 7) / 8, 256, 0, S(stream)>>>(d_x, rows, heads, hd, pos0, base, nullptr);
    return (int)cudaGetLastError();
}
void *q35_func_rope64(void) { return (void *)k_rope64; }
void *q35_func_rope64_dpos(void) { return (void *)k_rope64; }
void *q35_func_rope64_rows_dpos(void) { return (void *)k_rope64; }
int q35_launch_rope64_setenv(int *d_dyn, int pos, float base, void *stream) {
    k_rope_setenv<<<1, 1, 0, S(stream)>>>(d_dyn, pos, base);
    return (int)cudaGetLastError();
}

// ---- gated delta net (api.h:256-335) ----
int q35_launch_gdn_step_rows_chunk(float *d_state, int state_stride, const float *d_k, int k_stride,
                                   const float *d_v, int v_stride, const float *d_q, int q_stride, float *d_km,
                                   int km_stride, float *d_delta, int delta_stride, float *d_out, int out_stride,
                                   const float *d_gamma, int gamma_stride, const float *d_beta, int beta_stride,
                                   int heads, int nk, int kd, int vd, int rows, void *stream) {
    if (heads <= 0 || rows <= 0) return 0;
    if (vd != GDN_KD || kd != GDN_KD || nk <= 0 || nk > heads) return (int)cudaErrorInvalidValue;
    GdnArgs a{};
    a.state = d_state;
    a.state_head = state_stride;
    a.state_slot = 0;
    a.k = d_k; a.k_tok = k_stride; a.k_head = kd;
    a.q = d_q; a.q_tok = q_stride; a.q_head = kd;
    a.v = d_v; a.v_tok = v_stride; a.v_head = vd;
    a.km = d_km; a.km_tok = km_stride; a.km_head = vd;
    a.delta = d_delta; a.delta_tok = delta_stride; a.delta_head = vd;
    a.out = d_out; a.out_tok = out_stride; a.out_head = vd;
    a.gamma = d_gamma; a.g_tok = gamma_stride;
    a.beta = d_beta; a.b_tok = beta_stride;
    a.heads = heads; a.nk = nk; a.rows = rows;
    return gdn_launch(a, 1, S(stream));
}
int q35_launch_gdn_step_wy(float *d_state, int state_stride, const float *d_k, int k_stride, const float *d_v,
                           int v_stride, const float *d_q, int q_stride, float *d_km, int km_stride, float *d_delta,
                           int delta_stride, float *d_out, int out_stride, const float *d_gamma, int gamma_stride,
                           const float *d_beta, int beta_stride, int heads, int nk, int kd, int vd, int rows,
                           void *stream) {
    if (heads <= 0 || rows <= 0) return 0;
    if (vd != GDN_KD || kd != GDN_KD || nk <= 0 || nk > heads) return (int)cudaErrorInvalidValue;
    const int prc = gdn_prepare();
    if (prc) return prc;
    GdnArgs a{};
    a.state = d_state;
    a.state_head = state_stride;
    a.k = d_k; a.k_tok = k_stride; a.k_head = kd;
    a.q = d_q; a.q_tok = q_stride; a.q_head = kd;
    a.v = d_v; a.v_tok = v_stride; a.v_head = vd;
    a.km = d_km; a.km_tok = km_stride; a.km_head = vd;
    a.delta = d_delta; a.delta_tok = delta_stride; a.delta_head = vd;
    a.out = d_out; a.out_tok = out_stride; a.out_head = vd;
    a.gamma = d_gamma; a.g_tok = gamma_stride;
    a.beta = d_beta; a.b_tok = beta_stride;
    a.heads = heads; a.nk = nk; a.rows = rows;
    // the column-split kernel stages q / k rows with 16-byte async copies
    const bool al16 = !(reinterpret_cast<uintptr_t>(d_q) & 15u) && !(reinterpret_cast<uintptr_t>(d_k) & 15u) &&
                      !(q_stride & 3) && !(k_stride & 3);
    if (!al16) return gdn_wy_rows_launch(a, S(stream));
    // the Gram matrices of each 64-token chunk on the tensor cores, then the
    // column-split recurrence; without room for them (inside a capture) the
    // CUDA-core column split
    const int rc = wy_tc_launch(a, S(stream));
    return rc != -1 ? rc : gdn_wy_cols_launch(a, S(stream));
}
int q35_launch_gdn_step_rows(float *d_state, int state_stride, const float *d_k, int k_stride, const float *d_v,
                             int v_stride, const float *d_q, int q_stride, float *d_km, float *d_delta, float *d_out,
                             const float *d_gamma, const float *d_beta, int heads, int nk, int kd, int vd,
                             void *stream) {
    if (heads <= 0) return 0;
    if (vd != GDN_KD || kd != GDN_KD || nk <= 0 || nk > heads) return (int)cudaErrorInvalidValue;
    GdnArgs a{};
    a.state = d_state;
    a.state_head = state_stride;
    a.k = d_k; a.k_head = k_stride;
    a.q = d_q; a.q_head = q_stride;
    a.v = d_v; a.v_head = v_stride;
    a.km = d_km; a.km_head = vd;
    a.delta = d_delta; a.delta_head = vd;
    a.out = d_out; a.out_head = vd;
    a.gamma = d_gamma;
    a.beta = d_beta;
    a.heads = heads; a.nk = nk; a.rows = 1;
    return gdn_launch(a, 1, S(stream));
}
int q35_launch_gdn_step(float *d_state, const float *d_k, const float *d_v, const float *d_q, float *d_km,
                        float *d_delta, float *d_out, float gamma, float beta, int vd, void *stream) {
    if (vd != GDN_KD) return (int)cudaErrorInvalidValue;
    GdnArgs a{};
    a.state = d_state;
    a.k = d_k; a.q = d_q; a.v = d_v;
    a.km = d_km; a.delta = d_delta; a.out = d_out;
    a.gamma_imm = gamma;
    a.beta_imm = beta;
    a.heads = 1; a.nk = 1; a.rows = 1;
    return gdn_launch(a, 1, S(stream));
}
int q35_launch_gdn_gamma_rows(const float *d_a_raw, float *d_b_raw, const float *d_ssm_a, const float *d_dt_bias,
                              float *d_gamma, int nv, int tokens, int a_stride, int b_stride, int gamma_stride,
                              void *stream) {
    if (nv <= 0 || tokens <= 0) return 0;
    k_gdn_gamma<<<ew_grid((long long)nv * tokens, 128), 128, 0, S(stream)>>>(d_a_raw, d_b_raw, d_ssm_a, d_dt_bias,
                                                                            d_gamma, nv, tokens, a_stride, b_stride,
                                                                            gamma_stride);
    return (int)cudaGetLastError();
}
int q35_launch_gdn_gamma(const float *d_a_raw, float *d_b_raw, const float *d_ssm_a, const float *d_dt_bias,
                         float *d_gamma, int nv, void *stream) {
    return q35_launch_gdn_gamma_rows(d_a_raw, d_b_raw, d_ssm_a, d_dt_bias, d_gamma, nv, 1, nv, nv, nv, stream);
}

// ---- attention (api.h:337-415) ----
static int attn_api(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache, float *d_gout,
                    int len, const int *d_last_pos, int heads, int gqa, int hd, int kv_dim, float scale,
                    void *stream) {
    if (heads <= 0) return 0;
    if (hd != ATT_HD || gqa <= 0 || heads % gqa) return (int)cudaErrorInvalidValue;
    AttnArgs a{};
    a.q = d_q;
    a.gate = d_gate;
    a.q_tok = (long long)heads * hd;
    a.kc = d_kcache;
    a.vc = d_vcache;
    a.kv_slot = 0;
    a.kv_dim = kv_dim;
    a.last_pos = d_last_pos;
    a.len_imm = len;
    a.out = d_gout;
    a.out_tok = (long long)heads * hd;
    a.nsplit = 1;
    a.heads = heads;
    a.kv_heads = heads / gqa;
    a.scale = scale;
    return attn_launch(a, 1, d_last_pos ? 1 << 30 : len, S(stream));
}
int q35_launch_attn_decode(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                           float *, float *d_gout, int slot, int heads, int gqa, int hd, int kv_dim, float scale,
                           void *stream) {
    if (slot < 0) return (int)cudaErrorInvalidValue;
    return attn_api(d_q, d_gate, d_kcache, d_vcache, d_gout, slot + 1, nullptr, heads, gqa, hd, kv_dim, scale, stream);
}
int q35_launch_attn_decode_coal(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                                float *d_att, float *d_gout, int slot, int heads, int gqa, int hd, int kv_dim,
                                float scale, void *stream) {
    return q35_launch_attn_decode(d_q, d_gate, d_kcache, d_vcache, d_att, d_gout, slot, heads, gqa, hd, kv_dim, scale,
                                  stream);
}
int q35_launch_attn_decode_split2(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                                  float *d_att, float *d_gout, float *, int slot, int heads, int gqa, int hd,
                                  int kv_dim, float scale, int, void *stream) {
    return q35_launch_attn_decode(d_q, d_gate, d_kcache, d_vcache, d_att, d_gout, slot, heads, gqa, hd, kv_dim, scale,
                                  stream);
}
int q35_launch_attn_decode_dyn(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                               float *, float *d_gout, const int *d_slot, int heads, int gqa, int hd, int kv_dim,
                               float scale, void *stream) {
    if (!d_slot) return (int)cudaErrorInvalidValue;
    return attn_api(d_q, d_gate, d_kcache, d_vcache, d_gout, 0, d_slot, heads, gqa, hd, kv_dim, scale, stream);
}
int q35_launch_attn_decode_split_dyn(const float *d_q, const float *d_gate, const float *d_kcache,
                                     const float *d_vcache, float *d_att, float *d_gout, float *, const int *d_slot,
                                     int heads, int gqa, int hd, int kv_dim, float scale, int, void *stream) {
    return q35_launch_attn_decode_dyn(d_q, d_gate, d_kcache, d_vcache, d_att, d_gout, d_slot, heads, gqa, hd, kv_dim,
                                      scale, stream);
}
// rows r in [0, rows): attends to [0, slot0 + r], i.e. rows independent
// decode steps over a growing prefix (backend_cpu.zig:1059-1073)
__global__ void k_iota_len(int *len, int base, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) len[i] = base + i + 1;
}
int q35_launch_attn_chunk(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                          float *d_gout, int slot0, int rows, int heads, int gqa, int hd, int kv_dim, float scale,
                          void *stream) {
    if (rows <= 0 || heads <= 0) return 0;
    if (hd != ATT_HD || gqa <= 0 || heads % gqa || slot0 < 0) return (int)cudaErrorInvalidValue;
    for (int r = 0; r < rows; r++) {
        const long long off = (long long)r * heads * hd;
        int rc = attn_api(d_q + off, d_gate + off, d_kcache, d_vcache, d_gout + off, slot0 + r + 1, nullptr, heads, gqa,
                          hd, kv_dim, scale, stream);
        if (rc) return rc;
    }
    return 0;
}
int q35_attn_chunk_max_rows(int) { return 1 << 20; }

// Prefill-shaped causal attention over a chunk, in the CPU's operation
// order (the token-tiled kernels of attn.cuh); d_scores: the caller's
// workspace of rows x heads x scores_ld floats, scores_ld >= slot0 + rows
int q35b_attn_prefill(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                      float *d_gout, float *d_scores, long long scores_ld, int slot0, int rows, int heads, int gqa,
                      int hd, int kv_dim, float scale, void *stream) {
    if (rows <= 0 || heads <= 0) return 0;
    if (hd != ATT_HD || gqa <= 0 || heads % gqa || slot0 < 0 || !d_scores || scores_ld < (long long)slot0 + rows ||
        kv_dim < (heads / gqa) * hd || (kv_dim & 3) || (reinterpret_cast<uintptr_t>(d_kcache) & 15u) ||
        (reinterpret_cast<uintptr_t>(d_vcache) & 15u) || (reinterpret_cast<uintptr_t>(d_q) & 15u))
        return (int)cudaErrorInvalidValue;
    AttnXArgs a{};
    a.q = d_q;
    a.gate = d_gate;
    a.q_tok = (long long)heads * hd;
    a.kc = d_kcache;
    a.vc = d_vcache;
    a.kv_slot = 0;
    a.kv_dim = kv_dim;
    a.len_imm = slot0 + 1;
    a.len_step = 1;
    a.scores = d_scores;
    a.max_len = (int)scores_ld;
    a.out = d_gout;
    a.out_tok = (long long)heads * hd;
    a.heads = heads;
    a.kv_heads = heads / gqa;
    a.scale = scale;
    a.fam = 0;
    const int rc = attp_launch(a, rows, slot0 + rows, S(stream));
    return rc == -1 ? (int)cudaErrorInvalidValue : rc;
}
void *q35_func_attn_decode(void) { return (void *)k_attn_split<4>; }
void *q35_func_attn_decode_dyn(void) { return (void *)k_attn_split<4>; }
void *q35_func_attn_decode_coal(void) { return (void *)k_attn_split<4>; }
void *q35_func_attn_score_split(void) { return (void *)k_attn_split<4>; }
void *q35_func_attn_score_split_dyn(void) { return (void *)k_attn_split<4>; }
void *q35_func_attn_pv_split_dyn(void) { return (void *)k_attn_merge; }
void *q35_func_attn_softmax_dyn(void) { return (void *)k_attn_merge; }
void *q35_func_attn_reduce(void) { return (void *)k_attn_merge; }

// ---- device sampler (src/kernels/cuda/sample.cu:559-664; rules of
// src/sampler.zig): temperature, top-k, top-p, one xorshift64* draw ----
int q35_sample_scratch_ints(void) { return 16; }
int q35_sample_ctl_ints(void) { return SC_INTS; }
int q35_launch_sample_init(void **d_ctl, void **d_scratch) {
    if (!d_ctl || !d_scratch) return (int)cudaErrorInvalidValue;
    if (!*d_ctl) {
        if (cudaMalloc(d_ctl, SC_INTS * sizeof(int)) != cudaSuccess) {
            *d_ctl = nullptr;
            return (int)cudaGetLastError();
        }
        cudaMemset(*d_ctl, 0, SC_INTS * sizeof(int));
    }
    if (!*d_scratch) {  // the kernel keeps its working state on chip; the region is the contract's
        if (cudaMalloc(d_scratch, 16 * sizeof(int)) != cudaSuccess) {
            cudaFree(*d_ctl);
            *d_ctl = nullptr;
            return (int)cudaGetLastError();
        }
    }
    return 0;
}
void q35_launch_sample_deinit(void **d_ctl, void **d_scratch) {
    if (d_ctl && *d_ctl) { cudaFree(*d_ctl); *d_ctl = nullptr; }
    if (d_scratch && *d_scratch) { cudaFree(*d_scratch); *d_scratch = nullptr; }
}
int q35_launch_sample(const float *d_logits, int n, int *d_ctl, void *d_scratch, void *stream) {
    if (!d_logits || !d_ctl || !d_scratch || n <= 0) return (int)cudaErrorInvalidValue;
    const SmpArgs a{d_logits, n, n, 1, d_ctl, SC_INTS, nullptr, nullptr, nullptr, 0};
    return sample_launch(a, S(stream));
}
int q35b_sample_rows(const float *d_logits, long long ld, int n, int rows, int *d_ctl, long long ctl_ld, int advance,
                     int *d_tokens, void *stream) {
    if (rows < 0) return (int)cudaErrorInvalidValue;
    const SmpArgs a{d_logits, ld, n, rows, d_ctl, ctl_ld, nullptr, nullptr, d_tokens, advance ? 1 : 0};
    return sample_launch(a, S(stream));
}

// ---- codebooks (api.h:433-442): compiled into the kernels ----
int q35_launch_init_tables(void *) { return 0; }
unsigned long long q35_iq_tables_bytes(void) { return 16; }
int q35_iq_tables_ready(void) { return 1; }
void q35_launch_deinit_tables(void) {}

// ---- geometry (api.h:446-464) ----
int q35_quant_act_block_elems(int ttype) { return geom_of(ttype).family; }
int q35_quant_geom(int ttype, int *block_elems, int *block_bytes) {
    const Geom g = geom_of(ttype);
    if (!g.elems) return 0;
    if (block_elems) *block_elems = g.elems;
    if (block_bytes) *block_bytes = g.bytes;
    return 1;
}
int q35_mmq_dp4a_wants(int) { return 0; }
int q35_mmq_act_block_bytes(void) { return 288; }

// ---- additive API ----
// failure-detection self-test: a wait on an mbarrier nothing ever completes
__global__ void k_wait_probe(unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait(&bar, 0u, 150, limit_ns);  // never completes: gives up, records 150
}

int q35b_selftest_wait(int limit_ms, void *stream) {
    if (limit_ms <= 0 || limit_ms > 2000) return (int)cudaErrorInvalidValue;
    k_wait_probe<<<1, 32, 0, S(stream)>>>((unsigned long long)limit_ms * 1000000ull);
    const int rc = (int)cudaGetLastError();
    if (rc) return rc;
    return (int)cudaStreamSynchronize(S(stream));
}

int q35b_get_error(int *code) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_q35_error, sizeof(int));
    if (e != cudaSuccess) return (int)e;
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_q35_error, &zero, sizeof(int));
    if (code) *code = v;
    return (int)e;
}

int q35b_quantize_weight(int ttype, const float *d_src, void *d_dst, long long nblocks, void *stream) {
    if (!geom_of(ttype).elems) return (int)cudaErrorInvalidValue;
    if (nblocks <= 0) return 0;
    k_quantize_weight<<<(unsigned)((nblocks + 127) / 128), 128, 0, S(stream)>>>(ttype, d_src, (uint8_t *)d_dst,
                                                                                nblocks);
    return (int)cudaGetLastError();
}

int q35b_synth_fill(unsigned long long key, long long n, float k, float *d_dst, void *stream) {
    if (n < 0 || (n > 0 && !d_dst)) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    const long long blocks = std::min<long long>((n + 255) / 256, 148LL * 16);
    k_synth_fill<<<(unsigned)blocks, 256, 0, S(stream)>>>(key, n, k, d_dst);
    return (int)cudaGetLastError();
}

int q35b_mul_mat_vec_multi(int nmat, const void *const *d_w, const int *ttype, const long long *rows,
                           float *const *d_out, const long long *out_ld, const int *mode, const void *d_xq, int cols,
                           int tokens, void *stream) {
    if (nmat < 1 || nmat > GV_MAX_SEG) return (int)cudaErrorInvalidValue;
    GemvSegDesc s[GV_MAX_SEG];
    for (int i = 0; i < nmat; i++) s[i] = GemvSegDesc{d_w[i], d_out[i], rows[i], ttype[i], out_ld[i], mode ? mode[i] : 0};
    return gemv_launch(s, nmat, d_xq, cols, tokens, S(stream));
}

int q35b_mul_mat_vec_multi_ws(int nmat, const void *const *d_w, const int *ttype, const long long *rows,
                              float *const *d_out, const long long *out_ld, const int *mode, const void *d_xq,
                              int cols, int tokens, float *d_work, long long work_bytes, void *stream) {
    if (nmat < 1 || nmat > GV_MAX_SEG || work_bytes < 0 || (work_bytes > 0 && !d_work) ||
        (reinterpret_cast<uintptr_t>(d_work) & 3u))
        return (int)cudaErrorInvalidValue;
    GemvSegDesc s[GV_MAX_SEG];
    for (int i = 0; i < nmat; i++) s[i] = GemvSegDesc{d_w[i], d_out[i], rows[i], ttype[i], out_ld[i], mode ? mode[i] : 0};
    return gemv_launch(s, nmat, d_xq, cols, tokens, S(stream), 0, d_work, (size_t)work_bytes);
}

}  // extern "C"
