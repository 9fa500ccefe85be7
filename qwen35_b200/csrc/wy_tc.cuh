// wy_tc.cuh -- the WY chunked GDN prefill with its state-independent
// products on the tensor cores (sm_100a tcgen05, kind::tf32).
//
// Per 32-token chunk, the WY form needs the Gram matrices G_kk = K K^T and
// G_qk = Q K^T of the chunk's (l2-normalised) k and q rows (the A and M
// matrices before the per-head decays; `wy_chunk` in gdn.cuh).  They depend
// on neither the state nor the value head, so one pass computes them for
// every (chunk, k head) in parallel:
//   k_wy_gram: CTA per (pair of chunks, k head).  A = [K_0; K_1; Q_0; Q_1]
//   (4 x 32 rows x 128) is split into tf32 hi / lo parts (hi = x rounded to
//   tf32, lo = x - hi rounded to tf32) in the canonical K-major layout
//   (8-row x 16-byte core matrices, no swizzle); B = [K_0; K_1] is A's first
//   64 rows (same descriptors, N = 64).  One thread issues 16 K-steps x 3
//   `tcgen05.mma.cta_group::1.kind::tf32` (M = 128, N = 64, K = 8:
//   hi*hi + hi*lo + lo*hi, f32 accumulation in TMEM); each warp reads its
//   32 TMEM lanes x the 32 columns of its chunk back with `tcgen05.ld` and
//   stores one G block.
//   Dropping lo*lo leaves each product within ~2^-21 relative of the f32
//   product.
// The recurrence is the column-split WY kernel of gdn.cuh (k_gdn_wy_cols)
// with A_ts = exp(L_t - L_s) G_kk[t][s] (s < t) and M_ts = exp(L_t - L_s)
// G_qk[t][s] (s <= t) read from the pass's output instead of recomputed by
// each of a head's CTAs.  Both forms re-associate the per-token recurrence's
// sums; each stays within 1e-4 of it (tests).
#pragma once
#include "gdn.cuh"
#include "mmq.cuh"

namespace q35 {

constexpr int WYT_C = 2 * WY_C;                        // tokens per tensor-core tile (two chunks)
constexpr int WYT_SLICE_A = 128 * 32;                  // bytes of one K-slice of A (128 rows x 8 tf32)
constexpr int WYT_A = 16 * WYT_SLICE_A;                // 64 KB per part (hi or lo)
constexpr size_t WYT_GRAM_SMEM = (size_t)2 * WYT_A + 128;  // + barrier, TMEM slot
constexpr int WYT_G = 2 * WY_C * WY_C;                 // floats of G per (chunk, k head): G_kk then G_qk

// instruction descriptor: tf32 x tf32 -> f32, K-major A and B, M = 128, N = 64
__host__ __device__ constexpr uint32_t wyt_idesc() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

Q35_DEV void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

Q35_DEV uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

// byte offset of element e (0..127 along K) of row r in a canonical K-major
// operand stored as 16 K-slices of `rows` rows x 32 bytes
Q35_DEV int wyt_off(int r, int e, int slice_bytes) {
    return (e >> 3) * slice_bytes + (r >> 3) * 256 + ((e >> 2) & 1) * 128 + (r & 7) * 16 + (e & 3) * 4;
}

struct WyGramArgs {
    const float *q, *k;
    long long q_tok, k_tok;  // floats between tokens
    long long q_head, k_head;  // floats between k heads within a token
    int rows, nk;
    float *g;                // [chunk][k head][2][WY_C][WY_C]
};

__global__ void __launch_bounds__(128) k_wy_gram(const __grid_constant__ WyGramArgs a) {
    extern __shared__ __align__(128) uint8_t smg[];
    uint8_t *Ahi = smg, *Alo = Ahi + WYT_A;
    uint64_t *bar = reinterpret_cast<uint64_t *>(Alo + WYT_A);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 1);
    __shared__ int s_ok;
    const int p = blockIdx.x, kh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5;
    const int T0 = p * WYT_C;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(64)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // operands: thread = row of A; warps 0 / 1 hold the K rows of chunk 0 / 1
    // of the pair (also B's rows), warps 2 / 3 their Q rows; tokens past the
    // end are zero; eight 16-byte loads in flight per thread
    {
        const int r = tid, half = warp & 1, isq = warp >> 1, t = half * WY_C + (tid & 31);
        const bool live = T0 + t < a.rows;
        const float *src = isq ? a.q + (long long)(T0 + t) * a.q_tok + (long long)kh * a.q_head
                               : a.k + (long long)(T0 + t) * a.k_tok + (long long)kh * a.k_head;
#pragma unroll 1
        for (int e0 = 0; e0 < GDN_KD / 4; e0 += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++)
                v[u] = live ? reinterpret_cast<const float4 *>(src)[e0 + u] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float x[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    hi[w] = to_tf32(x[w]);
                    lo[w] = to_tf32(__fsub_rn(x[w], __uint_as_float(hi[w])));
                }
                // four consecutive K elements of one row are 16 contiguous bytes
                const int oa = wyt_off(r, 4 * (e0 + u), WYT_SLICE_A);
                *reinterpret_cast<uint4 *>(Ahi + oa) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4 *>(Alo + oa) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
    }
    fence_proxy_async();  // generic-proxy writes -> visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tid == 0) {
        const uint32_t idesc = wyt_idesc();
        for (int s = 0; s < 16; s++) {
            const uint64_t ah = umma_desc(Ahi + s * WYT_SLICE_A, 128, 256), al = umma_desc(Alo + s * WYT_SLICE_A, 128, 256);
            const uint64_t bh = ah, bl = al;  // B: the slice's first 64 rows
            umma_tf32(tmem, ah, bh, idesc, s > 0 ? 1u : 0u);
            umma_tf32(tmem, ah, bl, idesc, 1u);
            umma_tf32(tmem, al, bh, idesc, 1u);
        }
        umma_commit(bar);
    }
    if (tid == 0) s_ok = mbar_wait(bar, 0u, 170) ? 1 : 0;
    __syncthreads();
    const int half = warp & 1, chunk = 2 * p + half;
    if (s_ok && chunk * WY_C < a.rows) {
        tc_fence_after();
        // lanes 32w.. = this warp's rows; columns of its own chunk
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(half * WY_C), v);
        tmem_ld_wait();
        float *dst = a.g + ((long long)chunk * a.nk + kh) * WYT_G + (warp >> 1) * WY_C * WY_C + (tid & 31) * WY_C;
#pragma unroll
        for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4 *>(dst + i) = make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                                               __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(64) : "memory");
    }
}

// The Gram matrices live in a per-device buffer kept between calls, grown
// only outside stream capture (cudaMalloc would break a capture); -1 when it
// is too small during a capture (the caller then runs the CUDA-core form).
// Calls on one device share the buffer: order them (one stream, or events).
struct WyGramBuf {
    void *p = nullptr;
    size_t bytes = 0;
};
inline WyGramBuf &wy_gram_buf(int dev) {
    static WyGramBuf bufs[64];
    return bufs[dev & 63];
}

// bytes of Gram blocks a run of `rows` tokens needs
inline size_t wy_gram_bytes(int rows, int nk) {
    return (size_t)2 * ((rows + WYT_C - 1) / WYT_C) * nk * WYT_G * sizeof(float);
}

// gbuf / gbytes: the caller's Gram scratch (the engine's own), or null for a
// per-device buffer grown outside stream capture
inline int wy_tc_launch(const GdnArgs &a, cudaStream_t st, float *gbuf = nullptr, size_t gbytes = 0) {
    if (a.heads <= 0 || a.rows <= 0) return 0;
    if (a.nk <= 0 || a.q_head != GDN_KD || a.k_head != GDN_KD) return -1;
    static int ready = 0;
    if (!ready) {
        cudaError_t e = cudaFuncSetAttribute(k_wy_gram, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WYT_GRAM_SMEM);
        if (e != cudaSuccess) return (int)e;
        ready = 1;
    }
    const int npair = (a.rows + WYT_C - 1) / WYT_C;
    const size_t need = wy_gram_bytes(a.rows, a.nk);
    if (gbuf) {
        if (gbytes < need) return (int)cudaErrorInvalidValue;
        WyGramArgs g{a.q, a.k, a.q_tok, a.k_tok, a.q_head, a.k_head, a.rows, a.nk, gbuf};
        k_wy_gram<<<dim3((unsigned)npair, (unsigned)a.nk), 128, WYT_GRAM_SMEM, st>>>(g);
        const int rc = (int)cudaGetLastError();
        if (rc) return rc;
        return gdn_wy_cols_launch(a, st, gbuf);
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    WyGramBuf &b = wy_gram_buf(dev);
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
    WyGramArgs g{a.q, a.k, a.q_tok, a.k_tok, a.q_head, a.k_head, a.rows, a.nk, static_cast<float *>(b.p)};
    k_wy_gram<<<dim3((unsigned)npair, (unsigned)a.nk), 128, WYT_GRAM_SMEM, st>>>(g);
    const int rc = (int)cudaGetLastError();
    if (rc) return rc;
    return gdn_wy_cols_launch(a, st, static_cast<const float *>(b.p));
}

}  // namespace q35
