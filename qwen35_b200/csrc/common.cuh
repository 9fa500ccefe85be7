// common.cuh -- device helpers shared by every kernel of libq35b (sm_100a).
//
// Numerics contract: the library is built with -fmad=false, so no multiply
// and add are ever fused behind the source's back.  Where an operation order
// matters (block folds, norms, the GDN recurrence) the kernels spell it with
// __fmul_rn / __fadd_rn so the rounding sequence is visible in the source.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <utility>

#define Q35_DEV __device__ __forceinline__

namespace q35 {

// GGUF TensorType ids (the values of api.h / src/gguf.zig:87-122).
enum : int {
    TT_F32 = 0, TT_F16 = 1, TT_Q4_0 = 2, TT_Q4_1 = 3, TT_Q5_0 = 6, TT_Q5_1 = 7, TT_Q8_0 = 8, TT_Q4_K = 12, TT_Q5_K = 13,
    TT_Q6_K = 14, TT_Q8_K = 15, TT_IQ4_NL = 20, TT_IQ4_XS = 23, TT_BF16 = 30,
    // engine-internal: Q6_K blocks padded from 210 to 224 bytes (same field
    // offsets, 14 zero bytes after d), so that rows are 16-byte multiples for
    // TMA; not a GGUF type id
    TT_Q6_K_P = 0x1000 + 14,
};

// Q4_0 / Q4_1 / Q5_0 / Q5_1 (32-element blocks, Q8_0 activation): offsets of
// the fields in a block, GGUF layout (qs: element j < 16 in the low nibble of
// byte j, element j + 16 in the high nibble; qh: bit 4 of element j in bit j)
__host__ __device__ constexpr bool legacy_type(int tt) {
    return tt == TT_Q4_0 || tt == TT_Q4_1 || tt == TT_Q5_0 || tt == TT_Q5_1;
}
__host__ __device__ constexpr bool legacy_affine(int tt) { return tt == TT_Q4_1 || tt == TT_Q5_1; }  // d and min
__host__ __device__ constexpr bool legacy_five(int tt) { return tt == TT_Q5_0 || tt == TT_Q5_1; }    // qh plane
__host__ __device__ constexpr int legacy_qh_off(int tt) { return legacy_affine(tt) ? 4 : 2; }
__host__ __device__ constexpr int legacy_qs_off(int tt) {
    return (legacy_affine(tt) ? 4 : 2) + (legacy_five(tt) ? 4 : 0);
}

// Native block geometry of the weight types this library serves.
struct Geom { int elems, bytes, family; };  // family: 32 = Q8_0 act, 256 = Q8_K act
__host__ __device__ inline Geom geom_of(int tt) {
    switch (tt) {
    case TT_Q8_0: return {32, 34, 32};
    case TT_IQ4_NL: return {32, 18, 32};
    case TT_Q4_0: return {32, 18, 32};
    case TT_Q4_1: return {32, 20, 32};
    case TT_Q5_0: return {32, 22, 32};
    case TT_Q5_1: return {32, 24, 32};
    case TT_Q4_K: return {256, 144, 256};
    case TT_Q5_K: return {256, 176, 256};
    case TT_Q6_K: return {256, 210, 256};
    case TT_Q6_K_P: return {256, 224, 256};
    case TT_IQ4_XS: return {256, 136, 256};
    default: return {0, 0, 0};
    }
}

// Elements per f32 term of the ordered fold: one term per native block,
// except IQ4_XS, whose 256-element block contributes one term per 32-element
// sub-block (iq_kernels.c:967-1000: sumf += d1 * (sumi1 + sumi2) per sub-block)
__host__ __device__ inline int term_elems(int tt) { return tt == TT_IQ4_XS ? 32 : geom_of(tt).elems; }

// IQ4_XS block (256 elements, 136 bytes): d (f16) @0, scales_h (u16) @2,
// scales_l[4] @4, qs[128] @8; sub-block ib (32 elements) takes qs[16 ib ..
// 16 ib + 15] (element j in the low nibble, j + 16 in the high nibble, as
// IQ4_NL) and the 6-bit scale below, applied as ls - 32
// (iq_kernels.c:96-103, 978-979)
__host__ __device__ inline int iq4xs_ls(int scales_l_byte, int scales_h, int ib) {
    return ((scales_l_byte >> (4 * (ib & 1))) & 0xF) | (((scales_h >> (2 * ib)) & 3) << 4);
}

// ---------------------------------------------------------------------------
// error word: kernels that give up on a bounded wait record a site code here
// ---------------------------------------------------------------------------
// defined once: the library is a single translation unit (q35b.cu)
__device__ int g_q35_error;

Q35_DEV void set_error(int code) { atomicCAS(&g_q35_error, 0, code); }

Q35_DEV uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// f16 <-> f32
// ---------------------------------------------------------------------------
Q35_DEV float f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Round-to-nearest-even with inf/nan -> inf.  `sub_carry` is written when a
// subnormal rounds up into the smallest normal: 0x0400 is IEEE; the reference
// activation quantizer writes 0x0380 there (src/kernels/x86/kernels32.c:95)
// and the activation path keeps that value so its bytes match exactly.
__host__ __device__ inline uint16_t f32_to_f16_bits(float x, uint16_t sub_carry) {
#ifdef __CUDA_ARCH__
    const uint32_t u = __float_as_uint(x);
#else
    uint32_t u;
    memcpy(&u, &x, 4);
#endif
    const uint32_t sign = (u & 0x80000000u) >> 16;
    const uint32_t e = (u >> 23) & 0xFFu;
    const uint32_t m = u & 0x7FFFFFu;
    if (e >= 143u) return (uint16_t)(0x7C00u | sign);
    if (e >= 113u) {
        uint32_t keep = m >> 13;
        const uint32_t drop = m & 0x1FFFu;
        keep += (drop > 0x1000u) || (drop == 0x1000u && (keep & 1u));
        uint32_t e16 = e - 112u;
        if (keep >= 0x400u) { keep = 0; e16 += 1; }
        if (e16 > 30u) return (uint16_t)(0x7C00u | sign);
        return (uint16_t)(sign | (e16 << 10) | keep);
    }
    const uint32_t t = m | 0x800000u;
    const int s = (int)(126u - e);
    if (s >= 25) return (uint16_t)sign;
    uint32_t keep = t >> s;
    const uint32_t drop = t & ((1u << s) - 1u);
    const uint32_t mid = 1u << (s - 1);
    keep += (drop > mid) || (drop == mid && (keep & 1u));
    if (keep >= 0x400u) return (uint16_t)(sub_carry | sign);
    return (uint16_t)(sign | keep);
}

// ---------------------------------------------------------------------------
// loads of 2-byte aligned data (GGUF blocks are only 2-byte aligned)
// ---------------------------------------------------------------------------
Q35_DEV uint16_t ld_u16(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }

// N little-endian words starting at a 2-aligned SHARED address.  Reads one
// word past the end when p is 4-aligned, so staging buffers carry 16 bytes
// of padding.
template <int N>
Q35_DEV void lds_words_a2(const uint8_t *p, uint32_t (&w)[N]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *b = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 2u) * 8u;
    uint32_t r[N + 1];
#pragma unroll
    for (int i = 0; i <= N; i++) r[i] = b[i];
#pragma unroll
    for (int i = 0; i < N; i++) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}

// ---------------------------------------------------------------------------
// IQ4_NL codebook (src/iq_tables.zig:429-432) as four packed words, and a
// 16-entry byte lookup for four nibbles at once via two byte permutes.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) |
           ((uint32_t)(d & 0xFF) << 24);
}
constexpr uint32_t kIq4T0 = pack4(-127, -104, -83, -65);
constexpr uint32_t kIq4T1 = pack4(-49, -35, -22, -10);
constexpr uint32_t kIq4T2 = pack4(1, 13, 25, 38);
constexpr uint32_t kIq4T3 = pack4(53, 69, 89, 113);

// idx holds four 4-bit indices in the low nibble of each byte (0..15).
Q35_DEV uint32_t iq4_lookup4(uint32_t idx) {
    // selector nibbles: bit 0-2 of each index select one of 8 bytes of a table
    // half; gather the 4 indices' low 3 bits into the byte_perm selector
    const uint32_t s = (idx & 0x7u) | ((idx >> 4) & 0x70u) | ((idx >> 8) & 0x700u) | ((idx >> 12) & 0x7000u);
    const uint32_t lo = __byte_perm(kIq4T0, kIq4T1, s);
    const uint32_t hi = __byte_perm(kIq4T2, kIq4T3, s);
    // bit 3 of each index picks hi: selector byte k = k + 4*bit3
    const uint32_t b3 = (idx >> 3) & 0x01010101u;
    const uint32_t sel = 0x3210u | ((b3 & 1u) << 2) | (((b3 >> 8) & 1u) << 6) |
                         (((b3 >> 16) & 1u) << 10) | (((b3 >> 24) & 1u) << 14);
    return __byte_perm(lo, hi, sel);
}

// ---------------------------------------------------------------------------
// mbarrier / bulk-copy PTX (shared::cta addresses)
// ---------------------------------------------------------------------------
Q35_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

Q35_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
Q35_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
Q35_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

Q35_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
Q35_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t tx) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(tx)
                 : "memory");
}
Q35_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after ~2 s of wall time, records `site` in the error
// word and returns false.  Nothing in this library waits without a bound.
Q35_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, int site, uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u && globaltimer() - t0 > limit_ns) {
            set_error(site);
            return false;
        }
    }
}

// global -> shared bulk copy completing on `bar` (16-byte aligned, size % 16 == 0)
Q35_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// shared -> global bulk copy (16-byte aligned, size % 16 == 0) in a bulk
// group; bulk_s2g_wait_read() returns once the source shared memory has been
// read (the global writes complete on their own before the grid does)
Q35_DEV void bulk_s2g(void *dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
                 "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
Q35_DEV void bulk_s2g_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

Q35_DEV void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// programmatic dependent launch.  A kernel of the decode step calls
// pdl_trigger() first (its successor may then be scheduled while it runs) and
// pdl_wait() before its first access to memory an earlier kernel writes or
// reads; both are no-ops when the launch did not opt in.
// ---------------------------------------------------------------------------
Q35_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
Q35_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launches issued while this is set (the engine's step body) opt in to
// programmatic stream serialization; other launches are plain.
inline bool &pdl_enabled() {
    static thread_local bool on = false;
    return on;
}

// kernels launched through launch_k by this host thread (the engine reports
// the count of one step body)
inline long long &launch_count() {
    static thread_local long long n = 0;
    return n;
}

template <typename... KArgs, typename... Args>
inline int launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
    launch_count()++;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// block-wide sum (order is fixed for a given blockDim, not the CPU's serial
// order; used only where the reference's own device path also reduces)
// ---------------------------------------------------------------------------
Q35_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
Q35_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int NWARPS>
Q35_DEV float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.0f;
    if (NWARPS == 1) return red[0];
#pragma unroll
    for (int i = 0; i < NWARPS; i++) s = __fadd_rn(s, red[i]);
    return s;
}

// Sum of squares in the CPU's serial order: ((x0*x0 + x1*x1) + x2*x2) + ...
// (src/elementwise.zig:45-46).  One thread, one dependent add per element;
// `x` should be in shared memory (4-float reads keep the chain fed).
// The chain step for NC chains at once: add the 16 products p[] to every
// chain c[0..NC) in order, while forming the 16 products of b[] into q[]
#define Q35_SUMSQ_STEP(p, b, q)                                         \
    _Pragma("unroll") for (int k = 0; k < 4; k++) {                     \
        _Pragma("unroll") for (int h = 0; h < NC; h++) c[h] = __fadd_rn(c[h], p[4 * k]);     \
        q[4 * k] = __fmul_rn(b[k].x, b[k].x);                           \
        _Pragma("unroll") for (int h = 0; h < NC; h++) c[h] = __fadd_rn(c[h], p[4 * k + 1]); \
        q[4 * k + 1] = __fmul_rn(b[k].y, b[k].y);                       \
        _Pragma("unroll") for (int h = 0; h < NC; h++) c[h] = __fadd_rn(c[h], p[4 * k + 2]); \
        q[4 * k + 2] = __fmul_rn(b[k].z, b[k].z);                       \
        _Pragma("unroll") for (int h = 0; h < NC; h++) c[h] = __fadd_rn(c[h], p[4 * k + 3]); \
        q[4 * k + 3] = __fmul_rn(b[k].w, b[k].w);                       \
    }

// NC serial chains c[h] <- ((c[h] + x0*x0) + x1*x1) + ... over x[0..n)
// (the CPU's order, src/elementwise.zig:45-46), x in shared memory.  With
// x 16-byte aligned the first multiple of 32 elements runs software-
// pipelined in 16-element chunks, two per iteration (registers alternate,
// nothing is copied): while the adds of chunk c run, the products of chunk
// c+1 are formed and chunk c+2 is loaded, so the dependent adds are the
// critical path (one add latency per element).  Same operations, same order.
template <int NC>
Q35_DEV void sumsq_chains(float (&c)[NC], const float *x, int n) {
    int i = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && n >= 32) {
        const float4 *v = reinterpret_cast<const float4 *>(x);
        const int nc = (n / 32) * 2;  // even number of 16-element chunks
        float p[16], q[16];
        float4 b[4], cc[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float4 a = v[k];
            p[4 * k] = __fmul_rn(a.x, a.x);
            p[4 * k + 1] = __fmul_rn(a.y, a.y);
            p[4 * k + 2] = __fmul_rn(a.z, a.z);
            p[4 * k + 3] = __fmul_rn(a.w, a.w);
        }
#pragma unroll
        for (int k = 0; k < 4; k++) b[k] = v[4 + k];
        for (int ci = 0; ci < nc; ci += 2) {
            // p = products of chunk ci, b = values of chunk ci+1
            const int n2 = ci + 2 < nc ? ci + 2 : 0;  // past the end: re-read chunk 0, unused
#pragma unroll
            for (int k = 0; k < 4; k++) cc[k] = v[4 * n2 + k];
            Q35_SUMSQ_STEP(p, b, q)
            const int n3 = ci + 3 < nc ? ci + 3 : 0;
#pragma unroll
            for (int k = 0; k < 4; k++) b[k] = v[4 * n3 + k];
            Q35_SUMSQ_STEP(q, cc, p)
        }
        i = nc * 16;
    }
    for (; i < n; i++) {
        const float sq = __fmul_rn(x[i], x[i]);
#pragma unroll
        for (int h = 0; h < NC; h++) c[h] = __fadd_rn(c[h], sq);
    }
}
#undef Q35_SUMSQ_STEP

// Sum of squares in the CPU's serial order, one thread
Q35_DEV float serial_sumsq(const float *x, int n) {
    float c[1] = {0.0f};
    sumsq_chains<1>(c, x, n);
    return c[0];
}

// The serial sum continued from `s` over x[0..n) (one thread)
Q35_DEV float serial_sumsq_from(float s, const float *x, int n) {
    float c[1] = {s};
    sumsq_chains<1>(c, x, n);
    return c[0];
}

// ---------------------------------------------------------------------------
// The serial sum of squares by a whole CTA, bit-identical to serial_sumsq
// but with the latency of n / nwarps dependent adds instead of n.
//
// The f32 chain s_{i+1} = fl(s_i + fl(x_i * x_i)) stays within a few ulps of
// the exact prefix sum (all terms are >= 0; each add rounds by at most half
// an ulp of the running value).  So the row is cut into one segment per
// warp; a double-precision sum of the products (any order: it is only an
// estimate) gives the prefix at each segment's start, and warp w runs the
// chain over its segment from the 64 f32 values within 32 ulps of that
// estimate at once (32 lanes x 2 independent chains: the same instruction
// stream, so no more latency than one chain).  Then one thread stitches the
// segments in order: the candidate whose start is bit-equal to the true
// value reached so far holds the true value at the segment's end.  If the
// true value lies outside the window (possible for adversarial rows, e.g. a
// huge first element absorbing small ones), that segment is recomputed
// serially.  Either way the result is the serial chain's, bit for bit.
//
// x: n floats in shared memory, 16-byte aligned; called by every thread of
// the CTA (it synchronises); returns the sum in every thread.
// ---------------------------------------------------------------------------
constexpr int SPEC_MAX_WARPS = 8;
constexpr int SPEC_NC = 2;                // chains per lane
constexpr int SPEC_CAND = 32 * SPEC_NC;   // candidates per segment

Q35_DEV float cta_spec_sumsq(const float *x, int n) {
    __shared__ float s_res[SPEC_MAX_WARPS][SPEC_CAND];
    __shared__ double s_dsum[SPEC_MAX_WARPS];
    __shared__ uint32_t s_est[SPEC_MAX_WARPS];
    __shared__ float s_tot;
    const int nw = min((int)(blockDim.x >> 5), SPEC_MAX_WARPS);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int L = ((n + nw - 1) / nw + 31) & ~31;  // segment length, a multiple of 32
    const bool act = warp < nw;
    const int b0 = act ? min(n, warp * L) : n, b1 = act ? min(n, b0 + L) : n;
    // 1. the estimate: double sums of the products per segment
    double d = 0.0;
    for (int i = b0 + lane; i < b1; i += 32) d += (double)__fmul_rn(x[i], x[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (act && lane == 0) s_dsum[warp] = d;
    __syncthreads();
    if (act) {
        double pre = 0.0;
        for (int w = 0; w < warp; w++) pre += s_dsum[w];
        const uint32_t eb = __float_as_uint((float)pre);  // >= +0
        // 2. candidate chains: candidate j = lane + 32 h starts eb + j - 32
        //    ulps (clamped at +0); warp 0 starts at exactly 0 (eb = 0, j = 32)
        float c[SPEC_NC];
#pragma unroll
        for (int h = 0; h < SPEC_NC; h++) {
            const int bb = (int)eb + lane + 32 * h - SPEC_CAND / 2;
            c[h] = __uint_as_float(bb < 0 ? 0u : (uint32_t)bb);
        }
        sumsq_chains<SPEC_NC>(c, x + b0, b1 - b0);
#pragma unroll
        for (int h = 0; h < SPEC_NC; h++) s_res[warp][lane + 32 * h] = c[h];
        if (lane == 0) s_est[warp] = eb;
    }
    __syncthreads();
    // 3. stitch the segments in order
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int w = 0; w < nw; w++) {
            const int w0 = min(n, w * L), w1 = min(n, w0 + L);
            if (w0 >= w1) break;
            const int sb = (int)__float_as_uint(s);
            const int j = sb - (int)s_est[w] + SPEC_CAND / 2;
            if (j >= 0 && j < SPEC_CAND)
                s = s_res[w][j];  // that candidate started at exactly s (sb >= 0, so no clamping)
            else
                s = serial_sumsq_from(s, x + w0, w1 - w0);
        }
        s_tot = s;
    }
    __syncthreads();
    return s_tot;
}

// The same serial sum for a row in global memory, by a whole CTA: the row is
// copied into shared memory (`sm`, n floats, 16-byte aligned) in parallel,
// then thread 0 runs the chain.  Every thread returns the sum.
Q35_DEV float cta_serial_sumsq(const float *xg, int n, float *sm) {
    __shared__ float res;
    for (int i = threadIdx.x; i < n; i += blockDim.x) sm[i] = xg[i];
    __syncthreads();
    if (threadIdx.x == 0) res = serial_sumsq(sm, n);
    __syncthreads();
    return res;
}

// exp / log1p evaluated in double and rounded once to f32: within an ulp of
// the C library's correctly-rounded-in-practice expf/log1pf on the host.
Q35_DEV float exp_f(float x) { return (float)exp((double)x); }
Q35_DEV float log1p_f(float x) { return (float)log1p((double)x); }
Q35_DEV float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, exp_f(-x))); }
Q35_DEV float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f(-x))); }
Q35_DEV float softplus_f(float x) { return x > 20.0f ? x : log1p_f(exp_f(x)); }

}  // namespace q35

#define Q35_CHECK_LAUNCH() ((int)cudaGetLastError())
