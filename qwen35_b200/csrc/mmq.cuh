// mmq.cuh -- quantized matrix x many-token product on the 5th-generation
// tensor cores (tcgen05, sm_100a): batched decode and prefill.
//
//   y[t][r] = sum over blocks b, in block order, of  (dw[r][b] * dx[t][b]) * isum[r][t][b]
//
// isum is the exact int32 dot of the 32 int8 weights and activations of
// block b: one `tcgen05.mma.kind::i8` (M = 128 rows, N = TN tokens, K = 32)
// per block computes it for a 128 x TN tile, each block into its own TMEM
// accumulator region.  The f32 fold then runs on the CUDA cores in the
// reference scalar tier's order (kernels32.c:462), so the result is bit-exact
// with the CPU and with the decode GEMV -- the tensor core does the integer
// part only, where reordering is exact.  The fold is the arithmetic bound of
// this kernel (three rounded f32 operations per weight block and token), so
// it runs on packed f32x2 instructions and overlaps conversion, TMA and MMA
// (see k_mmq below).
#pragma once
#include "gemv_lpr.cuh"

namespace q35 {

constexpr int MMQ_M = 128;          // weight rows per tile (TMEM lanes)
// below this the decode GEMV is used; from 8 tokens a 16-token tile (rows
// past the tokens zero-filled by TMA, never stored) already beats the
// lane-per-row GEMV's 8-token passes (lm_head 1024 x 248320 Q8_0: 75 vs 131 us)
constexpr int MMQ_MIN_TOK = 8;
constexpr int MMQ_KB = 8;           // 32-element blocks per chunk (256 columns)
constexpr int MMQ_NS = 2;           // raw-chunk ring stages

struct MmqSeg {
    float *out;
    long long rows, out_ld;
    long long tile_begin;   // first row tile of this matrix
    int ttype, row_bytes, chunk_bytes, mode;
};

struct MmqArgs {
    CUtensorMap wmap[GV_MAX_SEG];   // weights: [rows][row_bytes/8] u64, box 128 rows x one chunk
    CUtensorMap xmap;               // activations: [ntok][act_row_bytes/8] u64, box 64 rows x 272 B
    MmqSeg seg[GV_MAX_SEG];
    int nseg;
    long long total_tiles;          // row tiles over all matrices
    int ntok, nchunk;
    int ntt;                        // token tiles (k_mmq walks row tiles x token tiles)
};

// ---- tcgen05 / descriptor helpers -----------------------------------------
// shared-memory matrix descriptor, K-major, no swizzle (version 1 = sm_100)
Q35_DEV uint64_t umma_desc(const void *smem_ptr, uint32_t lbo, uint32_t sbo) {
    const uint32_t a = smem_u32(smem_ptr);
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// instruction descriptor: s8 x s8 -> s32, K-major A and B, M = 128, N = TN
template <int TN>
__host__ __device__ constexpr uint32_t mmq_idesc() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(MMQ_M >> 4) << 24);
}

Q35_DEV void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
Q35_DEV void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
Q35_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
Q35_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 consecutive columns of 32-bit TMEM: register i = column c0 + i
Q35_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 16 / 8 consecutive columns
Q35_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
Q35_DEV void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
template <int N>
Q35_DEV void tmem_ldn(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 32) tmem_ld32(taddr, r);
    else if constexpr (N == 16) tmem_ld16(taddr, r);
    else tmem_ld8(taddr, r);
}
Q35_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// (float)d for |d| < 2^22, exactly: the integer placed in the mantissa of
// 1.5 * 2^23, which is then subtracted (both steps exact)
Q35_DEV float exact_i2f(int d) { return __fsub_rn(__int_as_float(0x4B400000 + d), 12582912.0f); }

// canonical K-major no-swizzle offset of row m, 16-byte half h of a 32-byte K slice
Q35_DEV int umma_off(int m, int h) { return (m >> 3) * 256 + h * 128 + (m & 7) * 16; }

// raw Q8_0 chunk row (8 blocks, 272 B at a 16-byte-aligned address) ->
// 8 operand rows + scales; `put(b, d, q)` receives block b's f16 scale and
// its 8 packed int8 words
template <class Put>
Q35_DEV void unpack_q8_0_chunk(const uint8_t *rp, Put put) {
    uint32_t W[68];
    const uint4 *s = reinterpret_cast<const uint4 *>(rp);
#pragma unroll
    for (int i = 0; i < 17; i++) {
        const uint4 v = s[i];
        W[4 * i] = v.x;
        W[4 * i + 1] = v.y;
        W[4 * i + 2] = v.z;
        W[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int o = 34 * k, w0 = o >> 2;
        uint32_t q[8];
        uint16_t d;
        if ((o & 3) == 0) {
            d = (uint16_t)(W[w0] & 0xFFFFu);
#pragma unroll
            for (int i = 0; i < 8; i++) q[i] = __funnelshift_r(W[w0 + i], W[w0 + i + 1], 16);
        } else {
            d = (uint16_t)(W[w0] >> 16);
#pragma unroll
            for (int i = 0; i < 8; i++) q[i] = W[w0 + 1 + i];
        }
        put(k, d, q);
    }
}

// raw IQ4_NL chunk row (8 blocks, 144 B) -> int8 codebook values: low
// nibbles are elements 0..15 of a block, high nibbles 16..31
template <class Put>
Q35_DEV void unpack_iq4_nl_chunk(const uint8_t *rp, Put put) {
    uint32_t W[36];
    const uint4 *s = reinterpret_cast<const uint4 *>(rp);
#pragma unroll
    for (int i = 0; i < 9; i++) {
        const uint4 v = s[i];
        W[4 * i] = v.x;
        W[4 * i + 1] = v.y;
        W[4 * i + 2] = v.z;
        W[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int o = 18 * k, w0 = o >> 2;
        uint32_t qs[4];
        uint16_t d;
        if ((o & 3) == 0) {
            d = (uint16_t)(W[w0] & 0xFFFFu);
#pragma unroll
            for (int i = 0; i < 4; i++) qs[i] = __funnelshift_r(W[w0 + i], W[w0 + i + 1], 16);
        } else {
            d = (uint16_t)(W[w0] >> 16);
#pragma unroll
            for (int i = 0; i < 4; i++) qs[i] = W[w0 + 1 + i];
        }
        uint32_t q[8];
#pragma unroll
        for (int i = 0; i < 4; i++) iq4_word(qs[i], q[i], q[4 + i]);
        put(k, d, q);
    }
}

Q35_DEV int mmq_find_seg(const MmqArgs &a, long long tile) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < GV_MAX_SEG; i++)
        if (i < a.nseg && tile >= a.seg[i].tile_begin) s = i;
    return s;
}

// packed f32 pairs (sub / mul .rn.f32x2, sm_100a): two IEEE
// round-to-nearest operations per instruction, lane for lane the scalar
// result.  A packed multiply whose result feeds a packed add can be
// contracted into a fused multiply-add (one rounding) by the code generator,
// so exact sums of products take their final add in scalar form.
Q35_DEV uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
Q35_DEV void f2_unpack(uint64_t v, float &lo, float &hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
Q35_DEV uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
Q35_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// (float)d0, (float)d1 for |d| < 2^22, exactly (exact_i2f on a pair)
Q35_DEV uint64_t f2_exact_i2f(uint32_t d0, uint32_t d1) {
    const uint64_t m = f2_pack(__int_as_float(0x4B400000 + (int)d0), __int_as_float(0x4B400000 + (int)d1));
    return f2_sub(m, f2_pack(12582912.0f, 12582912.0f));
}

// ---------------------------------------------------------------------------
// k_mmq: warp-specialised pipeline over 128-row x TN-token tiles; one
// persistent CTA per SM walks its tiles (w = blockIdx.x, + gridDim.x, ...)
// with every ring, buffer and TMEM half counting chunks across tiles
//   warp 0      TMA producer: raw weight + activation chunks, 2-stage ring
//   warp 1      TMEM owner; one lane issues the MMAs of a round (RB blocks)
//               into one of two TMEM halves and commits
//   warps 2-5   converters: raw chunk -> K-major operands + scales, into
//               operand buffer c % NB
//   warps 6-13  fold: thread = weight row = TMEM lane (quarter = warp % 4),
//               warps 6-9 the first half of the tokens, 10-13 the second;
//               reads a round's accumulators and folds them in block order
// so conversion of chunk c+1, the MMAs of round g+1 and the fold of round g
// run at once.  Hand-offs are mbarriers with bounded waits:
//   full / empty [stage]    TMA -> converters -> TMA
//   ready [buffer]          converters -> MMA issuer and fold (operands, scales)
//   opfree [buffer]         MMA completion (commit) -> converters (operands read)
//   tfull / tfree [half]    commit -> fold -> MMA issuer (TMEM half)
//   sfree [buffer]          fold -> converters (scales read)
// ---------------------------------------------------------------------------
constexpr int MMQ_THREADS = 448;  // 14 warps
// registers per thread of the MMQ kernels: all that one 448-thread CTA per
// SM can hold (14 warps x 32 x 144 = 64,512 of 65,536).  Left to the
// launch bound alone, ptxas stops at 128 and spills the fold's state at
// 64-token tiles; at 144 the K-quant kernels spill nothing and k_mmq<64>
// 12 bytes.
constexpr int MMQ_MAXNREG = 144;
static_assert(MMQ_THREADS * MMQ_MAXNREG <= 65536, "one CTA's registers");

template <int TN>
struct MmqPlan {
    static constexpr int RB = 256 / TN < MMQ_KB ? 256 / TN : MMQ_KB;  // blocks per round
    static constexpr int ROUNDS = MMQ_KB / RB;
    static constexpr int HALF = RB * TN;                             // TMEM columns per half
    static constexpr int TMEM_COLS = 2 * HALF < 32 ? 32 : 2 * HALF;
    static constexpr int W_STAGE = MMQ_M * 272;
    static constexpr int X_STAGE = TN * 272;
    static constexpr int A_BUF = MMQ_KB * MMQ_M * 32;
    static constexpr int B_BUF = MMQ_KB * TN * 32;
    // operand / scale buffers: chunks in flight between the converters and
    // the fold (3 where shared memory allows, so conversion runs two chunks ahead)
    static constexpr int NB = TN <= 32 ? 3 : 2;
    static constexpr int OFF_A = 0;                                   // [NB] A operands
    static constexpr int OFF_B = OFF_A + NB * A_BUF;                  // [NB] B operands
    static constexpr int OFF_DW = OFF_B + NB * B_BUF;                 // [NB][KB][128] f32
    static constexpr int OFF_DX = OFF_DW + NB * MMQ_KB * MMQ_M * 4;   // [NB][KB][TN] f32
    static constexpr int OFF_RAW = (OFF_DX + NB * MMQ_KB * TN * 4 + 1023) / 1024 * 1024;
    static constexpr int OFF_BAR = OFF_RAW + MMQ_NS * (W_STAGE + X_STAGE);
    static constexpr int SMEM = OFF_BAR + 256 + 1024;  // barriers (2 NS + 3 NB + 4) + TMEM slot, alignment slack
    static_assert(8 * (2 * MMQ_NS + 3 * NB + 4) + 4 <= 256, "barrier area");
    static_assert(SMEM <= 232448, "shared memory per CTA");
};

template <int TN>
__global__ void __maxnreg__(MMQ_MAXNREG) k_mmq(const __grid_constant__ MmqArgs a) {
    using P = MmqPlan<TN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *raw = sm + P::OFF_RAW;
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + P::OFF_BAR);  // [NS]
    uint64_t *empty = full + MMQ_NS;                                 // [NS]
    uint64_t *ready = empty + MMQ_NS;                                // [NB]
    uint64_t *opfree = ready + P::NB;                                // [NB]
    uint64_t *sfree = opfree + P::NB;                                // [NB]
    uint64_t *tfull = sfree + P::NB;                                 // [2]
    uint64_t *tfree = tfull + 2;                                     // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfree + 2);
    __shared__ volatile int s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int issued = 0, ncommit = 0;
    uint64_t *last_commit = nullptr;
    uint32_t last_parity = 0;
    // persistent: this CTA walks work items w = blockIdx.x, + gridDim.x, ...
    // (w = row tile * ntt + token tile); every role counts chunks `it`
    // across its items, so the rings, buffers and TMEM halves run on from
    // one tile into the next
    const long long nwork = a.total_tiles * a.ntt;

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < MMQ_NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 4);
        }
        for (int p = 0; p < P::NB; p++) {
            mbar_init(&ready[p], 4);
            mbar_init(&opfree[p], 1);
            mbar_init(&sfree[p], 8);
        }
        for (int h = 0; h < 2; h++) {
            mbar_init(&tfull[h], 1);
            mbar_init(&tfree[h], 8);
        }
        s_fail = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(P::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the activations (and a residual) belong to the previous kernel
    pdl_wait();

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint32_t xbytes = (uint32_t)(TN * 272);
            int it = 0;
            for (long long w = blockIdx.x; w < nwork && !s_fail; w += gridDim.x) {
                const long long tile = w / a.ntt;
                const int t0 = (int)(w - tile * a.ntt) * TN;
                const int si = mmq_find_seg(a, tile);
                const MmqSeg &sg = a.seg[si];
                const long long r0 = (tile - sg.tile_begin) * MMQ_M;
                const uint32_t wbytes = (uint32_t)(MMQ_M * sg.chunk_bytes);
                for (int c = 0; c < a.nchunk; c++, it++) {
                    const int s = it % MMQ_NS;
                    if (it >= MMQ_NS && (s_fail || !mbar_wait(&empty[s], (uint32_t)(((it / MMQ_NS) - 1) & 1), 121))) {
                        s_fail = 1;
                        break;
                    }
                    uint8_t *wst = raw + s * (P::W_STAGE + P::X_STAGE);
                    mbar_arrive_expect_tx(&full[s], wbytes + xbytes);
                    tma_load_2d(wst, &a.wmap[si], c * (sg.chunk_bytes / 8), (int)r0, &full[s]);
                    tma_load_2d(wst + P::W_STAGE, &a.xmap, c * 34, t0, &full[s]);
                    issued++;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        // lane 0 waits and issues; its verdict is shuffled to the warp so
        // the warp stays converged
        int g = 0, it = 0;
        bool ok = true;
        for (long long w = blockIdx.x; w < nwork && ok; w += gridDim.x) {
            for (int c = 0; c < a.nchunk && ok; c++, it++) {
                const int p = it % P::NB;
                const uint32_t use = (uint32_t)(it / P::NB);  // this buffer's use count
                if (lane == 0) ok = !s_fail && mbar_wait(&ready[p], use & 1u, 126);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                const uint8_t *sA = sm + P::OFF_A + p * P::A_BUF, *sB = sm + P::OFF_B + p * P::B_BUF;
                for (int r = 0; r < P::ROUNDS; r++, g++) {
                    const int h = g & 1;
                    if (lane == 0 && g >= 2) ok = !s_fail && mbar_wait(&tfree[h], (uint32_t)(((g >> 1) - 1) & 1), 127);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    tc_fence_after();
                    if (lane == 0) {
                        for (int kb = 0; kb < P::RB; kb++) {
                            const int b = r * P::RB + kb;
                            const uint64_t ad = umma_desc(sA + b * MMQ_M * 32, 128, 256);
                            const uint64_t bd = umma_desc(sB + b * TN * 32, 128, 256);
                            umma_i8(tmem + (uint32_t)(h * P::HALF + kb * TN), ad, bd, mmq_idesc<TN>(), 0u);
                        }
                        umma_commit(&tfull[h]);
                        last_commit = &tfull[h];
                        last_parity = (uint32_t)((g >> 1) & 1);
                        ncommit++;
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (lane == 0) {
                    umma_commit(&opfree[p]);
                    last_commit = &opfree[p];
                    last_parity = use & 1u;
                    ncommit++;
                }
                __syncwarp();
            }
        }
        if (!ok) s_fail = 1;
        // the last commit covers every MMA issued here: wait for its arrival
        // before the barriers' memory can go away
        if (ok && lane == 0 && ncommit > 0 && !mbar_wait(last_commit, last_parity, 130)) s_fail = 1;
        __syncwarp();
    } else if (warp < 6) {
        // ---------------- converters (thread = weight row; < TN: also a token row) ----------------
        const int ct = threadIdx.x - 64;
        int it = 0;
        bool ok = true;
        for (long long w = blockIdx.x; w < nwork && ok; w += gridDim.x) {
            const MmqSeg &sg = a.seg[mmq_find_seg(a, w / a.ntt)];
            for (int c = 0; c < a.nchunk; c++, it++) {
                const int s = it % MMQ_NS, p = it % P::NB;
                const uint32_t use = (uint32_t)(it / P::NB);
                // every lane waits (acquire); the warp votes so it breaks as one
                ok = !s_fail && mbar_wait(&full[s], (uint32_t)((it / MMQ_NS) & 1), 122);
                if (ok && use > 0)
                    ok = mbar_wait(&opfree[p], (use - 1) & 1u, 128) && mbar_wait(&sfree[p], (use - 1) & 1u, 129);
                if (!__all_sync(0xffffffffu, ok)) {
                    s_fail = 1;
                    ok = false;
                    break;
                }
                const uint8_t *wst = raw + s * (P::W_STAGE + P::X_STAGE);
                uint8_t *sA = sm + P::OFF_A + p * P::A_BUF, *sB = sm + P::OFF_B + p * P::B_BUF;
                float *sDW = reinterpret_cast<float *>(sm + P::OFF_DW) + p * MMQ_KB * MMQ_M;
                float *sDX = reinterpret_cast<float *>(sm + P::OFF_DX) + p * MMQ_KB * TN;
                auto putw = [&](int b, uint16_t d, const uint32_t (&wv)[8]) {
                    uint8_t *dst = sA + b * MMQ_M * 32;
                    *reinterpret_cast<uint4 *>(dst + umma_off(ct, 0)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                    *reinterpret_cast<uint4 *>(dst + umma_off(ct, 1)) = make_uint4(wv[4], wv[5], wv[6], wv[7]);
                    sDW[b * MMQ_M + ct] = f16_to_f32(d);
                };
                if (sg.ttype == TT_Q8_0)
                    unpack_q8_0_chunk(wst + ct * sg.chunk_bytes, putw);
                else
                    unpack_iq4_nl_chunk(wst + ct * sg.chunk_bytes, putw);
                if (ct < TN) {
                    auto putx = [&](int b, uint16_t d, const uint32_t (&wv)[8]) {
                        uint8_t *dst = sB + b * TN * 32;
                        *reinterpret_cast<uint4 *>(dst + umma_off(ct, 0)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                        *reinterpret_cast<uint4 *>(dst + umma_off(ct, 1)) = make_uint4(wv[4], wv[5], wv[6], wv[7]);
                        sDX[b * TN + ct] = f16_to_f32(d);
                    };
                    unpack_q8_0_chunk(wst + P::W_STAGE + ct * 272, putx);
                }
                // operands visible to the tensor core's (async) proxy
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&empty[s]);
                    mbar_arrive(&ready[p]);
                }
            }
        }
    } else {
        // ---------------- fold (thread = row = TMEM lane, half the tokens) ----------------
        constexpr int TH = TN / 2;            // tokens per fold warp
        const int q = warp & 3;               // TMEM lane quarter this warp may access
        const int fh = (warp - 6) >> 2;       // its token half
        const int row = q * 32 + lane;
        const uint64_t magic = f2_pack(12582912.0f, 12582912.0f);
        int g = 0, it = 0;
        for (long long w = blockIdx.x; w < nwork && !s_fail; w += gridDim.x) {
            const long long tile = w / a.ntt;
            const int t0 = (int)(w - tile * a.ntt) * TN;
            const MmqSeg &sg = a.seg[mmq_find_seg(a, tile)];
            const long long r0 = (tile - sg.tile_begin) * MMQ_M;
            uint64_t acc[TH / 2];
#pragma unroll
            for (int t = 0; t < TH / 2; t++) acc[t] = 0ull;
            for (int c = 0; c < a.nchunk; c++, it++) {
                const int p = it % P::NB;
                if (!__all_sync(0xffffffffu, !s_fail && mbar_wait(&ready[p], (uint32_t)(it / P::NB) & 1u, 123))) {
                    s_fail = 1;
                    break;
                }
                const float *sDW = reinterpret_cast<const float *>(sm + P::OFF_DW) + p * MMQ_KB * MMQ_M;
                const float *sDX = reinterpret_cast<const float *>(sm + P::OFF_DX) + p * MMQ_KB * TN + fh * TH;
                for (int r = 0; r < P::ROUNDS; r++, g++) {
                    const int h = g & 1;
                    if (!__all_sync(0xffffffffu, !s_fail && mbar_wait(&tfull[h], (uint32_t)((g >> 1) & 1), 124))) {
                        s_fail = 1;
                        break;
                    }
                    tc_fence_after();
                    // one block's TH columns per load, the next block's load in
                    // flight while the current one is folded
                    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * P::HALF + fh * TH);
                    uint32_t dA[TH], dB[TH];
                    tmem_ldn<TH>(tbase, dA);
                    tmem_ld_wait();
#pragma unroll
                    for (int kb = 0; kb < P::RB; kb++) {
                        uint32_t(&d)[TH] = (kb & 1) ? dB : dA;
                        if (kb + 1 < P::RB) tmem_ldn<TH>(tbase + (uint32_t)((kb + 1) * TN), (kb & 1) ? dA : dB);
                        const int b = r * P::RB + kb;
                        const float dw = sDW[b * MMQ_M + row];
                        const uint64_t dw2 = f2_pack(dw, dw);
                        const uint64_t *dx2 = reinterpret_cast<const uint64_t *>(sDX + b * TN);
#pragma unroll
                        for (int i = 0; i < TH; i += 2) {
                            // sumf += dw * dx * (float)sumi for a pair of tokens: the
                            // products on packed f32x2, the sum in scalar adds (a
                            // packed multiply feeding a packed add may be contracted
                            // into one fused multiply-add, which rounds once)
                            const uint64_t f = f2_sub(f2_pack(__int_as_float(0x4B400000 + (int)d[i]),
                                                              __int_as_float(0x4B400000 + (int)d[i + 1])),
                                                      magic);
                            float a0, a1, p0, p1;
                            f2_unpack(acc[i / 2], a0, a1);
                            f2_unpack(f2_mul(f2_mul(dw2, dx2[i / 2]), f), p0, p1);
                            acc[i / 2] = f2_pack(__fadd_rn(a0, p0), __fadd_rn(a1, p1));
                        }
                        tmem_ld_wait();
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tfree[h]);
                }
                if (__any_sync(0xffffffffu, s_fail != 0)) break;
                if (lane == 0) mbar_arrive(&sfree[p]);
            }
            // outputs: row `row` of this tile, tokens t0 + fh*TH .. + TH - 1
            const long long rr = r0 + row;
            if (!s_fail && rr < sg.rows) {
                const int nt = min(TN, a.ntok - t0) - fh * TH;
#pragma unroll
                for (int i = 0; i < TH; i += 2) {
                    float v0, v1;
                    f2_unpack(acc[i / 2], v0, v1);
                    const long long tk = t0 + fh * TH + i;
                    if (i < nt) {
                        float *o = sg.out + tk * sg.out_ld + rr;
                        *o = sg.mode == GV_ADD ? __fadd_rn(*o, v0) : v0;
                    }
                    if (i + 1 < nt) {
                        float *o = sg.out + (tk + 1) * sg.out_ld + rr;
                        *o = sg.mode == GV_ADD ? __fadd_rn(*o, v1) : v1;
                    }
                }
            }
        }
    }
    __syncthreads();
    if (s_fail) {
        // a wait gave up: let this CTA's own copies and MMAs land (bounded)
        // before its shared memory and TMEM are released
        if (warp == 0 && lane == 0)
            for (int c = issued > MMQ_NS ? issued - MMQ_NS : 0; c < issued; c++)
                if (!mbar_wait(&full[c % MMQ_NS], (uint32_t)((c / MMQ_NS) & 1), 125)) break;
        if (warp == 1 && lane == 0 && ncommit > 0) mbar_wait(last_commit, last_parity, 125);
        if (threadIdx.x == 0) set_error(120);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P::TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// K-quant weights (Q4_K, Q5_K) x Q8_K activations.  A 256-element block has
// 8 sub-blocks with 6-bit scales sc_j and mins m_j (kernels256.c:474-498,
// 605-629):  isum = sum_j sc_j * dot_j,  summs = sum_j m_j * bsum_j,
// sumf += (dy*d)*isum - (dy*dmin)*summs.  One MMA per sub-block (K = 32) into
// its own TN-column TMEM region; the fold forms isum / summs in exact integer
// arithmetic (any order), then the f32 step in the reference's order.
// Chunk = one 256-element block.  Same warp roles and hand-offs as k_mmq;
// the converters also copy the Q8_K activation rows (292 B, 4-byte aligned)
// straight from global memory, their loads issued before the weight wait.
// A round is 4 sub-blocks at TN = 64 (two rounds per block, TMEM halves of
// 256 columns), all 8 otherwise.
//
// Q6_K (224-byte padded blocks, kernels256.c:720-738): 16 groups of 16
// elements with signed 8-bit scales s_g, isum = sum_g s_g * dot16_g, sumf +=
// (d*dy)*isum.  The converters fold the scale into the weight, w = s_g * q
// (q = 6-bit value - 32, so -4064 <= w <= 4096), and split it into two int8
// digits, w = 64*hi + lo with hi = w >> 6 in [-64, 64] and lo = w & 63; the
// MMAs of all sub-blocks of a block accumulate the hi digits into one TMEM
// region H and the lo digits into L, so isum = 64*H + L exactly (|isum| <
// 2^27) and the fold reads two values per block and token.  A chunk is half
// a block (4 sub-blocks x 2 digits = the 8 operand tiles of one buffer); the
// raw stage holds the whole block and is released after its second half.
// ---------------------------------------------------------------------------
struct MmqkArgs {
    CUtensorMap wmap[GV_MAX_SEG];   // weights: [rows][row_bytes/8] u64, box 128 rows x one block
    MmqSeg seg[GV_MAX_SEG];
    int nseg;
    long long total_tiles;
    const uint8_t *xq;              // Q8_K activation rows
    long long xq_ld;
    int ntok, nblk;                 // tokens, 256-element blocks per row
    // split-K (one segment): CTA z takes blocks [nblk*z/Z, nblk*(z+1)/Z) and
    // writes each block's f32 term to terms[(block*ntok + token)*rows + row]
    // for k_mmq_term_sum to add in block order; null: fold and write here
    float *terms;
};

// Q6: raw stages sized for padded Q6_K (224 bytes per row and block); the
// Q4_K / Q5_K instances keep 176-byte stages and the larger L1 that leaves
template <int TN, bool Q6>
struct MmqkPlan {
    static constexpr int RB = TN == 64 ? 4 : 8;     // sub-blocks per round
    static constexpr int ROUNDS = 8 / RB;
    static constexpr int HALF = RB * TN;             // TMEM columns per half
    static constexpr int TMEM_COLS = 2 * HALF;
    static constexpr int NB = TN == 64 ? 2 : 3;      // operand / scale buffers
    static constexpr int NS = 3;                     // raw weight stages
    static constexpr int W_STAGE = MMQ_M * (Q6 ? 224 : 176);  // one block of 128 rows
    static constexpr int A_BUF = 8 * MMQ_M * 32;
    static constexpr int B_BUF = 8 * TN * 32;
    // per buffer: A | B | sc[128][8] u8 | mn[128][8] u8 | d[128] dmin[128] f32 | dy[TN] f32 | bs[TN][8] i32
    static constexpr int OB_A = 0, OB_B = A_BUF, OB_SC = OB_B + B_BUF, OB_MN = OB_SC + MMQ_M * 8;
    static constexpr int OB_D = OB_MN + MMQ_M * 8, OB_DY = OB_D + 2 * MMQ_M * 4, OB_BS = OB_DY + TN * 4;
    static constexpr int BUF = (OB_BS + TN * 32 + 1023) / 1024 * 1024;
    static constexpr int OFF_RAW = NB * BUF;
    static constexpr int OFF_BAR = OFF_RAW + NS * W_STAGE;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;
    static_assert(8 * (2 * NS + 3 * NB + 4) + 4 <= 256, "barrier area");
    static_assert(SMEM <= 232448, "shared memory per CTA");
};

template <int TN, bool Q6>
__global__ void __maxnreg__(MMQ_MAXNREG) k_mmq_kq(const __grid_constant__ MmqkArgs a) {
    using P = MmqkPlan<TN, Q6>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *raw = sm + P::OFF_RAW;
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + P::OFF_BAR);  // [NS]
    uint64_t *empty = full + P::NS;                                  // [NS]
    uint64_t *ready = empty + P::NS;                                 // [NB]
    uint64_t *opfree = ready + P::NB;                                // [NB]
    uint64_t *sfree = opfree + P::NB;                                // [NB]
    uint64_t *tfull = sfree + P::NB;                                 // [2]
    uint64_t *tfree = tfull + 2;                                     // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfree + 2);
    __shared__ volatile int s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int issued = 0, ncommit = 0;
    uint64_t *last_commit = nullptr;
    uint32_t last_parity = 0;
    const long long tile = blockIdx.x;
    const int t0 = blockIdx.y * TN;
    int sgi = 0;
#pragma unroll
    for (int i = 1; i < GV_MAX_SEG; i++)
        if (i < a.nseg && tile >= a.seg[i].tile_begin) sgi = i;
    const MmqSeg &sg = a.seg[sgi];
    const long long r0 = (tile - sg.tile_begin) * MMQ_M;
    const bool q6 = Q6 && sg.ttype == TT_Q6_K_P;
    const int kb0 = (int)((long long)a.nblk * blockIdx.z / gridDim.z);
    const int nb = (int)((long long)a.nblk * (blockIdx.z + 1) / gridDim.z) - kb0;  // blocks of this CTA
    const int nch = q6 ? 2 * nb : nb;  // chunks: blocks, or half blocks for Q6_K

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < P::NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 4);
        }
        for (int p = 0; p < P::NB; p++) {
            mbar_init(&ready[p], 4);
            mbar_init(&opfree[p], 1);
            mbar_init(&sfree[p], 8);
        }
        for (int h = 0; h < 2; h++) {
            mbar_init(&tfull[h], 1);
            mbar_init(&tfree[h], 8);
        }
        s_fail = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(P::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint32_t wbytes = (uint32_t)(MMQ_M * sg.chunk_bytes);
            for (int c = 0; c < nb; c++) {
                const int s = c % P::NS;
                if (c >= P::NS &&
                    (s_fail || !mbar_wait(&empty[s], (uint32_t)(((c / P::NS) - 1) & 1), 131))) {
                    s_fail = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], wbytes);
                tma_load_2d(raw + s * P::W_STAGE, &a.wmap[sgi], (kb0 + c) * (sg.chunk_bytes / 8), (int)r0, &full[s]);
                issued++;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        int g = 0;
        bool ok = true;
        const uint32_t idesc = mmq_idesc<TN>();
        if (q6) {
            // chunk c = half c & 1 of block c >> 1; block b into TMEM half b & 1
            for (int c = 0; c < 2 * nb && ok; c++) {
                const int p = c % P::NB, b = c >> 1, hb = c & 1, h = b & 1;
                const uint32_t use = (uint32_t)(c / P::NB);
                if (lane == 0) ok = !s_fail && mbar_wait(&ready[p], use & 1u, 136);
                if (lane == 0 && ok && hb == 0 && b >= 2)
                    ok = !s_fail && mbar_wait(&tfree[h], (uint32_t)(((b >> 1) - 1) & 1), 137);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint8_t *buf = sm + p * P::BUF;
                    for (int kb = 0; kb < 4; kb++) {
                        const uint64_t bd = umma_desc(buf + P::OB_B + kb * TN * 32, 128, 256);
                        for (int dg = 0; dg < 2; dg++) {
                            const uint64_t ad = umma_desc(buf + P::OB_A + (2 * kb + dg) * MMQ_M * 32, 128, 256);
                            umma_i8(tmem + (uint32_t)(h * P::HALF + dg * TN), ad, bd, idesc, (hb | kb) ? 1u : 0u);
                        }
                    }
                    umma_commit(&opfree[p]);
                    last_commit = &opfree[p];
                    last_parity = use & 1u;
                    ncommit++;
                    if (hb) {
                        umma_commit(&tfull[h]);
                        last_commit = &tfull[h];
                        last_parity = (uint32_t)((b >> 1) & 1);
                        ncommit++;
                    }
                }
                __syncwarp();
            }
        }
        for (int c = 0; c < nb && ok && !q6; c++) {
            const int p = c % P::NB;
            const uint32_t use = (uint32_t)(c / P::NB);
            if (lane == 0) ok = !s_fail && mbar_wait(&ready[p], use & 1u, 136);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const uint8_t *buf = sm + p * P::BUF;
            for (int r = 0; r < P::ROUNDS; r++, g++) {
                const int h = g & 1;
                if (lane == 0 && g >= 2) ok = !s_fail && mbar_wait(&tfree[h], (uint32_t)(((g >> 1) - 1) & 1), 137);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) {
                    for (int kb = 0; kb < P::RB; kb++) {
                        const int j = r * P::RB + kb;
                        const uint64_t ad = umma_desc(buf + P::OB_A + j * MMQ_M * 32, 128, 256);
                        const uint64_t bd = umma_desc(buf + P::OB_B + j * TN * 32, 128, 256);
                        umma_i8(tmem + (uint32_t)(h * P::HALF + kb * TN), ad, bd, idesc, 0u);
                    }
                    umma_commit(&tfull[h]);
                    last_commit = &tfull[h];
                    last_parity = (uint32_t)((g >> 1) & 1);
                    ncommit++;
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) {
                umma_commit(&opfree[p]);
                last_commit = &opfree[p];
                last_parity = use & 1u;
                ncommit++;
            }
            __syncwarp();
        }
        if (!ok) s_fail = 1;
        if (ok && lane == 0 && ncommit > 0 && !mbar_wait(last_commit, last_parity, 138)) s_fail = 1;
        __syncwarp();
    } else if (warp < 6) {
        // ---------------- converters ----------------
        // weights: thread ct = row ct; activations: thread ct = token ct % TN,
        // sub-blocks [SPT*(ct/TN), SPT*(ct/TN) + SPT)
        const int ct = threadIdx.x - 64;
        const bool q5 = sg.ttype == TT_Q5_K;
        constexpr int SPT = TN / 16;
        const int tk = ct % TN, hq = ct / TN;
        const bool live = t0 + tk < a.ntok;
        // activation words of block c + 1 are loaded (into registers) while
        // block c is converted: a global round trip per block would
        // otherwise sit on the converters' critical path
        // sw: the f32 d bits, then the 16 int16 bsums as 8 words
        uint32_t xw[SPT * 8], nxw[SPT * 8], xsw[9], nxsw[9];
        // (Q6_K: chunk c is elements 128*(c & 1).. of block c >> 1, and only
        // the threads with SPT * hq < 4 have sub-blocks in it)
        const bool xact = !q6 || SPT * hq < 4;
        auto fetch = [&](int c, uint32_t (&w)[SPT * 8], uint32_t (&sw)[9]) {
            const int cb = kb0 + (q6 ? c >> 1 : c);
            const uint8_t *src = a.xq + (long long)(t0 + tk) * a.xq_ld + (long long)cb * 292;
            const bool on = live && c < nch && xact;
            const int xo = 4 + (q6 ? 128 * (c & 1) : 0) + 32 * SPT * hq;
#pragma unroll
            for (int i = 0; i < SPT * 8; i++)
                w[i] = on ? reinterpret_cast<const uint32_t *>(src + xo)[i] : 0u;
#pragma unroll
            for (int i = 0; i < 9; i++) sw[i] = 0u;
            if (hq == 0 && live && c < nch) {
                sw[0] = *reinterpret_cast<const uint32_t *>(src);
#pragma unroll
                for (int i = 0; i < 8; i++) sw[1 + i] = reinterpret_cast<const uint32_t *>(src + 260)[i];
            }
        };
        fetch(0, xw, xsw);
        for (int c = 0; c < nch; c++) {
            const int cb = q6 ? c >> 1 : c;  // block of this chunk = its raw stage
            const int s = cb % P::NS, p = c % P::NB;
            const uint32_t use = (uint32_t)(c / P::NB);
            fetch(c + 1, nxw, nxsw);
            bool ok = !s_fail && mbar_wait(&full[s], (uint32_t)((cb / P::NS) & 1), 132);
            if (ok && use > 0)
                ok = mbar_wait(&opfree[p], (use - 1) & 1u, 139) && mbar_wait(&sfree[p], (use - 1) & 1u, 140);
            if (!__all_sync(0xffffffffu, ok)) {
                s_fail = 1;
                break;
            }
            uint8_t *buf = sm + p * P::BUF;
            // activations into the B operands and per-token values
#pragma unroll
            for (int jj = 0; jj < SPT; jj++) {
                if (!xact) break;
                uint8_t *dst = buf + P::OB_B + (SPT * hq + jj) * TN * 32;
                *reinterpret_cast<uint4 *>(dst + umma_off(tk, 0)) =
                    make_uint4(xw[8 * jj], xw[8 * jj + 1], xw[8 * jj + 2], xw[8 * jj + 3]);
                *reinterpret_cast<uint4 *>(dst + umma_off(tk, 1)) =
                    make_uint4(xw[8 * jj + 4], xw[8 * jj + 5], xw[8 * jj + 6], xw[8 * jj + 7]);
            }
            if (q6) {
                if (hq == 0) reinterpret_cast<uint32_t *>(buf + P::OB_DY)[tk] = xsw[0];
                // weights: row ct, half c & 1 of the raw block -> hi / lo digit tiles
                const uint8_t *rp = raw + s * P::W_STAGE + ct * sg.chunk_bytes;
                const int hb = c & 1;
                uint32_t QL[16], QH[8];
                const uint4 *v4 = reinterpret_cast<const uint4 *>(rp + 64 * hb);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint4 v = v4[i];
                    QL[4 * i] = v.x;
                    QL[4 * i + 1] = v.y;
                    QL[4 * i + 2] = v.z;
                    QL[4 * i + 3] = v.w;
                }
                const uint4 *h4 = reinterpret_cast<const uint4 *>(rp + 128 + 32 * hb);
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const uint4 v = h4[i];
                    QH[4 * i] = v.x;
                    QH[4 * i + 1] = v.y;
                    QH[4 * i + 2] = v.z;
                    QH[4 * i + 3] = v.w;
                }
                const uint2 scw = *reinterpret_cast<const uint2 *>(rp + 192 + 8 * hb);  // scales[8*hb .. +7]
                reinterpret_cast<float *>(buf + P::OB_D)[ct] = f16_lo(*reinterpret_cast<const uint32_t *>(rp + 208));
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    // sub-block k of the half: element l = ql[64*hb + 32*(k & 1) + l]
                    // (low nibble for k < 2, high for k >= 2) | qh bits 2k, 2k+1
                    const int sa = (int)(int8_t)(((2 * k < 4 ? scw.x : scw.y) >> (8 * ((2 * k) & 3))) & 0xFFu);
                    const int sb = (int)(int8_t)(((2 * k + 1 < 4 ? scw.x : scw.y) >> (8 * ((2 * k + 1) & 3))) & 0xFFu);
                    uint32_t hi[8], lo[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const uint32_t ql = QL[8 * (k & 1) + i];
                        const uint32_t v = ((k < 2 ? ql : ql >> 4) & 0x0F0F0F0Fu) |
                                           (((QH[i] >> (2 * k)) & 0x03030303u) << 4);
                        const int sc = i < 4 ? sa : sb;  // elements 0..15 | 16..31
                        uint32_t hw = 0u, lw = 0u;
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int w = ((int)((v >> (8 * e)) & 0xFFu) - 32) * sc;
                            hw |= (uint32_t)((w >> 6) & 0xFF) << (8 * e);
                            lw |= (uint32_t)(w & 63) << (8 * e);
                        }
                        hi[i] = hw;
                        lo[i] = lw;
                    }
                    uint8_t *dh = buf + P::OB_A + (2 * k) * MMQ_M * 32;
                    uint8_t *dl = dh + MMQ_M * 32;
                    *reinterpret_cast<uint4 *>(dh + umma_off(ct, 0)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4 *>(dh + umma_off(ct, 1)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                    *reinterpret_cast<uint4 *>(dl + umma_off(ct, 0)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    *reinterpret_cast<uint4 *>(dl + umma_off(ct, 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                }
            } else {
            if (hq == 0) {
                reinterpret_cast<uint32_t *>(buf + P::OB_DY)[tk] = xsw[0];
                int xbs[8];
#pragma unroll
                for (int j = 0; j < 8; j++)
                    xbs[j] = (int)(int16_t)(xsw[1 + j] & 0xFFFFu) + (int)(int16_t)(xsw[1 + j] >> 16);
                int4 *bsd = reinterpret_cast<int4 *>(buf + P::OB_BS + tk * 32);
                bsd[0] = make_int4(xbs[0], xbs[1], xbs[2], xbs[3]);
                bsd[1] = make_int4(xbs[4], xbs[5], xbs[6], xbs[7]);
            }
            // weights: row ct of the raw block
            {
                const uint8_t *rp = raw + s * P::W_STAGE + ct * sg.chunk_bytes;
                uint32_t W[44];
                const uint4 *v4 = reinterpret_cast<const uint4 *>(rp);
#pragma unroll
                for (int i = 0; i < 9; i++) {
                    const uint4 v = v4[i];
                    W[4 * i] = v.x;
                    W[4 * i + 1] = v.y;
                    W[4 * i + 2] = v.z;
                    W[4 * i + 3] = v.w;
                }
                if (q5) {
#pragma unroll
                    for (int i = 9; i < 11; i++) {
                        const uint4 v = v4[i];
                        W[4 * i] = v.x;
                        W[4 * i + 1] = v.y;
                        W[4 * i + 2] = v.z;
                        W[4 * i + 3] = v.w;
                    }
                }
                float *dd = reinterpret_cast<float *>(buf + P::OB_D);
                dd[ct] = f16_lo(W[0]);
                dd[MMQ_M + ct] = f16_hi(W[0]);
                uint32_t scw[2] = {0u, 0u}, mnw[2] = {0u, 0u};
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    int sc, mn;
                    kq_scale_min_w(j, W + 1, sc, mn);
                    scw[j >> 2] |= (uint32_t)sc << (8 * (j & 3));
                    mnw[j >> 2] |= (uint32_t)mn << (8 * (j & 3));
                    const int cq = j >> 1;
                    uint32_t o[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const uint32_t ql = q5 ? W[12 + 8 * cq + i] : W[4 + 8 * cq + i];
                        uint32_t v = (j & 1) ? (ql >> 4) & 0x0F0F0F0Fu : ql & 0x0F0F0F0Fu;
                        if (q5) v |= ((W[4 + i] >> j) & 0x01010101u) << 4;
                        o[i] = v;
                    }
                    uint8_t *dst = buf + P::OB_A + j * MMQ_M * 32;
                    *reinterpret_cast<uint4 *>(dst + umma_off(ct, 0)) = make_uint4(o[0], o[1], o[2], o[3]);
                    *reinterpret_cast<uint4 *>(dst + umma_off(ct, 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                }
                *reinterpret_cast<uint2 *>(buf + P::OB_SC + ct * 8) = make_uint2(scw[0], scw[1]);
                *reinterpret_cast<uint2 *>(buf + P::OB_MN + ct * 8) = make_uint2(mnw[0], mnw[1]);
            }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (!q6 || (c & 1)) mbar_arrive(&empty[s]);  // Q6_K: the stage after the block's second half
                mbar_arrive(&ready[p]);
            }
#pragma unroll
            for (int i = 0; i < SPT * 8; i++) xw[i] = nxw[i];
#pragma unroll
            for (int i = 0; i < 9; i++) xsw[i] = nxsw[i];
        }
    } else {
        // ---------------- fold (thread = row = TMEM lane, half the tokens) ----------------
        constexpr int TH = TN / 2;
        const int q = warp & 3;
        const int fh = (warp - 6) >> 2;
        const int row = q * 32 + lane;
        float acc[TH];
#pragma unroll
        for (int t = 0; t < TH; t++) acc[t] = 0.0f;
        int g = 0;
        for (int c = 0; c < nch && q6; c++) {
            // Q6_K: after the second half of block b, isum = 64*H + L
            const int p = c % P::NB, b = c >> 1, h = b & 1;
            if (!__all_sync(0xffffffffu, !s_fail && mbar_wait(&ready[p], (uint32_t)(c / P::NB) & 1u, 133))) {
                s_fail = 1;
                break;
            }
            if (c & 1) {
                if (!__all_sync(0xffffffffu, !s_fail && mbar_wait(&tfull[h], (uint32_t)((b >> 1) & 1), 134))) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * P::HALF + fh * TH);
                uint32_t dH[TH], dL[TH];
                tmem_ldn<TH>(tbase, dH);
                tmem_ldn<TH>(tbase + (uint32_t)TN, dL);
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tfree[h]);
                const uint8_t *buf = sm + p * P::BUF;
                const float dw = reinterpret_cast<const float *>(buf + P::OB_D)[row];
                const float *dy = reinterpret_cast<const float *>(buf + P::OB_DY) + fh * TH;
                const long long tb = (long long)(kb0 + b) * a.ntok + t0 + fh * TH;
#pragma unroll
                for (int i = 0; i < TH; i++) {
                    const int is = 64 * (int)dH[i] + (int)dL[i];
                    const float term = __fmul_rn(__fmul_rn(dw, dy[i]), __int2float_rn(is));
                    if (!a.terms)
                        acc[i] = __fadd_rn(acc[i], term);
                    else if (r0 + row < sg.rows && t0 + fh * TH + i < a.ntok)
                        a.terms[(tb + i) * sg.rows + r0 + row] = term;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sfree[p]);
        }
        for (int c = 0; c < nb && !q6; c++) {
            const int p = c % P::NB;
            if (!__all_sync(0xffffffffu, !s_fail && mbar_wait(&ready[p], (uint32_t)(c / P::NB) & 1u, 133))) {
                s_fail = 1;
                break;
            }
            const uint8_t *buf = sm + p * P::BUF;
            const uint2 scw = *reinterpret_cast<const uint2 *>(buf + P::OB_SC + row * 8);
            int is[TH];
#pragma unroll
            for (int t = 0; t < TH; t++) is[t] = 0;
            for (int r = 0; r < P::ROUNDS; r++, g++) {
                const int h = g & 1;
                if (!__all_sync(0xffffffffu, !s_fail && mbar_wait(&tfull[h], (uint32_t)((g >> 1) & 1), 134))) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * P::HALF + fh * TH);
                uint32_t dA[TH], dB[TH];
                tmem_ldn<TH>(tbase, dA);
                tmem_ld_wait();
#pragma unroll
                for (int kb = 0; kb < P::RB; kb++) {
                    uint32_t(&d)[TH] = (kb & 1) ? dB : dA;
                    if (kb + 1 < P::RB) tmem_ldn<TH>(tbase + (uint32_t)((kb + 1) * TN), (kb & 1) ? dA : dB);
                    const int j = r * P::RB + kb;
                    const int sc = (int)(((j < 4 ? scw.x : scw.y) >> (8 * (j & 3))) & 0xFFu);
#pragma unroll
                    for (int i = 0; i < TH; i++) is[i] += sc * (int)d[i];
                    tmem_ld_wait();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tfree[h]);
            }
            if (__any_sync(0xffffffffu, s_fail != 0)) break;
            // d = dy*d_w; dmin = dy*dmin_w; sumf += d*isum - dmin*summs
            const uint2 mnw = *reinterpret_cast<const uint2 *>(buf + P::OB_MN + row * 8);
            const float *dd = reinterpret_cast<const float *>(buf + P::OB_D);
            const float dw = dd[row], dmw = dd[MMQ_M + row];
            const float *dy = reinterpret_cast<const float *>(buf + P::OB_DY) + fh * TH;
            const int4 *bs = reinterpret_cast<const int4 *>(buf + P::OB_BS) + fh * TH * 2;
            int mn[8];
#pragma unroll
            for (int j = 0; j < 8; j++) mn[j] = (int)(((j < 4 ? mnw.x : mnw.y) >> (8 * (j & 3))) & 0xFFu);
            const long long tb = (long long)(kb0 + c) * a.ntok + t0 + fh * TH;
#pragma unroll
            for (int i = 0; i < TH; i++) {
                const int4 b0 = bs[2 * i], b1 = bs[2 * i + 1];
                const int ms = mn[0] * b0.x + mn[1] * b0.y + mn[2] * b0.z + mn[3] * b0.w + mn[4] * b1.x +
                               mn[5] * b1.y + mn[6] * b1.z + mn[7] * b1.w;
                const float d = __fmul_rn(dy[i], dw), dm = __fmul_rn(dy[i], dmw);
                const float term = __fsub_rn(__fmul_rn(d, __int2float_rn(is[i])), __fmul_rn(dm, __int2float_rn(ms)));
                if (!a.terms)
                    acc[i] = __fadd_rn(acc[i], term);
                else if (r0 + row < sg.rows && t0 + fh * TH + i < a.ntok)
                    a.terms[(tb + i) * sg.rows + r0 + row] = term;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sfree[p]);
        }
        const long long rr = r0 + row;
        if (!s_fail && rr < sg.rows && !a.terms) {
            const int nt = min(TN, a.ntok - t0) - fh * TH;
#pragma unroll
            for (int i = 0; i < TH; i++) {
                if (i < nt) {
                    float *o = sg.out + (long long)(t0 + fh * TH + i) * sg.out_ld + rr;
                    *o = sg.mode == GV_ADD ? __fadd_rn(*o, acc[i]) : acc[i];
                }
            }
        }
    }
    __syncthreads();
    if (s_fail) {
        if (warp == 0 && lane == 0)
            for (int c = issued > P::NS ? issued - P::NS : 0; c < issued; c++)
                if (!mbar_wait(&full[c % P::NS], (uint32_t)((c / P::NS) & 1), 135)) break;
        if (warp == 1 && lane == 0 && ncommit > 0) mbar_wait(last_commit, last_parity, 135);
        if (threadIdx.x == 0) set_error(130);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P::TMEM_COLS)
                     : "memory");
    }
}

// split-K epilogue: y[t][r] = sum over blocks b, in block order from 0.0f,
// of terms[b][t][r] (the fold of k_mmq_kq, operation for operation), then
// written or added to the output like the unsplit kernel.  When a kernel has
// recorded an error (k_mmq_kq gives up a bounded wait with code 130 and
// leaves some term slots unwritten), nothing is written: the output keeps
// its previous contents, as after a failed unsplit launch.
__global__ void k_mmq_term_sum(const float *__restrict__ terms, int nblk, int ntok, long long rows, float *out,
                               long long out_ld, int mode) {
    pdl_trigger();
    pdl_wait();
    if (*(volatile int *)&g_q35_error != 0) return;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)ntok * rows) return;
    const long long t = i / rows, r = i - t * rows;
    const long long stride = (long long)ntok * rows;
    const float *p = terms + i;
    float acc = 0.0f;
    for (int b = 0; b < nblk; b++) acc = __fadd_rn(acc, p[b * stride]);
    float *o = out + t * out_ld + r;
    *o = mode == GV_ADD ? __fadd_rn(*o, acc) : acc;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
inline bool mmq_encode(CUtensorMap *m, const void *base, long long rows, long long row_stride, int row_bytes,
                       int box_bytes, int box_rows) {
    const auto fn = lpr_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_stride};
    const cuuint32_t box[2] = {(cuuint32_t)(box_bytes / 8), (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline int mmq_prepare() {
    static int done = 0;
    if (done) return 0;
    const cudaError_t es[] = {
        cudaFuncSetAttribute(k_mmq<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqPlan<64>::SMEM),
        cudaFuncSetAttribute(k_mmq<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqPlan<32>::SMEM),
        cudaFuncSetAttribute(k_mmq<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqPlan<16>::SMEM),
        cudaFuncSetAttribute(k_mmq_kq<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqkPlan<64, false>::SMEM),
        cudaFuncSetAttribute(k_mmq_kq<32, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqkPlan<32, false>::SMEM),
        cudaFuncSetAttribute(k_mmq_kq<16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqkPlan<16, false>::SMEM),
        cudaFuncSetAttribute(k_mmq_kq<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqkPlan<64, true>::SMEM),
        cudaFuncSetAttribute(k_mmq_kq<32, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqkPlan<32, true>::SMEM),
        cudaFuncSetAttribute(k_mmq_kq<16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqkPlan<16, true>::SMEM)};
    for (cudaError_t e : es)
        if (e != cudaSuccess) return (int)e;
    done = 1;
    return 0;
}

// token tile of k_mmq / k_mmq_kq: the widest of 64 / 32 / 16 that still gives
// half the SMs a tile (the fold work per tile scales with the tile's tokens,
// so narrower tiles spread a short matrix over more SMs, but every token tile
// streams the weights again; measured on B200, half the SMs beat all of them
// and a quarter at batch 32 / 64) and is not wider than the tokens rounded up
// to 16; 16 when none qualifies
#ifndef Q35_MMQ_TILE_SM_DIV
#define Q35_MMQ_TILE_SM_DIV 2
#endif
inline int mmq_q32_token_tile(long long row_tiles, int ntok) {
    const long long sms = gemv_sm_count() / Q35_MMQ_TILE_SM_DIV;
    const int ntok16 = (ntok + 15) / 16 * 16;
    for (int tn : {64, 32})
        if (tn <= ntok16 && row_tiles * ((ntok + tn - 1) / tn) >= sms) return tn;
    return 16;
}

// split-K factor for one segment of `tiles` row tiles: when the widest
// token tile leaves more than half the SMs idle, K is split over CTAs (at
// least 2 blocks each, at most 16 splits, one wave) if the caller's term
// buffer holds nblk x ntok x rows floats; 1 = no split.  Only up to
// MMQ_SPLIT_MAX_TOK tokens: the terms are written and read back once
// (8 bytes per block, token and row against 144-224 weight bytes per block
// and row), so past 32 tokens their traffic outweighs the weights' and the
// split stops paying (measured on B200: 27B ffn_down 101 -> 52 us at 16
// tokens, 101 -> 83 at 32, none at 64)
constexpr int MMQ_SPLIT_MAX_TOK = 32;
inline int mmq_kq_split(long long tiles, long long rows, int ntok, int nblk, size_t terms_bytes, int &tn) {
    if (ntok > MMQ_SPLIT_MAX_TOK) return 1;
    const long long sms = gemv_sm_count();
    const int wide = ntok > 32 ? 64 : ntok > 16 ? 32 : 16;
    const long long ctas = tiles * ((ntok + wide - 1) / wide);
    if (2 * ctas > sms || (size_t)nblk * ntok * rows * sizeof(float) > terms_bytes) return 1;
    const long long ks = std::min<long long>(std::min<long long>(sms / ctas, nblk / 2), 16);
    if (ks < 2) return 1;
    tn = wide;
    return (int)ks;
}

// K-quant (Q4_K / Q5_K / Q6_K in 224-byte blocks) weights x Q8_K activations;
// -1 when not eligible.  terms / terms_bytes: the caller's scratch for split-K
// (null: never split)
inline int mmq_kq_launch(const GemvSegDesc *segs, int nseg, const void *xq, int cols, int ntok, cudaStream_t st,
                         long long xq_ld, float *terms = nullptr, size_t terms_bytes = 0) {
    const long long act_row = (long long)(cols / 256) * 292;
    const long long ld = xq_ld > 0 ? xq_ld : act_row;
    if ((reinterpret_cast<uintptr_t>(xq) & 3u) || (ld & 3)) return -1;
    MmqkArgs a{};
    long long tiles = 0;
    for (int i = 0; i < nseg; i++) {
        const int tt = segs[i].ttype;
        if (tt != TT_Q4_K && tt != TT_Q5_K && tt != TT_Q6_K_P) return -1;
        const Geom g = geom_of(tt);
        const int rb = cols / 256 * g.bytes;
        if (rb % 16 || (reinterpret_cast<uintptr_t>(segs[i].w) & 15u)) return -1;
        MmqSeg &s = a.seg[i];
        s.out = segs[i].out;
        s.rows = segs[i].rows;
        s.out_ld = segs[i].out_ld;
        s.ttype = tt;
        s.row_bytes = rb;
        s.chunk_bytes = g.bytes;  // 144 / 176 / 224
        s.mode = segs[i].mode;
        s.tile_begin = tiles;
        tiles += (s.rows + MMQ_M - 1) / MMQ_M;
        if (!mmq_encode(&a.wmap[i], segs[i].w, s.rows, rb, rb, s.chunk_bytes, MMQ_M)) return -1;
    }
    if (tiles == 0) return 0;
    a.nseg = nseg;
    a.total_tiles = tiles;
    a.xq = reinterpret_cast<const uint8_t *>(xq);
    a.xq_ld = ld;
    a.ntok = ntok;
    a.nblk = cols / 256;
    Q35_TRY_RC(mmq_prepare());
    int tn = mmq_q32_token_tile(tiles, ntok);
    const int ks = (terms && nseg == 1) ? mmq_kq_split(tiles, a.seg[0].rows, ntok, a.nblk, terms_bytes, tn) : 1;
    a.terms = ks > 1 ? terms : nullptr;
    const dim3 grid((unsigned)tiles, (unsigned)((ntok + tn - 1) / tn), (unsigned)ks);
    bool q6 = false;
    for (int i = 0; i < nseg; i++) q6 = q6 || segs[i].ttype == TT_Q6_K_P;
    int rc;
    if (q6) {
        if (tn == 16)
            rc = launch_k(k_mmq_kq<16, true>, grid, dim3(MMQ_THREADS), (size_t)MmqkPlan<16, true>::SMEM, st, a);
        else if (tn == 32)
            rc = launch_k(k_mmq_kq<32, true>, grid, dim3(MMQ_THREADS), (size_t)MmqkPlan<32, true>::SMEM, st, a);
        else
            rc = launch_k(k_mmq_kq<64, true>, grid, dim3(MMQ_THREADS), (size_t)MmqkPlan<64, true>::SMEM, st, a);
    } else {
        if (tn == 16)
            rc = launch_k(k_mmq_kq<16, false>, grid, dim3(MMQ_THREADS), (size_t)MmqkPlan<16, false>::SMEM, st, a);
        else if (tn == 32)
            rc = launch_k(k_mmq_kq<32, false>, grid, dim3(MMQ_THREADS), (size_t)MmqkPlan<32, false>::SMEM, st, a);
        else
            rc = launch_k(k_mmq_kq<64, false>, grid, dim3(MMQ_THREADS), (size_t)MmqkPlan<64, false>::SMEM, st, a);
    }
    if (rc || ks == 1) return rc;
    const long long n = (long long)ntok * a.seg[0].rows;
    return launch_k(k_mmq_term_sum, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, (const float *)terms,
                    a.nblk, ntok, a.seg[0].rows, a.seg[0].out, a.seg[0].out_ld, a.seg[0].mode);
}

// Tensor-core path for >= MMQ_MIN_TOK tokens of Q8_0 / IQ4_NL (Q8_0
// activation at a 16-byte multiple stride) or Q4_K / Q5_K / padded Q6_K (Q8_K
// activation) weights with 16-byte-aligned rows.  Returns -1 (nothing launched) when not
// eligible.
inline int mmq_launch(const GemvSegDesc *segs, int nseg, const void *xq, int cols, int ntok, cudaStream_t st,
                      long long xq_ld, float *terms, size_t terms_bytes) {
    if (ntok < MMQ_MIN_TOK || nseg < 1 || nseg > GV_MAX_SEG || cols <= 0 || cols % 256 != 0) return -1;
    if (geom_of(segs[0].ttype).family == 256)
        return mmq_kq_launch(segs, nseg, xq, cols, ntok, st, xq_ld, terms, terms_bytes);
    const long long act_row = (long long)(cols / 32) * 34;
    const long long ld = xq_ld > 0 ? xq_ld : act_row;
    if ((reinterpret_cast<uintptr_t>(xq) & 15u) || (ld & 15)) return -1;
    MmqArgs a{};
    long long tiles = 0;
    for (int i = 0; i < nseg; i++) {
        const int tt = segs[i].ttype;
        if (tt != TT_Q8_0 && tt != TT_IQ4_NL) return -1;
        const Geom g = geom_of(tt);
        const int rb = cols / g.elems * g.bytes;
        if (rb % 16 || (reinterpret_cast<uintptr_t>(segs[i].w) & 15u)) return -1;
        MmqSeg &s = a.seg[i];
        s.out = segs[i].out;
        s.rows = segs[i].rows;
        s.out_ld = segs[i].out_ld;
        s.ttype = tt;
        s.row_bytes = rb;
        s.chunk_bytes = 256 / g.elems * g.bytes;  // 272 / 144
        s.mode = segs[i].mode;
        s.tile_begin = tiles;
        tiles += (s.rows + MMQ_M - 1) / MMQ_M;
        if (!mmq_encode(&a.wmap[i], segs[i].w, s.rows, rb, rb, s.chunk_bytes, MMQ_M)) return -1;
    }
    if (tiles == 0) return 0;
    const int tn = mmq_q32_token_tile(tiles, ntok);
    if (!mmq_encode(&a.xmap, xq, ntok, ld, (int)act_row, 272, tn)) return -1;
    a.nseg = nseg;
    a.total_tiles = tiles;
    a.ntok = ntok;
    a.nchunk = cols / 256;
    a.ntt = (ntok + tn - 1) / tn;
    Q35_TRY_RC(mmq_prepare());
    // persistent: one CTA per SM (shared memory and TMEM allow one) walks
    // the tiles, so one tile's fold overlaps the next tile's loads
    const long long nwork = tiles * a.ntt;
    const dim3 grid((unsigned)std::min<long long>(nwork, gemv_sm_count()));
    if (tn == 16) return launch_k(k_mmq<16>, grid, dim3(MMQ_THREADS), (size_t)MmqPlan<16>::SMEM, st, a);
    if (tn == 32) return launch_k(k_mmq<32>, grid, dim3(MMQ_THREADS), (size_t)MmqPlan<32>::SMEM, st, a);
    return launch_k(k_mmq<64>, grid, dim3(MMQ_THREADS), (size_t)MmqPlan<64>::SMEM, st, a);
}

}  // namespace q35
