// sample.cuh -- device sampler: temperature -> top-k -> top-p -> one draw,
// with the selection rules of the reference's Sampler.sample
// (src/sampler.zig:67-190), for one or many logits rows in one launch.
//
// The rules (sampler.zig):
//   * temperature <= 0: greedy, the first index of the maximum;
//   * terms e_i = exp(f32((x_i - max) / T)), mass in f64;
//   * top-k: the k-th largest VALUE is a threshold, ties at it all kept;
//   * top-p: the threshold is raised to the value at which the descending
//     order's cumulative mass first reaches p of the mass top-k kept;
//   * draw: coin = top 24 bits of one xorshift64* word / 2^24, the first
//     surviving index (increasing order) with coin < acc / sum, else the
//     last survivor, else 0.
//
// B200 layout: one thread-block cluster of SMP_CS CTAs per row.  Each CTA
// holds a contiguous slice of the row in shared memory, each thread a
// contiguous chunk of that slice, and the chunk's exp terms sit beside it in
// shared memory (one evaluation per element).  Every selection is exact and
// order-independent: the max, the top-k radix select over order-preserving
// 32-bit keys (integer histograms, shared-memory atomics, summed over the
// cluster through distributed shared memory), and the top-p threshold found
// by the same 4-pass radix descent over integer masses (each term rounded to
// a multiple of 2^-44; a sum of 2^18 terms stays below 2^62).  The f64 mass
// sums are chunked in a fixed order (thread chunks in index order, then
// threads, warps and CTAs in order), so a row always gives the same token;
// they agree with the reference's one sequential f64 sum to about n * 2^-53
// relative, so the drawn index differs from the sequential walk's only when
// the coin falls within that distance of a cumulative boundary.
//
// Control block per row: 16 int32 in the reference's layout (sample.cu:
// vocab, temperature bits, top_k, top_p bits, rng lo / hi in, token out,
// rng lo / hi out, threshold bits out, flags out).  The state is read before
// anything is written, and the CTA of rank 0 writes the outputs after the
// cluster's last barrier.
#pragma once
#include <climits>

#include "common.cuh"

namespace q35 {

constexpr int SMP_CS = 16;         // CTAs per cluster (non-portable size): one cluster per logits row
constexpr int SMP_THREADS = 512;
constexpr int SMP_EPT = 32;        // logits per thread at most
constexpr long long SMP_MAX_N = (long long)SMP_CS * SMP_THREADS * SMP_EPT;  // 262144
constexpr int SMP_WARPS = SMP_THREADS / 32;

enum : int {
    SC_VOCAB = 0, SC_TEMP = 1, SC_TOPK = 2, SC_TOPP = 3, SC_RNG_LO = 4, SC_RNG_HI = 5, SC_TOKEN = 6,
    SC_RNG_OUT_LO = 7, SC_RNG_OUT_HI = 8, SC_THRESH = 9, SC_FLAGS = 10, SC_INTS = 16
};

struct SmpArgs {
    const float *logits;
    long long ld;            // floats between rows
    int n, rows;
    int *ctl;                // control blocks
    long long ctl_ld;        // ints between control blocks
    const int *tok_slot;     // optional: row r uses block tok_slot[run_end ? run_end[r] - 1 : r]
    const int *run_end;
    int *tok_out;            // optional: token of row r also to tok_out[r]
    int advance;             // 1: the advanced PRNG state also replaces the input state
};

// exchange area of one CTA, read by the others through distributed shared
// memory; two of them alternate so one cluster barrier per exchange suffices
struct SmpXch {
    float f;
    int i0, i1, pad;
    double d;
    uint32_t hist[256];
    unsigned long long mass[256];
};

Q35_DEV void smp_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
Q35_DEV int smp_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return (int)r;
}
Q35_DEV uint32_t smp_remote(const void *p, int rank) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(p), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
Q35_DEV uint32_t dsm_u32(const void *p, int rank) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(smp_remote(p, rank)) : "memory");
    return v;
}
Q35_DEV unsigned long long dsm_u64(const void *p, int rank) {
    unsigned long long v;
    asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(smp_remote(p, rank)) : "memory");
    return v;
}
Q35_DEV float dsm_f32(const float *p, int rank) { return __uint_as_float(dsm_u32(p, rank)); }
Q35_DEV double dsm_f64(const double *p, int rank) { return __longlong_as_double((long long)dsm_u64(p, rank)); }

// order-preserving key of a float (larger float -> larger key) and back
Q35_DEV uint32_t smp_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return b ^ ((b >> 31) ? 0xFFFFFFFFu : 0x80000000u);
}
Q35_DEV float smp_unkey(uint32_t k) { return __uint_as_float(k ^ ((k >> 31) ? 0x80000000u : 0xFFFFFFFFu)); }

// xorshift64* (sampler.zig:60-70)
Q35_DEV uint64_t smp_xs64(uint64_t &s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s * 0x2545F4914F6CDD1DULL;
}

constexpr double SMP_FIX = 17592186044416.0;  // 2^44: integer mass units per unit of mass

__global__ void __launch_bounds__(SMP_THREADS, 1) k_sample(SmpArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ SmpXch xch[2];
    __shared__ uint32_t s_tot[256];
    __shared__ unsigned long long s_mtot[256];
    __shared__ double s_part[SMP_THREADS];
    __shared__ double s_wex[SMP_WARPS];
    __shared__ float s_wf[SMP_WARPS];
    __shared__ int s_wi[SMP_WARPS];
    __shared__ int s_sel[2];
    __shared__ long long s_acc;
    extern __shared__ float xs[];

    const int row = blockIdx.y, cr = smp_rank(), tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int blk = row;
    if (a.tok_slot) blk = a.tok_slot[a.run_end ? a.run_end[row] - 1 : row];
    int *ctl = a.ctl + a.ctl_ld * blk;
    const float T = __int_as_float(ctl[SC_TEMP]);
    const int topk = ctl[SC_TOPK];
    const float topp = __int_as_float(ctl[SC_TOPP]);
    uint64_t rng = ((uint64_t)(uint32_t)ctl[SC_RNG_HI] << 32) | (uint64_t)(uint32_t)ctl[SC_RNG_LO];
    const int n = a.n;
    const bool greedy = !(T > 0.0f);
    const bool use_k = !greedy && topk > 0 && topk < n;
    const bool use_p = !greedy && topp > 0.0f && topp < 1.0f;

    // this CTA's slice of the row; this thread's chunk of it (padded to an
    // odd stride in shared memory, so a warp's chunk walks hit distinct banks)
    const int slice = (n + SMP_CS - 1) / SMP_CS;
    const int lo = cr * slice;
    const int cnt = max(0, min(n, lo + slice) - lo);
    const int cpt = (slice + SMP_THREADS - 1) / SMP_THREADS;
    const int stride = cpt | 1;
    const int c0 = tid * cpt;
    const int len = max(0, min(cnt, c0 + cpt) - c0);
    const float *xr = a.logits + a.ld * row + lo;
    for (int i = tid; i < cnt; i += SMP_THREADS) {
        const int t = i / cpt;
        xs[t * stride + (i - t * cpt)] = xr[i];
    }
    __syncthreads();
    const float *my = xs + tid * stride;
    const int g0 = lo + c0;
    int buf = 0;

    // ---- max and its first index (sampler.zig:71-90) ----
    float m = -INFINITY;
    int mi = INT_MAX;
    for (int j = 0; j < len; j++)
        if (my[j] > m) {
            m = my[j];
            mi = g0 + j;
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, o);
        const int oi = __shfl_xor_sync(0xffffffffu, mi, o);
        if (om > m || (om == m && oi < mi)) {
            m = om;
            mi = oi;
        }
    }
    if (lane == 0) {
        s_wf[warp] = m;
        s_wi[warp] = mi;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < SMP_WARPS; w++)
            if (s_wf[w] > m || (s_wf[w] == m && s_wi[w] < mi)) {
                m = s_wf[w];
                mi = s_wi[w];
            }
        xch[buf].f = m;
        xch[buf].i0 = mi;
    }
    smp_cluster_sync();
    float maxv = -INFINITY;
    int amax = INT_MAX;
    for (int r = 0; r < SMP_CS; r++) {
        const float rm = dsm_f32(&xch[buf].f, r);
        const int ri = (int)dsm_u32(&xch[buf].i0, r);
        if (rm > maxv || (rm == maxv && ri < amax)) {
            maxv = rm;
            amax = ri;
        }
    }
    buf ^= 1;
    // greedy: nothing beats -FLT_MAX -> index 0 (sampler.zig:72-79)
    int token = (maxv > -3.402823466e38f && amax != INT_MAX) ? amax : 0;
    float thresh = -3.402823466e38f;  // top-k off: keep v >= -FLT_MAX

    if (!greedy) {
        // ---- top-k: the k-th largest value by a 4-pass radix select ----
        if (use_k) {
            uint32_t prefix = 0, mask = 0;
            int rank = topk;
            for (int pass = 0; pass < 4; pass++) {
                const int shift = 24 - 8 * pass;
                SmpXch &X = xch[buf];
                for (int b = tid; b < 256; b += SMP_THREADS) X.hist[b] = 0;
                __syncthreads();
                for (int j = 0; j < len; j++) {
                    const uint32_t key = smp_key(my[j]);
                    if ((key & mask) == prefix) atomicAdd(&X.hist[(key >> shift) & 255u], 1u);
                }
                smp_cluster_sync();
                for (int b = tid; b < 256; b += SMP_THREADS) {
                    uint32_t s = 0;
                    for (int r = 0; r < SMP_CS; r++) s += dsm_u32(&X.hist[b], r);
                    s_tot[b] = s;
                }
                __syncthreads();
                if (tid == 0) {
                    int acc = 0, chosen = 0, cacc = 0;
                    for (int d = 255; d >= 0; d--) {
                        const int c = (int)s_tot[d];
                        if (c == 0) continue;
                        if (acc + c >= rank) {
                            chosen = d;
                            cacc = acc;
                            break;
                        }
                        acc += c;
                    }
                    s_sel[0] = chosen;
                    s_sel[1] = cacc;
                }
                __syncthreads();
                prefix |= (uint32_t)s_sel[0] << shift;
                mask |= 255u << shift;
                rank -= s_sel[1];
                buf ^= 1;
            }
            thresh = smp_unkey(prefix);
        }

        // ---- exp terms of the survivors, once, beside the chunk ----
        float *e = xs + SMP_THREADS * stride + tid * stride;
        for (int j = 0; j < len; j++) e[j] = !(my[j] < thresh) ? exp_f(__fdiv_rn(__fsub_rn(my[j], maxv), T)) : 0.0f;

        // fixed-order f64 sum of one value per thread over the cluster:
        // thread values -> warps (lane order) -> CTA (warp order) -> ranks
        // (rank order); also each thread's exclusive prefix in that order
        auto cluster_scan = [&](double v, double &excl) -> double {
            s_part[tid] = v;
            __syncthreads();
            if (lane == 0) {
                double p = 0.0;
                for (int l = 0; l < 32; l++) {
                    const double x = s_part[warp * 32 + l];
                    s_part[warp * 32 + l] = p;
                    p += x;
                }
                s_wex[warp] = p;
            }
            __syncthreads();
            if (tid == 0) {
                double p = 0.0;
                for (int w = 0; w < SMP_WARPS; w++) {
                    const double x = s_wex[w];
                    s_wex[w] = p;
                    p += x;
                }
                xch[buf].d = p;
            }
            smp_cluster_sync();
            double rex = 0.0, tot = 0.0;
            for (int r = 0; r < SMP_CS; r++) {
                const double x = dsm_f64(&xch[buf].d, r);
                if (r < cr) rex += x;
                tot += x;
            }
            excl = rex + (s_wex[warp] + s_part[tid]);
            buf ^= 1;
            __syncthreads();  // s_part / s_wex are rewritten by the next scan
            return tot;
        };

        // ---- top-p: raise the threshold (sampler.zig:125-165) ----
        if (use_p) {
            double st = 0.0, ex;
            for (int j = 0; j < len; j++)
                if (!(my[j] < thresh)) st += (double)e[j];
            const double total = cluster_scan(st, ex);
            if (total > 0.0) {
                uint32_t prefix = 0, mask = 0;
                // integer mass of all survivors over the cluster (exact),
                // then the target: p of it
                unsigned long long sfix = 0;
                for (int j = 0; j < len; j++)
                    if (!(my[j] < thresh)) sfix += (unsigned long long)__double2ll_rn((double)e[j] * SMP_FIX);
                {
                    SmpXch &X = xch[buf];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) sfix += __shfl_xor_sync(0xffffffffu, sfix, o);
                    if (tid == 0) X.mass[0] = 0;
                    __syncthreads();
                    if (lane == 0) atomicAdd(&X.mass[0], sfix);
                    smp_cluster_sync();
                    sfix = 0;
                    for (int r = 0; r < SMP_CS; r++) sfix += dsm_u64(&X.mass[0], r);
                    buf ^= 1;
                }
                long long need = __double2ll_rn((double)sfix * (double)topp);
                bool found_all = true;
                for (int pass = 0; pass < 4; pass++) {
                    const int shift = 24 - 8 * pass;
                    SmpXch &X = xch[buf];
                    for (int b = tid; b < 256; b += SMP_THREADS) X.mass[b] = 0;
                    __syncthreads();
                    for (int j = 0; j < len; j++)
                        if (!(my[j] < thresh)) {
                            const uint32_t key = smp_key(my[j]);
                            if ((key & mask) == prefix)
                                atomicAdd(&X.mass[(key >> shift) & 255u],
                                          (unsigned long long)__double2ll_rn((double)e[j] * SMP_FIX));
                        }
                    smp_cluster_sync();
                    for (int b = tid; b < 256; b += SMP_THREADS) {
                        unsigned long long s = 0;
                        for (int r = 0; r < SMP_CS; r++) s += dsm_u64(&X.mass[b], r);
                        s_mtot[b] = s;
                    }
                    __syncthreads();
                    if (tid == 0) {
                        long long acc = 0;
                        int chosen = -1;
                        long long cacc = 0;
                        for (int d = 255; d >= 0; d--) {
                            const long long c = (long long)s_mtot[d];
                            if (c == 0) continue;
                            if (acc + c >= need) {
                                chosen = d;
                                cacc = acc;
                                break;
                            }
                            acc += c;
                        }
                        s_sel[0] = chosen;
                        s_acc = cacc;
                    }
                    __syncthreads();
                    if (s_sel[0] < 0) {
                        found_all = false;
                        buf ^= 1;
                        break;
                    }
                    prefix |= (uint32_t)s_sel[0] << shift;
                    mask |= 255u << shift;
                    need -= s_acc;
                    buf ^= 1;
                }
                if (found_all) {
                    const float cut = smp_unkey(prefix);
                    if (cut > thresh) thresh = cut;
                }
            }
        }

        // ---- mass and the draw (sampler.zig:167-190) ----
        double s = 0.0;
        int last = -1;
        for (int j = 0; j < len; j++)
            if (!(my[j] < thresh)) {
                s += (double)e[j];
                last = g0 + j;
            }
        double pre;
        const double sum = cluster_scan(s, pre);
        if (rng == 0) rng = 0x9E3779B97F4A7C15ULL;
        const uint64_t word = smp_xs64(rng);
        const double coin = (double)((float)(word >> 40) / 16777216.0f);
        int found = INT_MAX;
        double acc = pre;
        for (int j = 0; j < len && found == INT_MAX; j++)
            if (!(my[j] < thresh)) {
                acc += (double)e[j];
                if (coin < acc / sum) found = g0 + j;
            }
        // first crossing and last survivor over the cluster
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            found = min(found, __shfl_xor_sync(0xffffffffu, found, o));
            last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
        }
        if (lane == 0) {
            s_wi[warp] = found;
            s_part[warp] = (double)last;
        }
        __syncthreads();
        if (tid == 0) {
            int f = INT_MAX, l = -1;
            for (int w = 0; w < SMP_WARPS; w++) {
                f = min(f, s_wi[w]);
                l = max(l, (int)s_part[w]);
            }
            xch[buf].i0 = f;
            xch[buf].i1 = l;
        }
        smp_cluster_sync();
        int f = INT_MAX, l = -1;
        for (int r = 0; r < SMP_CS; r++) {
            f = min(f, (int)dsm_u32(&xch[buf].i0, r));
            l = max(l, (int)dsm_u32(&xch[buf].i1, r));
        }
        buf ^= 1;
        token = f != INT_MAX ? f : (l >= 0 ? l : 0);
    }
    // no CTA leaves while another may still read its shared memory
    smp_cluster_sync();
    if (cr == 0 && tid == 0) {
        ctl[SC_TOKEN] = token;
        if (!greedy) {
            ctl[SC_RNG_OUT_LO] = (int)(uint32_t)(rng & 0xFFFFFFFFu);
            ctl[SC_RNG_OUT_HI] = (int)(uint32_t)(rng >> 32);
            if (a.advance) {
                ctl[SC_RNG_LO] = (int)(uint32_t)(rng & 0xFFFFFFFFu);
                ctl[SC_RNG_HI] = (int)(uint32_t)(rng >> 32);
            }
        }
        ctl[SC_THRESH] = __float_as_int(thresh);
        ctl[SC_FLAGS] = (greedy ? 1 : 0) | (use_k ? 2 : 0) | (use_p ? 4 : 0);
        if (a.tok_out) a.tok_out[row] = token;
    }
}

inline size_t sample_smem(int n) {
    const int slice = (n + SMP_CS - 1) / SMP_CS;
    const int cpt = (slice + SMP_THREADS - 1) / SMP_THREADS;
    return 2 * (size_t)SMP_THREADS * (size_t)(cpt | 1) * sizeof(float);  // the chunks, then their terms
}

inline int sample_launch(const SmpArgs &a, cudaStream_t st) {
    if (a.rows <= 0) return 0;
    if (a.n <= 0 || a.n > SMP_MAX_N || !a.logits || !a.ctl || a.ld < a.n || a.ctl_ld < SC_INTS)
        return (int)cudaErrorInvalidValue;
    static int ready = 0;
    const size_t smem = sample_smem(a.n);
    if (!ready) {
        cudaError_t r = cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sample_smem((int)SMP_MAX_N));
        if (r == cudaSuccess) r = cudaFuncSetAttribute(k_sample, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (r != cudaSuccess) return (int)r;
        ready = 1;
    }
    launch_count()++;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(SMP_CS, (unsigned)a.rows);
    cfg.blockDim = dim3(SMP_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = SMP_CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int clusters_ok = -1;  // can a 16-CTA cluster of this kernel be resident at all
    if (clusters_ok < 0) {
        int nc = 0;
        const cudaError_t r = cudaOccupancyMaxActiveClusters(&nc, k_sample, &cfg);
        if (r != cudaSuccess) return (int)r;
        clusters_ok = nc > 0;
    }
    if (!clusters_ok) return (int)cudaErrorInvalidClusterSize;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return (int)cudaLaunchKernelEx(&cfg, k_sample, a);
}

}  // namespace q35
