// tp.cuh -- tensor-parallel collectives of the engine (NCCL over NVLink).
//
// A TP rank runs the ordinary engine on its shard (head / ffn / vocab slices,
// see qwen35_b200/tp.py).  Two exchanges per decode step and layer pair:
//   * after each row-parallel projection (attn_output, ssm_out, ffn_down) the
//     partial [n][hidden] sums are all-reduced, then added to the residual
//     stream, which every rank holds whole and identical;
//   * the lm_head's rank-local (max, index) pairs are all-gathered and the
//     global greedy token is the largest value, ties to the smaller index
//     (the first maximum, as the single-GPU argmax).
// NCCL is loaded at run time (dlopen "libnccl.so.2"): in a process that has
// already initialised torch.distributed this resolves to the same library
// instance, so the library neither links nor ships a second NCCL.
//
// The row-parallel all-reduce has a second form that replaces the NCCL call
// and the residual add with one kernel over NVLink peer memory
// (k_tp_allreduce_add): every rank's partial-sum, residual and flag buffers
// are mapped into every rank (CUDA IPC), rank q owns hidden columns
// [q h/N, (q+1) h/N) of every token, pulls that slice of all N partials with
// plain peer loads, sums them in rank order (so every rank computes the same
// bits), adds the residual and stores the result into every rank's residual
// with plain peer stores.  Epoch flags (release / acquire at system scope)
// order the two exchanges; every wait is bounded and records an error code
// instead of hanging.
#pragma once
#include <dlfcn.h>
#include <nccl.h>

#include "common.cuh"

namespace q35 {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    bool ok = false;
};

inline NcclApi &nccl_api() {
    static NcclApi a;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
            a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
            a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
            a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
            a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
            a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.all_gather && a.comm_destroy;
        }
    }
    return a;
}

// x[i] += part[i] (the all-reduced row-parallel output into the residual)
__global__ void k_add_rows(float *x, const float *part, long long n) {
    pdl_trigger();
    pdl_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], part[i]);
}

// per row: (max value bits, first index of the max + offset) of n logits
__global__ void __launch_bounds__(1024) k_argmax_pair(const float *x, long long row_stride, int n, int offset,
                                                      int *pair) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *xr = x + (long long)blockIdx.x * row_stride;
    float bv = -INFINITY;
    int bi = n;
    for (int i = threadIdx.x; i < n; i += 1024) {
        const float v = xr[i];
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 32; w++)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
                bv = sv[w];
                bi = si[w];
            }
        pair[2 * blockIdx.x] = __float_as_int(bv);
        pair[2 * blockIdx.x + 1] = (bi >= n ? 0 : bi) + offset;
    }
}

// all[p][r][2] from every rank -> out[r]: the largest value, ties to the
// smaller (global) index
__global__ void k_argmax_combine(const int *all, int nrun, int nranks, int *out) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= nrun) return;
    float bv = __int_as_float(all[2 * r]);
    int bi = all[2 * r + 1];
    for (int p = 1; p < nranks; p++) {
        const float v = __int_as_float(all[((long long)p * nrun + r) * 2]);
        const int i = all[((long long)p * nrun + r) * 2 + 1];
        if (v > bv || (v == bv && i < bi)) {
            bv = v;
            bi = i;
        }
    }
    out[r] = bi;
}

// ---------------------------------------------------------------------------
// peer all-reduce + residual add (see the header)
// ---------------------------------------------------------------------------
constexpr int TP_MAX = 8;
constexpr int TP_FLAG_WORDS = 2 * TP_MAX;  // per rank: ready[TP_MAX], done[TP_MAX]

struct TpPeers {
    float *part[TP_MAX];  // every rank's partial sums [n][hidden] (this rank's own included)
    float *x[TP_MAX];     // every rank's residual stream [n][hidden]
    int *flags[TP_MAX];   // every rank's flag words
};

struct TpArArgs {
    TpPeers pe;
    int *state;                    // this rank: [0] epoch (calls completed), [1] CTA arrivals
    int rank, nranks, hidden, n;
    unsigned long long limit_ns;   // bound of every wait
};

Q35_DEV void st_release_sys(int *p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
Q35_DEV int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// wait until flags[0..n) all reach `target`; false (error recorded) past the limit
Q35_DEV bool tp_wait_all(const int *flags, int n, int target, unsigned long long limit_ns, int site) {
    const uint64_t t0 = globaltimer();
    for (int p = 0; p < n; p++) {
        while (ld_acquire_sys(flags + p) < target) {
            if (globaltimer() - t0 > limit_ns) {
                set_error(site);
                return false;
            }
            __nanosleep(100);
        }
    }
    return true;
}

Q35_DEV float4 f4_add(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// x[t][c] += sum over ranks p (in order) of part_p[t][c], on every rank.
// 1. once this rank's partials are complete (the dependency wait), raise
//    ready[rank] on every rank, then wait for every rank's ready;
// 2. for the owned columns, read the N partials (peer loads), sum them in
//    rank order, add the residual and store the result into every rank's
//    residual (peer stores);
// 3. the last CTA to finish raises done[rank] on every rank and waits for
//    every rank's done: past it, no rank reads this rank's partials any more
//    and every rank's share of this rank's residual has landed.
__global__ void __launch_bounds__(256) k_tp_allreduce_add(const __grid_constant__ TpArArgs a) {
    pdl_wait();
    __shared__ int s_ok;
    const int target = a.state[0] + 1;  // read by every CTA before any arrives below
    const int *my = a.pe.flags[a.rank];
    if (blockIdx.x == 0 && (int)threadIdx.x < a.nranks) {
        __threadfence_system();
        st_release_sys(a.pe.flags[threadIdx.x] + a.rank, target);
    }
    if (threadIdx.x == 0) s_ok = tp_wait_all(my, a.nranks, target, a.limit_ns, 150) ? 1 : 0;
    __syncthreads();
    const int hs4 = a.hidden / a.nranks / 4, c0 = a.rank * (a.hidden / a.nranks);
    const long long items = (long long)a.n * hs4;
    if (s_ok) {
        for (long long i = blockIdx.x * 256LL + threadIdx.x; i < items; i += (long long)gridDim.x * 256) {
            const int t = (int)(i / hs4), j = c0 + 4 * (int)(i - (long long)t * hs4);
            const long long off = (long long)t * a.hidden + j;
            float4 s = __ldcg(reinterpret_cast<const float4 *>(a.pe.part[0] + off));
            for (int p = 1; p < a.nranks; p++) s = f4_add(s, __ldcg(reinterpret_cast<const float4 *>(a.pe.part[p] + off)));
            const float4 xv = f4_add(__ldcg(reinterpret_cast<const float4 *>(a.pe.x[a.rank] + off)), s);
            for (int p = 0; p < a.nranks; p++) __stcg(reinterpret_cast<float4 *>(a.pe.x[p] + off), xv);
        }
    }
    __threadfence_system();
    __syncthreads();
    pdl_trigger();
    if (threadIdx.x == 0) {
        if (atomicAdd(a.state + 1, 1) == (int)gridDim.x - 1) {
            __threadfence_system();
            a.state[1] = 0;
            a.state[0] = target;
            for (int p = 0; p < a.nranks; p++) st_release_sys(a.pe.flags[p] + TP_MAX + a.rank, target);
            tp_wait_all(my + TP_MAX, a.nranks, target, a.limit_ns, 151);
        }
    }
}

inline int tp_ar_launch(const TpArArgs &a, cudaStream_t st) {
    if (a.n <= 0) return 0;
    const long long items = (long long)a.n * (a.hidden / a.nranks / 4);
    const int grid = (int)std::min<long long>(std::max<long long>((items + 255) / 256, 1), 64);
    return launch_k(k_tp_allreduce_add, dim3((unsigned)grid), dim3(256), 0, st, a);
}

}  // namespace q35
