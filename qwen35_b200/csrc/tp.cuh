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

}  // namespace q35
