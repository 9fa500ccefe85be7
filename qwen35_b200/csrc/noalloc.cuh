// noalloc.cuh -- split-KV decode attention whose partials live in a fixed
// device array, so the call allocates no device memory.
//
// Who needs it: a host that sizes its weights and KV slots to fill HBM at
// start-up has no room left for a per-call partials buffer, and a decode loop
// that is latency-bound cannot afford cudaMalloc / cudaFree (both may
// synchronize the device).  The reference's split-KV entry points take a
// caller-allocated partials buffer; this backend's q35_launch_attn_decode_split2
// ignores that buffer and runs a single split.  This entry point is the
// split-KV path that needs no buffer from the caller.
//
// The scratch is one file-scope array per device, NA_MAX_HEADS query heads x
// NA_MAX_SPLITS splits of (256 partial sums + max + sum) floats, 4.2 MB.
// Its address is looked up once per device with that device current (the
// first call on a device does this set-up; a caller that captures streams
// makes that first call before capturing).  Every call on a device shares the
// array and leaves its partials there; nothing in it has to start at zero,
// because the merge reads only partials the same call's split kernel wrote
// first.  Two calls that can run at the same time on one device (unordered
// streams, or host threads on different streams) race on the array: order
// them on one stream or with events.
#pragma once
#include <algorithm>
#include <mutex>

#include "attn.cuh"
#include "api.cuh"

namespace q35 {

constexpr int NA_MAX_HEADS = 64;
constexpr int NA_MAX_SPLITS = 64;
constexpr int NA_MAX_DEVICES = 64;
constexpr long long NA_ACC_FLOATS = (long long)NA_MAX_HEADS * NA_MAX_SPLITS * ATT_HD;
constexpr long long NA_ML_FLOATS = (long long)NA_MAX_HEADS * NA_MAX_SPLITS * 2;

static __device__ __align__(256) float g_na_scratch[NA_ACC_FLOATS + NA_ML_FLOATS];

static float *g_na_ptr[NA_MAX_DEVICES];
static std::mutex g_na_mu;

static int na_scratch(float **out) {
    int dev = -1;
    int rc = (int)cudaGetDevice(&dev);
    if (rc) return rc;
    if (dev < 0 || dev >= NA_MAX_DEVICES) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_na_mu);
    if (!g_na_ptr[dev]) {
        void *p = nullptr;
        rc = (int)cudaGetSymbolAddress(&p, g_na_scratch);
        if (rc) return rc;
        g_na_ptr[dev] = static_cast<float *>(p);
    }
    *out = g_na_ptr[dev];
    return 0;
}

}  // namespace q35

extern "C" {

// Same arguments and result as q35_launch_attn_decode (minus the unused
// score buffer): out = softmax(q . K[0..slot] * scale) V * sigmoid(gate).
// The context is cut into at most NA_MAX_SPLITS equal ranges of whole 32-
// position groups, so long contexts spread over many CTAs.
int q35b_attn_decode_noalloc(const float *d_q, const float *d_gate, const float *d_kcache, const float *d_vcache,
                             float *d_gout, int slot, int heads, int gqa, int hd, int kv_dim, float scale,
                             void *stream) {
    using namespace q35;
    if (heads <= 0) return 0;
    if (slot < 0 || hd != ATT_HD || gqa <= 0 || heads % gqa) return (int)cudaErrorInvalidValue;
    if (heads > NA_MAX_HEADS) return (int)cudaErrorInvalidValue;
    float *scratch = nullptr;
    int rc = na_scratch(&scratch);
    if (rc) return rc;
    const int len = slot + 1;
    const int groups = (len + 31) / 32;
    const int nsplit = std::min(NA_MAX_SPLITS, (len + ATT_SPLIT - 1) / ATT_SPLIT);
    const int split_len = 32 * ((groups + nsplit - 1) / nsplit);
    AttnArgs a{};
    a.q = d_q;
    a.gate = d_gate;
    a.q_tok = (long long)heads * hd;
    a.kc = d_kcache;
    a.vc = d_vcache;
    a.kv_slot = 0;
    a.kv_dim = kv_dim;
    a.len_imm = len;
    a.out = d_gout;
    a.out_tok = (long long)heads * hd;
    a.part_acc = scratch;
    a.part_ml = scratch + NA_ACC_FLOATS;
    a.nsplit = (len + split_len - 1) / split_len;
    a.split_len = split_len;
    a.heads = heads;
    a.kv_heads = heads / gqa;
    a.scale = scale;
    return attn_launch(a, 1, len, S(stream));
}

}  // extern "C"
