"""ctypes bindings to the CPU oracle (oracle/_build/liboracle.so).

Test infrastructure: the oracle is the checker, never the thing measured or
shipped.  `load_oracle()` builds it with make when the .so is missing (gcc is
present on both this container and the GPU box).
"""
import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_SO = os.path.join(ORACLE_DIR, "_build", "liboracle.so")
REF_SO = os.path.join(ORACLE_DIR, "_ref", "libq35ref.so")

TT = {"F32": 0, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14,
      "Q8_K": 15, "IQ4_NL": 20, "IQ4_XS": 23}
GEOM = {8: (32, 34), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 20: (32, 18), 12: (256, 144),
        13: (256, 176), 14: (256, 210), 23: (256, 136)}

f32p = ctypes.POINTER(ctypes.c_float)
u8p = ctypes.POINTER(ctypes.c_uint8)
i32p = ctypes.POINTER(ctypes.c_int)


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("n_layers", "full_attention_interval", "hidden",
                                             "n_heads", "n_kv_heads", "head_dim", "n_ff", "vocab")] + \
               [("rms_eps", ctypes.c_float), ("rope_freq_base", ctypes.c_float)] + \
               [(n, ctypes.c_int) for n in ("gdn_n_heads", "gdn_num_k_heads", "gdn_head_dim",
                                             "conv_kernel")]


def _declare(lib):
    V, I, F = None, ctypes.c_int, ctypes.c_float
    sig = {
        "q35o_f16_to_f32": (F, [ctypes.c_uint16]),
        "q35o_f32_to_f16": (ctypes.c_uint16, [F]),
        "q35o_quantize_q8_0": (V, [I, f32p, u8p]),
        "q35o_quantize_q8_K": (V, [I, f32p, u8p]),
        "q35o_quantize_act": (V, [I, I, f32p, u8p]),
        "q35o_quantize_weight": (V, [I, I, f32p, u8p]),
        "q35o_synth_fill": (V, [ctypes.c_uint64, ctypes.c_longlong, F, f32p]),
        "q35o_dequant_row": (V, [I, u8p, f32p, I]),
        "q35o_vec_dot": (F, [I, I, u8p, u8p]),
        "q35o_block_isum": (ctypes.c_int32, [I, u8p, u8p]),
        "q35o_matvec_q": (V, [I, u8p, u8p, f32p, I, I, I]),
        "q35o_matvec_f32": (V, [f32p, f32p, f32p, I, I, I]),
        "q35o_matvec_w16": (V, [I, ctypes.c_void_p, f32p, f32p, I, I, I]),
        "q35o_matvec": (V, [I, u8p, f32p, f32p, I, I, I]),
        "q35o_rmsnorm": (V, [f32p, f32p, f32p, I, F]),
        "q35o_rmsnorm_rows": (V, [f32p, f32p, f32p, I, I, F]),
        "q35o_l2norm": (V, [f32p, I]),
        "q35o_l2norm_qk_scale": (V, [f32p, I, I, I, F]),
        "q35o_silu": (F, [F]),
        "q35o_sigmoid": (F, [F]),
        "q35o_softplus": (F, [F]),
        "q35o_softmax": (V, [f32p, I]),
        "q35o_swiglu": (V, [f32p, f32p, I]),
        "q35o_mul_silu": (V, [f32p, f32p, I]),
        "q35o_mul_sigmoid": (V, [f32p, f32p, I]),
        "q35o_rope64": (V, [f32p, I, F]),
        "q35o_rope64_rows": (V, [f32p, I, I, I, I, F]),
        "q35o_conv_step": (V, [f32p, f32p, f32p, I]),
        "q35o_gdn_gamma": (V, [f32p, f32p, f32p, f32p, f32p, I]),
        "q35o_gdn_fused": (V, [f32p, f32p, f32p, f32p, f32p, f32p, f32p, F, F, I, I]),
        "q35o_gdn_step_rows": (V, [f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, I, I, I, I]),
        "q35o_deinterleave_qg": (V, [f32p, f32p, f32p, I, I]),
        "q35o_attn_decode": (V, [f32p, f32p, f32p, f32p, f32p, f32p, I, I, I, I, I, F]),
        "q35o_argmax": (I, [f32p, I]),
        "q35o_sample": (I, [f32p, I, F, I, F, ctypes.POINTER(ctypes.c_uint64), f32p]),
        "q35o_kth_largest": (F, [f32p, I, I]),
        "q35o_model_create": (ctypes.c_void_p, [ctypes.POINTER(Config), I, I]),
        "q35o_model_destroy": (V, [ctypes.c_void_p]),
        "q35o_model_set_threads": (V, [ctypes.c_void_p, I]),
        "q35o_model_set_tensor": (I, [ctypes.c_void_p, ctypes.c_char_p, I, ctypes.c_void_p, I, I]),
        "q35o_model_check": (I, [ctypes.c_void_p]),
        "q35o_model_reset": (V, [ctypes.c_void_p]),
        "q35o_forward": (f32p, [ctypes.c_void_p, I, I]),
        "q35o_layer_out": (f32p, [ctypes.c_void_p, I]),
        "q35o_generate": (I, [ctypes.c_void_p, i32p, I, I, i32p]),
        "q35o_time_decode": (ctypes.c_double, [ctypes.c_void_p, I, I, I, i32p]),
        "q35o_kernel_tier": (ctypes.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None
_LIB_CR = None


def load_oracle(cr_exp=False):
    """The oracle library; cr_exp: the build with correctly rounded exp /
    log1p (the device's arithmetic) instead of the C library's expf / log1pf"""
    global _LIB, _LIB_CR
    if cr_exp:
        if _LIB_CR is None:
            so = os.path.join(ORACLE_DIR, "_build", "liboracle_crexp.so")
            if not os.path.exists(so):
                subprocess.run(["make", "-C", ORACLE_DIR], check=True, capture_output=True)
            _LIB_CR = _declare(ctypes.CDLL(so))
        return _LIB_CR
    if _LIB is None:
        if not os.path.exists(ORACLE_SO):
            subprocess.run(["make", "-C", ORACLE_DIR], check=True, capture_output=True)
        _LIB = _declare(ctypes.CDLL(ORACLE_SO))
    return _LIB


def load_ref():
    """The reference's own x86 kernels (built only where the reference tree
    exists); None when absent."""
    if not os.path.exists(REF_SO):
        return None
    return _declare(ctypes.CDLL(REF_SO))


def fp(a):
    return a.ctypes.data_as(f32p)


def bp(a):
    return a.ctypes.data_as(u8p)


def ip(a):
    return a.ctypes.data_as(i32p)


def row_bytes(tt, cols):
    e, b = GEOM[tt]
    return cols // e * b


def act_row_bytes(tt, cols):
    e, _ = GEOM[tt]
    return cols // 32 * 34 if e == 32 else cols // 256 * 292


def quantize_weight(lib, tt, w):
    """w: [rows, cols] f32 -> packed bytes [rows, row_bytes]"""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    out = np.zeros((rows, row_bytes(tt, cols)), dtype=np.uint8)
    lib.q35o_quantize_weight(tt, rows * cols, fp(w), bp(out))
    return out


def quantize_act(lib, tt, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None]
    t, cols = x.shape
    out = np.zeros((t, act_row_bytes(tt, cols)), dtype=np.uint8)
    for i in range(t):
        lib.q35o_quantize_act(tt, cols, fp(x[i]), bp(out[i]))
    return out


def dequant(lib, tt, wq, cols):
    rows = wq.shape[0]
    out = np.zeros((rows, cols), dtype=np.float32)
    for r in range(rows):
        lib.q35o_dequant_row(tt, bp(np.ascontiguousarray(wq[r])), fp(out[r]), cols)
    return out


def matvec_q(lib, tt, wq, xq, rows, cols, tokens):
    out = np.zeros((tokens, rows), dtype=np.float32)
    lib.q35o_matvec_q(tt, bp(np.ascontiguousarray(wq)), bp(np.ascontiguousarray(xq)), fp(out),
                      rows, cols, tokens)
    return out


def oracle_model(synth, threads=1, max_seq=512, cr_exp=False):
    """CPU oracle engine over the exact packed bytes of a SyntheticModel
    (copied device -> host).  Returns (lib, handle, keepalive)."""
    lib = load_oracle(cr_exp)
    c = synth.cfg
    cfg = Config(c.n_layers, c.full_attention_interval, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim, c.n_ff,
                 c.vocab, c.rms_eps, c.rope_freq_base, c.gdn_n_heads, c.gdn_num_k_heads, c.gdn_head_dim,
                 c.conv_kernel)
    m = lib.q35o_model_create(ctypes.byref(cfg), max_seq, threads)
    keep = []
    for name in synth.tensors:
        tt, rows, cols, arr = synth.host(name)
        arr = np.ascontiguousarray(arr)
        keep.append(arr)
        rc = lib.q35o_model_set_tensor(m, name.encode(), tt, arr.ctypes.data, rows, cols)
        assert rc == 0, name
    assert lib.q35o_model_check(m) == 0
    return lib, m, keep


def oracle_forward(lib, m, token, pos, vocab):
    p = lib.q35o_forward(m, token, pos)
    return np.ctypeslib.as_array(p, shape=(vocab,)).copy()


def oracle_layer_out(lib, m, li, hidden):
    p = lib.q35o_layer_out(m, li)
    return np.ctypeslib.as_array(p, shape=(hidden,)).copy()


class OracleSampler:
    """Sampler.sample (src/sampler.zig) through the oracle: the PRNG state
    lives here, as in the reference's Sampler struct"""

    def __init__(self, lib, temperature=0.0, top_k=0, top_p=0.0, seed=0):
        self.lib, self.t, self.k, self.p = lib, float(temperature), int(top_k), float(top_p)
        self.state = ctypes.c_uint64(seed if seed else 0x9E3779B97F4A7C15)

    def sample(self, logits):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        scratch = np.empty(max(1, x.size), np.float32)
        return int(self.lib.q35o_sample(fp(x), x.size, self.t, self.k, self.p, ctypes.byref(self.state),
                                        fp(scratch)))
