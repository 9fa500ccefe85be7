"""Qwen3.5 hybrid model configs, the GGUF tensor plan and the seeded
synthetic-value generator, with no dependency on torch or on libq35b.

Tensor names and shapes follow the GGUF layout the reference engine loads
(src/engine.zig:826-993): linear weights are [rows = out, cols = in],
`blk.N.ssm_conv1d.weight` is [conv_dim, 4] f32, norms are pre-folded (1 + w).

The synthetic generator (`synth_key`, `synth_k`, `synth_vector`) is the
host-side statement of the library's `q35b_synth_fill`: a CPU process (the
reference arm of the benchmark) builds the same weight values from it that
the GPU run builds on the device, so both decode identical bytes.
"""
import dataclasses

import numpy as np

from . import lib as _lib
from .lib import TT


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    n_layers: int
    hidden: int
    n_ff: int
    vocab: int
    n_heads: int
    n_kv_heads: int
    gdn_n_heads: int
    gdn_num_k_heads: int
    head_dim: int = 256
    gdn_head_dim: int = 128
    full_attention_interval: int = 4
    rms_eps: float = 1e-6
    rope_freq_base: float = 1e7
    conv_kernel: int = 4
    # weight type per role
    quant: tuple = ()

    def qtype(self, role):
        d = dict(self.quant)
        return TT[d.get(role, d.get("bulk", "Q8_0"))]

    def is_full(self, li):
        f = self.full_attention_interval
        return f > 0 and li % f == f - 1

    @property
    def conv_dim(self):
        return 2 * self.gdn_num_k_heads * self.gdn_head_dim + self.gdn_n_heads * self.gdn_head_dim

    def c_config(self):
        return _lib.Config(self.n_layers, self.full_attention_interval, self.hidden, self.n_heads, self.n_kv_heads,
                           self.head_dim, self.n_ff, self.vocab, self.rms_eps, self.rope_freq_base,
                           self.gdn_n_heads, self.gdn_num_k_heads, self.gdn_head_dim, self.conv_kernel)


# 0.8B (all Q8_0), 4B (mixed), 27B (Q4_K, Q6_K output)
CONFIGS = {
    "0.8b": ModelConfig("qwen3.5-0.8b-q8_0", 24, 1024, 3584, 248320, 8, 2, 16, 16,
                        quant=(("bulk", "Q8_0"),)),
    "4b": ModelConfig("qwen3.5-4b-mixed", 32, 2560, 9216, 248320, 16, 4, 32, 16,
                      quant=(("bulk", "IQ4_NL"), ("ffn_down", "Q5_K"), ("ssm_alpha", "Q8_0"),
                             ("ssm_beta", "Q8_0"), ("output", "Q6_K"))),
    "27b": ModelConfig("qwen3.5-27b-q4_k", 64, 5120, 17408, 248320, 24, 4, 48, 16,
                       quant=(("bulk", "Q4_K"), ("output", "Q6_K"))),
    # small shapes for parity tests (same head sizes, fewer/narrower layers)
    "tiny": ModelConfig("tiny-q8_0", 4, 256, 512, 2048, 2, 1, 2, 2, quant=(("bulk", "Q8_0"),)),
    "tiny-mixed": ModelConfig("tiny-mixed", 8, 512, 1024, 4096, 4, 1, 4, 2,
                              quant=(("bulk", "IQ4_NL"), ("ffn_down", "Q5_K"), ("ssm_alpha", "Q8_0"),
                                     ("ssm_beta", "Q8_0"), ("output", "Q6_K"), ("attn_output", "Q4_K"))),
    # tensor-parallel parity cases: every head count splits two ways
    "tiny-tp": ModelConfig("tiny-tp-q8_0", 4, 256, 1024, 2048, 4, 2, 4, 2, quant=(("bulk", "Q8_0"),)),
    "tiny-tp-mixed": ModelConfig("tiny-tp-mixed", 4, 512, 1024, 4096, 4, 2, 8, 4,
                                 quant=(("bulk", "IQ4_NL"), ("ffn_down", "Q5_K"), ("ssm_alpha", "Q8_0"),
                                        ("ssm_beta", "Q8_0"), ("output", "Q6_K"), ("attn_output", "Q4_K"))),
    # the 27B TP-8 shapes in small: one kv head replicated on both ranks, an
    # odd count of ffn blocks (3 -> 2 + 1), Q4_K bulk with a Q6_K lm_head
    # (GDN value heads in pairs: ssm_out columns in whole 256-blocks)
    # the legacy 32-element families (Q4_0 / Q4_1 / Q5_0 / Q5_1) in one model
    "tiny-legacy": ModelConfig("tiny-legacy", 8, 512, 1024, 4096, 4, 1, 4, 2,
                               quant=(("bulk", "Q4_0"), ("attn_qkv", "Q5_0"), ("ffn_down", "Q5_1"),
                                      ("ffn_up", "Q4_1"), ("attn_output", "Q5_1"), ("output", "Q4_1"))),
    # the 27B layer shapes (hidden 5120, ffn 17408, 24 q / 4 kv heads, 48 GDN
    # value heads over 16 k heads, Q4_K with a Q6_K lm_head) in 4 layers
    # (3 GDN + 1 attention) and a 32768-entry vocab: TP parity against the
    # oracle at the shapes the 27B benchmark splits
    "27b-4l": ModelConfig("qwen3.5-27b-shape-4layer", 4, 5120, 17408, 32768, 24, 4, 48, 16,
                          quant=(("bulk", "Q4_K"), ("output", "Q6_K"))),
    "tiny-tp-rep": ModelConfig("tiny-tp-rep", 4, 512, 768, 4096, 4, 1, 8, 4,
                               quant=(("bulk", "Q4_K"), ("output", "Q6_K"))),
}


def tensor_plan(cfg):
    """[(name, role, ttype, rows, cols, init)] in GGUF naming.  init is one of
    'w' (N(0, 0.02)), 'norm' (1 + N(0, 0.02)), 'conv', 'ssm_a', 'dt'."""
    h, nv, kd = cfg.hidden, cfg.gdn_n_heads, cfg.gdn_head_dim
    q_dim, kv_dim = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    P = []

    def lin(name, role, rows, cols):
        P.append((name, role, cfg.qtype(role), rows, cols, "w"))

    def vec(name, n, init):
        P.append((name, init, TT["F32"], 1, n, init))

    lin("token_embd.weight", "token_embd", cfg.vocab, h)
    if "output" in dict(cfg.quant):
        lin("output.weight", "output", cfg.vocab, h)
    vec("output_norm.weight", h, "norm")
    for li in range(cfg.n_layers):
        b = f"blk.{li}."
        vec(b + "attn_norm.weight", h, "norm")
        vec(b + "post_attention_norm.weight", h, "norm")
        if cfg.is_full(li):
            lin(b + "attn_q.weight", "attn_q", 2 * q_dim, h)
            lin(b + "attn_k.weight", "attn_k", kv_dim, h)
            lin(b + "attn_v.weight", "attn_v", kv_dim, h)
            lin(b + "attn_output.weight", "attn_output", h, q_dim)
            vec(b + "attn_q_norm.weight", cfg.head_dim, "norm")
            vec(b + "attn_k_norm.weight", cfg.head_dim, "norm")
        else:
            lin(b + "attn_qkv.weight", "attn_qkv", cfg.conv_dim, h)
            lin(b + "attn_gate.weight", "attn_gate", nv * kd, h)
            lin(b + "ssm_alpha.weight", "ssm_alpha", nv, h)
            lin(b + "ssm_beta.weight", "ssm_beta", nv, h)
            lin(b + "ssm_out.weight", "ssm_out", h, nv * kd)
            vec(b + "ssm_conv1d.weight", cfg.conv_dim * 4, "conv")
            vec(b + "ssm_dt.bias", nv, "dt")
            vec(b + "ssm_a", nv, "ssm_a")
            vec(b + "ssm_norm.weight", kd, "norm")
        lin(b + "ffn_gate.weight", "ffn_gate", cfg.n_ff, h)
        lin(b + "ffn_up.weight", "ffn_up", cfg.n_ff, h)
        lin(b + "ffn_down.weight", "ffn_down", h, cfg.n_ff)
    return P


# ---------------------------------------------------------------------------
# seeded synthetic values (q35b_synth_fill, restated in numpy for vectors)
# ---------------------------------------------------------------------------
SYNTH_STD = np.float32(37837.227)  # standard deviation of four summed 16-bit uniforms
SIGMA = {"w": 0.02, "norm": 0.02, "conv": 0.5, "dt": 0.5}


def synth_key(seed, index):
    """stream key of tensor `index` of the plan"""
    return (int(seed) * 1000003 + int(index)) & (2**64 - 1)


def synth_k(sigma):
    """f32 multiplier that maps the centred Irwin-Hall sum to N(0, sigma^2)"""
    return float(np.float32(sigma) / SYNTH_STD)


def synth_hash_np(key, n):
    """splitmix64 finalizer over key * 0x9E37.. + i * 0xD1B5.. (uint64, wrapping)"""
    i = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(key) * np.uint64(0x9E3779B97F4A7C15) + i * np.uint64(0xD1B54A32D192ED03)
        z ^= z >> np.uint64(30)
        z *= np.uint64(0xBF58476D1CE4E5B9)
        z ^= z >> np.uint64(27)
        z *= np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    return z


def synth_normal_np(key, n, sigma):
    """the values q35b_synth_fill(key, n, synth_k(sigma)) writes"""
    z = synth_hash_np(key, n)
    m = np.uint64(0xFFFF)
    s = ((z & m) + ((z >> np.uint64(16)) & m) + ((z >> np.uint64(32)) & m) + (z >> np.uint64(48))).astype(np.int64)
    return (s - 131070).astype(np.float32) * np.float32(synth_k(sigma))


def synth_vector(key, n, init):
    """f32 vector tensors of the plan (norm / conv / dt / ssm_a), on the host"""
    if init == "norm":
        return np.float32(1.0) + synth_normal_np(key, n, SIGMA["norm"])
    if init in ("conv", "dt"):
        return synth_normal_np(key, n, SIGMA[init])
    if init == "ssm_a":
        u = (synth_hash_np(key, n) >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)
        return -np.exp(u * np.float32(2.0) - np.float32(1.0))
    raise ValueError(init)
