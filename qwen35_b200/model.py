"""Qwen3.5 hybrid model configs, seeded synthetic weights and the batched
engine, on top of libq35b's C ABI.

Tensor names and shapes follow the GGUF layout the reference engine loads
(src/engine.zig:826-993): linear weights are [rows = out, cols = in],
`blk.N.ssm_conv1d.weight` is [conv_dim, 4] f32, norms are pre-folded (1 + w).
Weights are generated on the device from a seeded generator and packed by
the library's device encoders (`q35b_quantize_weight`): Q8_0 is the
reference's own weight quantizer, IQ4_NL / K-quants are deterministic
encoders of this library (the reference has none).
"""
import ctypes
import dataclasses

import torch

from . import lib as _lib
from .lib import GEOM, TT, check


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


def packed_bytes(tt, rows, cols):
    if tt == TT["F32"]:
        return rows * cols * 4
    e, b = GEOM[tt]
    return rows * (cols // e) * b


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class SyntheticModel:
    """Seeded synthetic weights, generated and packed on the GPU."""

    def __init__(self, cfg, seed=0, device="cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.tensors = {}  # name -> (ttype, rows, cols, uint8/float32 device tensor)
        L = _lib.load()
        gen = torch.Generator(device=self.device)
        for i, (name, role, tt, rows, cols, init) in enumerate(tensor_plan(cfg)):
            gen.manual_seed(seed * 1000003 + i)
            n = rows * cols
            if init == "w":
                f = torch.randn(n, generator=gen, device=self.device, dtype=torch.float32) * 0.02
                e, b = GEOM[tt]
                out = torch.empty(n // e * b, dtype=torch.uint8, device=self.device)
                check(L.q35b_quantize_weight(tt, f.data_ptr(), out.data_ptr(), n // e, _stream()), name)
                del f
            elif init == "norm":
                out = 1.0 + 0.02 * torch.randn(n, generator=gen, device=self.device)
            elif init == "conv":
                out = 0.5 * torch.randn(n, generator=gen, device=self.device)
            elif init == "dt":
                out = 0.5 * torch.randn(n, generator=gen, device=self.device)
            elif init == "ssm_a":
                out = -torch.exp(torch.rand(n, generator=gen, device=self.device) * 2.0 - 1.0)
            else:
                raise ValueError(init)
            self.tensors[name] = (tt, rows, cols, out)
        torch.cuda.synchronize(self.device)

    def weight_bytes(self):
        return sum(t.numel() * t.element_size() for (_, _, _, t) in self.tensors.values())

    def host(self, name):
        tt, rows, cols, t = self.tensors[name]
        return tt, rows, cols, t.cpu().numpy()


class Engine:
    """Batched decode engine (q35b_engine) over a SyntheticModel."""

    def __init__(self, model, n_slots, max_seq, max_batch, tp_id=None):
        """model: a SyntheticModel, or a tp.ShardModel (then `tp_id`, the
        NCCL id of q35b_tp_unique_id shared by all ranks, is required and every
        rank constructs its engine at the same time)"""
        self.L = _lib.load()
        self.model = model
        self.cfg = model.cfg
        self.max_batch = max_batch
        self.n_slots = n_slots
        self.max_seq = max_seq
        cc = self.cfg.c_config()
        h = ctypes.c_void_p()
        check(self.L.q35b_engine_create(ctypes.addressof(cc), n_slots, max_seq, max_batch, ctypes.byref(h)), "create")
        self.h = h
        if getattr(model, "P", 1) > 1:
            if tp_id is None:
                raise ValueError("a tensor-parallel shard needs the NCCL id")
            idbuf = ctypes.create_string_buffer(bytes(tp_id), len(tp_id))
            check(self.L.q35b_engine_set_tp(h, model.P, model.p, model.vocab_local, model.vocab_offset,
                                            ctypes.cast(idbuf, ctypes.c_void_p)), "set_tp")
        for name, (tt, rows, cols, t) in model.tensors.items():
            check(self.L.q35b_engine_set_tensor(h, name.encode(), tt, t.data_ptr(), rows, cols), name)
        check(self.L.q35b_engine_finalize(h), "finalize")
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        check(self.L.q35b_engine_device_inputs(h, *[ctypes.byref(p) for p in ptrs]), "device_inputs")
        self.d_tokens, self.d_slots, self.d_pos, self.d_next = [p.value for p in ptrs]

    def close(self):
        if self.h:
            self.L.q35b_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset_slot(self, slot, stream=None):
        check(self.L.q35b_engine_reset_slot(self.h, slot, _stream(stream)), "reset_slot")

    def step_host(self, tokens, slots, pos, stream=None):
        n = len(tokens)
        arr = ctypes.c_int * n
        t, s, p, nx = arr(*tokens), arr(*slots), arr(*pos), arr()
        check(self.L.q35b_engine_step_host(self.h, n, t, s, p, nx, _stream(stream)), "step_host")
        return list(nx)

    def forward(self, tokens, slots, pos, run_end, stream=None):
        """one forward over runs (q35b_engine_forward); returns the next token
        of every run"""
        n, nrun = len(tokens), len(run_end)
        arr = ctypes.c_int * n
        nx = (ctypes.c_int * nrun)()
        check(self.L.q35b_engine_forward(self.h, n, arr(*tokens), arr(*slots), arr(*pos), nrun,
                                         (ctypes.c_int * nrun)(*run_end), nx, _stream(stream)), "forward")
        return list(nx)

    def set_prefill_wy(self, on):
        check(self.L.q35b_engine_set_prefill_wy(self.h, 1 if on else 0), "set_prefill_wy")

    def prefill(self, slot, tokens, pos0=0, stream=None):
        """prompt prefill of one slot (q35b_engine_prefill); returns the greedy
        token after the last prompt token"""
        nx = ctypes.c_int(0)
        check(self.L.q35b_engine_prefill(self.h, slot, (ctypes.c_int * len(tokens))(*tokens), len(tokens), pos0,
                                         ctypes.byref(nx), _stream(stream)), "prefill")
        return nx.value

    def step(self, d_tokens, d_slots, d_pos, d_next, d_logits=None, use_graph=True, stream=None):
        """device int32 tensors (n,) -> writes d_next (and d_logits n x vocab)"""
        n = d_tokens.numel()
        check(self.L.q35b_engine_step(self.h, n, d_tokens.data_ptr(), d_slots.data_ptr(), d_pos.data_ptr(),
                                      d_next.data_ptr() if d_next is not None else None,
                                      d_logits.data_ptr() if d_logits is not None else None,
                                      1 if use_graph else 0, _stream(stream)), "step")

    def set_probe(self, on):
        check(self.L.q35b_engine_set_probe(self.h, 1 if on else 0), "set_probe")

    def layer_out(self, li, n):
        """residual stream after layer li for the last step (probe on), (n, hidden)"""
        p = self.L.q35b_engine_layer_out(self.h, li)
        if not p:
            return None
        torch.cuda.synchronize()
        return device_view(p, n * self.cfg.hidden, torch.float32).view(n, self.cfg.hidden).clone()

    def serve(self, prompts, n_gen, max_batch=None, stream=None):
        """continuous batching: prompts list[list[int]], n_gen list[int] ->
        (list[list[int]] generated, steps)"""
        nseq = len(prompts)
        flat = [t for p in prompts for t in p]
        offs, o = [], 0
        for p in prompts:
            offs.append(o)
            o += len(p)
        ooffs, oo = [], 0
        for g in n_gen:
            ooffs.append(oo)
            oo += g
        I = ctypes.c_int
        LL = ctypes.c_longlong
        c_prompts = (I * max(1, len(flat)))(*flat)
        c_poff = (LL * nseq)(*offs)
        c_plen = (I * nseq)(*[len(p) for p in prompts])
        c_ngen = (I * nseq)(*n_gen)
        c_out = (I * max(1, oo))()
        c_ooff = (LL * nseq)(*ooffs)
        steps = LL()
        check(self.L.q35b_serve(self.h, nseq, c_prompts, c_poff, c_plen, c_ngen, c_out, c_ooff,
                                max_batch or self.max_batch, ctypes.byref(steps), _stream(stream)), "serve")
        res = [list(c_out[ooffs[i]:ooffs[i] + n_gen[i]]) for i in range(nseq)]
        return res, steps.value


class _CudaArray:
    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def device_view(ptr, n, dtype=torch.float32):
    """zero-copy torch view of library-owned device memory"""
    ts = {torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, n, ts), device="cuda")
