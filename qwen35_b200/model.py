"""Seeded synthetic weights and the batched engine, on top of libq35b's C
ABI (configs and the tensor plan: `configs.py`).

Weights are generated on the device from a seeded generator and packed by
the library's device encoders (`q35b_quantize_weight`): Q8_0 is the
reference's own weight quantizer, IQ4_NL / K-quants are deterministic
encoders of this library (the reference has none).
"""
import ctypes

import numpy as np
import torch

from . import lib as _lib
from .configs import CONFIGS, ModelConfig, synth_k, synth_key, synth_vector, tensor_plan  # noqa: F401
from .lib import GEOM, TT, check


def packed_bytes(tt, rows, cols):
    if tt == TT["F32"]:
        return rows * cols * 4
    e, b = GEOM[tt]
    return rows * (cols // e) * b


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class SyntheticModel:
    """Seeded synthetic weights, generated and packed on the GPU.

    gen="torch": torch's device generator (the test models).  gen="synth":
    the library's q35b_synth_fill for the linear weights and the host
    generator of `configs.synth_vector` for the f32 vectors; a CPU process
    rebuilds exactly these values from `configs` alone (the benchmark's
    reference arm decodes the same bytes)."""

    def __init__(self, cfg, seed=0, device="cuda", gen="torch"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.tensors = {}  # name -> (ttype, rows, cols, uint8/float32 device tensor)
        L = _lib.load()
        if gen == "synth":
            self._init_synth(L, seed)
            return
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

    def _init_synth(self, L, seed):
        for i, (name, role, tt, rows, cols, init) in enumerate(tensor_plan(self.cfg)):
            n = rows * cols
            key = synth_key(seed, i)
            if init == "w":
                f = torch.empty(n, dtype=torch.float32, device=self.device)
                check(L.q35b_synth_fill(key, n, synth_k(0.02), f.data_ptr(), _stream()), name)
                e, b = GEOM[tt]
                out = torch.empty(n // e * b, dtype=torch.uint8, device=self.device)
                check(L.q35b_quantize_weight(tt, f.data_ptr(), out.data_ptr(), n // e, _stream()), name)
                del f
            else:
                out = torch.from_numpy(synth_vector(key, n, init)).to(self.device)
            self.tensors[name] = (tt, rows, cols, out)
        torch.cuda.synchronize(self.device)

    def checksum(self):
        """sum of the packed bytes as little-endian 64-bit words, mod 2^64,
        over every tensor in plan order (padded to 8 bytes with zeros)"""
        acc = 0
        for name in self.tensors:
            t = self.tensors[name][3].reshape(-1).view(torch.uint8)
            pad = (-t.numel()) % 8
            if pad:
                t = torch.cat([t, torch.zeros(pad, dtype=torch.uint8, device=t.device)])
            acc = (acc + int(t.view(torch.int64).sum().item())) & (2**64 - 1)
        return acc

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

    def ipc_handles(self):
        """this rank's CUDA IPC handles for the peer all-reduce (bytes)"""
        buf = ctypes.create_string_buffer(192)
        check(self.L.q35b_engine_ipc_handles(self.h, ctypes.cast(buf, ctypes.c_void_p), 192), "ipc_handles")
        return buf.raw

    def set_peers(self, handles):
        """map every rank's buffers (handles: the ranks' ipc_handles() in
        rank order) and switch to the peer all-reduce"""
        raw = b"".join(handles)
        buf = ctypes.create_string_buffer(raw, len(raw))
        check(self.L.q35b_engine_set_peers(self.h, ctypes.cast(buf, ctypes.c_void_p), len(raw)), "set_peers")

    def set_allreduce(self, peer):
        check(self.L.q35b_engine_set_allreduce(self.h, 1 if peer else 0), "set_allreduce")

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

    def set_sampling(self, on):
        """device sampler (per-slot parameters) instead of the greedy argmax"""
        check(self.L.q35b_engine_set_sampling(self.h, 1 if on else 0), "set_sampling")

    def set_sampler(self, slot, temperature=0.0, top_k=0, top_p=0.0, seed=0):
        check(self.L.q35b_engine_set_sampler(self.h, slot, float(temperature), int(top_k), float(top_p),
                                             int(seed)), "set_sampler")

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
