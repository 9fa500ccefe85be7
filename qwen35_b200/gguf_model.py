"""GGUF checkpoints for the engine.

`GGUFModel(path)` reads a Qwen3.5 GGUF file the way the reference's loader
does (src/engine.zig:810-993 over src/gguf.zig): the model configuration from
the `qwen35.*` metadata keys, the decoder's tensors by their GGUF names, the
packed quantized blocks uploaded exactly as stored.  There are no value
transforms: the GGUF already holds the RMSNorm weights folded (1 + w), ssm_a
as -exp(A_log) and the conv taps channel-major, which is what the engine
applies (src/engine.zig:10-22).  Trailing next-token-prediction layers
(`qwen35.nextn_predict_layers`) are not part of the decoder and are skipped,
as in the reference.  The result plugs into `Engine(model, ...)` like a
`SyntheticModel`.

`write_gguf(model, path)` writes a model's tensors and configuration in the
same layout (used to round-trip the synthetic models through the loader).
"""
import collections
import dataclasses
import warnings

import numpy as np
import torch

from .model import TT, ModelConfig, tensor_plan

ARCH = "qwen35"
LINEAR_TYPES = {TT["Q8_0"], TT["IQ4_NL"], TT["Q4_K"], TT["Q5_K"], TT["Q6_K"], TT["Q4_0"], TT["Q4_1"], TT["Q5_0"],
                TT["Q5_1"]}
F16, BF16 = 1, 30


def _get(reader, key):
    f = reader.fields.get(key)
    if f is None:
        return None
    v = f.contents()
    return v


def read_config(reader):
    """ModelConfig from the file's metadata (src/engine.zig:820-868)"""
    g = lambda k: _get(reader, f"{ARCH}.{k}")  # noqa: E731
    cfg = dict(n_layers=0, hidden=0, n_ff=0, vocab=0, n_heads=0, n_kv_heads=0, gdn_n_heads=0, gdn_num_k_heads=0)
    if g("block_count") is not None:
        cfg["n_layers"] = int(g("block_count"))
        nextn = g("nextn_predict_layers")
        if nextn is not None and 0 < int(nextn) < cfg["n_layers"]:
            cfg["n_layers"] -= int(nextn)
    for key, name in (("embedding_length", "hidden"), ("feed_forward_length", "n_ff"),
                      ("attention.head_count", "n_heads"), ("attention.head_count_kv", "n_kv_heads"),
                      ("attention.key_length", "head_dim"), ("full_attention_interval", "full_attention_interval"),
                      ("ssm.state_size", "gdn_head_dim"), ("ssm.conv_kernel", "conv_kernel"),
                      ("ssm.group_count", "gdn_num_k_heads")):
        if g(key) is not None:
            cfg[name] = int(g(key))
    if g("attention.layer_norm_rms_epsilon") is not None:
        cfg["rms_eps"] = float(g("attention.layer_norm_rms_epsilon"))
    if g("rope.freq_base") is not None:
        cfg["rope_freq_base"] = float(g("rope.freq_base"))
    kd = cfg.get("gdn_head_dim", 128)
    if g("ssm.inner_size") is not None:
        cfg["gdn_n_heads"] = int(g("ssm.inner_size")) // kd
    rot = g("rope.dimension_count")
    if rot is not None and int(rot) != 64:
        raise ValueError(f"rotary dimension {int(rot)}: this backend rotates dims 0..63 of each head")
    vocab = _get(reader, "tokenizer.ggml.vocab_size")
    if vocab is not None:
        cfg["vocab"] = int(vocab)
    else:
        emb = [t for t in reader.tensors if t.name == "token_embd.weight"]
        if emb:
            cfg["vocab"] = int(emb[0].shape[1])
    name = _get(reader, "general.name") or "gguf"
    return ModelConfig(name=str(name), **cfg)


class GGUFModel:
    """A GGUF file's decoder tensors on the device, keyed by GGUF name."""

    def __init__(self, path, device="cuda"):
        from gguf import GGUFReader
        reader = GGUFReader(path)
        self.cfg = read_config(reader)
        self.device = torch.device(device)
        plan = {p[0]: p[2] for p in tensor_plan(self.cfg)}
        plan.setdefault("output.weight", TT["Q8_0"])  # optional: tied to token_embd when absent
        eos = _get(reader, "tokenizer.ggml.eos_token_id")
        self.eos_token_id = None if eos is None else int(eos)
        self.tensors = {}
        for t in reader.tensors:
            if t.name not in plan:
                continue  # next-token-prediction layers and tensors the decoder does not use
            tt = int(t.tensor_type)
            dims = [int(d) for d in t.shape]  # GGUF order: dims[0] = columns
            cols = dims[0]
            rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
            if plan[t.name] == TT["F32"]:
                # norm weights, conv taps, dt bias, ssm_a: f32 vectors (src/backend_cpu.zig:1196-1212)
                if tt == TT["F32"]:
                    arr = np.asarray(t.data, dtype=np.float32).reshape(-1)
                elif tt == F16:
                    arr = np.asarray(t.data).view(np.float16).astype(np.float32).reshape(-1)
                elif tt == BF16:
                    arr = (np.asarray(t.data).view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(-1)
                else:
                    raise ValueError(f"{t.name}: vector tensor of GGUF type {tt} (expected F32, F16 or BF16)")
                dev = torch.from_numpy(np.array(arr, dtype=np.float32)).to(self.device)
                self.tensors[t.name] = (TT["F32"], 1, arr.size, dev)
            elif tt in LINEAR_TYPES:
                raw = np.asarray(t.data).view(np.uint8).reshape(-1)
                with warnings.catch_warnings():  # the file's read-only map, copied by .to()
                    warnings.simplefilter("ignore", UserWarning)
                    dev = torch.from_numpy(raw).to(self.device, copy=True)
                self.tensors[t.name] = (tt, rows, cols, dev)
            else:
                raise ValueError(f"{t.name}: GGUF tensor type {tt} is not supported by this backend "
                                 "(linear layers: Q8_0, IQ4_NL, Q4_K, Q5_K, Q6_K, Q4_0, Q4_1, Q5_0, Q5_1)")
        missing = sorted(set(plan) - set(self.tensors) - {"output.weight"})
        if missing:
            raise ValueError(f"GGUF file lacks {len(missing)} decoder tensors, e.g. {missing[:3]}")
        self.cfg = dataclasses.replace(self.cfg, quant=self._quant_map())

    def _quant_map(self):
        """The file's weight types as a ModelConfig.quant: the most common
        linear type as 'bulk', each role that differs from it by name"""
        roles = collections.defaultdict(set)
        for name, role, *_ in tensor_plan(self.cfg):
            if name in self.tensors and self.tensors[name][0] != TT["F32"]:
                roles[role].add(self.tensors[name][0])
        if "output.weight" in self.tensors:
            roles["output"].add(self.tensors["output.weight"][0])
        inv = {v: k for k, v in TT.items()}
        count = collections.Counter(t for ts in roles.values() for t in ts)
        bulk = count.most_common(1)[0][0]
        quant = [("bulk", inv[bulk])]
        for role in sorted(roles):
            ts = roles[role]
            if len(ts) > 1:
                raise ValueError(f"weights of role {role} come in several types {sorted(ts)}")
            if ts != {bulk} or role == "output":
                quant.append((role, inv[next(iter(ts))]))
        return tuple(quant)

    def weight_bytes(self):
        return sum(t.numel() * t.element_size() for (_, _, _, t) in self.tensors.values())

    def host(self, name):
        tt, rows, cols, t = self.tensors[name]
        return tt, rows, cols, t.cpu().numpy()


def write_gguf(model, path, extra_metadata=None):
    """Write `model` (cfg + tensors, host-copied) as a qwen35 GGUF file.
    extra_metadata: {key: int | float | str} added after (or replacing) the
    configuration keys, e.g. next-token-prediction layer counts."""
    import gguf
    c = model.cfg
    kv = {
        "general.name": c.name,
        f"{ARCH}.block_count": c.n_layers,
        f"{ARCH}.embedding_length": c.hidden,
        f"{ARCH}.feed_forward_length": c.n_ff,
        f"{ARCH}.attention.head_count": c.n_heads,
        f"{ARCH}.attention.head_count_kv": c.n_kv_heads,
        f"{ARCH}.attention.key_length": c.head_dim,
        f"{ARCH}.full_attention_interval": c.full_attention_interval,
        f"{ARCH}.attention.layer_norm_rms_epsilon": float(c.rms_eps),
        f"{ARCH}.ssm.state_size": c.gdn_head_dim,
        f"{ARCH}.ssm.conv_kernel": c.conv_kernel,
        f"{ARCH}.ssm.inner_size": c.gdn_n_heads * c.gdn_head_dim,
        f"{ARCH}.ssm.group_count": c.gdn_num_k_heads,
        f"{ARCH}.rope.freq_base": float(c.rope_freq_base),
        f"{ARCH}.rope.dimension_count": 64,
        "tokenizer.ggml.vocab_size": c.vocab,
    }
    kv.update(extra_metadata or {})
    w = gguf.GGUFWriter(path, ARCH)
    for key, v in kv.items():
        if isinstance(v, str):
            w.add_string(key, v)
        elif isinstance(v, float):
            w.add_float32(key, v)
        else:
            w.add_uint32(key, int(v))
    for name, (tt, rows, cols, t) in model.tensors.items():
        arr = t.cpu().numpy() if hasattr(t, "cpu") else np.asarray(t)
        if tt == TT["F32"]:
            w.add_tensor(name, np.ascontiguousarray(arr, dtype=np.float32).reshape(-1))
        else:
            raw = np.ascontiguousarray(arr).view(np.uint8).reshape(rows, -1)
            w.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType(tt))  # byte shape -> element shape
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
