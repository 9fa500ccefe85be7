"""GGUF checkpoints: the loader (qwen35_b200/gguf_model.py, after the
reference's src/engine.zig:810-993) over files written by `write_gguf`.

CPU: metadata -> configuration, every tensor's bytes through a round trip,
next-token-prediction layers skipped, f16 / bf16 vectors widened, the
errors the reference's loader raises (missing tensor, unsupported type).
GPU: an engine over the loaded file decodes the same greedy tokens as one
over the in-memory model it was written from.
"""
import dataclasses

import numpy as np
import pytest
import torch

import oracle_lib as ol
from qwen35_b200.gguf_model import GGUFModel, write_gguf
from qwen35_b200.model import CONFIGS, TT, tensor_plan


class _HostModel:
    """cfg + tensors {name: (tt, rows, cols, numpy array)}"""

    def __init__(self, cfg, tensors):
        self.cfg, self.tensors = cfg, tensors


def _host_model(cfg_name, seed=1):
    cfg = CONFIGS[cfg_name]
    O = ol.load_oracle()
    rng = np.random.default_rng(seed)
    tensors = {}
    for name, _, tt, rows, cols, init in tensor_plan(cfg):
        if init == "w":
            w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
            tensors[name] = (tt, rows, cols, ol.quantize_weight(O, tt, w))
        else:
            tensors[name] = (tt, rows, cols, rng.standard_normal(rows * cols).astype(np.float32))
    return _HostModel(cfg, tensors)


def _same_bytes(a, b):
    return np.array_equal(np.asarray(a).view(np.uint8).reshape(-1), np.asarray(b).view(np.uint8).reshape(-1))


@pytest.mark.parametrize("cfg_name", ["tiny", "tiny-mixed"])
def test_round_trip(tmp_path, cfg_name):
    m = _host_model(cfg_name)
    path = str(tmp_path / "m.gguf")
    write_gguf(m, path)
    g = GGUFModel(path, device="cpu")
    # metadata floats are f32 in the file, as the engine reads them
    assert g.cfg == dataclasses.replace(m.cfg, rms_eps=float(np.float32(m.cfg.rms_eps)), quant=g.cfg.quant)
    assert dict(g.cfg.quant) == dict(m.cfg.quant)  # weight types per role, read back from the tensors
    assert set(g.tensors) == set(m.tensors)
    for name, (tt, rows, cols, arr) in m.tensors.items():
        gt, gr, gc, t = g.tensors[name]
        assert (gt, gr, gc) == (tt, rows, cols), name
        assert _same_bytes(t.numpy(), arr), name


def test_nextn_layers_skipped(tmp_path):
    m = _host_model("tiny")
    n = m.cfg.n_layers
    extra = dict(m.tensors)
    # a trailing full-attention prediction layer, as the 27B file carries
    for name in list(m.tensors):
        if name.startswith(f"blk.{n - 1}."):
            extra[name.replace(f"blk.{n - 1}.", f"blk.{n}.")] = m.tensors[name]
    extra[f"blk.{n}.nextn.enorm"] = (TT["F32"], 1, m.cfg.hidden, np.ones(m.cfg.hidden, np.float32))
    path = str(tmp_path / "m.gguf")
    write_gguf(_HostModel(m.cfg, extra), path,
               extra_metadata={"qwen35.block_count": n + 1, "qwen35.nextn_predict_layers": 1})
    g = GGUFModel(path, device="cpu")
    assert g.cfg.n_layers == n
    assert set(g.tensors) == set(m.tensors)


def test_half_vectors_widened(tmp_path):
    m = _host_model("tiny")
    h = m.cfg.hidden
    vals = ((np.arange(h) % 256) / 16.0 - 8.0).astype(np.float32)  # 8 significant bits: exact in f16 and bf16
    t = dict(m.tensors)
    t["output_norm.weight"] = (1, 1, h, vals.astype(np.float16))  # GGML F16
    t["blk.0.attn_norm.weight"] = (30, 1, h, (vals.view(np.uint32) >> 16).astype(np.uint16))  # GGML BF16
    path = str(tmp_path / "m.gguf")
    write_gguf(_HostModel(m.cfg, t), path)
    g = GGUFModel(path, device="cpu")
    for name in ("output_norm.weight", "blk.0.attn_norm.weight"):
        tt, rows, cols, d = g.tensors[name]
        assert (tt, rows, cols) == (TT["F32"], 1, h)
        assert np.array_equal(d.numpy(), vals), name


def test_missing_tensor_raises(tmp_path):
    m = _host_model("tiny")
    t = {k: v for k, v in m.tensors.items() if k != "blk.1.ssm_a"}
    path = str(tmp_path / "m.gguf")
    write_gguf(_HostModel(m.cfg, t), path)
    with pytest.raises(ValueError, match="lacks 1 decoder tensors"):
        GGUFModel(path, device="cpu")


def test_unsupported_linear_type_raises(tmp_path):
    m = _host_model("tiny")
    t = dict(m.tensors)
    tt, rows, cols, _ = t["blk.0.ffn_up.weight"]
    t["blk.0.ffn_up.weight"] = (1, rows, cols, np.zeros((rows, cols), np.float16))  # F16 matrix
    path = str(tmp_path / "m.gguf")
    write_gguf(_HostModel(m.cfg, t), path)
    with pytest.raises(ValueError, match="not supported"):
        GGUFModel(path, device="cpu")


def test_rotary_dim_checked(tmp_path):
    m = _host_model("tiny")
    path = str(tmp_path / "m.gguf")
    write_gguf(m, path, extra_metadata={"qwen35.rope.dimension_count": 32})
    with pytest.raises(ValueError, match="rotary dimension"):
        GGUFModel(path, device="cpu")


@pytest.mark.gpu
@pytest.mark.parametrize("cfg_name", ["tiny", "tiny-mixed"])
def test_gguf_engine_tokens(tmp_path, cfg_name):
    """the engine over a GGUF file == the engine over the model it was written from"""
    from qwen35_b200 import model as q35
    cfg = CONFIGS[cfg_name]
    synth = q35.SyntheticModel(cfg, seed=3)
    path = str(tmp_path / "m.gguf")
    write_gguf(synth, path)
    loaded = GGUFModel(path, device="cuda")
    prompt = [int(x) for x in np.random.default_rng(3).integers(0, cfg.vocab, 12)]
    runs = []
    for mdl in (synth, loaded):
        eng = q35.Engine(mdl, n_slots=1, max_seq=64, max_batch=4)
        eng.reset_slot(0)
        tok = eng.prefill(0, prompt)
        toks = [tok]
        for i in range(16):
            tok = eng.step_host([tok], [0], [len(prompt) + i])[0]
            toks.append(tok)
        eng.close()
        runs.append(toks)
    torch.cuda.synchronize()
    assert runs[0] == runs[1]
