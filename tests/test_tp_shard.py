"""Tensor-parallel sharding on CPU: every rank's shard of every tensor is a
byte gather of the whole tensor, and the P shards reassemble it exactly."""
import numpy as np
import pytest
import torch

from qwen35_b200 import tp
from qwen35_b200.lib import GEOM, TT
from qwen35_b200.model import CONFIGS, packed_bytes, tensor_plan


def fake_tensors(cfg, seed=0):
    """random bytes / floats with the packed sizes of every tensor"""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, role, tt, rows, cols, init in tensor_plan(cfg):
        if tt == TT["F32"]:
            t = torch.randn(rows * cols, generator=g)
        else:
            t = torch.randint(0, 256, (packed_bytes(tt, rows, cols),), generator=g, dtype=torch.int32).to(torch.uint8)
        out[name] = (tt, rows, cols, t)
    return out


@pytest.mark.parametrize("cfg_name,P", [("tiny-tp", 2), ("tiny-tp-mixed", 2), ("tiny-tp-mixed", 4)])
def test_shards_reassemble(cfg_name, P):
    cfg = CONFIGS[cfg_name]
    if cfg.n_kv_heads % P or cfg.gdn_num_k_heads % P or cfg.n_heads % P:
        pytest.skip("does not split")
    full = fake_tensors(cfg)
    shards = [tp.shard_tensors(cfg, full, P, p) for p in range(P)]
    plan = [tp.shard_plan(cfg, P, p) for p in range(P)]
    for name, (tt, rows, cols, t) in full.items():
        kind = plan[0][name][0]
        if kind == "whole":
            for s in shards:
                assert torch.equal(s[name][3], t)
            continue
        if kind in ("rows", "rows4", "vec"):
            width = 4 if kind == "rows4" else (1 if kind == "vec" else None)
            if kind == "rows":
                rb = tt == TT["F32"] and cols * 4 or cols // GEOM[tt][0] * GEOM[tt][1]
                rec = torch.zeros(rows, rb, dtype=torch.uint8)
                for p in range(P):
                    idx = plan[p][name][1]
                    rec[idx] = shards[p][name][3].view(torch.uint8).reshape(len(idx), rb)
                assert torch.equal(rec.reshape(-1), t.view(torch.uint8))
            else:
                n = t.numel() // width
                rec = torch.zeros(n, width)
                for p in range(P):
                    idx = plan[p][name][1]
                    rec[idx] = shards[p][name][3].reshape(len(idx), width)
                assert torch.equal(rec.reshape(-1), t)
        else:  # cols
            e, b = GEOM[tt]
            nb = cols // e
            rec = torch.zeros(rows, nb, b, dtype=torch.uint8)
            for p in range(P):
                blocks = sorted({c // e for c in plan[p][name][1]})
                rec[:, blocks] = shards[p][name][3].reshape(rows, len(blocks), b)
            assert torch.equal(rec.reshape(-1), t)


def test_gdn_head_map_stays_local():
    """value head h = p + P*i uses k head h % nk = p + P*(i % (nk/P)): the
    local index i % (nk/P) of a k head this rank holds"""
    for nv, nk, P in [(48, 16, 2), (48, 16, 4), (32, 16, 8), (16, 16, 2), (4, 2, 2)]:
        for p in range(P):
            vh = list(range(p, nv, P))
            kh = list(range(p, nk, P))
            for i, h in enumerate(vh):
                assert kh[i % (nk // P)] == h % nk


def test_local_config_and_rejects():
    cfg = CONFIGS["27b"]
    loc = tp.local_config(cfg, 4)
    assert (loc.n_heads, loc.n_kv_heads, loc.gdn_n_heads, loc.gdn_num_k_heads, loc.n_ff) == (6, 1, 12, 4, 4352)
    assert loc.vocab == cfg.vocab and loc.hidden == cfg.hidden
    with pytest.raises(ValueError):
        tp.local_config(cfg, 8)  # 4 kv heads do not split 8 ways
