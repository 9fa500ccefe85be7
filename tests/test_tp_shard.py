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


@pytest.mark.parametrize("cfg_name,P", [("tiny-tp", 2), ("tiny-tp-mixed", 2), ("tiny-tp-mixed", 4),
                                         ("tiny-tp-rep", 2)])
def test_shards_reassemble(cfg_name, P):
    """replicated kv heads write the same rows from several ranks; uneven ffn
    shards still cover every block once"""
    cfg = CONFIGS[cfg_name]
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
    """the local value head l (global h) reads local k head l % (nk/P), which
    is global k head h % nk, for head groups of 1 (32-element blocks) and 2
    (256-element blocks)"""
    import dataclasses
    for nv, nk, P, ssm_out in [(48, 16, 2, "Q4_K"), (48, 16, 4, "Q4_K"), (48, 16, 8, "Q4_K"), (32, 16, 8, "IQ4_NL"),
                               (16, 16, 2, "Q8_0"), (4, 2, 2, "Q8_0"), (8, 4, 2, "Q4_K"), (32, 16, 4, "Q5_K")]:
        cfg = dataclasses.replace(CONFIGS["27b"], gdn_n_heads=nv, gdn_num_k_heads=nk,
                                  quant=(("bulk", "Q4_K"), ("ssm_out", ssm_out)))
        seen = []
        for p in range(P):
            vh, kh = tp.gdn_heads(cfg, P, p)
            assert len(vh) == nv // P and len(kh) == nk // P
            for l, h in enumerate(vh):
                assert kh[l % (nk // P)] == h % nk
            if GEOM[TT[ssm_out]][0] == 256:  # whole ssm_out blocks: heads in aligned pairs
                assert all(vh[2 * i] % 2 == 0 and vh[2 * i + 1] == vh[2 * i] + 1 for i in range(len(vh) // 2))
            seen += vh
        assert sorted(seen) == list(range(nv))


def test_local_config_and_rejects():
    cfg = CONFIGS["27b"]
    loc = tp.local_config(cfg, 4)
    assert (loc.n_heads, loc.n_kv_heads, loc.gdn_n_heads, loc.gdn_num_k_heads, loc.n_ff) == (6, 1, 12, 4, 4352)
    assert loc.vocab == cfg.vocab and loc.hidden == cfg.hidden
    # TP 8: 4 kv heads replicated on rank pairs, 68 ffn blocks as 9,9,9,9,8,8,8,8
    locs = [tp.local_config(cfg, 8, p) for p in range(8)]
    assert [c.n_ff for c in locs] == [2304] * 4 + [2048] * 4
    assert all((c.n_heads, c.n_kv_heads, c.gdn_n_heads, c.gdn_num_k_heads) == (3, 1, 6, 2) for c in locs)
    assert [tp.kv_heads(cfg, 8, p) for p in range(8)] == [[0], [0], [1], [1], [2], [2], [3], [3]]
    # every rank's q heads read only the kv head it holds (GQA group = H / KV)
    for p in range(8):
        grp = cfg.n_heads // cfg.n_kv_heads
        assert {h // grp for h in range(p * 3, p * 3 + 3)} == set(tp.kv_heads(cfg, 8, p))
    assert sum(tp.ffn_range(cfg, 8, p)[1] - tp.ffn_range(cfg, 8, p)[0] for p in range(8)) == cfg.n_ff
    with pytest.raises(ValueError):
        tp.local_config(cfg, 16)  # 24 q heads do not split 16 ways
    with pytest.raises(ValueError):
        tp.local_config(CONFIGS["tiny-tp-mixed"], 3)


class _FakeEngine:
    """stands in for model.Engine in the handle exchange: this rank's IPC
    handle bytes, and the list set_peers receives"""

    def __init__(self, rank):
        self.rank = rank
        self.peers = None

    def ipc_handles(self):
        return bytes([self.rank + 1]) * 192

    def set_peers(self, handles):
        self.peers = list(handles)


def _peers_worker(rank, world, port, out_dir):
    import datetime
    import os

    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        eng = _FakeEngine(rank)
        tp.connect_peers(dist, eng)
        with open(os.path.join(out_dir, f"r{rank}"), "wb") as f:
            f.write(b"".join(eng.peers))
    finally:
        dist.destroy_process_group()


def test_connect_peers_exchanges_handles_in_rank_order():
    """tp.connect_peers over a world-size-3 gloo group: every rank's engine
    receives all ranks' handles, in rank order (the order the peer
    all-reduce indexes its peer table by)"""
    import os
    import socket
    import tempfile

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_peers_worker, args=(3, port, d), nprocs=3, start_method="spawn")
        expect = b"".join(bytes([r + 1]) * 192 for r in range(3))
        for r in range(3):
            assert open(os.path.join(d, f"r{r}"), "rb").read() == expect
