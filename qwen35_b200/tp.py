"""Tensor parallelism (Megatron-style) for the batched engine: the shard of
each GGUF tensor a rank holds, and the rank-local model config.

Rank p of P holds
  * column-parallel projections (their output rows): attention q heads
    [p*H/P, (p+1)*H/P) (attn_q rows are per head [q_h | gate_h]) and kv heads
    likewise; GDN value heads h = p + P*i and k heads kh = p + P*i, so the
    reference's value-head -> k-head map h % nk (src/backend_cpu.zig:1006)
    becomes i % (nk/P) locally; ffn gate / up rows [p*F/P, (p+1)*F/P);
  * row-parallel projections (their input columns, whole quant blocks):
    attn_output over its q heads, ssm_out over its value heads, ffn_down over
    its ffn rows -- their outputs are partial sums, all-reduced before the
    residual add;
  * the lm_head rows [p*V/P, (p+1)*V/P) (a greedy token is the max over the
    ranks' local maxima); the embedding table and all norms whole.

Shards are plain byte gathers of the packed tensors, so a rank's engine runs
exactly the single-GPU kernels on smaller shapes.
"""
import dataclasses

import torch

from .lib import GEOM, TT


def check_tp(cfg, P):
    """raise ValueError unless `cfg` splits evenly P ways"""
    need = [("n_heads", cfg.n_heads), ("n_kv_heads", cfg.n_kv_heads), ("gdn_n_heads", cfg.gdn_n_heads),
            ("gdn_num_k_heads", cfg.gdn_num_k_heads), ("n_ff", cfg.n_ff), ("vocab", cfg.vocab)]
    for what, n in need:
        if n % P:
            raise ValueError(f"{what}={n} does not split {P} ways")
    if (cfg.n_ff // P) % 256:
        raise ValueError("ffn shard must be whole 256-element blocks")
    if cfg.gdn_n_heads % cfg.gdn_num_k_heads:
        raise ValueError("gdn_n_heads must be a multiple of gdn_num_k_heads")


def local_config(cfg, P):
    """the rank-local model config (vocab stays whole: it sizes the embedding)"""
    check_tp(cfg, P)
    return dataclasses.replace(cfg, n_heads=cfg.n_heads // P, n_kv_heads=cfg.n_kv_heads // P,
                               gdn_n_heads=cfg.gdn_n_heads // P, gdn_num_k_heads=cfg.gdn_num_k_heads // P,
                               n_ff=cfg.n_ff // P)


def _row_bytes(tt, cols):
    if tt == TT["F32"]:
        return cols * 4
    e, b = GEOM[tt]
    return cols // e * b


def gather_rows(t, tt, rows, cols, idx):
    """rows `idx` of a packed [rows, cols] tensor (uint8 or f32 storage)"""
    rb = _row_bytes(tt, cols)
    by = t.view(torch.uint8).reshape(rows, rb)
    ix = torch.as_tensor(idx, dtype=torch.long, device=t.device)
    out = by.index_select(0, ix).reshape(-1)
    return out.view(torch.float32) if tt == TT["F32"] else out


def gather_cols(t, tt, rows, cols, col_idx):
    """columns `col_idx` (whole quant blocks, in order) of a packed tensor"""
    if tt == TT["F32"]:
        ix = torch.as_tensor(col_idx, dtype=torch.long, device=t.device)
        return t.reshape(rows, cols).index_select(1, ix).reshape(-1)
    e, b = GEOM[tt]
    blocks = sorted({c // e for c in col_idx})
    if len(blocks) * e != len(col_idx) or any(c % e for c in col_idx[::e]):
        raise ValueError("column shard must be whole blocks")
    by = t.view(torch.uint8).reshape(rows, cols // e, b)
    ix = torch.as_tensor(blocks, dtype=torch.long, device=t.device)
    return by.index_select(1, ix).reshape(-1)


def _heads(first, count, size):
    return [first * size + i for i in range(count * size)]


def shard_plan(cfg, P, p):
    """{name: (kind, index list)}: 'rows' / 'cols' gathers, 'whole' copies"""
    H, KV, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    nv, nk, kd = cfg.gdn_n_heads, cfg.gdn_num_k_heads, cfg.gdn_head_dim
    F, V = cfg.n_ff, cfg.vocab
    hq = list(range(p * H // P, (p + 1) * H // P))
    hkv = list(range(p * KV // P, (p + 1) * KV // P))
    vh = list(range(p, nv, P))
    kh = list(range(p, nk, P))
    qrows = [r for h in hq for r in range(2 * hd * h, 2 * hd * (h + 1))]
    kvrows = [r for h in hkv for r in range(hd * h, hd * (h + 1))]
    qcols = [c for h in hq for c in range(hd * h, hd * (h + 1))]
    # GDN conv channels / qkv rows: [q: nk*kd | k: nk*kd | v: nv*kd]
    gq = [c for h in kh for c in range(kd * h, kd * (h + 1))]
    gk = [nk * kd + c for c in gq]
    gv = [2 * nk * kd + c for h in vh for c in range(kd * h, kd * (h + 1))]
    vcols = [c for h in vh for c in range(kd * h, kd * (h + 1))]
    frows = list(range(p * F // P, (p + 1) * F // P))
    vrows = list(range(p * V // P, (p + 1) * V // P))
    plan = {"token_embd.weight": ("whole", None), "output_norm.weight": ("whole", None),
            "output.weight": ("rows", vrows)}
    for li in range(cfg.n_layers):
        b = f"blk.{li}."
        plan[b + "attn_norm.weight"] = ("whole", None)
        plan[b + "post_attention_norm.weight"] = ("whole", None)
        if cfg.is_full(li):
            plan[b + "attn_q.weight"] = ("rows", qrows)
            plan[b + "attn_k.weight"] = ("rows", kvrows)
            plan[b + "attn_v.weight"] = ("rows", kvrows)
            plan[b + "attn_output.weight"] = ("cols", qcols)
            plan[b + "attn_q_norm.weight"] = ("whole", None)
            plan[b + "attn_k_norm.weight"] = ("whole", None)
        else:
            plan[b + "attn_qkv.weight"] = ("rows", gq + gk + gv)
            plan[b + "attn_gate.weight"] = ("rows", vcols)
            plan[b + "ssm_alpha.weight"] = ("rows", vh)
            plan[b + "ssm_beta.weight"] = ("rows", vh)
            plan[b + "ssm_out.weight"] = ("cols", vcols)
            plan[b + "ssm_conv1d.weight"] = ("rows4", gq + gk + gv)  # [conv_dim][4] f32
            plan[b + "ssm_dt.bias"] = ("vec", vh)
            plan[b + "ssm_a"] = ("vec", vh)
            plan[b + "ssm_norm.weight"] = ("whole", None)
        plan[b + "ffn_gate.weight"] = ("rows", frows)
        plan[b + "ffn_up.weight"] = ("rows", frows)
        plan[b + "ffn_down.weight"] = ("cols", frows)
    return plan


def shard_tensors(cfg, tensors, P, p):
    """{name: (tt, rows, cols, tensor)} of rank p from the whole model's
    tensors (same form).  A tied lm_head (no output.weight) is cut from
    token_embd."""
    plan = shard_plan(cfg, P, p)
    out = {}
    for name, (kind, idx) in plan.items():
        src = name
        if name == "output.weight" and name not in tensors:
            src = "token_embd.weight"
        tt, rows, cols, t = tensors[src]
        if kind == "whole":
            out[name] = (tt, rows, cols, t)
        elif kind == "rows":
            out[name] = (tt, len(idx), cols, gather_rows(t, tt, rows, cols, idx))
        elif kind == "cols":
            out[name] = (tt, rows, len(idx), gather_cols(t, tt, rows, cols, idx))
        elif kind == "rows4":  # conv taps: [conv_dim, 4] stored as one f32 row
            taps = t.reshape(-1, 4).index_select(0, torch.as_tensor(idx, dtype=torch.long, device=t.device))
            out[name] = (tt, 1, taps.numel(), taps.reshape(-1))
        elif kind == "vec":
            v = t.reshape(-1).index_select(0, torch.as_tensor(idx, dtype=torch.long, device=t.device))
            out[name] = (tt, 1, v.numel(), v)
        else:
            raise ValueError(kind)
    return out


class ShardModel:
    """rank p's tensors and local config, usable wherever a SyntheticModel is"""

    def __init__(self, model, P, p):
        self.full_cfg = model.cfg
        self.cfg = local_config(model.cfg, P)
        self.P, self.p = P, p
        self.vocab_offset = p * model.cfg.vocab // P
        self.vocab_local = model.cfg.vocab // P
        self.tensors = shard_tensors(model.cfg, model.tensors, P, p)
