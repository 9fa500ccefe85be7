"""Tensor parallelism (Megatron-style) for the batched engine: the shard of
each GGUF tensor a rank holds, and the rank-local model config.

Rank p of P holds
  * column-parallel projections (their output rows): attention q heads
    [p*H/P, (p+1)*H/P) (attn_q rows are per head [q_h | gate_h]) and kv heads
    likewise -- with fewer kv heads than ranks (27B: 4 kv heads at TP 8) each
    kv head is replicated on the P/KV ranks whose q heads read it, so a rank
    holds exactly one; GDN value heads in groups of g = max(1, B/128)
    heads, B the block width of ssm_out's type (g = 2 for 256-element K-quant
    blocks, so a rank's ssm_out columns are whole blocks): rank p holds value
    heads h = g*(p + P*i) + u and k heads likewise, and the reference's
    value-head -> k-head map h % nk (src/backend_cpu.zig:1006) becomes the
    local l % (nk/P) (it holds when nk is a multiple of g*P); ffn gate / up rows
    in whole 256-row blocks, as even as the block count allows (27B at TP 8:
    68 blocks -> 9,9,9,9,8,8,8,8);
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


FFN_BLOCK = 256  # ffn split unit: one K-quant block of ffn_down's columns


def gdn_group(cfg):
    """value heads per ssm_out column block (1 for 32-element blocks, 2 for
    256-element K-quant blocks over 128-wide heads)"""
    tt = cfg.qtype("ssm_out")
    if tt == TT["F32"]:
        return 1
    return max(1, GEOM[tt][0] // cfg.gdn_head_dim)


def gdn_heads(cfg, P, p):
    """(value heads, k heads) of rank p, ascending"""
    g = gdn_group(cfg)
    vh = [g * (p + P * i) + u for i in range(cfg.gdn_n_heads // (g * P)) for u in range(g)]
    kh = [g * (p + P * i) + u for i in range(cfg.gdn_num_k_heads // (g * P)) for u in range(g)]
    return vh, kh


def check_tp(cfg, P):
    """raise ValueError unless `cfg` splits P ways"""
    g = gdn_group(cfg)
    need = [("n_heads", cfg.n_heads, P), ("gdn_n_heads", cfg.gdn_n_heads, g * P),
            ("gdn_num_k_heads", cfg.gdn_num_k_heads, g * P), ("vocab", cfg.vocab, P)]
    for what, n, m in need:
        if n % m:
            raise ValueError(f"{what}={n} does not split {P} ways (in groups of {m // P})")
    if cfg.n_kv_heads % P and P % cfg.n_kv_heads:
        raise ValueError(f"n_kv_heads={cfg.n_kv_heads} neither splits {P} ways nor replicates evenly")
    if cfg.n_ff % FFN_BLOCK or cfg.n_ff // FFN_BLOCK < P:
        raise ValueError(f"n_ff={cfg.n_ff} is not {P} or more whole {FFN_BLOCK}-row blocks")
    if cfg.gdn_n_heads % cfg.gdn_num_k_heads:
        raise ValueError("gdn_n_heads must be a multiple of gdn_num_k_heads")


def ffn_range(cfg, P, p):
    """[first, end) ffn rows of rank p: whole blocks, the first n_blocks % P
    ranks one block more"""
    nb = cfg.n_ff // FFN_BLOCK
    base, extra = divmod(nb, P)
    first = p * base + min(p, extra)
    count = base + (1 if p < extra else 0)
    return first * FFN_BLOCK, (first + count) * FFN_BLOCK


def kv_heads(cfg, P, p):
    """the kv heads rank p holds: KV/P contiguous heads, or (KV < P) the one
    its q heads read"""
    KV = cfg.n_kv_heads
    if KV % P == 0:
        return list(range(p * KV // P, (p + 1) * KV // P))
    return [p // (P // KV)]


def local_config(cfg, P, p=0):
    """the rank-local model config (vocab stays whole: it sizes the
    embedding); only n_ff can differ between ranks"""
    check_tp(cfg, P)
    f0, f1 = ffn_range(cfg, P, p)
    return dataclasses.replace(cfg, n_heads=cfg.n_heads // P, n_kv_heads=len(kv_heads(cfg, P, p)),
                               gdn_n_heads=cfg.gdn_n_heads // P, gdn_num_k_heads=cfg.gdn_num_k_heads // P,
                               n_ff=f1 - f0)


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
    check_tp(cfg, P)
    H, hd = cfg.n_heads, cfg.head_dim
    nv, nk, kd = cfg.gdn_n_heads, cfg.gdn_num_k_heads, cfg.gdn_head_dim
    V = cfg.vocab
    hq = list(range(p * H // P, (p + 1) * H // P))
    hkv = kv_heads(cfg, P, p)
    vh, kh = gdn_heads(cfg, P, p)
    qrows = [r for h in hq for r in range(2 * hd * h, 2 * hd * (h + 1))]
    kvrows = [r for h in hkv for r in range(hd * h, hd * (h + 1))]
    qcols = [c for h in hq for c in range(hd * h, hd * (h + 1))]
    # GDN conv channels / qkv rows: [q: nk*kd | k: nk*kd | v: nv*kd]
    gq = [c for h in kh for c in range(kd * h, kd * (h + 1))]
    gk = [nk * kd + c for c in gq]
    gv = [2 * nk * kd + c for h in vh for c in range(kd * h, kd * (h + 1))]
    vcols = [c for h in vh for c in range(kd * h, kd * (h + 1))]
    frows = list(range(*ffn_range(cfg, P, p)))
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
        self.cfg = local_config(model.cfg, P, p)
        self.P, self.p = P, p
        self.vocab_offset = p * model.cfg.vocab // P
        self.vocab_local = model.cfg.vocab // P
        self.tensors = shard_tensors(model.cfg, model.tensors, P, p)


def shared_nccl_id(dist, device):
    """the engine communicator's NCCL id, made on rank 0 by q35b_tp_unique_id
    and broadcast over the process group `dist` (every rank calls this)"""
    import ctypes

    from . import lib
    buf = torch.zeros(128, dtype=torch.uint8, device=device)
    if dist.get_rank() == 0:
        raw = ctypes.create_string_buffer(128)
        rc = lib.load().q35b_tp_unique_id(ctypes.cast(raw, ctypes.c_void_p), 128)
        if rc != 0:
            raise RuntimeError(f"q35b_tp_unique_id failed: {rc}")
        buf.copy_(torch.frombuffer(bytearray(raw.raw), dtype=torch.uint8))
    dist.broadcast(buf, 0)
    return buf.cpu().numpy().tobytes()


def connect_peers(dist, eng):
    """exchange the engines' IPC handles over the process group `dist` and
    map every rank's buffers, switching `eng` to the peer all-reduce (every
    rank calls this, after its engine is built)"""
    mine = eng.ipc_handles()
    allh = [None] * dist.get_world_size()
    dist.all_gather_object(allh, mine)
    eng.set_peers(allh)
    dist.barrier()

