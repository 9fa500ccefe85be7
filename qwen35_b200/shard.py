"""Sequence sharding over ranks: one process per GPU, each an independent
replica of the model serving a subset of the sequences.  Requests are
independent, so there is no collective on the data path; the only
cross-rank traffic is the timing reduction (max over ranks) and, for
serving, gathering the finished token lists on rank 0.

The reference engine is single-sequence and single-GPU; this is the
multi-GPU layer its batched successor needs (cost-balanced placement, then
continuous batching per rank through q35b_serve).
"""


def seq_cost(prompt_len, n_gen):
    """tokens a sequence pushes through the decode step (prefill one token
    per step, then generation)"""
    return int(prompt_len) + int(n_gen)


def shard_sequences(costs, world):
    """Longest-first greedy bin packing: visit sequences by descending cost
    (ties by index) and give each to the rank with the least load so far
    (ties by rank).  Returns one ascending index list per rank.  Deterministic,
    so every rank computes the same plan without communicating."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i))
    load = [0] * world
    out = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += int(costs[i])
    return [sorted(s) for s in out]


def max_over_ranks(value, dist, device="cpu"):
    """the largest `value` over all ranks (a float); `dist` None = one rank"""
    if dist is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_outputs(local, shard, n_total, dist, rank):
    """rank 0 gets every sequence's token list in the original order.
    `local[k]` belongs to sequence `shard[k]`.  Uses gather_object, which the
    NCCL and gloo backends both provide."""
    if dist is None:
        res = [None] * n_total
        for k, i in enumerate(shard):
            res[i] = local[k]
        return res
    pairs = list(zip(shard, local))
    got = [None] * dist.get_world_size() if rank == 0 else None
    dist.gather_object(pairs, got, dst=0)
    if rank != 0:
        return None
    res = [None] * n_total
    for part in got:
        for i, toks in part:
            res[i] = toks
    return res
