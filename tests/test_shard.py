"""Multi-GPU host logic on CPU: sequence sharding, max-over-ranks timing and
output gathering, run as world-size-2 gloo process groups on 127.0.0.1.
No GPU is needed (the data path has no collective; only these do)."""
import datetime
import os
import socket
import tempfile

import pytest
import torch.multiprocessing as mp

from qwen35_b200.shard import gather_outputs, max_over_ranks, seq_cost, shard_sequences


def test_shard_covers_and_balances():
    import numpy as np
    rng = np.random.default_rng(0)
    prompts = rng.integers(64, 2049, 64)
    costs = [seq_cost(p, 256) for p in prompts]
    for world in (1, 2, 4, 8):
        plan = shard_sequences(costs, world)
        flat = sorted(i for s in plan for i in s)
        assert flat == list(range(64))
        loads = [sum(costs[i] for i in s) for s in plan]
        # longest-first greedy: the spread is at most one sequence's cost
        assert max(loads) - min(loads) <= max(costs)
        assert plan == shard_sequences(costs, world)  # deterministic


def test_shard_more_ranks_than_sequences():
    plan = shard_sequences([5, 3], 4)
    assert plan == [[0], [1], [], []]
    with pytest.raises(ValueError):
        shard_sequences([1], 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir, mode):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        if mode == "ok":
            costs = [seq_cost(p, g) for p, g in [(3, 5), (11, 2), (6, 7), (1, 4), (8, 3)]]
            shard = shard_sequences(costs, world)[rank]
            local = [[i, i * 10] for i in shard]  # stand-in token lists
            res = gather_outputs(local, shard, len(costs), dist, rank)
            m = max_over_ranks(0.5 + rank, dist)
            with open(os.path.join(out_dir, f"r{rank}"), "w") as f:
                f.write(f"{m}\n{res}\n")
        else:
            # rank 1 leaves between steps without joining the next collective;
            # rank 0's collective must end with an error, not hang
            if rank == 1:
                os._exit(0)
            try:
                max_over_ranks(1.0, dist)
                status = "returned"
            except Exception as e:  # gloo raises on the process-group timeout
                status = "error:" + type(e).__name__
            with open(os.path.join(out_dir, "r0"), "w") as f:
                f.write(status)
            # the group is broken: leave without running its destructor
            os._exit(0)
    finally:
        if mode == "ok":
            dist.destroy_process_group()


def test_gloo_two_ranks_shard_gather_max():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d, "ok"), nprocs=2, start_method="spawn")
        for r in range(2):
            lines = open(os.path.join(d, f"r{r}")).read().splitlines()
            assert float(lines[0]) == 1.5
        assert open(os.path.join(d, "r0")).read().splitlines()[1] == str([[i, i * 10] for i in range(5)])
        assert open(os.path.join(d, "r1")).read().splitlines()[1] == "None"


def test_gloo_missing_rank_is_an_error_not_a_hang():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_worker, args=(2, _free_port(), d, "leave"), nprocs=2, start_method="spawn",
                                 join=False)
        import time
        deadline = time.time() + 120
        while not ctx.join(timeout=5):
            assert time.time() < deadline, "ranks did not finish"
        status = open(os.path.join(d, "r0")).read()
        assert status.startswith("error:"), status
