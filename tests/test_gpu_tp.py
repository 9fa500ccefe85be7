"""Tensor-parallel decode on 2 GPUs: two ranks, each running the engine on
its shard, against one GPU running the whole model and against the CPU oracle
stepping the whole model; the row-parallel all-reduce both through NCCL and
through the peer all-reduce kernel (identical bits at two ranks).

Row-parallel partial sums are added in a different order than the single
GPU's one serial fold, so the comparison is by tolerance: the residual
stream after every layer within 1e-3 relative L2 (the BASELINE per-layer
bar) and the same greedy tokens.  Cases: even head splits (Q8_0 and mixed
precision), one kv head replicated on both ranks with an odd count of ffn
blocks, and the 27B layer shapes (Q4_K, Q6_K lm_head, 4 kv heads split, 48
GDN value heads in pairs).  Skipped with fewer than 2 GPUs.

At the 27B shapes the reassociated partial sums (one rounding apart from the
single GPU's fold) now and then flip the rounding of an int8 activation
quantization downstream; the sharp attention of a random-weight model turns
such a flip into a percent-level change of the following layers.  Two CPU
builds that differ only in the last ulp of expf part the same way there (1.5e-2
measured on this model, same tokens), so that case is held to identical greedy
tokens and the envelope of such rounding differences (5e-2), the small cases to
1e-3."""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N_STEPS = 14


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(eng, cfg, prompt, n_layers, n_steps):
    toks, probes = [], []
    last = None
    eng.reset_slot(0)
    for pos in range(n_steps):
        t = prompt[pos] if pos < len(prompt) else last
        last = eng.step_host([t], [0], [pos])[0]
        toks.append(last)
        probes.append(np.stack([eng.layer_out(li, 1)[0].cpu().numpy() for li in range(n_layers)]))
    return toks, np.stack(probes)


def _run_oracle(full, prompt, n_steps):
    """the CPU oracle over the full model's bytes, on the same token sequence"""
    from oracle_lib import oracle_forward, oracle_layer_out, oracle_model
    cfg = full.cfg
    O, m, keep = oracle_model(full, threads=min(16, os.cpu_count() or 1), max_seq=64)
    toks, probes = [], []
    last = None
    for pos in range(n_steps):
        t = prompt[pos] if pos < len(prompt) else last
        lc = oracle_forward(O, m, t, pos, cfg.vocab)
        last = int(np.argmax(lc))
        toks.append(last)
        probes.append(np.stack([oracle_layer_out(O, m, li, cfg.hidden) for li in range(cfg.n_layers)]))
    O.q35o_model_destroy(m)
    return toks, np.stack(probes)


def _worker(rank, world, port, out_dir, cfg_name, n_steps):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", rank))
    from qwen35_b200 import tp
    from qwen35_b200 import model as q35
    cfg = q35.CONFIGS[cfg_name]
    full = q35.SyntheticModel(cfg, seed=21)
    shard = tp.ShardModel(full, world, rank)
    uid = tp.shared_nccl_id(dist, torch.device("cuda", rank))
    eng = q35.Engine(shard, n_slots=2, max_seq=64, max_batch=4, tp_id=uid)
    eng.set_probe(True)
    prompt = [int(v) for v in np.random.default_rng(21).integers(0, cfg.vocab, 6)]
    toks, probes = _run(eng, cfg, prompt, cfg.n_layers, n_steps)
    np.save(os.path.join(out_dir, f"probe{rank}.npy"), probes)
    np.save(os.path.join(out_dir, f"toks{rank}.npy"), np.array(toks))
    # the same steps with the peer all-reduce (one kernel over NVLink peer
    # memory instead of the NCCL call and the residual add)
    tp.connect_peers(dist, eng)
    ptoks, pprobes = _run(eng, cfg, prompt, cfg.n_layers, n_steps)
    np.save(os.path.join(out_dir, f"pprobe{rank}.npy"), pprobes)
    np.save(os.path.join(out_dir, f"ptoks{rank}.npy"), np.array(ptoks))
    dist.barrier()  # no rank unmaps or frees while another may still read it
    eng.close()  # its graphs hold NCCL work: released before the process group
    if rank == 0:
        ref = q35.Engine(full, n_slots=2, max_seq=64, max_batch=4)
        ref.set_probe(True)
        rt, rp = _run(ref, cfg, prompt, cfg.n_layers, n_steps)
        ref.close()
        np.save(os.path.join(out_dir, "probe_ref.npy"), rp)
        np.save(os.path.join(out_dir, "toks_ref.npy"), np.array(rt))
        ot, op = _run_oracle(full, prompt, n_steps)
        np.save(os.path.join(out_dir, "probe_oracle.npy"), op)
        np.save(os.path.join(out_dir, "toks_oracle.npy"), np.array(ot))
    dist.barrier()
    dist.destroy_process_group()


def _worst(a, b):
    worst = 0.0
    for s in range(a.shape[0]):
        for li in range(a.shape[1]):
            x, y = a[s, li].astype(np.float64), b[s, li].astype(np.float64)
            worst = max(worst, np.linalg.norm(x - y) / max(np.linalg.norm(y), 1e-30))
    return worst


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("cfg_name,n_steps,bound", [("tiny-tp", N_STEPS, 1e-3), ("tiny-tp-mixed", N_STEPS, 1e-3),
                                                    ("tiny-tp-rep", N_STEPS, 1e-3), ("27b-4l", 10, 5e-2)])
def test_tp2_matches_single_gpu_and_oracle(cfg_name, n_steps, bound):
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d, cfg_name, n_steps), nprocs=2, start_method="spawn")
        p0, p1, pr, po = (np.load(os.path.join(d, f)) for f in ("probe0.npy", "probe1.npy", "probe_ref.npy",
                                                                "probe_oracle.npy"))
        t0, t1, tr, to = (np.load(os.path.join(d, f)) for f in ("toks0.npy", "toks1.npy", "toks_ref.npy",
                                                                "toks_oracle.npy"))
        # the ranks hold one residual stream, bit for bit
        assert np.array_equal(p0.view(np.uint32), p1.view(np.uint32))
        assert np.array_equal(t0, t1)
        # the peer all-reduce: at two ranks its rank-order sum p0 + p1 and the
        # residual add are NCCL's sum and k_add_rows bit for bit
        q0, q1 = (np.load(os.path.join(d, f)) for f in ("pprobe0.npy", "pprobe1.npy"))
        u0, u1 = (np.load(os.path.join(d, f)) for f in ("ptoks0.npy", "ptoks1.npy"))
        assert np.array_equal(q0.view(np.uint32), q1.view(np.uint32))
        assert np.array_equal(q0.view(np.uint32), p0.view(np.uint32))
        assert np.array_equal(u0, t0) and np.array_equal(u1, t1)
        # the single GPU is the oracle's (bit-exact engine); TP follows both
        # within the per-layer bar, with the same greedy tokens
        w_ref, w_or = _worst(p0, pr), _worst(p0, po)
        print(f"{cfg_name}: TP-2 vs one GPU {w_ref:.3e}, vs oracle {w_or:.3e}; tokens {list(t0)}")
        assert w_ref < bound, w_ref
        assert w_or < bound, w_or
        assert np.array_equal(t0, tr)
        assert np.array_equal(t0, to)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_peer_allreduce_waits_are_bounded():
    """the peer all-reduce's waits end: run as rank 0 of two whose rank 1
    never runs (its flags are words nothing sets), the kernel gives up after
    1 ms per wait and records error 150; the context stays usable"""
    import ctypes
    from qwen35_b200 import lib
    L = lib.load()
    code = ctypes.c_int(-1)
    assert L.q35b_get_error(ctypes.byref(code)) == 0
    assert L.q35b_tp_selftest_timeout(1_000_000, None) == 0
    assert L.q35b_get_error(ctypes.byref(code)) == 0
    assert code.value == 150
    x = torch.ones(1024, device="cuda")
    assert float((x * 2).sum()) == 2048.0

