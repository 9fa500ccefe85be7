"""Decode throughput of the B200 backend (libq35b) on the reference's headline
metric: decode tokens/s at batch 1 / 64 (0.8B Q8_0, 4B IQ4_NL), GEMV HBM GB/s
against the measured peak.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (`value`): the 0.8B-shaped Q8_0 model,
batch 1: every sequence is prefilled with a 128-token prompt of seeded random
ids, then K greedy decode steps are timed.  Weights are seeded synthetic
(N(0, 0.02), packed on the device); 0.8 GB of weights per step is larger than
L2 (126 MB), so no flush is needed between steps.  Multi-GPU (torchrun): one
process per GPU, each an independent replica with its own sequences (weak
scaling, no collective on the data path); the timed region is bracketed by a
barrier and device syncs and the max over ranks is reported.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
PUBLISHED_08B_Q8_0_B1 = 121.84  # reference CUDA backend, RTX 4090 D (docs/cuda-bench-0.8b.md:17)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "25"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        # nvidia-smi takes longer to start than a short timed region lasts:
        # begin timing only once it is writing samples
        t0 = time.time()
        while time.time() - t0 < 5.0 and self.proc.poll() is None:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.02)
        self.skip = 0
        try:
            with open(self.path) as f:
                self.skip = sum(1 for _ in f)  # samples from before the timed region
        except OSError:
            pass

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = open(self.path).readlines()
        lines = lines[getattr(self, "skip", 0):] or lines[-1:]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def nvsmi_id(local):
    """nvidia-smi --id for this rank's device: its PCI bus id, matched through
    torch's device properties (CUDA_VISIBLE_DEVICES may renumber devices)."""
    import torch
    p = torch.cuda.get_device_properties(local)
    try:
        return "%08X:%02X:%02X.0" % (int(p.pci_domain_id), int(p.pci_bus_id), int(p.pci_device_id))
    except Exception:
        return str(local)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def make_prompts(rng, n, length, vocab):
    return [[int(t) for t in rng.integers(0, vocab, length)] for _ in range(n)]


class Run:
    """one model + engine on this rank, prefilled and ready to decode"""

    def __init__(self, cfg_name, batch, prompt_len, extra_steps, seed, gen="torch"):
        import numpy as np
        import torch

        from qwen35_b200 import model as q35
        self.torch = torch
        self.cfg = q35.CONFIGS[cfg_name]
        self.synth = q35.SyntheticModel(self.cfg, seed=seed, gen=gen)
        self.batch = batch
        self.max_seq = prompt_len + extra_steps + 8
        self.eng = q35.Engine(self.synth, n_slots=batch, max_seq=self.max_seq, max_batch=batch)
        rng = np.random.default_rng(seed + 17)
        self.prompts = make_prompts(rng, batch, prompt_len, self.cfg.vocab)
        for s in range(batch):
            self.eng.reset_slot(s)
        nxt = None
        for pos in range(prompt_len):
            nxt = self.eng.step_host([p[pos] for p in self.prompts], list(range(batch)), [pos] * batch)
        self.pos = prompt_len
        self.last = nxt
        # device-resident inputs for the timed decode loop
        L = self.eng.L
        h = self.eng.h
        i32 = torch.int32
        q35.device_view(self.eng.d_tokens, batch, i32).copy_(torch.tensor(nxt, dtype=i32))
        q35.device_view(self.eng.d_slots, batch, i32).copy_(torch.arange(batch, dtype=i32))
        q35.device_view(self.eng.d_pos, batch, i32).fill_(self.pos)
        torch.cuda.synchronize()
        self.L, self.h = L, h
        self.stream = torch.cuda.current_stream()

    def dev_steps(self, k):
        s = ctypes.c_void_p(self.stream.cuda_stream)
        for _ in range(k):
            rc = self.L.q35b_engine_step_dev(self.h, self.batch, self.max_seq, 1, s)
            assert rc == 0, rc
            rc = self.L.q35b_engine_advance(self.h, self.batch, s)
            assert rc == 0, rc
            self.pos += 1

    def host_steps(self, k, toks):
        """end-to-end through the public host-buffer API"""
        slots = list(range(self.batch))
        for _ in range(k):
            toks = self.eng.step_host(toks, slots, [self.pos] * self.batch)
            self.pos += 1
        return toks

    def launches_per_step(self):
        return int(self.L.q35b_engine_launches_per_step(self.h)) + 1  # + the feedback kernel

    def close(self):
        self.eng.close()


def time_decode(run, steps, warmup, dist):
    torch = run.torch
    run.dev_steps(warmup)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("q35_timed")
    e0.record(run.stream)
    run.dev_steps(steps)
    e1.record(run.stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    return e0.elapsed_time(e1)


def time_e2e(run, steps, warmup, dist):
    torch = run.torch
    toks = [int(t) for t in run.last]
    toks = run.host_steps(warmup, toks)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    run.host_steps(steps, toks)
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1e3
    if dist:
        dist.barrier()
    return ms


def time_prefill(cfg_name, ntok, chunk, seed, dist, wy=False, nvtx=False):
    """one prompt of ntok seeded tokens through q35b_engine_prefill (runs of
    `chunk` tokens: tensor-core projections, chunked GDN recurrence, causal
    attention), CUDA events on the stream the engine runs on"""
    import numpy as np
    import torch

    from qwen35_b200 import model as q35
    synth = q35.SyntheticModel(q35.CONFIGS[cfg_name], seed=seed)
    eng = q35.Engine(synth, n_slots=1, max_seq=ntok + 8, max_batch=chunk)
    eng.set_prefill_wy(wy)
    prompt = [int(t) for t in np.random.default_rng(seed + 5).integers(0, synth.cfg.vocab, ntok)]
    eng.reset_slot(0)
    eng.prefill(0, prompt)  # warm-up
    eng.reset_slot(0)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if nvtx:
        torch.cuda.nvtx.range_push("q35_timed")
    e0.record(st)
    eng.prefill(0, prompt, stream=st)
    e1.record(st)
    torch.cuda.synchronize()
    if nvtx:
        torch.cuda.nvtx.range_pop()
    ms = max_over_ranks(e0.elapsed_time(e1), dist)
    eng.close()
    del synth
    torch.cuda.empty_cache()
    return ms


SERVE_SEQS, SERVE_PROMPT, SERVE_GEN = 64, (64, 2048), 256


def time_serve(cfg_name, seed, dist, world, rank, wy=False):
    """continuous batching of SERVE_SEQS sequences (seeded
    prompt lengths uniform in SERVE_PROMPT, SERVE_GEN greedy tokens each)
    through q35b_serve, the sequences sharded over the ranks (every rank
    serves its share of the fixed set: strong scaling).  Returns (ms of this
    rank, prompt tokens and generated tokens of the whole set)."""
    import numpy as np
    import torch

    from qwen35_b200 import model as q35
    cfg = q35.CONFIGS[cfg_name]
    rng = np.random.default_rng(seed + 41)
    lens = rng.integers(SERVE_PROMPT[0], SERVE_PROMPT[1] + 1, SERVE_SEQS)
    prompts = [[int(t) for t in rng.integers(0, cfg.vocab, n)] for n in lens]
    mine = list(range(rank, SERVE_SEQS, world))
    synth = q35.SyntheticModel(cfg, seed=seed)
    nslot = len(mine)
    eng = q35.Engine(synth, n_slots=nslot, max_seq=SERVE_PROMPT[1] + SERVE_GEN + 8, max_batch=256)
    eng.set_prefill_wy(wy)
    eng.serve([prompts[mine[0]][:40]], [4], max_batch=nslot)  # warm-up (graphs, attributes)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    out, steps = eng.serve([prompts[i] for i in mine], [SERVE_GEN] * nslot, max_batch=nslot, stream=st)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    assert all(len(o) == SERVE_GEN for o in out)
    eng.close()
    del synth
    torch.cuda.empty_cache()
    return ms, int(sum(lens)), SERVE_SEQS * SERVE_GEN


def time_tp_decode(cfg_name, batch, ctx, steps, warmup, seed, dist, world, rank):
    """batch-`batch` greedy decode at `ctx` context, tensor-parallel over all
    `world` ranks (one engine per rank on its shard, NCCL all-reduce of the
    row-parallel partials; world 1 is the whole model on one GPU).  The
    context is synthetic: every slot steps from position `ctx` over the
    engine's zeroed KV pools and a zero GDN state, which reads and writes the
    same bytes per step as after a real prefill (values do not change the
    work) without prefilling batch x ctx prompt tokens.  With several ranks
    the steps are timed twice on one engine: the row-parallel all-reduce
    through NCCL, then through the peer all-reduce kernel.  Returns (ms for
    `steps` steps with the peer all-reduce -- NCCL's at one rank -- max over
    ranks; the NCCL form's ms or None; this rank's weight bytes)."""
    import numpy as np
    import torch

    from qwen35_b200 import model as q35
    from qwen35_b200 import tp
    cfg = q35.CONFIGS[cfg_name]
    m = q35.SyntheticModel(cfg, seed=seed)  # same seed on every rank: one model
    uid = None
    if world > 1:
        m = tp.ShardModel(m, world, rank)
        torch.cuda.empty_cache()
        uid = tp.shared_nccl_id(dist, "cuda")
    wbytes = sum(t.numel() * t.element_size() for (_, _, _, t) in m.tensors.values())
    max_seq = ctx + warmup + steps + 8
    eng = q35.Engine(m, n_slots=batch, max_seq=max_seq, max_batch=batch, tp_id=uid)
    i32 = torch.int32
    toks = np.random.default_rng(seed + 3).integers(0, cfg.vocab, batch)
    q35.device_view(eng.d_tokens, batch, i32).copy_(torch.tensor(toks, dtype=i32))
    q35.device_view(eng.d_slots, batch, i32).copy_(torch.arange(batch, dtype=i32))
    q35.device_view(eng.d_pos, batch, i32).fill_(ctx)
    st = torch.cuda.current_stream()
    s = ctypes.c_void_p(st.cuda_stream)

    def run(k):
        for _ in range(k):
            rc = eng.L.q35b_engine_step_dev(eng.h, batch, max_seq, 1, s)
            assert rc == 0, rc
            rc = eng.L.q35b_engine_advance(eng.h, batch, s)
            assert rc == 0, rc

    def timed():
        # every timed run starts at the same context (a second run on the
        # engine would otherwise step past max_seq)
        q35.device_view(eng.d_pos, batch, i32).fill_(ctx)
        run(warmup)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("q35_timed")
        e0.record(st)
        run(steps)
        e1.record(st)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1), dist)

    ms, ms_nccl = timed(), None
    if world > 1:
        ms_nccl = ms
        tp.connect_peers(dist, eng)
        ms = timed()
        dist.barrier()  # no rank unmaps or frees while another may still read it
    eng.close()  # its graphs hold NCCL work: released before the process group
    del m
    torch.cuda.empty_cache()
    return ms, ms_nccl, wbytes


def max_over_ranks(v, dist):
    """largest value over ranks (NCCL all-reduce on this rank's device)"""
    from qwen35_b200.shard import max_over_ranks as mor
    return mor(v, dist, "cuda")


def gemv_roofline(run, reps=20):
    """the dominant launch of the batch-1 step, timed alone with CUDA events:
    the tied lm_head GEMV over token_embd (vocab x hidden Q8_0, 270 MB > L2)."""
    torch = run.torch
    import numpy as np
    L = run.L
    tt, rows, cols, w = run.synth.tensors["token_embd.weight"]
    e, b = {8: (32, 34), 20: (32, 18), 12: (256, 144), 13: (256, 176), 14: (256, 210)}[tt]
    fam = 32 if e == 32 else 256
    x = torch.randn(cols, device="cuda")
    xq = torch.zeros(cols // fam * (34 if fam == 32 else 292), dtype=torch.uint8, device="cuda")
    s = ctypes.c_void_p(run.stream.cuda_stream)
    if fam == 32:
        L.q35_launch_quantize_q8_0(x.data_ptr(), xq.data_ptr(), cols // 32, s)
    else:
        L.q35_launch_quantize_q8_K(x.data_ptr(), xq.data_ptr(), cols // 256, s)
    out = torch.zeros(rows, device="cuda")
    for _ in range(3):
        assert L.q35_launch_mul_mat_vec(w.data_ptr(), xq.data_ptr(), out.data_ptr(), rows, cols, 1, tt, s) == 0
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    # NVTX range that an ncu capture of this kernel selects
    torch.cuda.nvtx.range_push("q35_roofline")
    for a, c in ev:
        a.record(run.stream)
        L.q35_launch_mul_mat_vec(w.data_ptr(), xq.data_ptr(), out.data_ptr(), rows, cols, 1, tt, s)
        c.record(run.stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = float(np.mean([a.elapsed_time(c) for a, c in ev]))
    algo = rows * (cols // e) * b + xq.numel() + rows * 4
    # the library takes the lane-per-row kernel for 16-byte-aligned rows of
    # these types, the block-splitting one otherwise
    lpr = tt in (8, 20, 12, 13) and cols % 256 == 0 and w.data_ptr() % 16 == 0
    kname = "k_gemv_lpr<1>" if lpr else "k_gemv<1>"
    return {"kernel": "%s (lm_head, %dx%d %s)" % (kname, rows, cols, {8: "Q8_0", 20: "IQ4_NL", 12: "Q4_K",
                                                                     13: "Q5_K", 14: "Q6_K"}[tt]),
            "bytes": algo, "ms": ms, "gbs": algo / (ms * 1e-3) / 1e9}


def measured_traffic(kernel):
    """DRAM bytes per launch of the roofline kernel from the committed ncu
    summary (profiles/*.json), when the summary covers this kernel"""
    p = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
    except (OSError, ValueError):
        return None
    e = d.get(kernel)
    return float(e["dram_bytes_per_launch"]) if e else None


def host_weights(lib, cfg_name, seed):
    """The headline model's weights built on the host, with no GPU and no
    libq35b: the oracle's restatement of q35b_synth_fill (same keys, same
    f32 bits) and of the reference's Q8_0 weight quantizer
    (src/quant_dequant.zig:1404-1425; the device encoder gives the same bytes),
    f32 vectors from the same host generator.  Returns (cfg, {name: (ttype,
    rows, cols, array)}, checksum), the checksum as SyntheticModel.checksum."""
    import numpy as np

    from qwen35_b200 import configs  # shapes and the host generator only: no torch, no libq35b
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as ol
    cfg = configs.CONFIGS[cfg_name]
    plan = configs.tensor_plan(cfg)
    scratch = np.empty(max(r * c for (_, _, _, r, c, init) in plan if init == "w"), np.float32)
    tensors, acc = {}, 0
    for i, (name, role, tt, rows, cols, init) in enumerate(plan):
        key, n = configs.synth_key(seed, i), rows * cols
        if init == "w":
            lib.q35o_synth_fill(key, n, configs.synth_k(0.02), ol.fp(scratch))
            e, b = ol.GEOM[tt]
            out = np.empty(n // e * b, np.uint8)
            lib.q35o_quantize_weight(tt, n, ol.fp(scratch), ol.bp(out))
        else:
            out = configs.synth_vector(key, n, init)
        tensors[name] = (tt, rows, cols, out)
        raw = out.view(np.uint8).reshape(-1)
        pad = (-raw.size) % 8
        if pad:
            raw = np.concatenate([raw, np.zeros(pad, np.uint8)])
        acc = (acc + int(raw.view("<u8").sum(dtype=np.uint64))) & (2**64 - 1)
    return cfg, tensors, acc


def _cpu_model(lib, cfg, tensors, threads, max_seq):
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as ol
    c = cfg
    ccfg = ol.Config(c.n_layers, c.full_attention_interval, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim, c.n_ff,
                     c.vocab, c.rms_eps, c.rope_freq_base, c.gdn_n_heads, c.gdn_num_k_heads, c.gdn_head_dim,
                     c.conv_kernel)
    m = lib.q35o_model_create(ctypes.byref(ccfg), max_seq, threads)
    for name, (tt, rows, cols, arr) in tensors.items():
        assert arr.flags["C_CONTIGUOUS"], name
        assert lib.q35o_model_set_tensor(m, name.encode(), tt, arr.ctypes.data, rows, cols) == 0
    assert lib.q35o_model_check(m) == 0
    return m


def cpu_model_name():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuDecode:
    """The reference's CPU path for the headline workload: the reference's own
    x86 C kernels (oracle/_ref/libq35ref.so, compiled from the reference
    sources; the C restatement when the reference tree was absent at build
    time) under the restated engine loop and row-parallel pool
    (src/pool.zig:468-533), over the same weights and the same 128-token
    prompt as the GPU arm, prefilled with all host threads."""

    def __init__(self, seed, prompt_len, max_steps):
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import numpy as np

        import oracle_lib as ol
        self.ref = os.path.exists(ol.REF_SO)
        self.lib = ol._declare(ctypes.CDLL(ol.REF_SO)) if self.ref else ol.load_oracle()
        self.cores = os.cpu_count() or 1
        self.cfg, self.tensors, self.checksum = host_weights(self.lib, "0.8b", seed)
        self.m = _cpu_model(self.lib, self.cfg, self.tensors, self.cores, prompt_len + max_steps + 8)
        prompt = make_prompts(np.random.default_rng(seed + 17), 1, prompt_len, self.cfg.vocab)[0]
        logits = None
        for i, t in enumerate(prompt):
            logits = self.lib.q35o_forward(self.m, t, i)
        self.tok = int(np.argmax(np.ctypeslib.as_array(logits, shape=(self.cfg.vocab,))))
        self.pos = prompt_len
        self.prompt_len = prompt_len
        self.buf = (ctypes.c_int * (max_steps + 1))()

    def decode(self, n, threads=None):
        """n greedy decode steps; seconds (wall, CPU)"""
        if n <= 0:
            return 0.0
        if threads is not None:
            self.lib.q35o_model_set_threads(self.m, threads)
        dt = self.lib.q35o_time_decode(self.m, self.tok, self.pos, n, self.buf)
        self.tok = int(self.buf[n - 1])
        self.pos += n
        return dt

    def kind(self):
        return "reference" if self.ref else "port"

    def what(self):
        return ("reference x86 C kernels compiled from the reference sources" if self.ref
                else "C restatement") + ", restated engine loop"

    def close(self):
        self.lib.q35o_model_destroy(self.m)


def cpu_baseline(args, seconds_target=10.0, seconds_1t=4.0):
    """bounded sample of the headline workload on this host's cores: all
    threads, then one thread (decode steps sized to about seconds_target /
    seconds_1t of CPU time)"""
    cd = CpuDecode(args.seed, args.prompt, 64 + 48)
    try:
        dt1 = cd.decode(1, cd.cores)
        n = int(max(2, min(64, seconds_target / max(dt1, 1e-3))))
        dt = cd.decode(n)
        t1 = cd.decode(1, 1)
        n1 = int(max(2, min(48, seconds_1t / max(t1, 1e-3))))
        dt_1 = cd.decode(n1)
        return {"value": n / dt, "unit": "tokens/s", "cores": cd.cores, "kind": cd.kind(),
                "value_1_thread": n1 / dt_1, "cpu": cpu_model_name(), "weights_checksum": "%016x" % cd.checksum,
                "sample": f"0.8B Q8_0 batch 1, the GPU arm's {args.prompt}-token prompt and weights, {n} timed "
                          f"decode tokens on {cd.cores} threads, then {n1} on 1 thread ({cd.what()})"}
    finally:
        cd.close()


def run_reference_arm(args, rank):
    """`--impl reference`: the reference's CPU implementation of the path on
    this box's host cores, on the headline workload (same weights, same
    128-token prompt, same decode positions as the GPU arm); rank 0 only.
    Loads no GPU code: the weights are built on the host (host_weights)."""
    if rank != 0:
        return
    cd = CpuDecode(args.seed, args.prompt, args.warmup + args.steps + 48)
    cd.decode(args.warmup)
    dt = cd.decode(args.steps)
    v = args.steps / dt
    t1 = cd.decode(1, 1)
    n1 = int(max(2, min(24, 4.0 / max(t1, 1e-3))))
    v1 = n1 / cd.decode(n1)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> int32, f32", "data": "synthetic",
        "config": CONFIG_08B,
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cd.cores, "kind": cd.kind(),
                         "value_1_thread": v1, "cpu": cpu_model_name(), "weights_checksum": "%016x" % cd.checksum,
                         "sample": f"0.8B Q8_0 batch 1, {args.prompt}-token prompt, decode positions "
                                   f"{args.prompt}..{args.prompt + args.warmup + args.steps - 1} ({args.warmup} "
                                   f"warm-up + {args.steps} timed on {cd.cores} threads; then {n1} steps on 1 "
                                   f"thread for value_1_thread), {cd.what()}"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    cd.close()


# ---------------------------------------------------------------------------
# isolated kernel sweeps (BASELINE configs 2 and 3): `--sweep gemv|gdn|all`
# ---------------------------------------------------------------------------
SWEEP_TYPES = ("Q8_0", "IQ4_NL", "Q4_K", "Q5_K", "Q6_K")
SWEEP_SHAPES = ((1024, 6144), (1024, 3584), (3584, 1024), (2048, 1024), (1024, 248320))  # [in, out]
SWEEP_TOKENS = (1, 8, 64, 512)
ROTATE_BYTES = 3 * 126 * 2**20  # distinct weight bytes cycled through: 3x L2


def _timed_loop(torch, launch, n_rot, target_ms=40.0):
    """average device time of one launch: `reps` launches cycling through
    n_rot weight copies are captured in one CUDA graph (so host-side launch
    cost does not gap the stream), the graph is replayed, and CUDA events on
    the replay stream time 3 replays.  launch(i, stream) issues launch i."""
    st = torch.cuda.current_stream()
    for i in range(3):
        launch(i % n_rot, st)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(3):
        launch(i % n_rot, st)
    e1.record(st)
    torch.cuda.synchronize()
    est = max(e0.elapsed_time(e1) / 3, 1e-3)
    reps = int(min(400, max(8, target_ms / est)))
    reps = max(reps, n_rot) if n_rot <= 400 else reps
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        cs = torch.cuda.current_stream()
        for i in range(reps):
            launch(i % n_rot, cs)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(3):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (3 * reps)
    del g
    return ms, reps


def sweep_gemv(L, hbm, only=None):
    """quantized matvec / MMQ over BASELINE config 2: seeded N(0,1) f32
    weights [in, out] encoded on the device (q35b_quantize_weight), f32
    N(0,1) activations quantized by the activation quantizer of the weight's
    family, timed through q35_launch_mul_mat_vec.  Weight copies are rotated
    so that at least 3x L2 of distinct weight bytes pass between reuses.
    only: "TYPE:INxOUT:TOKENS" runs that one case."""
    import numpy as np
    import torch
    from qwen35_b200.lib import GEOM, TT
    st = torch.cuda.current_stream()
    s = ctypes.c_void_p(st.cuda_stream)
    g = torch.Generator(device="cuda")
    shapes, types, tokens = SWEEP_SHAPES, SWEEP_TYPES, SWEEP_TOKENS
    if only is not None:  # one case, any shape and token count
        o_t, o_shape, o_tok = only.split(":")
        o_in, o_out = (int(v) for v in o_shape.split("x"))
        shapes, types, tokens = [(o_in, o_out)], [o_t], [int(o_tok)]
    for cols, rows in shapes:
        for tname in types:
            cases = [t for t in tokens if only is None or only == f"{tname}:{cols}x{rows}:{t}"]
            if not cases:
                continue
            tt = TT[tname]
            e, b = GEOM[tt]
            row_bytes = cols // e * b
            mbytes = rows * row_bytes
            pitch = (mbytes + 255) // 256 * 256
            n_rot = max(2, -(-ROTATE_BYTES // mbytes))
            g.manual_seed(1000 + rows + cols + tt)
            wf = torch.randn(rows * cols, device="cuda", generator=g)
            wq = torch.empty(n_rot * pitch, dtype=torch.uint8, device="cuda")
            assert L.q35b_quantize_weight(tt, wf.data_ptr(), wq.data_ptr(), rows * cols // e, s) == 0
            del wf
            for i in range(1, n_rot):
                wq[i * pitch:i * pitch + mbytes].copy_(wq[:mbytes])
            fam = 32 if e == 32 else 256
            abytes = cols // fam * (34 if fam == 32 else 292)
            for ntok in cases:
                x = torch.randn(ntok * cols, device="cuda", generator=g)
                xq = torch.empty(ntok * abytes, dtype=torch.uint8, device="cuda")
                quant = L.q35_launch_quantize_q8_0 if fam == 32 else L.q35_launch_quantize_q8_K
                assert quant(x.data_ptr(), xq.data_ptr(), ntok * cols // fam, s) == 0
                out = torch.empty(ntok * rows, device="cuda")
                base = wq.data_ptr()

                def launch(i, ls):
                    rc = L.q35_launch_mul_mat_vec(base + i * pitch, xq.data_ptr(), out.data_ptr(), rows, cols,
                                                  ntok, tt, ctypes.c_void_p(ls.cuda_stream))
                    assert rc == 0, rc

                ms, reps = _timed_loop(torch, launch, n_rot)
                algo = mbytes + ntok * cols * 4 + ntok * rows * 4
                ops = 2.0 * rows * cols * ntok
                # the library's routing: tensor-core MMQ from 8 tokens (MMQ_MIN_TOK)
                if ntok >= 8 and tname != "Q6_K":
                    path = "k_mmq" if tname in ("Q8_0", "IQ4_NL") else "k_mmq_kq"
                elif ntok >= 8:
                    path = "k_repack_q6k + k_mmq_kq"  # raw 210-byte rows, repacked per call
                elif tname != "Q6_K":
                    path = "k_gemv_lpr"
                else:
                    path = "k_gemv"
                line = {"sweep": "gemv", "type": tname, "in": cols, "out": rows, "tokens": ntok,
                        "kernel": path, "us": ms * 1e3, "weight_bytes": mbytes, "algo_bytes": algo,
                        "gbs": algo / (ms * 1e-3) / 1e9, "frac_hbm": algo / (ms * 1e-3) / 1e9 / hbm,
                        "int8_tops": ops / (ms * 1e-3) / 1e12, "rotated_copies": n_rot, "reps": reps}
                print(json.dumps(line), flush=True)
                del x, xq, out
            del wq
            torch.cuda.empty_cache()


WY_FORM = ("WY, 32-token chunks: Gram matrices on tcgen05 kind::tf32 (3xTF32, k_wy_gram), "
           "column-split recurrence (k_gdn_wy_cols)")


def sweep_gdn(L, hbm, only=None):
    """gated delta-net in isolation: 16 heads, dk = dv =
    128, f32 state, q/k L2-normalised, beta = sigmoid(N(0,1)), gamma =
    exp(-softplus(N(0,1))), causal conv k=4 over 6144 channels.  Decode step
    at batch 1/16/64 (conv step + delta-rule step, each sequence its own
    state); prefill of one sequence of 512/2048/8192 tokens, exact per-token
    kernel and the WY chunked form; a ragged batch of 32 sequences with
    lengths uniform in 64..4096 (one WY launch per sequence).  `only` = a
    prefill length: that WY prefill alone (a small case to profile)."""
    import numpy as np
    import torch
    st = torch.cuda.current_stream()
    s = ctypes.c_void_p(st.cuda_stream)
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    H, D, CH = 16, 128, 6144
    F = torch.nn.functional

    def qk(n):
        return F.normalize(torch.randn(n, D, device="cuda", generator=g), dim=1).contiguous()

    for B in (1, 16, 64) if only is None else ():
        nh = H * B
        # rotate states so >= 3x L2 of distinct state passes between reuses
        sbytes = nh * D * D * 4
        n_rot = max(2, -(-ROTATE_BYTES // sbytes))
        state = torch.randn(n_rot, nh * D * D, device="cuda", generator=g) * 0.01
        k, q, v = qk(nh), qk(nh), torch.randn(nh, D, device="cuda", generator=g)
        q.mul_(1.0 / np.sqrt(D))
        gamma = torch.exp(-F.softplus(torch.randn(nh, device="cuda", generator=g)))
        beta = torch.sigmoid(torch.randn(nh, device="cuda", generator=g))
        km, delta, out = (torch.empty(nh, D, device="cuda") for _ in range(3))
        conv = torch.randn(n_rot, B * CH * 3, device="cuda", generator=g)
        wconv = torch.randn(B * CH * 4, device="cuda", generator=g)
        y = torch.randn(B * CH, device="cuda", generator=g)

        def launch(i, ls):
            s = ctypes.c_void_p(ls.cuda_stream)
            assert L.q35_launch_conv_step(conv[i].data_ptr(), y.data_ptr(), wconv.data_ptr(), B * CH, s) == 0
            assert L.q35_launch_gdn_step_rows(state[i].data_ptr(), D * D, k.data_ptr(), D, v.data_ptr(), D,
                                              q.data_ptr(), D, km.data_ptr(), delta.data_ptr(), out.data_ptr(),
                                              gamma.data_ptr(), beta.data_ptr(), nh, nh, D, D, s) == 0

        ms, reps = _timed_loop(torch, launch, n_rot)
        algo = 2 * sbytes + B * CH * (3 * 2 + 4 + 2) * 4 + nh * D * 4 * 6
        print(json.dumps({"sweep": "gdn", "mode": "decode", "batch": B, "heads": nh, "us": ms * 1e3,
                          "algo_bytes": algo, "gbs": algo / (ms * 1e-3) / 1e9,
                          "frac_hbm": algo / (ms * 1e-3) / 1e9 / hbm, "launches": 2, "rotated_copies": n_rot,
                          "reps": reps}), flush=True)
        del state, conv
        torch.cuda.empty_cache()

    def prefill(rows, wy, state):
        k, q, v = qk(rows * H).view(rows, H * D), qk(rows * H).view(rows, H * D), \
            torch.randn(rows, H * D, device="cuda", generator=g)
        q.mul_(1.0 / np.sqrt(D))
        gamma = torch.exp(-F.softplus(torch.randn(rows, H, device="cuda", generator=g)))
        beta = torch.sigmoid(torch.randn(rows, H, device="cuda", generator=g))
        km, delta, out = (torch.empty(rows, H * D, device="cuda") for _ in range(3))
        fn = L.q35_launch_gdn_step_wy if wy else L.q35_launch_gdn_step_rows_chunk
        keep = (k, q, v, gamma, beta, km, delta, out)

        def launch(_i, ls):
            assert fn(state.data_ptr(), D * D, k.data_ptr(), H * D, v.data_ptr(), H * D, q.data_ptr(), H * D,
                      km.data_ptr(), H * D, delta.data_ptr(), H * D, out.data_ptr(), H * D, gamma.data_ptr(), H,
                      beta.data_ptr(), H, H, H, D, D, rows, ctypes.c_void_p(ls.cuda_stream)) == 0
        return launch, keep

    state = torch.zeros(H * D * D, device="cuda")
    for rows in (512, 2048, 8192) if only is None else (int(only),):
        for wy in (False, True) if only is None else (True,):
            launch, keep = prefill(rows, wy, state)
            ms, reps = _timed_loop(torch, launch, 1, target_ms=100.0)
            print(json.dumps({"sweep": "gdn", "mode": "prefill", "form": WY_FORM if wy else
                              "exact per-token", "seq_len": rows, "us": ms * 1e3,
                              "tokens_per_s": rows / (ms * 1e-3), "reps": reps}), flush=True)
            del keep
    if only is not None:
        return
    # ragged: 32 sequences, lengths U[64, 4096], each its own state
    lens = np.random.default_rng(3).integers(64, 4097, 32)
    states = torch.zeros(32, H * D * D, device="cuda")
    runs = [prefill(int(n), True, states[i]) for i, n in enumerate(lens)]

    def ragged(_i, ls):
        for launch, _k in runs:
            launch(0, ls)

    ms, reps = _timed_loop(torch, ragged, 1, target_ms=200.0)
    print(json.dumps({"sweep": "gdn", "mode": "ragged prefill", "form": WY_FORM, "sequences": 32,
                      "tokens": int(lens.sum()), "us": ms * 1e3, "tokens_per_s": float(lens.sum()) / (ms * 1e-3),
                      "launches": 32, "reps": reps}), flush=True)


METRIC = "decode tokens/s at batch 1/64 (0.8B Q8_0, 4B IQ4_NL); GEMV HBM GB/s vs peak"
CONFIG_08B = {"workload": "0.8B-Q8_0 greedy decode, batch 1, 128-token prompt (BASELINE config 1)",
              "model": "qwen3.5-0.8b-q8_0 (24 layers LLLFx6, hidden 1024, ffn 3584, vocab 248320)",
              "global_batch": 1, "seq_len": 128, "parallelism": "replicas (sequence-sharded, no collective)",
              "l2": "weights 0.80 GB per step > 126 MB L2: no flush needed"}


# the batched-decode matrices of the 4B and 27B configs on the tensor-core
# MMQ, as the engine lays them out (Q6_K repacked to 224-byte blocks):
# (type, in, out)
MMQ_SWEEP = (("Q4_K", 5120, 17408), ("Q4_K", 17408, 5120), ("Q6_K_P", 5120, 248320),
             ("Q5_K", 9216, 2560), ("Q6_K_P", 2560, 248320))
MMQ_SWEEP_TOKENS = (16, 32, 64)


def sweep_mmq(L, hbm, only=None):
    """k_mmq_kq over MMQ_SWEEP at batch 16 / 32 / 64 through
    q35b_mul_mat_vec_multi (the engine's entry), weights rotated past 3x L2.
    only: "TYPE:INxOUT:TOKENS" runs that one case."""
    import torch
    from qwen35_b200.lib import GEOM, TT
    st = torch.cuda.current_stream()
    s = ctypes.c_void_p(st.cuda_stream)
    g = torch.Generator(device="cuda")
    for tname, cols, rows in MMQ_SWEEP:
        padded = tname == "Q6_K_P"
        tt = TT["Q6_K"] if padded else TT[tname]
        code = 0x1000 + tt if padded else tt
        e, b = GEOM[tt]
        nblk = rows * cols // e
        bb = 224 if padded else b
        mbytes = nblk * bb
        cases = [t for t in MMQ_SWEEP_TOKENS if only is None or only == f"{tname}:{cols}x{rows}:{t}"]
        if not cases:
            continue
        pitch = (mbytes + 255) // 256 * 256
        n_rot = max(2, -(-ROTATE_BYTES // mbytes))
        g.manual_seed(2000 + rows + cols + tt)
        wf = torch.randn(rows * cols, device="cuda", generator=g)
        raw = torch.empty(nblk * b, dtype=torch.uint8, device="cuda")
        assert L.q35b_quantize_weight(tt, wf.data_ptr(), raw.data_ptr(), nblk, s) == 0
        del wf
        wq = torch.zeros(n_rot * pitch, dtype=torch.uint8, device="cuda")
        first = wq[:mbytes].view(nblk, bb)
        first[:, :b].copy_(raw.view(nblk, b))
        del raw
        for i in range(1, n_rot):
            wq[i * pitch:i * pitch + mbytes].copy_(wq[:mbytes])
        for ntok in cases:
            x = torch.randn(ntok * cols, device="cuda", generator=g)
            xq = torch.empty(ntok * (cols // 256) * 292, dtype=torch.uint8, device="cuda")
            assert L.q35_launch_quantize_q8_K(x.data_ptr(), xq.data_ptr(), ntok * cols // 256, s) == 0
            out = torch.empty(ntok * rows, device="cuda")
            base = wq.data_ptr()
            T, R, LD, M = (ctypes.c_int * 1)(code), (ctypes.c_longlong * 1)(rows), \
                (ctypes.c_longlong * 1)(rows), (ctypes.c_int * 1)(0)
            O = (ctypes.c_void_p * 1)(out.data_ptr())

            def launch(i, ls):
                W = (ctypes.c_void_p * 1)(base + i * pitch)
                rc = L.q35b_mul_mat_vec_multi(1, W, T, R, O, LD, M, xq.data_ptr(), cols, ntok,
                                              ctypes.c_void_p(ls.cuda_stream))
                assert rc == 0, rc

            # split-K through q35b_mul_mat_vec_multi_ws (the engine passes its
            # own workspace the same way); used only where the rule allows
            work = torch.empty((cols // 256) * ntok * rows, dtype=torch.float32, device="cuda")

            def launch_ws(i, ls):
                W = (ctypes.c_void_p * 1)(base + i * pitch)
                rc = L.q35b_mul_mat_vec_multi_ws(1, W, T, R, O, LD, M, xq.data_ptr(), cols, ntok,
                                                 work.data_ptr(), work.numel() * 4, ctypes.c_void_p(ls.cuda_stream))
                assert rc == 0, rc

            for split, fn in ((False, launch), (True, launch_ws)):
                ms, reps = _timed_loop(torch, fn, n_rot)
                algo = mbytes + ntok * (cols // 256) * 292 + ntok * rows * 4
                line = {"sweep": "mmq", "type": tname, "in": cols, "out": rows, "tokens": ntok,
                        "kernel": "k_mmq_kq" + (" + k_mmq_term_sum (workspace given)" if split else ""),
                        "us": ms * 1e3, "weight_bytes": mbytes, "algo_bytes": algo,
                        "gbs": algo / (ms * 1e-3) / 1e9, "frac_hbm": algo / (ms * 1e-3) / 1e9 / hbm,
                        "int8_tops": 2.0 * rows * cols * ntok / (ms * 1e-3) / 1e12, "rotated_copies": n_rot,
                        "reps": reps}
                print(json.dumps(line), flush=True)
            del x, xq, out, work
        del wq, first
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--no-variants", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--sweep", choices=["gemv", "gdn", "mmq", "prefill", "decode", "all"], default=None,
                    help="isolated kernel sweeps (BASELINE configs 2 / 3; mmq: the 4B / 27B batched-decode "
                         "matrices) or one engine workload alone (prefill, decode; inside the NVTX range "
                         "q35_timed) instead of the decode bench")
    ap.add_argument("--sweep-case", default=None, help="--sweep gemv|mmq: one case, TYPE:INxOUT:TOKENS; --sweep gdn: one WY "
                    "prefill length; --sweep prefill: MODEL:TOKENS:CHUNK[:exact]; --sweep decode: MODEL:BATCH")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # a CPU run: no process group, no CUDA context, no libq35b
        run_reference_arm(args, rank)
        return
    import torch
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        dist = tdist
    else:
        torch.cuda.set_device(0)

    from qwen35_b200.build import build
    if rank == 0:
        build()
    if dist:
        dist.barrier()
    pk, pk_kind = peaks()
    if args.sweep:
        from qwen35_b200 import lib as qlib
        L = qlib.load()
        hbm = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
        if args.sweep in ("gemv", "all"):
            sweep_gemv(L, hbm, args.sweep_case)
        if args.sweep in ("gdn", "all"):
            sweep_gdn(L, hbm, args.sweep_case)
        if args.sweep in ("mmq", "all"):
            sweep_mmq(L, hbm, args.sweep_case)
        if args.sweep == "decode":
            # one model's batched decode steps alone (the variants' timing,
            # inside the NVTX range q35_timed for a launch list)
            f = (args.sweep_case or "4b:64").split(":")
            r = Run(f[0], int(f[1]), args.prompt, 2 * (args.warmup + args.steps) + 8, seed=args.seed)
            vms = time_decode(r, args.steps, args.warmup, None)
            print(json.dumps({"sweep": "decode", "model": r.cfg.name, "batch": r.batch, "steps": args.steps,
                              "ms_per_step": vms / args.steps,
                              "value": r.batch * args.steps / (vms * 1e-3), "unit": "tokens/s"}))
            r.close()
        if args.sweep == "prefill":
            # one engine prefill (the prefill variants' timing, inside the NVTX
            # range q35_timed for a launch list)
            f = (args.sweep_case or "4b:512:256").split(":")
            wy = not (len(f) > 3 and f[3] == "exact")
            pms = time_prefill(f[0], int(f[1]), int(f[2]), args.seed, None, wy, nvtx=True)
            print(json.dumps({"sweep": "prefill", "model": f[0], "prefill_tokens": int(f[1]), "chunk": int(f[2]),
                              "gdn": "chunked WY" if wy else "per-token (exact)", "ms": pms,
                              "value": int(f[1]) / (pms * 1e-3), "unit": "prefill tokens/s"}))
        return
    extra = 2 * (args.warmup + args.steps) + 8

    # ---------------- headline: 0.8B Q8_0, batch 1 ----------------
    run = Run("0.8b", 1, args.prompt, extra, seed=args.seed + rank, gen="synth")
    clocks = ClockSampler(nvsmi_id(local))
    clocks.start()
    ms = time_decode(run, args.steps, args.warmup, dist)
    clk = clocks.stop()
    ms = max_over_ranks(ms, dist)
    e2e_ms = max_over_ranks(time_e2e(run, args.steps, args.warmup, dist), dist)
    launches = run.launches_per_step() * args.steps
    wsum = run.synth.checksum()
    roof = gemv_roofline(run) if rank == 0 else None
    value = world * run.batch * args.steps / (ms * 1e-3)
    e2e_val = world * run.batch * args.steps / (e2e_ms * 1e-3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(args)
    run.close()
    del run
    torch.cuda.empty_cache()

    variants = []
    if not args.no_variants:
        for cfg_name, batch in (("0.8b", 64), ("4b", 1), ("4b", 64)):
            ksteps = min(args.steps, 32)
            r = Run(cfg_name, batch, args.prompt, 2 * (args.warmup + ksteps) + 8, seed=args.seed + rank)
            vms = max_over_ranks(time_decode(r, ksteps, args.warmup, dist), dist)
            variants.append({"model": r.cfg.name, "batch_per_gpu": batch, "steps": ksteps,
                             "ms_per_step": vms / ksteps,
                             "value": world * batch * ksteps / (vms * 1e-3), "unit": "tokens/s"})
            r.close()
            del r
            torch.cuda.empty_cache()
        # 27B tensor-parallel over every rank of this run (strong scaling: the
        # batch of 32 sequences at 4096 context is fixed)
        ksteps = min(args.steps, 16)
        tms, tms_nccl, wb = time_tp_decode("27b", 32, 4096, ksteps, args.warmup, args.seed, dist, world, rank)
        tpv = {"model": "qwen3.5-27b-q4_k", "tp": world, "batch": 32, "context": 4096,
               "context_fill": "synthetic (zero KV / GDN state, positions at 4096)",
               "steps": ksteps, "ms_per_step": tms / ksteps, "value": 32 * ksteps / (tms * 1e-3),
               "unit": "tokens/s", "scaling": "strong", "weight_bytes_per_rank": wb}
        if tms_nccl is not None:
            tpv["allreduce"] = "peer (k_tp_allreduce_add: NVLink peer loads / stores, residual add fused)"
            tpv["nccl_ms_per_step"] = tms_nccl / ksteps
            tpv["nccl_value"] = 32 * ksteps / (tms_nccl * 1e-3)
        variants.append(tpv)
        for wy in (False, True):
            sms, sp, sg = time_serve("4b", args.seed, dist, world, rank, wy)
            sms = max_over_ranks(sms, dist)
            variants.append({"model": "qwen3.5-4b-mixed", "workload": "continuous batching (BASELINE config 4): %d "
                             "sequences, prompts uniform in %d..%d tokens, %d greedy tokens each, sharded by "
                             "sequence over the ranks" % (SERVE_SEQS, SERVE_PROMPT[0], SERVE_PROMPT[1], SERVE_GEN),
                             "gdn": "chunked WY for prompt runs >= 16 tokens" if wy else "per-token (exact)",
                             "ms": sms, "value": SERVE_SEQS * SERVE_GEN / (sms * 1e-3), "unit": "generated tokens/s",
                             "prompt_tokens": sp, "generated_tokens": sg,
                             "total_tokens_per_s": (sp + sg) / (sms * 1e-3),
                             "scaling": "strong"})
        for cfg_name, ntok, chunk in (("0.8b", 512, 256), ("4b", 512, 256)):
            for wy in (False, True):
                pms = time_prefill(cfg_name, ntok, chunk, args.seed + rank, dist, wy)
                variants.append({"model": cfg_name, "prefill_tokens": ntok, "chunk": chunk,
                                 "gdn": "chunked WY" if wy else "per-token (exact)", "ms": pms,
                                 "value": world * ntok / (pms * 1e-3), "unit": "prefill tokens/s"})

    if rank == 0:
        hbm = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / world / PUBLISHED_08B_Q8_0_B1,
            "dtype": "int8 x int8 -> int32 block dots, f32 fold/state/KV", "data": "synthetic",
            "config": dict(CONFIG_08B, global_batch=world),
            "clocks": clk,
            "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": 12 * world,
                    "d2h_bytes_per_step": 4 * world},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "achieved": roof["gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": roof["gbs"] / hbm, "traffic": measured_traffic(roof["kernel"]),
                         "kernel": roof["kernel"],
                         "algorithmic_bytes_per_launch": roof["bytes"], "avg_launch_ms": roof["ms"],
                         "peak_source": f"{pk_kind} (MEASURED_PEAKS.json hbm_gbs)" if pk_kind == "measured"
                         else "fallback 6.65 TB/s"},
            "cpu_baseline": cpu,
            "weights_checksum": "%016x" % wsum,
            "variants": variants,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
