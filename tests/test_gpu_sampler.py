"""The device sampler against the oracle's restatement of the reference's
Sampler.sample (src/sampler.zig:67-190) on the same logits and seeds: the
same token and the same PRNG state after every draw.

The oracle is the build with correctly rounded exp (the device's
arithmetic), so both sides sum the same f32 terms; the device sums them in a
fixed chunked order and finds the top-p cut from exact integer masses, which
could move a draw only if the coin fell within ~1e-16 (f64 sums) or ~1e-8
(top-p masses) of a cumulative boundary."""
import ctypes

import numpy as np
import pytest
import torch

from oracle_lib import OracleSampler, load_oracle, oracle_forward, oracle_model

pytestmark = pytest.mark.gpu

S = None


@pytest.fixture(scope="module")
def L():
    from qwen35_b200 import lib
    return lib.load()


@pytest.fixture(scope="module")
def O():
    return load_oracle(cr_exp=True)


def ok(rc):
    assert rc == 0, f"cuda error {rc}"


def ctl_block(temperature, top_k, top_p, state, n):
    b = np.zeros(16, np.int32)
    b[0] = n
    b[1] = np.float32(temperature).view(np.int32)
    b[2] = top_k
    b[3] = np.float32(top_p).view(np.int32)
    b[4] = np.uint32(state & 0xFFFFFFFF).view(np.int32)
    b[5] = np.uint32(state >> 32).view(np.int32)
    return b


def state_of(blk, out=True):
    lo, hi = (blk[7], blk[8]) if out else (blk[4], blk[5])
    return int(np.int32(lo).view(np.uint32)) | (int(np.int32(hi).view(np.uint32)) << 32)


def _logit_cases(rng):
    n = 248320
    yield "vocab N(0,3)", (rng.standard_normal(n) * 3).astype(np.float32)
    x = (rng.standard_normal(n) * 2).astype(np.float32)
    x[rng.choice(n, 5, replace=False)] = 14.0  # a few dominant ties
    yield "vocab, tied peaks", x
    yield "small, rounded (ties)", np.round(rng.standard_normal(1000) * 2, 1).astype(np.float32)
    x = rng.standard_normal(3001).astype(np.float32)
    x[::7] = -np.inf
    yield "-inf entries", x
    yield "all equal", np.full(517, 0.25, np.float32)
    yield "n = 1", np.array([3.0], np.float32)


PARAMS = [(0.0, 0, 0.0), (1.0, 0, 0.0), (0.7, 40, 0.0), (1.3, 0, 0.9), (0.8, 50, 0.95), (1.0, 1, 0.0),
          (2.0, 0, 0.3), (1.0, 5000, 0.5)]


def test_sample_matches_oracle(L, O):
    """q35_launch_sample (the reference's single-row entry point): token and
    PRNG state out, every case x parameter set x 3 seeds, and the greedy
    branch's first-index tie rule"""
    rng = np.random.default_rng(0)
    d_ctl = torch.zeros(16, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(16, dtype=torch.int32, device="cuda")
    checked = 0
    for name, x in _logit_cases(rng):
        dx = torch.from_numpy(x).cuda()
        for (t, k, p) in PARAMS:
            for seed in (1, 12345, 2**63 + 77):
                blk = ctl_block(t, k, p, seed, x.size)
                d_ctl.copy_(torch.from_numpy(blk))
                ok(L.q35_launch_sample(dx.data_ptr(), x.size, d_ctl.data_ptr(), scratch.data_ptr(), S))
                got = d_ctl.cpu().numpy()
                ref = OracleSampler(O, t, k, p, seed)
                want = ref.sample(x)
                assert int(got[6]) == want, (name, t, k, p, seed)
                if t > 0:
                    assert state_of(got) == ref.state.value, (name, t, k, p, seed)
                checked += 1
    assert checked == 6 * len(PARAMS) * 3


def test_stream_of_draws_and_rows(L, O):
    """q35b_sample_rows over 6 rows, each with its own parameters and seed,
    advancing the state in place: 25 successive calls follow 6 oracle
    samplers draw for draw"""
    rng = np.random.default_rng(1)
    rows, n = 6, 50000
    x = (rng.standard_normal((rows, n)) * 2.5).astype(np.float32)
    params = [(1.0, 0, 0.0), (0.6, 20, 0.0), (1.2, 0, 0.8), (0.9, 100, 0.9), (0.0, 0, 0.0), (1.0, 3, 0.0)]
    ctl = np.stack([ctl_block(t, k, p, 1000 + r, n) for r, (t, k, p) in enumerate(params)])
    d_ctl = torch.from_numpy(ctl).cuda()
    refs = [OracleSampler(O, t, k, p, 1000 + r) for r, (t, k, p) in enumerate(params)]
    dx = torch.from_numpy(x).cuda()
    toks = torch.zeros(rows, dtype=torch.int32, device="cuda")
    for step in range(25):
        ok(L.q35b_sample_rows(dx.data_ptr(), n, n, rows, d_ctl.data_ptr(), 16, 1, toks.data_ptr(), S))
        got = toks.cpu().numpy()
        for r in range(rows):
            assert int(got[r]) == refs[r].sample(x[r]), (step, r)
        blk = d_ctl.cpu().numpy()
        for r in range(rows):
            if params[r][0] > 0:
                assert state_of(blk[r], out=False) == refs[r].state.value
        x[:, step % n] += 0.5  # the logits move between calls
        dx.copy_(torch.from_numpy(x))


def test_sample_rejects_bad_input(L):
    d = torch.zeros(16, dtype=torch.int32, device="cuda")
    x = torch.zeros(10, device="cuda")
    assert L.q35_launch_sample(x.data_ptr(), 0, d.data_ptr(), d.data_ptr(), S) != 0
    assert L.q35_launch_sample(x.data_ptr(), 300000, d.data_ptr(), d.data_ptr(), S) != 0
    assert L.q35b_sample_rows(x.data_ptr(), 10, 10, 1, d.data_ptr(), 8, 0, None, S) != 0


def test_engine_sampling_matches_oracle(O):
    """the engine with sampling on: two sequences decode side by side in one
    step (one with temperature / top-k / top-p, one greedy), every draw made
    inside the step from the slot's device-resident state; the oracle engine
    (correctly rounded exp) and oracle samplers give the same tokens"""
    from qwen35_b200 import model as q35
    cfg = q35.CONFIGS["tiny-mixed"]
    synth = q35.SyntheticModel(cfg, seed=17)
    eng = q35.Engine(synth, n_slots=2, max_seq=48, max_batch=2)
    eng.set_sampling(True)
    samplers = [(1.1, 30, 0.9, 4242), (0.0, 0, 0.0, 0)]
    for slot, (t, k, p, seed) in enumerate(samplers):
        eng.reset_slot(slot)
        eng.set_sampler(slot, t, k, p, seed)
    oracles = []
    for slot, (t, k, p, seed) in enumerate(samplers):
        Om, m, keep = oracle_model(synth, threads=4, max_seq=48, cr_exp=True)
        oracles.append((m, keep, OracleSampler(Om, t, k, p, seed)))
    rng = np.random.default_rng(17)
    prompts = [[int(v) for v in rng.integers(0, cfg.vocab, 5)] for _ in samplers]
    toks_g = [[], []]
    toks_c = [[], []]
    cur = [prompts[0][0], prompts[1][0]]
    for pos in range(24):
        nxt = eng.step_host(cur, [0, 1], [pos, pos])
        for s in range(2):
            m, keep, smp = oracles[s]
            lc = oracle_forward(Om, m, cur[s], pos, cfg.vocab)
            tc = smp.sample(lc)
            toks_g[s].append(nxt[s])
            toks_c[s].append(tc)
            cur[s] = prompts[s][pos + 1] if pos + 1 < len(prompts[s]) else nxt[s]
        assert nxt == [toks_c[0][-1], toks_c[1][-1]], pos
    for m, keep, _ in oracles:
        Om.q35o_model_destroy(m)
    eng.close()
