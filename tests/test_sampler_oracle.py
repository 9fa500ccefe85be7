"""The oracle's sampler (q35o_sample) pinned against the reference's own
sampler tests (src/sampler.zig:263-411), restated: greedy ties, determinism of
the stream, the top-k tail exclusion, the k-th largest value with float ties,
top-p's nucleus and its threshold against a sorted cumulative prefix, top-p
off values, k >= n.  CPU only."""
import numpy as np
import pytest

from oracle_lib import OracleSampler, fp, load_oracle


@pytest.fixture(scope="module")
def L():
    return load_oracle()


def test_greedy_picks_max_ties_low_index(L):  # sampler.zig:263-267
    s = OracleSampler(L, temperature=0.0, seed=1)
    assert s.sample([1.0, 3.0, 2.0, 3.0, -1.0]) == 1


def test_temperature_stream_deterministic(L):  # sampler.zig:269-287
    lg = [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8]
    a, b = OracleSampler(L, 0.8, seed=42), OracleSampler(L, 0.8, seed=42)
    assert [a.sample(lg) for _ in range(20)] == [b.sample(lg) for _ in range(20)]


def test_top_k_excludes_tail(L):  # sampler.zig:289-299
    s = OracleSampler(L, 1.0, top_k=1, seed=7)
    assert all(s.sample([0.0, 0.0, 0.0, 0.0, 10.0, 0.0]) == 4 for _ in range(200))


@pytest.mark.parametrize("vals,ranks", [
    ([5, 1, 9, 3, 7, 2, 8, 4, 6], {0: 9, 1: 8, 7: 2, 8: 1}),   # sampler.zig:301-318
    ([3, 1, 3, 2, 3, 0, 3], {0: 3, 3: 3, 4: 2, 6: 0}),          # sampler.zig:320-333
])
def test_kth_largest(L, vals, ranks):
    for r, want in ranks.items():
        a = np.array(vals, np.float32)
        assert L.q35o_kth_largest(fp(a), a.size, r) == want


def test_top_p_keeps_nucleus(L):  # sampler.zig:335-347
    lg = [-20, -20, -20, -20, 10, 10, 10, -20, -20]
    s = OracleSampler(L, 1.0, top_p=0.5, seed=11)
    assert all(s.sample(lg) in (4, 5, 6) for _ in range(300))


def test_top_p_threshold_is_sorted_cumulative_prefix(L):  # sampler.zig:349-394
    lg = np.array([-3, -1, 0.5, 0.5, 2, 2, 2, -1, 4, 0.1, -0.2, 1], np.float32)
    mx = lg.max()
    order = np.sort(lg)[::-1]
    total = float(np.exp((lg - mx).astype(np.float64)).sum())
    for p in (0.1, 0.25, 0.5, 0.75, 0.9):
        acc, want = 0.0, order[-1]
        for v in order:
            acc += float(np.exp(np.float64(v - mx)))
            if acc >= total * p:
                want = v
                break
        s = OracleSampler(L, 1.0, top_p=p, seed=5)
        drawn = [lg[s.sample(lg)] for _ in range(400)]
        assert min(drawn) >= want


def test_top_p_off_values_match_no_top_p(L):  # sampler.zig:396-408
    lg = [0.3, -1.2, 2.0, 0.4, 1.1, -0.6, 0.0, 0.9]
    for p in (0.0, -1.0, 1.0, 2.0):
        a, b = OracleSampler(L, 0.9, seed=21), OracleSampler(L, 0.9, top_p=p, seed=21)
        assert [a.sample(lg) for _ in range(50)] == [b.sample(lg) for _ in range(50)]


def test_top_k_at_least_n_is_pure_temperature(L):  # sampler.zig:410-414
    lg = [0.0, 1.0, 2.0, 3.0]
    a, b = OracleSampler(L, 1.0, top_k=100, seed=3), OracleSampler(L, 1.0, seed=3)
    assert [a.sample(lg) for _ in range(50)] == [b.sample(lg) for _ in range(50)]


def test_draw_frequencies_follow_softmax(L):
    """the draw walks cumulative softmax mass: frequencies over many draws
    match exp(x / T) / sum (a check of the restatement, not a reference test)"""
    lg = np.array([0.0, 1.0, 2.0, 0.5], np.float32)
    s = OracleSampler(L, 0.7, seed=99)
    cnt = np.bincount([s.sample(lg) for _ in range(20000)], minlength=4) / 20000
    p = np.exp(lg / 0.7) / np.exp(lg / 0.7).sum()
    assert np.abs(cnt - p).max() < 0.015
