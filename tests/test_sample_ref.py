"""The CPU restatement of the device sampler (oracle/sample_ref.py): its
limits (top_k = 1 and a near-zero temperature give the argmax), its
filters (top-k, top-p never draw outside the kept set) and its
distribution (empirical frequencies within 5 sigma of the softmax)."""
from __future__ import annotations

import numpy as np

from oracle import sample_ref as S


def test_limits_are_greedy():
    rng = np.random.default_rng(1)
    for i in range(20):
        lg = rng.standard_normal(3000).astype(np.float32)
        am = int(np.argmax(lg))
        assert S.sample(lg, 0.8, 1.0, 1, seed=i, pos=i) == am
        assert S.sample(lg, 1e-3, 1.0, 0, seed=i, pos=i) == am


def test_filters_keep_only_the_top():
    p = np.array([0.5, 0.3, 0.15, 0.05], np.float64)
    lg = np.log(p).astype(np.float32)
    got = {S.sample(lg, 1.0, 0.75, 0, seed=3, pos=k) for k in range(400)}
    assert got <= {0, 1} and len(got) == 2
    got = {S.sample(lg, 1.0, 1.0, 2, seed=4, pos=k) for k in range(400)}
    assert got <= {0, 1} and len(got) == 2
    got = {S.sample(lg, 1.0, 1.0, 3, seed=5, pos=k) for k in range(400)}
    assert got <= {0, 1, 2} and 2 in got


def test_distribution_matches_softmax():
    lg = np.array([1.0, 0.5, 0.0, -0.5, -1.0, 2.0, 0.25, -2.0], np.float32)
    T = 0.9
    n = 4000
    counts = np.zeros(lg.size)
    for k in range(n):
        counts[S.sample(lg, T, 1.0, 0, seed=11, stream=2, pos=k)] += 1
    e = np.exp((lg - lg.max()) / T)
    prob = e / e.sum()
    sigma = np.sqrt(n * prob * (1 - prob))
    assert np.all(np.abs(counts - n * prob) <= 5 * sigma + 1)


def test_draws_are_functions_of_seed_stream_position():
    lg = np.random.default_rng(2).standard_normal(500).astype(np.float32)
    a = [S.sample(lg, 1.0, 0.95, 0, seed=7, stream=s, pos=p) for s in range(3) for p in range(5)]
    b = [S.sample(lg, 1.0, 0.95, 0, seed=7, stream=s, pos=p) for s in range(3) for p in range(5)]
    assert a == b
    c = [S.sample(lg, 1.0, 0.95, 0, seed=8, stream=s, pos=p) for s in range(3) for p in range(5)]
    assert a != c
