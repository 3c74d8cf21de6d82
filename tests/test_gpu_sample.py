"""Device sampling (aion_set_sampler) against its CPU restatement
(oracle/sample_ref.py) on the same logits: every draw must be the same
token.  The logits come from the device after each step
(aion_read_logits / aion_decode_batch), so the comparison is exact; the
stream is also checked against the oracle's forward of the sampled tokens
(logits within 1e-4 of the largest).  A multi-step launch must draw what
step-by-step launches draw, and top_k = 1 must give the greedy stream."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import sample_ref as S

pytestmark = pytest.mark.gpu

SP = dict(temperature=0.9, top_p=0.9, top_k=50, seed=123)


def test_batch1_draws_match_restatement(cuda, oracle, tiny_path):
    import aion_b200 as A
    n = 24
    with A.Model(tiny_path) as m:
        m.set_sampler(**SP)
        m.decode_async(1, 1, 0)
        logits = [m.read_logits()]
        for i in range(1, n):
            m.decode_async(1)
            logits.append(m.read_logits())
        toks = m.tokens(n)
        m.reset()
        m.decode_async(n, 1, 0)              # the same draws from one launch
        assert m.tokens(n) == toks
    om = oracle.open(tiny_path)
    for i in range(n - 1):
        assert toks[i + 1] == S.sample(logits[i], SP["temperature"], SP["top_p"], SP["top_k"], SP["seed"], 0, i), i
        want = om.forward(toks[i], i)
        assert np.abs(logits[i] - want).max() <= 1e-4 * np.abs(want).max()
    om.close()
    assert len(set(toks)) > 4                # it does sample


def test_top_k_one_is_greedy(cuda, tiny_path, golden_tiny):
    import aion_b200 as A
    with A.Model(tiny_path) as m:
        m.set_sampler(temperature=1.3, top_k=1, seed=9)
        toks, _ = m.generate(64)
        m.set_sampler()                      # back to greedy
        g, _ = m.generate(64)
    assert toks == golden_tiny["w4a16_tokens"][:64] == g


def test_batch_draws_match_restatement(cuda, tiny_path):
    import aion_b200 as A
    nb, steps = 6, 10
    first = [1, 7, 100, 5000, 31000, 2]
    with A.Model(tiny_path, max_batch=8) as m:
        m.set_sampler(**SP)
        toks, pos = list(first), [0] * nb
        rows = [list(first)]
        for s in range(steps):
            t, lg = m.decode_batch(toks, pos, 1, want_logits=True)
            for b in range(nb):
                assert t[1, b] == S.sample(lg[b], SP["temperature"], SP["top_p"], SP["top_k"], SP["seed"], b,
                                           pos[b]), (s, b)
            toks = list(t[1])
            pos = [p + 1 for p in pos]
            rows.append(toks)
        whole, _ = m.decode_batch(first, [0] * nb, steps)
    assert whole.tolist() == rows


def test_sampler_rejects_bad_parameters(cuda, tiny_path):
    import aion_b200 as A
    with A.Model(tiny_path) as m:
        for kw in (dict(temperature=1.0, top_p=0.0), dict(temperature=1.0, top_p=1.5),
                   dict(temperature=1.0, top_k=-1), dict(temperature=float("inf"))):
            with pytest.raises(A.AionError):
                m.set_sampler(**kw)
