"""Lock-step batched decode (aion_decode_batch) against the oracle.

Each sequence of a batch is checked on its own against the oracle's
token-by-token forward (src/kernel_simd.c:1014-1169, greedy pick of
:1236-1243): the greedy tokens must be identical and the last step's logits
within 1e-4 of the largest logit (24-bit fixed-point activations per group
of 32, fp32 accumulate; the measured gap is about 1e-6).  Batches of 5, 17
and 32 sequences cover one, three and four blocks of eight with padding;
sequences continue from KV caches of different lengths written by
aion_prefill (the prefill's own bf16 error bounds that case at 1e-3).  The
7B case must reproduce the reference engine's W4A16 stream in every slot.
"""
from __future__ import annotations

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu

REL = 1e-4


def oracle_stream(oracle, path, first, steps, prompt=()):
    om = oracle.open(path)
    for pos, t in enumerate(prompt):
        om.forward(int(t), pos)
    pos, tok, toks, logits = len(prompt), int(first), [], None
    for _ in range(steps):
        toks.append(tok)
        logits = om.forward(tok, pos)
        tok = int(np.argmax(logits))
        pos += 1
    om.close()
    return toks, tok, logits


def rel_err(got, want):
    return float(np.abs(got - want).max() / np.abs(want).max())


@pytest.mark.parametrize("n,steps", [(5, 24), (17, 12), (32, 8)])
def test_batch_from_position_zero(cuda, oracle, tiny_path, n, steps):
    import aion_b200 as A
    first = [(1 + 977 * b) % cases.TINY[5] for b in range(n)]
    with A.Model(tiny_path, max_batch=32) as m:
        toks, lg = m.decode_batch(first, [0] * n, steps, want_logits=True)
    for b in range(n):
        want, pick, wl = oracle_stream(oracle, tiny_path, first[b], steps)
        assert list(toks[:steps, b]) == want, b
        assert toks[steps, b] == pick
        assert rel_err(lg[b], wl) <= REL, b


def test_batch_continues_prefilled_caches(cuda, oracle, tiny_path, golden_tiny):
    """Sequences 0-1 hold 9 prompt tokens, 2-5 hold 6: one batch continues
    all six from their own positions."""
    import aion_b200 as A
    base = golden_tiny["w4a16_tokens"]
    p6 = np.array([[base[(5 * s + t) % len(base)] for t in range(6)] for s in range(6)], np.int32)
    p9 = np.array([[base[(11 * s + t + 3) % len(base)] for t in range(9)] for s in range(2)], np.int32)
    steps = 16
    with A.Model(tiny_path, max_batch=8) as m:
        l6 = m.prefill(p6)
        l9 = m.prefill(p9)
        first = [int(np.argmax(l9[0])), int(np.argmax(l9[1]))] + [int(np.argmax(l6[s])) for s in range(2, 6)]
        pos0 = [9, 9, 6, 6, 6, 6]
        toks, lg = m.decode_batch(first, pos0, steps, want_logits=True)
    prompts = [p9[0], p9[1]] + [p6[s] for s in range(2, 6)]
    for b in range(6):
        want, pick, wl = oracle_stream(oracle, tiny_path, first[b], steps, prompts[b])
        assert list(toks[:steps, b]) == want, b
        assert toks[steps, b] == pick
        assert rel_err(lg[b], wl) <= 1e-3, b


def test_batch_rejects_bad_calls(cuda, tiny_path):
    import aion_b200 as A
    with A.Model(tiny_path, max_batch=4) as m:
        with pytest.raises(A.AionError):
            m.decode_batch([1] * 5, [0] * 5, 2)          # more sequences than held
        with pytest.raises(A.AionError):
            m.decode_batch([1], [cases.TINY[6] - 1], 2)  # runs past max_pos
        with pytest.raises(A.AionError):
            m.decode_batch([cases.TINY[5]], [0], 1)      # token out of range
        toks, _ = m.decode_batch([1], [0], 4)            # the context still works
        assert toks.shape == (5, 1)


def test_batch_7b_matches_reference_stream(ckpt7b, golden_7b):
    """The first 64 tokens against the reference's stream; then 200 tokens
    against the batch-1 path, so that each head's positions span several
    rounds of the attention warps (8 positions x 11 warps a round) and each
    CTA takes several (sequence, head) units."""
    import aion_b200 as A
    want = golden_7b["w4a16_tokens"][:64]
    with A.Model(ckpt7b, max_batch=9, max_pos=256) as m:
        toks, _ = m.decode_batch([1] * 9, [0] * 9, 199)
        one, _ = m.generate(200)
    for b in range(9):
        assert list(toks[:64, b]) == want, b
        assert list(toks[:200, b]) == one, b
