"""Batched prefill (aion_prefill) against the oracle's token-by-token forward.

A prefill of n_tok tokens is n_tok forward steps with forced tokens, so the
oracle runs those steps (src/kernel_simd.c:1014 per token) for each
sequence.  Tolerances: the last position's logits within 1e-3 relative of
the oracle's (the prefill's products are bf16 x bf16 split in two parts
each, about 2^-16 relative per product, fp32 accumulate); the KV caches it
leaves are checked by continuing the greedy decode from them, which must
give the oracle's tokens.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-3


def rel_err(got: np.ndarray, want: np.ndarray) -> float:
    return float(np.abs(got - want).max() / np.abs(want).max())


def oracle_stream(oracle, path, prompt, extra):
    """Oracle logits after `prompt` and the greedy tokens that follow."""
    om = oracle.open(path)
    logits = None
    for pos, tok in enumerate(prompt):
        logits = om.forward(int(tok), pos)
    last = logits.copy()
    toks, pos = [], len(prompt)
    tok = int(np.argmax(logits))
    for _ in range(extra):
        toks.append(tok)
        logits = om.forward(tok, pos)
        tok = int(np.argmax(logits))
        pos += 1
    om.close()
    return last, toks


@pytest.mark.parametrize("n_seq,n_tok", [(1, 1), (2, 64), (3, 100)])
def test_prefill_matches_oracle(cuda, oracle, tiny_path, golden_tiny, n_seq, n_tok):
    import aion_b200 as A
    base = golden_tiny["w4a16_tokens"]
    prompts = np.array([[base[(7 * s + t) % len(base)] for t in range(n_tok)] for s in range(n_seq)], np.int32)
    with A.Model(tiny_path, max_batch=4) as m:
        logits = m.prefill(prompts)
        for s in range(n_seq):
            want, cont = oracle_stream(oracle, tiny_path, prompts[s], 8)
            assert rel_err(logits[s], want) <= REL
            # Continue the greedy stream from the KV cache the prefill wrote.
            m.set_sequence(s)
            m.decode_async(8, int(np.argmax(logits[s])), n_tok)
            got = m.tokens(n_tok + 8)[n_tok:]
            assert got == cont


def test_prefill_rejects_too_many_sequences(cuda, tiny_path):
    import aion_b200 as A
    with A.Model(tiny_path, max_batch=2) as m:
        with pytest.raises(A.AionError):
            m.prefill(np.ones((3, 4), np.int32))
