"""Model-level parity on the GPU (tiny Llama-2: dim 288, 6 layers, vocab
32000, seq 256; seed-0 random weights, int4 by the quantize.c arithmetic).

Tolerances:
  - logits: max|l - l_oracle| / max|l_oracle| <= 1e-3 per step (fp32
    accumulate; the reorderings of the GPU sums stay near 1e-6);
  - greedy token streams: identical to the reference's own streams
    (tests/golden/tiny.json, from src/kernel_simd.c), all 256 steps;
  - W4A8 logits: bit-identical to the reference order (the exponentials
    follow the host C library's expf, tabulated where it is not correctly
    rounded).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-3


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.fixture(scope="module")
def model(cuda, tiny_path):
    import aion_b200 as A
    m = A.Model(tiny_path)
    yield m
    m.close()


@pytest.fixture(scope="module")
def model_w4a8(cuda, tiny_path):
    import aion_b200 as A
    m = A.Model(tiny_path, mode="w4a8")
    yield m
    m.close()


def test_config(model):
    assert model.config.as_tuple() == (288, 768, 6, 6, 6, 32000, 256)


def test_generate_matches_reference_stream(model, golden_tiny):
    toks, secs = model.generate(256)
    assert toks == golden_tiny["w4a16_tokens"]
    assert secs > 0


def test_forward_logits_track_oracle(model, oracle, tiny_path, golden_tiny):
    om = oracle.open(tiny_path)
    toks = golden_tiny["w4a16_tokens"]
    worst = 0.0
    for pos in range(256):
        got = model.transformer(toks[pos], pos)
        want = om.forward(toks[pos], pos)
        worst = max(worst, rel_err(got, want))
        if pos + 1 < 256:
            assert int(np.argmax(got)) == toks[pos + 1]
    assert worst <= REL
    om.close()


def test_w4a8_generate_matches_reference_stream(model_w4a8, golden_tiny):
    toks, _ = model_w4a8.generate(256)
    assert toks == golden_tiny["w4a8_tokens"]


def test_w4a8_logits_match_oracle(model_w4a8, oracle, tiny_path, golden_tiny):
    """W4A8 follows the reference's operation order end to end (integer group
    dots, sequential epilogues, 4-lane RMSNorm sums, sequential attention and
    softmax sums, the host's expf): every logit agrees bit for bit."""
    om = oracle.open(tiny_path)
    toks = golden_tiny["w4a8_tokens"]
    equal = total = 0
    for pos in range(64):
        got = model_w4a8.transformer(toks[pos], pos)
        want = om.forward(toks[pos], pos, mode=1)
        assert rel_err(got, want) <= 1e-6
        equal += int((got.view(np.uint32) == want.view(np.uint32)).sum())
        total += got.size
    assert equal == total
    om.close()


def test_graph_and_eager_agree(cuda, tiny_path, golden_tiny):
    import aion_b200 as A
    toks = golden_tiny["w4a16_tokens"]
    with A.Model(tiny_path, use_graph=True) as g, A.Model(tiny_path, use_graph=False) as e:
        for pos in range(8):
            assert (g.transformer(toks[pos], pos).view(np.uint32) == e.transformer(toks[pos], pos).view(np.uint32)).all()


def test_generate_is_repeatable(model):
    a, _ = model.generate(32)
    b, _ = model.generate(32)
    assert a == b


def test_bad_arguments(model):
    import aion_b200 as A
    for tok, pos in ((-1, 0), (32000, 0), (1, 256), (1, -1)):
        with pytest.raises(A.AionError) as e:
            model.transformer(tok, pos)
        assert e.value.code == "ARG"
    with pytest.raises(A.AionError):
        model.generate(257)


def test_max_pos_bounds(cuda, tiny_path):
    import aion_b200 as A
    with pytest.raises(A.AionError) as e:
        A.Model(tiny_path, max_pos=257)
    assert e.value.code == "ARG"
    with A.Model(tiny_path, max_pos=16) as m:
        toks, _ = m.generate(16)
        assert len(toks) == 16
