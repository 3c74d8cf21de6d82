"""The fp32 path (the reference CLI without "int4": load_checkpoint and the
fp32 branch of transformer(), src/kernel_simd.c:906-936, 1014-1169) against
the reference's own fp32 run and the oracle's bit-exact restatement of it.

Tolerances: the 256-token greedy stream of the tiny fp32 model equals the
reference's (tests/golden/tiny.json, from its CLI and its engine); logits
are within 1e-5 of the largest logit of the oracle's (fp32 weights and
activations, fp32 accumulate in a different order).  A file with a negative
vocab_size (a separate classifier appended) runs the tied classifier, as
the reference does."""
from __future__ import annotations

import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-5


def test_f32_stream_matches_reference(cuda, tiny_f32_path, golden_tiny):
    import aion_b200 as A
    with A.Model(tiny_f32_path) as m:
        assert m.mode == "f32"
        toks, _ = m.generate(256)
    assert toks == golden_tiny["f32_tokens"] == golden_tiny["f32_cli_tokens"]


def test_f32_logits_match_oracle(cuda, oracle, tiny_f32_path, golden_tiny):
    import aion_b200 as A
    stream = golden_tiny["f32_tokens"][:48]
    om = oracle.open(tiny_f32_path)
    with A.Model(tiny_f32_path) as m:
        for pos, tok in enumerate(stream):
            got = m.transformer(tok, pos)
            want = om.forward(tok, pos)
            assert np.abs(got - want).max() <= REL * np.abs(want).max(), pos
    om.close()


def test_f32_unshared_classifier_file_is_tied(cuda, oracle, workdir, tiny_f32_path, golden_tiny):
    """vocab_size < 0 announces wcls after the RoPE tables; like
    load_checkpoint (src/kernel_simd.c:910), the loader takes abs() and the
    logits still come from the embedding table."""
    import aion_b200 as A
    data = bytearray(tiny_f32_path.read_bytes())
    hdr = np.frombuffer(bytes(data[:28]), np.int32).copy()
    hdr[5] = -hdr[5]
    data[:28] = hdr.tobytes()
    wcls = np.random.default_rng(7).standard_normal(abs(int(hdr[5])) * int(hdr[0])).astype(np.float32)
    p = workdir / "tiny_f32_wcls.bin"
    p.write_bytes(bytes(data) + wcls.tobytes())
    with A.Model(p) as m:
        toks, _ = m.generate(64)
    assert toks == golden_tiny["f32_tokens"][:64]
    om = oracle.open(p)
    otoks, _, _ = om.generate(64)
    om.close()
    assert otoks.tolist() == toks


def test_f32_cli_prints_the_reference_stream(cuda, tiny_f32_path, golden_tiny, tmp_path):
    from aion_b200.build import CLI
    r = subprocess.run([str(CLI), str(tiny_f32_path), "256", "1"], capture_output=True, text=True, check=True,
                       cwd=tmp_path)
    got = [int(line.split()[1]) for line in r.stdout.strip().splitlines()]
    assert got == golden_tiny["f32_cli_tokens"]
    assert "Float32" in r.stderr


def test_f32_rejects_int4_only_features(cuda, tiny_f32_path):
    import aion_b200 as A
    with pytest.raises(A.AionError):
        A.Model(tiny_f32_path, mode="w4a8")
    with A.Model(tiny_f32_path, max_batch=2) as m:
        with pytest.raises(A.AionError):
            m.prefill(np.ones((1, 4), np.int32))
        with pytest.raises(A.AionError):
            m.decode_batch([1], [0], 2)
