"""The oracle is pinned to the reference: every check here compares the C
restatement (oracle/aion_oracle.c) with fixtures produced by the
reference's own code (tests/golden/make_golden.py), bit for bit.  CPU only."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

import cases


def test_tiny_checkpoint_matches_reference_quantizer(built, workdir, golden_tiny):
    """Product synthesizer -> fp32 file (hash) -> product quantizer == quantize.c output."""
    import aion_b200 as A
    f32 = workdir / "tiny_f32.bin"
    A.synth_checkpoint(f32, cases.TINY, cases.SEEDS["tiny"], int4=False)
    assert hashlib.sha256(f32.read_bytes()).hexdigest() == golden_tiny["fp32_sha"]
    q = workdir / "tiny_int4_from_f32.bin"
    A.quantize_file(f32, q)
    assert hashlib.sha256(q.read_bytes()).hexdigest() == golden_tiny["int4_sha"]
    assert q.stat().st_size == golden_tiny["int4_bytes"] == A.checkpoint_bytes(cases.TINY)


def test_synth_is_thread_count_invariant(built, workdir):
    import aion_b200 as A
    a, b = workdir / "t1.bin", workdir / "t8.bin"
    cfg = (64, 96, 2, 4, 2, 512, 16)
    A.synth_checkpoint(a, cfg, 9, int4=True, threads=1)
    A.synth_checkpoint(b, cfg, 9, int4=True, threads=8)
    assert a.read_bytes() == b.read_bytes()
    assert a.stat().st_size == A.checkpoint_bytes(cfg)


@pytest.mark.parametrize("name", sorted(cases.quantizer_kat_inputs()))
def test_quantizer_kats(oracle, golden_kat, name):
    import aion_b200 as A
    w = cases.quantizer_kat_inputs()[name]
    want = golden_kat["quantizer"][name]
    for packed, scales in (oracle.quantize_buffer(w), A.quantize_buffer(w)):
        assert packed.tolist() == want["packed"]
        assert scales.view(np.uint32).tolist() == want["scales_hex"]


def test_quantizer_zero_group_scale_is_one(oracle):
    packed, scales = oracle.quantize_buffer(np.zeros(32, np.float32))
    assert scales[0] == 1.0 and (packed == 0x88).all()


@pytest.mark.parametrize("name", sorted(cases.actquant_kat_inputs()))
def test_actquant_kats(oracle, golden_kat, name):
    x = cases.actquant_kat_inputs()[name]
    qx, xs = oracle.quantize_activations(x)
    want = golden_kat["actquant"][name]
    assert qx.tolist() == want["qx"]
    assert xs.view(np.uint32).tolist() == want["xs_hex"]


@pytest.mark.parametrize("shape", cases.MATVEC_7B + cases.MATVEC_EDGE, ids=lambda s: f"{s[0]}x{s[1]}")
def test_matvec_kats(oracle, golden_kat, shape):
    import aion_b200 as A
    d, n = shape
    want = golden_kat["matvec"][f"{d}x{n}"]
    w = cases.matrix(d, n, want["seed"])
    packed, scales = A.quantize_buffer(w)
    assert cases.sha(packed) == want["packed_sha"] and cases.sha(scales) == want["scales_sha"]
    x = cases.vector(n, want["seed"])
    assert cases.sha(oracle.matvec_w4a16(x, scales, packed, n, d)) == want["w4a16_sha"]
    assert cases.sha(oracle.matvec_w4a8(x, scales, packed, n, d)) == want["w4a8_sha"]


def test_tiny_w4a16_stream_and_logits(oracle, tiny_path, golden_tiny):
    m = oracle.open(tiny_path)
    toks, gaps, logits = m.generate(256, dump_logits=True)
    assert toks.tolist() == golden_tiny["w4a16_tokens"] == golden_tiny["w4a16_cli_tokens"]
    assert [cases.sha(l) for l in logits] == golden_tiny["w4a16_logits_sha"]
    m.close()


def test_tiny_w4a8_stream_and_logits(oracle, tiny_path, golden_tiny):
    m = oracle.open(tiny_path)
    toks, gaps, logits = m.generate(256, mode=1, dump_logits=True)
    assert toks.tolist() == golden_tiny["w4a8_tokens"]
    assert [cases.sha(l) for l in logits] == golden_tiny["w4a8_logits_sha"]
    m.close()


def test_tiny_f32_stream_and_logits(oracle, tiny_f32_path, golden_tiny):
    """The fp32 path (the reference CLI without "int4"): the oracle's
    restatement of matmul_block_4x4 gives the reference's logits bit for bit."""
    m = oracle.open(tiny_f32_path)
    toks, gaps, logits = m.generate(256, dump_logits=True)
    assert toks.tolist() == golden_tiny["f32_tokens"] == golden_tiny["f32_cli_tokens"]
    assert [cases.sha(l) for l in logits] == golden_tiny["f32_logits_sha"]
    m.close()


def test_oracle_matches_live_reference_on_fresh_seeds(oracle):
    """Where the reference build is present, compare on inputs not in the fixtures."""
    from oracle.oracle import Reference, ref_available
    if not ref_available():
        pytest.skip("reference build not present")
    ref = Reference()
    for seed in range(3):
        d, n = 37, 96 * (seed + 1)
        w = cases.matrix(d, n, 500 + seed)
        p_ref, s_ref = ref.quantize_buffer(w)
        p, s = oracle.quantize_buffer(w)
        assert (p == p_ref).all() and (s.view(np.uint32) == s_ref.view(np.uint32)).all()
        x = cases.vector(n, 700 + seed) * np.float32(3.0)
        assert (oracle.matvec_w4a16(x, s, p, n, d).view(np.uint32) ==
                ref.matmul_int4_scalar(x, s, p, n, d).view(np.uint32)).all()
        assert (oracle.matvec_w4a8(x, s, p, n, d).view(np.uint32) ==
                ref.matmul_w4a8(x, s, p, n, d).view(np.uint32)).all()
        nw = np.abs(cases.vector(n, 900 + seed)).astype(np.float32)
        assert (oracle.rmsnorm(x, nw).view(np.uint32) == ref.rmsnorm(x, nw).view(np.uint32)).all()
