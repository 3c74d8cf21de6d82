"""Generates the golden fixtures of tests/golden/ from the REFERENCE itself.

Run in a container that has the reference tree (the binaries of
oracle/_ref/ are built from it by `make -C oracle`):

    python tests/golden/make_golden.py [--7b]

Every expected value here comes from the reference's own code: the
`quantize` binary and quantize_buffer() of quantize.c, and the functions of
src/kernel_simd.c through oracle/_ref/libaionref.so (its CLI for the token
stream).  The fixtures are hashes and short token lists; the tests check the
oracle restatement against them, and the GPU path against the oracle.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import aion_b200 as A  # noqa: E402
import cases  # noqa: E402
from oracle.oracle import REF_DIR, Reference  # noqa: E402

OUT = Path(__file__).resolve().parent


def file_sha(p: Path) -> str:
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for b in iter(lambda: f.read(1 << 24), b""):
            h.update(b)
    return h.hexdigest()


def model_fixture(ref: Reference, path: Path, steps: int, w4a8_steps: int, threads: int, cli: bool) -> dict:
    out = {}
    if cli:
        r = subprocess.run([str(REF_DIR / "kernel_simd"), str(path), str(steps), str(threads), "int4", "scalar"],
                           capture_output=True, text=True, check=True, cwd=tempfile.gettempdir())
        out["w4a16_cli_tokens"] = [int(l.split()[1]) for l in r.stdout.strip().splitlines()]
    ref.open(path, threads=threads, scalar=True)
    t0 = time.time()
    toks, gaps, logits = ref.generate(steps, dump_logits=True)
    out["w4a16_seconds"] = time.time() - t0
    out["w4a16_tokens"] = toks.tolist()
    out["w4a16_gaps"] = [float(g) for g in gaps]
    out["w4a16_logits_sha"] = [cases.sha(l) for l in logits]
    out["w4a16_logits_head"] = [[float(v) for v in l[:4]] for l in logits[:4]]
    toks8, gaps8, logits8 = ref.generate(w4a8_steps, w4a8=True, dump_logits=True)
    out["w4a8_tokens"] = toks8.tolist()
    out["w4a8_gaps"] = [float(g) for g in gaps8]
    out["w4a8_logits_sha"] = [cases.sha(l) for l in logits8]
    return out


def f32_fixture(ref: Reference, path: Path, steps: int) -> dict:
    """The reference's fp32 path on the fp32 file: its CLI (no "int4" flag,
    one thread) and the same loop through the harness with logits."""
    r = subprocess.run([str(REF_DIR / "kernel_simd"), str(path), str(steps), "1"], capture_output=True, text=True,
                       check=True, cwd=tempfile.gettempdir())
    out = {"f32_cli_tokens": [int(l.split()[1]) for l in r.stdout.strip().splitlines()]}
    ref.open_f32(path, threads=1)
    toks, gaps, logits = ref.generate(steps, dump_logits=True)
    out["f32_tokens"] = toks.tolist()
    out["f32_gaps"] = [float(g) for g in gaps]
    out["f32_logits_sha"] = [cases.sha(l) for l in logits]
    return out


def kat_fixture(ref: Reference) -> dict:
    kat: dict = {"quantizer": {}, "actquant": {}, "matvec": {}}
    for name, w in cases.quantizer_kat_inputs().items():
        packed, scales = ref.quantize_buffer(w)
        kat["quantizer"][name] = {"packed": packed.tolist(), "scales_hex": scales.view(np.uint32).tolist()}
    for name, x in cases.actquant_kat_inputs().items():
        qx, xs = ref.quantize_activations(x)
        kat["actquant"][name] = {"qx": qx.tolist(), "xs_hex": xs.view(np.uint32).tolist()}
    for d, n in cases.MATVEC_7B + cases.MATVEC_EDGE:
        seed = cases.case_seed(d, n)
        w = cases.matrix(d, n, seed)
        packed, scales = ref.quantize_buffer(w)
        x = cases.vector(n, seed)
        y16 = ref.matmul_int4_scalar(x, scales, packed, n, d)
        y8 = ref.matmul_w4a8(x, scales, packed, n, d)
        kat["matvec"][f"{d}x{n}"] = {
            "seed": seed,
            "packed_sha": cases.sha(packed), "scales_sha": cases.sha(scales),
            "w4a16_sha": cases.sha(y16), "w4a8_sha": cases.sha(y8),
            "w4a16_head": [float(v) for v in y16[:4]], "w4a8_head": [float(v) for v in y8[:4]],
        }
    return kat


# Short-prefix prefill case of bench.py's prefill leg: the first PROMPT_TOK
# tokens of its sequences 0 and 1 (uniform random tokens, seed 2), then
# PREFILL_EXTRA greedy steps.  The reference runs them as forced decode
# steps (transformer() at positions 0.. of one KV cache per sequence).
PREFILL_SEED, PREFILL_SEQ, PREFILL_TOK, PROMPT_TOK, PREFILL_EXTRA = 2, 32, 512, 8, 3
N_PROBE = 64


def prefill_fixture(ref: Reference, path: Path, threads: int) -> dict:
    ref.open(path, threads=threads, scalar=True)
    vocab = ref.vocab
    prompts = np.random.default_rng(PREFILL_SEED).integers(0, vocab, (PREFILL_SEQ, PREFILL_TOK)).astype(np.int32)
    probe = np.random.default_rng(7).choice(vocab, N_PROBE, replace=False)
    logits = lambda: np.ctypeslib.as_array(ref.L.ref_logits(), (vocab,)).copy()  # noqa: E731
    out = {"prompt_tokens": PROMPT_TOK, "extra_steps": PREFILL_EXTRA, "seed": PREFILL_SEED,
           "probe_index": [int(i) for i in probe], "sequences": []}
    for s in range(2):
        p = prompts[s, :PROMPT_TOK]
        for pos, t in enumerate(p):
            ref.L.ref_forward(int(t), pos)
        lg = logits()
        srt = np.sort(lg)
        toks = [int(np.argmax(lg))]
        for i in range(PREFILL_EXTRA):
            ref.L.ref_forward(toks[-1], PROMPT_TOK + i)
            toks.append(int(np.argmax(logits())))
        out["sequences"].append({"prompt": p.tolist(), "tokens": toks, "logits_sha": cases.sha(lg),
                                 "max_abs": float(np.abs(lg).max()), "gap": float(srt[-1] - srt[-2]),
                                 "probe": [float(lg[i]) for i in probe]})
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--7b", dest="b7", action="store_true", help="also the 7B stream (needs ~5 GB disk, minutes)")
    ap.add_argument("--threads", type=int, default=7)
    ap.add_argument("--tmp", default=tempfile.gettempdir())
    ap.add_argument("--f32-only", action="store_true", help="only add the fp32-path keys to tiny.json")
    ap.add_argument("--f32-child", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--7b-prefill", dest="b7_prefill", action="store_true",
                    help="only (re)write the short-prefix prefill case of 7b.json")
    args = ap.parse_args()
    ref = Reference()
    tmp = Path(args.tmp)
    if args.f32_child:
        print(json.dumps(f32_fixture(ref, Path(args.f32_child), 256)))
        return
    if args.b7_prefill:
        p7 = tmp / "aion_7b_int4.bin"
        if not p7.exists():
            A.synth_checkpoint(p7, cases.LLAMA7B, cases.SEEDS["7b"], int4=True)
        b7 = json.loads((OUT / "7b.json").read_text())
        assert file_sha(p7) == b7["int4_sha"]
        code = ("import sys, json; sys.path.insert(0, %r); sys.path.insert(0, %r);"
                "from tests.golden.make_golden import prefill_fixture; from oracle.oracle import Reference;"
                "print(json.dumps(prefill_fixture(Reference(), %r, %d)))"
                % (str(ROOT), str(ROOT / "tests"), str(p7), args.threads))
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True)
        b7["prefill_short"] = json.loads(r.stdout.strip().splitlines()[-1])
        (OUT / "7b.json").write_text(json.dumps(b7))
        print("7b.json prefill_short written; gaps", [q["gap"] for q in b7["prefill_short"]["sequences"]])
        return
    f32 = tmp / "aion_tiny_f32.bin"
    if args.f32_only:
        A.synth_checkpoint(f32, cases.TINY, cases.SEEDS["tiny"], int4=False)
        tiny = json.loads((OUT / "tiny.json").read_text())
        assert file_sha(f32) == tiny["fp32_sha"]
        # The reference engine is process-global: the fp32 run goes in a child.
        r = subprocess.run([sys.executable, __file__, "--f32-child", str(f32)], capture_output=True, text=True,
                           check=True)
        tiny.update(json.loads(r.stdout.strip().splitlines()[-1]))
        (OUT / "tiny.json").write_text(json.dumps(tiny))
        print("tiny.json fp32 keys written; min gap", min(tiny["f32_gaps"]))
        return

    (OUT / "kat.json").write_text(json.dumps(kat_fixture(ref)))
    print("kat.json written")

    q = tmp / "aion_tiny_int4_ref.bin"
    A.synth_checkpoint(f32, cases.TINY, cases.SEEDS["tiny"], int4=False)
    subprocess.run([str(REF_DIR / "quantize"), str(f32), str(q)], check=True, capture_output=True)
    tiny = {"config": list(cases.TINY), "seed": cases.SEEDS["tiny"], "fp32_sha": file_sha(f32),
            "int4_sha": file_sha(q), "int4_bytes": q.stat().st_size}
    tiny.update(model_fixture(ref, q, 256, 256, args.threads, cli=True))
    r = subprocess.run([sys.executable, __file__, "--f32-child", str(f32)], capture_output=True, text=True, check=True)
    tiny.update(json.loads(r.stdout.strip().splitlines()[-1]))
    (OUT / "tiny.json").write_text(json.dumps(tiny))
    print("tiny.json written; min gap", min(tiny["w4a16_gaps"]))

    if args.b7:
        p7 = tmp / "aion_7b_int4.bin"
        if not p7.exists():
            A.synth_checkpoint(p7, cases.LLAMA7B, cases.SEEDS["7b"], int4=True)
        b7 = {"config": list(cases.LLAMA7B), "seed": cases.SEEDS["7b"], "int4_sha": file_sha(p7),
              "int4_bytes": p7.stat().st_size}
        # The reference engine is process-global: run the 7B model in a child.
        code = ("import sys, json; sys.path.insert(0, %r); sys.path.insert(0, %r);"
                "from tests.golden.make_golden import model_fixture; from oracle.oracle import Reference;"
                "print(json.dumps(model_fixture(Reference(), %r, 64, 64, %d, cli=False)))"
                % (str(ROOT), str(ROOT / "tests"), str(p7), args.threads))
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True)
        b7.update(json.loads(r.stdout.strip().splitlines()[-1]))
        (OUT / "7b.json").write_text(json.dumps(b7))
        print("7b.json written; min gap", min(b7["w4a16_gaps"]))


if __name__ == "__main__":
    main()
