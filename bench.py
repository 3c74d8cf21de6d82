#!/usr/bin/env python
"""Benchmark: Llama-2-7B-shape int4 (W4A16) greedy decode, batch 1, on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl aion|reference] [--matvec]

Workload: the 7B shape (dim 4096, hidden 11008, 32 layers, 32 heads, vocab
32000) with seed-1 random-init N(0, 0.02) weights quantized by the
quantize.c arithmetic, fp32 activations and KV cache; greedy decode from
BOS=1 over the 512-token workload.  One step = one decode token; the K
timed steps run in one persistent decode launch (split where the stream
restarts).  W warm-up tokens take positions 0..W-1, the K timed tokens
continue the same greedy stream (a new sequence starts from BOS at
position 0 after 512 tokens).  The weights
(4.13 GB per token) are far larger than L2, so every step streams them
from HBM.

N > 1: independent replicas, one per GPU (the 7B path does not shard;
"scaling": "weak"); value = N * K / (max over ranks of the timed region).

--impl reference times the reference's own CPU int4 path (oracle/_ref,
built from the reference's src/kernel_simd.c; scalar int4 kernel, host
thread pool) on the same workload, bounded to a few minutes.
--matvec times the isolated matvec shapes only (for profiling).
The JSON line also carries "prefill": the batched-prefill workload on the
same model (32 sequences x 512 uniform random tokens, seed 2, through every
layer at once on the tensor cores, then 128 greedy decode steps per
sequence), with its own roofline against the measured bf16 peak
(--no-prefill skips it).
--tp13b runs the 13B-shape model (dim 5120, hidden 13824, 40 layers, seed 3)
tensor-parallel over the N ranks of the launch (one process per GPU): greedy
decode of a 256-token workload from BOS, one sequence, "scaling": "strong".
--profile-layers L runs the same path on a 7B-shape checkpoint truncated to
L layers (same seed and shapes; for ncu captures that must stay small, never
for the reported metric).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG_7B = (4096, 11008, 32, 32, 32, 32000, 2048)
SEED_7B = 1
CFG_13B = (5120, 13824, 40, 40, 40, 32000, 2048)
SEED_13B = 3
TP_TOKENS = 256
BATCH_13B = 16
BOS = 1
WORKLOAD_TOKENS = 512
WEIGHT_BYTES_PER_TOKEN = 4_129_423_360          # 0.625 B x 6,607,077,376 weights


def weight_bytes_per_token(layers: int) -> int:
    """int4 weight bytes one token streams (0.625 B per weight: nibble +
    1/32 fp32 scale): per layer wq, wk, wv, wo, w1, w2, w3; plus the
    classifier (the tied embedding)."""
    dim, hid, vocab = CFG_7B[0], CFG_7B[1], CFG_7B[5]
    return int(0.625 * (layers * (4 * dim * dim + 3 * dim * hid) + vocab * dim))
MATVEC_SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes per token of the decode kernel's weight stream, measured once
# with ncu (dram__bytes_read.sum + dram__bytes_write.sum of an 8-step 7B
# launch, minus its K/V reads): 1.0001 x the algorithmic weight bytes.
DRAM_WEIGHT_BYTES_PER_TOKEN = 4.1296e9


def matvec_bytes(d: int, n: int) -> int:
    """Algorithmic bytes of one d x n int4 matvec: packed + scales + x + y."""
    return int(0.625 * d * n) + 4 * n + 4 * d


def hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def ckpt_dir() -> Path:
    d = Path(os.environ.get("AION_CKPT_DIR", Path(tempfile.gettempdir()) / "aion_ckpt"))
    d.mkdir(parents=True, exist_ok=True)
    return d


def ensure_7b(rank: int, layers: int = 0, writer: str = "aion") -> Path:
    """Writes the seeded 7B int4 checkpoint once per host (rank 0); with
    layers > 0, the same shapes truncated to that many layers.  writer
    "aion" uses the library's synthesizer; "reference" runs
    oracle/_ref/synth_ckpt, the same generator feeding the reference's own
    quantize_buffer (quantize.c), so the reference arm loads nothing of the
    product library.  Both write identical bytes (tests/test_oracle.py)."""
    cfg = CFG_7B if layers <= 0 else (CFG_7B[0], CFG_7B[1], layers) + CFG_7B[3:]
    name = "llama2_7b_seed1.int4" if layers <= 0 else f"llama2_7b_shape_{layers}l_seed1.int4"
    path = ckpt_dir() / name
    done = path.with_suffix(".done")
    if rank == 0 and not done.exists():
        tmp = path.with_suffix(".tmp")
        if writer == "reference":
            subprocess.run([str(ROOT / "oracle" / "_ref" / "synth_ckpt"), str(tmp), *map(str, cfg), str(SEED_7B)],
                           check=True)
        else:
            import aion_b200 as A
            A.synth_checkpoint(tmp, cfg, SEED_7B, int4=True)
        tmp.rename(path)
        done.write_text("ok")
    while not done.exists():
        time.sleep(1.0)
    return path


def config_7b(world: int, layers: int = 0) -> dict:
    """The workload's config dict, identical in both arms."""
    return {"workload": "llama2-7b-shape W4A16 greedy decode, batch 1, 512-token workload",
            "dim": CFG_7B[0], "hidden": CFG_7B[1], "layers": layers if layers > 0 else CFG_7B[2],
            "heads": CFG_7B[3], "vocab": CFG_7B[5], "seed": SEED_7B, "parallelism": f"replicas x{world}",
            "l2": "weights 4.13 GB/token > L2 (no flush needed)"}


def ensure_13b(rank: int) -> Path:
    """Writes the seeded 13B int4 checkpoint once per host (rank 0)."""
    import aion_b200 as A
    path = ckpt_dir() / "llama2_13b_seed3.int4"
    done = path.with_suffix(".done")
    if rank == 0 and not done.exists():
        tmp = path.with_suffix(".tmp")
        A.synth_checkpoint(tmp, CFG_13B, SEED_13B, int4=True)
        tmp.rename(path)
        done.write_text("ok")
    while not done.exists():
        time.sleep(1.0)
    return path


class Clocks:
    """Samples SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except FileNotFoundError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i] and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


_REF_ENGINE = None


def cpu_reference_decode(path: Path, warmup: int, max_tokens: int, budget_s: float, w4a8: bool = False) -> dict:
    """The reference's own CPU int4 path (scalar int4 kernel, pthread pool)
    on the 7B checkpoint: tokens/s over a bounded sample of the workload.
    w4a8: the reference's quantize_activations_neon + matmul_w4a8_neon
    wired into its forward pass by oracle/ref_harness.c (through the scalar
    NEON shim on x86 hosts)."""
    global _REF_ENGINE
    from oracle.oracle import REF_DIR, Oracle, Reference
    cores = os.cpu_count() or 1
    threads = max(1, cores - 1)       # T = cores oversubscribes the spin barrier
    if (REF_DIR / "libaionref.so").exists():
        if _REF_ENGINE is None:       # the reference engine is process-global: open once
            _REF_ENGINE = Reference().open(path, threads=threads, scalar=True)
        ref = _REF_ENGINE
        fwd = ref.L.ref_forward_w4a8 if w4a8 else ref.L.ref_forward
        logits = lambda: np.ctypeslib.as_array(ref.L.ref_logits(), (CFG_7B[5],))  # noqa: E731
        kind = "reference"
    else:
        orc = Oracle()
        orc.set_threads(threads)
        m = orc.open(path)
        fwd = lambda t, p: m.o.L.orc_forward(m.h, t, p, 0)  # noqa: E731
        logits = lambda: np.ctypeslib.as_array(m.o.L.orc_logits(m.h), (CFG_7B[5],))  # noqa: E731
        kind = "port"
    tok = BOS
    for pos in range(warmup):
        fwd(tok, pos)
        tok = int(np.argmax(logits()))
    n, t0 = 0, time.perf_counter()
    pos = warmup
    while n < max_tokens and (time.perf_counter() - t0) < budget_s:
        fwd(tok, pos)
        tok = int(np.argmax(logits()))
        pos += 1
        n += 1
    secs = time.perf_counter() - t0
    what = ("reference W4A8 functions (quantize_activations_neon + matmul_w4a8_neon via the scalar NEON shim)"
            if w4a8 else "reference scalar int4 path")
    return {"value": n / secs, "unit": "tok/s", "cores": threads, "kind": kind, "tokens": n, "seconds": secs,
            "sample": f"7B {'W4A8' if w4a8 else 'W4A16'} greedy decode from BOS, {n} tokens at positions "
                      f"{warmup}..{warmup + n - 1} after {warmup} warm-up tokens; {what}, {threads} pthreads on "
                      f"{cores} host cores"}


def run_reference_arm(args) -> None:
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    path = ensure_7b(0, writer="reference")
    cb = cpu_reference_decode(path, args.warmup, args.steps, budget_s=args.ref_budget)
    line = {"metric": "Llama-2-7B int4 decode tok/s (batch 1)", "value": cb["value"], "unit": "tok/s",
            "n_gpus": world, "steps": cb["tokens"], "warmup": args.warmup,
            "ms_per_step": 1000.0 / cb["value"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 weights, fp32 activations", "data": "synthetic",
            "config": config_7b(world),
            "impl": "reference",
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PREFILL_SEQ, PREFILL_TOK, PREFILL_DECODE, PREFILL_SEED = 32, 512, 128, 2


def bf16_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured (sustained)"
        except Exception:
            pass
    return 1400.0, "fallback (sustained)"


def prefill_parity(model) -> dict | None:
    """The short-prefix case of this leg against the reference (committed
    fixture from the reference engine, tests/golden/7b.json "prefill_short"):
    the first tokens of sequences 0 and 1 of the prefill workload through
    model.prefill, then lock-step greedy steps; the last-position logits at
    the fixture's probe indices within 1e-3 of max |logit|, and every
    token identical.  Runs after the timed regions."""
    fx = json.loads((ROOT / "tests" / "golden" / "7b.json").read_text()).get("prefill_short")
    if not fx:
        return None
    seqs, n, extra = fx["sequences"], fx["prompt_tokens"], fx["extra_steps"]
    logits = model.prefill(np.array([q["prompt"] for q in seqs], np.int32))
    first = np.argmax(logits, axis=1).astype(np.int32)
    toks, _ = model.decode_batch(first, np.full(len(seqs), n, np.int32), extra)
    idx = np.array(fx["probe_index"])
    err = max(float(np.abs(logits[i][idx] - np.array(q["probe"], np.float32)).max() / q["max_abs"])
              for i, q in enumerate(seqs))
    return {"case": f"{len(seqs)} sequences x {n} prompt tokens of the workload, then {extra} greedy steps",
            "tokens_compared": (extra + 1) * len(seqs),
            "identical": all(toks[:, i].tolist() == q["tokens"] for i, q in enumerate(seqs)),
            "logit_rel_err_max": err, "logit_rel_tol": 1e-3}


def prefill_leg(model, layers: int, stream, device: int) -> dict:
    """32 x 512 prefill then 128 decode steps per sequence, timed with CUDA
    events on the model's stream."""
    import torch
    dim, hid, vocab = CFG_7B[0], CFG_7B[1], CFG_7B[5]
    toks = np.random.default_rng(PREFILL_SEED).integers(0, vocab, (PREFILL_SEQ, PREFILL_TOK)).astype(np.int32)
    model.prefill(toks)                   # warm-up at full size: buffers, tensor maps, module load
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    logits = model.prefill(toks)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    rows = PREFILL_SEQ * PREFILL_TOK
    lin_flops = 2.0 * rows * layers * (4 * dim * dim + 3 * dim * hid) + 2.0 * PREFILL_SEQ * vocab * dim
    attn_flops = PREFILL_SEQ * layers * 2.0 * (PREFILL_TOK * (PREFILL_TOK + 1) / 2) * dim * 2
    tflops = (lin_flops + attn_flops) / (ms * 1e-3) / 1e12
    peak, kind = bf16_peak()
    # The 128 decode steps of all 32 sequences in lock step (one launch).
    first = np.argmax(logits, axis=1).astype(np.int32)
    pos0 = np.full(PREFILL_SEQ, PREFILL_TOK, np.int32)
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    toks_out, _ = model.decode_batch(first, pos0, PREFILL_DECODE)
    d1.record(stream)
    torch.cuda.synchronize()
    dms = d0.elapsed_time(d1)
    wb = weight_bytes_per_token(layers)
    kvb = sum(kv_step_bytes(layers, dim, [PREFILL_TOK + i] * PREFILL_SEQ) for i in range(PREFILL_DECODE))
    dgbs = (wb * PREFILL_DECODE + kvb) / (dms * 1e-3) / 1e9
    hpeak, hkind = hbm_peak()
    return {"workload": f"{PREFILL_SEQ} x {PREFILL_TOK} uniform random tokens (seed {PREFILL_SEED}) prefill, "
                        f"then {PREFILL_DECODE} greedy decode steps of all {PREFILL_SEQ} sequences in lock step",
            "prefill_ms": ms, "prefill_tok_s": rows / (ms * 1e-3),
            "roofline": {"kernel": "prefill (k_gemm_bf16_tn dominant)", "bound": "tensor",
                         "achieved": tflops, "peak": peak, "peak_kind": kind, "unit": "TFLOP/s",
                         "frac": tflops / peak, "algorithmic_flops": lin_flops + attn_flops,
                         "note": "algorithmic bf16-equivalent flops; the kernels issue 3x the linear MMA work "
                                 "(two-part bf16 operands)"},
            "decode_ms": dms, "decode_tok_s": PREFILL_SEQ * PREFILL_DECODE / (dms * 1e-3),
            "decode_roofline": {"kernel": "k_decode_batch<4> (lock-step batch of 32)", "bound": "hbm",
                                "achieved": dgbs, "peak": hpeak, "peak_kind": hkind, "unit": "GB/s",
                                "frac": dgbs / hpeak, "weight_bytes_per_step": wb,
                                "kv_bytes_per_step_avg": kvb / PREFILL_DECODE},
            "decode_stream_head": toks_out[:8, 0].tolist(),
            "parity": prefill_parity(model) if layers == CFG_7B[2] else None}


def kv_step_bytes(layers: int, kv_dim: int, positions) -> int:
    """KV-cache bytes one decode step reads and writes: per sequence at
    position p and layer, K and V rows 0..p read (fp32) and row p written."""
    return sum(layers * 2 * kv_dim * 4 * (p + 2) for p in positions)


def isolated_matvecs(device: int, reps: int, shapes=None) -> dict:
    """GB/s of the W4A16 matvec kernel on the isolated 7B shapes, rotating over
    enough distinct weight copies to exceed 2x L2 so every launch reads HBM."""
    import torch
    import aion_b200 as A
    rng = np.random.default_rng(5)
    out = {}
    for d, n in shapes or MATVEC_SHAPES:
        copies = max(2, int(np.ceil(2 * 126e6 / (0.625 * d * n))) + 1)
        mats = []
        for _ in range(copies):
            packed = rng.integers(0, 256, d * n // 2, dtype=np.uint8)
            scales = (rng.random(d * n // 32, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
            mats.append(A.QMatrix(scales, packed, d, n, device=device))
        x = torch.randn(n, device=f"cuda:{device}")
        y = torch.empty(d, device=f"cuda:{device}")
        for m in mats:
            m.matvec_w4a16(x, y)
        torch.cuda.synchronize()
        # Eager: one ctypes call per launch (includes the host's launch cost).
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            for m in mats:
                m.matvec_w4a16(x, y)
        e1.record()
        torch.cuda.synchronize()
        eager_ms = e0.elapsed_time(e1) / (reps * copies)
        # Kernel time: the same launches captured once in a CUDA graph and
        # replayed, so the host's launch rate does not limit the GPU.
        side = torch.cuda.Stream(device=f"cuda:{device}")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for m in mats:
                m.matvec_w4a16(x, y, stream=side)
        g.replay()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * copies)
        out[f"{d}x{n}"] = {"us": ms * 1e3, "GBps": matvec_bytes(d, n) / (ms * 1e-3) / 1e9,
                           "frac": matvec_bytes(d, n) / (ms * 1e-3) / 1e9 / hbm_peak()[0],
                           "eager_us": eager_ms * 1e3,
                           "eager_GBps": matvec_bytes(d, n) / (eager_ms * 1e-3) / 1e9}
        del g
        for m in mats:
            m.free()
    return out


def run_fp32(args, local: int) -> None:
    """7B-shape fp32 llama2.c checkpoint (the reference's fp32 path): batch-1
    greedy decode from BOS, one persistent launch, weights 4 bytes each."""
    import torch
    import aion_b200 as A
    L = args.profile_layers if args.profile_layers > 0 else CFG_7B[2]
    cfg = (CFG_7B[0], CFG_7B[1], L) + CFG_7B[3:]
    path = ckpt_dir() / f"llama2_7b_shape_{L}l_seed1.f32"
    done = path.with_suffix(".done")
    if not done.exists():
        tmp = path.with_suffix(".tmp")
        A.synth_checkpoint(tmp, cfg, SEED_7B, int4=False)
        tmp.rename(path)
        done.write_text("ok")
    model = A.Model(path, device=local, max_pos=args.steps + args.warmup + 1)
    assert model.mode == "f32"
    stream = torch.cuda.ExternalStream(model.stream_ptr(), device=f"cuda:{local}")
    model.decode_async(args.warmup, BOS, 0)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    model.decode_async(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    dim, hid, vocab = CFG_7B[0], CFG_7B[1], CFG_7B[5]
    wb = 4 * (L * (4 * dim * dim + 3 * dim * hid) + vocab * dim)
    gbs = wb * args.steps / (ms * 1e-3) / 1e9
    peak, kind = hbm_peak()
    print(json.dumps({
        "metric": "Llama-2-7B fp32 decode tok/s (batch 1, fp32 checkpoint)", "value": args.steps / (ms * 1e-3),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"llama2-7b-shape fp32 greedy decode from BOS, {L} layers", "layers": L, "seed": 1},
        "roofline": {"kernel": "k_decode<F32> (persistent decode, fp32 tiles)", "bound": "hbm", "achieved": gbs,
                     "peak": peak, "peak_kind": kind, "unit": "GB/s", "frac": gbs / peak, "bytes_per_token": wb},
        "gpu_launches": 1, "clocks": clk, "token_stream_head": model.tokens(min(16, args.warmup + args.steps))}), flush=True)
    model.close()


def run_batch(args, local: int) -> None:
    """7B-shape lock-step batched decode: args.batch sequences from BOS,
    args.steps greedy steps each (positions 0..steps-1), one launch."""
    import torch
    import aion_b200 as A
    nb = args.batch
    path = ensure_7b(0, args.profile_layers)
    model = A.Model(path, device=local, max_batch=nb, max_pos=args.steps + args.warmup + 1)
    L = model.config.n_layers
    stream = torch.cuda.ExternalStream(model.stream_ptr(), device=f"cuda:{local}")
    model.decode_batch([BOS] * nb, [0] * nb, args.warmup)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    toks, _ = model.decode_batch([BOS] * nb, [0] * nb, args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    dim = CFG_7B[0]
    wb = weight_bytes_per_token(L)
    kvb = sum(kv_step_bytes(L, dim, [i] * nb) for i in range(args.steps))
    gbs = (wb * args.steps + kvb) / (ms * 1e-3) / 1e9
    peak, kind = hbm_peak()
    parity = None
    gold = ROOT / "tests" / "golden" / "7b.json"
    if gold.exists() and args.profile_layers <= 0:
        want = json.loads(gold.read_text())["w4a16_tokens"]
        k = min(len(want), args.steps + 1)
        parity = {"tokens_compared": k, "identical_in_every_slot": all(
            list(toks[:k, b]) == want[:k] for b in range(nb))}
    print(json.dumps({
        "metric": f"Llama-2-7B int4 decode tok/s (batch {nb}, lock step)", "value": nb * args.steps / (ms * 1e-3),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "s4 weights x s8 activation digits (24-bit fixed point per group, int32 tensor-core dot), "
                 "fp32 accumulate",
        "data": "synthetic",
        "config": {"workload": f"llama2-7b-shape W4A16 greedy decode of {nb} sequences from BOS, positions "
                               f"0..{args.steps - 1}", "layers": L, "seed": 1, "parallelism": "replicas x1"},
        "roofline": {"kernel": f"k_decode_batch<{(nb + 7) // 8}>", "bound": "hbm", "achieved": gbs, "peak": peak,
                     "peak_kind": kind, "unit": "GB/s", "frac": gbs / peak,
                     "weight_bytes_per_step": wb, "kv_bytes_per_step_avg": kvb / args.steps},
        "e2e": {"value": nb * args.steps / wall, "unit": "tok/s", "h2d_bytes_per_step": 8 * nb / args.steps,
                "d2h_bytes_per_step": 4 * nb * (args.steps + 1) / args.steps},
        "gpu_launches": 1, "clocks": clk, "parity": parity}), flush=True)
    model.close()


def tp13b_leg(args, world, rank, local, pg, barrier, max_over_ranks):
    """13B-shape decode, tensor-parallel over the launch's ranks (TP = N,
    one process per GPU): batch 1 and batch 16 over the 256-token workload.
    Returns the sub-object of the JSON line on rank 0 (None elsewhere)."""
    import torch
    import aion_b200 as A
    path = ensure_13b(rank)
    barrier()
    model = A.Model(path, device=local, tp_size=world, tp_rank=rank, max_pos=TP_TOKENS, max_batch=BATCH_13B)
    if world > 1:
        handles = [None] * world
        pg.all_gather_object(handles, model.tp_handle())
        model.tp_connect(handles)
    stream = torch.cuda.ExternalStream(model.stream_ptr(), device=f"cuda:{local}")
    steps = min(args.steps, TP_TOKENS - args.warmup)
    model.decode_async(args.warmup, BOS, 0)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    model.decode_async(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    toks = model.tokens(args.warmup + steps)
    dim, hid, L, vocab = CFG_13B[0], CFG_13B[1], CFG_13B[2], CFG_13B[5]
    wbytes = int(0.625 * (L * (4 * dim * dim + 3 * dim * hid) + vocab * dim)) // world
    gbs = wbytes * steps / (ms * 1e-3) / 1e9
    peak, kind = hbm_peak()
    # Batch-16 decode of the same 256-token workload, all sequences from BOS
    # (tensor-parallel over the same ranks; per-GPU bytes below).
    model.decode_batch([BOS] * BATCH_13B, [0] * BATCH_13B, 4)   # warm-up
    torch.cuda.synchronize()
    barrier()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(stream)
    btoks, _ = model.decode_batch([BOS] * BATCH_13B, [0] * BATCH_13B, TP_TOKENS - 1)
    b1.record(stream)
    torch.cuda.synchronize()
    barrier()
    bms = max_over_ranks(b0.elapsed_time(b1))
    nst = TP_TOKENS - 1
    kvb = sum(kv_step_bytes(L, dim, [i] * BATCH_13B) for i in range(nst)) // world
    bgbs = (wbytes * nst + kvb) / (bms * 1e-3) / 1e9
    batch = {"workload": f"batch {BATCH_13B} greedy decode of {TP_TOKENS} tokens from BOS (lock step)",
             "value": BATCH_13B * nst / (bms * 1e-3), "unit": "tok/s", "ms_per_step": bms / nst,
             "roofline": {"kernel": "k_decode_batch<2>", "bound": "hbm", "achieved": bgbs, "peak": peak,
                          "peak_kind": kind, "unit": "GB/s", "frac": bgbs / peak,
                          "bytes_per_step_per_gpu": wbytes + kvb // nst},
             "same_stream_as_batch1": bool((btoks[:16, 0] == np.array(toks[:16])).all())}
    model.close()
    if rank != 0:
        return None
    return {
        "metric": "Llama-2-13B int4 decode tok/s (batch 1, tensor-parallel)", "value": steps / (ms * 1e-3),
        "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": ms / steps,
        "higher_is_better": True, "scaling": "strong",
        "dtype": "s4 weights x s8 activation digits (int32 tensor-core dot), fp32 accumulate",
        "config": {"workload": f"llama2-13b-shape W4A16 greedy decode, batch 1, {TP_TOKENS}-token workload",
                   "dim": dim, "hidden": hid, "layers": L, "vocab": vocab, "seed": SEED_13B,
                   "parallelism": f"tp{world}"},
        "roofline": {"kernel": "k_decode<W4A16> (persistent decode, in-kernel NVLink exchange)", "bound": "hbm",
                     "achieved": gbs, "peak": peak, "peak_kind": kind, "unit": "GB/s",
                     "frac": gbs / peak, "bytes_per_token_per_gpu": wbytes},
        "gpu_launches": 1, "clocks": clk,
        "token_stream_head": toks[:16], "batch16": batch}


def w4a8_leg(path: Path, device: int, steps: int, warmup: int, cpu: bool) -> dict:
    """7B W4A8 greedy decode, batch 1 (activations quantized per group of 32
    to int8 before every matmul, as the reference's W4A8 functions): the same
    persistent launch and timing as the W4A16 headline, its own roofline, and
    the reference's W4A8 path on the host cores beside it."""
    import torch
    import aion_b200 as A
    steps = min(steps, WORKLOAD_TOKENS - warmup)
    model = A.Model(path, device=device, mode="w4a8", max_pos=WORKLOAD_TOKENS)
    stream = torch.cuda.ExternalStream(model.stream_ptr(), device=f"cuda:{device}")
    model.decode_async(warmup, BOS, 0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    model.decode_async(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    toks = model.tokens(warmup + steps)
    model.close()
    L = CFG_7B[2]
    wb = weight_bytes_per_token(L)
    gbs = wb * steps / (ms * 1e-3) / 1e9
    peak, kind = hbm_peak()
    parity = None
    gold = ROOT / "tests" / "golden" / "7b.json"
    if gold.exists():
        want = json.loads(gold.read_text()).get("w4a8_tokens", [])
        k = min(len(want), len(toks))
        parity = {"tokens_compared": k, "identical": toks[:k] == want[:k]}
    out = {"workload": f"llama2-7b-shape W4A8 greedy decode from BOS, batch 1, positions {warmup}..{warmup + steps - 1}",
           "value": steps / (ms * 1e-3), "unit": "tok/s", "ms_per_step": ms / steps, "steps": steps,
           "warmup": warmup,
           "dtype": "s4 weights x s8 activations (reference per-group quantization), int32 group dots, fp32 row sums",
           "roofline": {"kernel": "k_decode<W4A8> (persistent decode, all steps)", "bound": "hbm", "achieved": gbs,
                        "peak": peak, "peak_kind": kind, "unit": "GB/s", "frac": gbs / peak,
                        "bytes_per_token": wb},
           "gpu_launches": 1, "parity": parity}
    if cpu:
        cb = cpu_reference_decode(path, 2, 200, budget_s=15.0, w4a8=True)
        out["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=WORKLOAD_TOKENS - 3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["aion", "reference"], default="aion")
    ap.add_argument("--matvec", action="store_true", help="isolated matvec shapes only")
    ap.add_argument("--shape", default=None, help="with --matvec: one shape, e.g. 32000x4096")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-matvec", action="store_true", help="skip the isolated matvec shapes")
    ap.add_argument("--no-prefill", action="store_true", help="skip the batched-prefill leg")
    ap.add_argument("--no-w4a8", action="store_true", help="skip the W4A8 decode leg")
    ap.add_argument("--no-tp13b", action="store_true", help="skip the 13B tensor-parallel leg")
    ap.add_argument("--ref-budget", type=float, default=120.0, help="seconds of timed reference decode")
    ap.add_argument("--tp13b", action="store_true", help="13B shape, tensor-parallel over the launch's ranks")
    ap.add_argument("--batch", type=int, default=0, help="7B lock-step batched decode of this many sequences")
    ap.add_argument("--fp32", action="store_true", help="7B-shape fp32 checkpoint (the reference's fp32 path)")
    ap.add_argument("--profile-layers", type=int, default=0,
                    help="profiling only: 7B shapes truncated to this many layers")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        run_reference_arm(args)
        return

    import torch
    import aion_b200 as A

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local}"))
        pg = dist

    def barrier():
        if pg:
            pg.barrier()

    def max_over_ranks(v: float) -> float:
        if not pg:
            return v
        t = torch.tensor([v], device=f"cuda:{local}", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    if args.tp13b:
        res = tp13b_leg(args, world, rank, local, pg, barrier, max_over_ranks)
        if rank == 0:
            res["data"] = "synthetic"
            res["vs_baseline"] = None
            print(json.dumps(res), flush=True)
        if pg:
            pg.destroy_process_group()
        return

    if args.batch > 0:
        if rank == 0:
            run_batch(args, local)
        return

    if args.fp32:
        if rank == 0:
            run_fp32(args, local)
        return

    if args.matvec:
        shapes = [tuple(int(v) for v in args.shape.split("x"))] if args.shape else None
        res = isolated_matvecs(local, reps=max(args.steps, 1), shapes=shapes)
        if rank == 0:
            print(json.dumps({"metric": "int4 matvec HBM GB/s (isolated 7B shapes)", "matvec": res}), flush=True)
        return

    path = ensure_7b(rank, args.profile_layers)
    do_prefill = not args.no_prefill and rank == 0
    model = A.Model(path, device=local, max_batch=PREFILL_SEQ if do_prefill else 1,
                    max_pos=PREFILL_TOK + PREFILL_DECODE if do_prefill else 0)
    L = model.config.n_layers
    stream = torch.cuda.ExternalStream(model.stream_ptr(), device=f"cuda:{local}")

    def decode(count: int, start_pos: int) -> int:
        """Enqueues `count` greedy steps from start_pos, restarting from BOS
        at position 0 after the 512-token workload; returns kernel launches."""
        launches, pos = 0, start_pos
        while count > 0:
            if pos >= WORKLOAD_TOKENS:
                pos = 0
            n = min(count, WORKLOAD_TOKENS - pos)
            if pos == 0:
                model.decode_async(n, BOS, 0)
                launches += 2            # k_set_step + k_decode
            else:
                model.decode_async(n)
                launches += 1
            count -= n
            pos += n
        return launches

    # Warm-up: positions 0..W-1 of the greedy stream.
    decode(args.warmup, 0)
    torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    launches = decode(args.steps, args.warmup)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms_local = e0.elapsed_time(e1)
    ms = max_over_ranks(ms_local)
    tok_s = world * args.steps / (ms * 1e-3)
    stream_tokens = model.tokens(min(args.warmup + args.steps, WORKLOAD_TOKENS))

    # Parity sanity: the stream against the reference's 7B stream, where recorded.
    parity = None
    gold = ROOT / "tests" / "golden" / "7b.json"
    if gold.exists() and args.profile_layers <= 0:
        want = json.loads(gold.read_text())["w4a16_tokens"]
        k = min(len(want), len(stream_tokens))
        parity = {"tokens_compared": k, "identical": stream_tokens[:k] == want[:k]}

    # Roofline of the decode kernel (one persistent launch runs all steps):
    # algorithmic bytes = int4 weights of every token (+ KV cache reads,
    # reported separately), over the CUDA-event time of the launches.
    dim, hid, vocab = CFG_7B[0], CFG_7B[1], CFG_7B[5]
    kv_bytes = 0
    pos = args.warmup
    for _ in range(args.steps):
        if pos >= WORKLOAD_TOKENS:
            pos = 0
        kv_bytes += 2 * L * dim * 4 * (pos + 1)
        pos += 1
    wbytes = weight_bytes_per_token(L)
    weights_gbs = wbytes * args.steps / (ms_local * 1e-3) / 1e9
    peak, peak_kind = hbm_peak()
    traffic = (DRAM_WEIGHT_BYTES_PER_TOKEN * args.steps + kv_bytes
               if args.profile_layers <= 0 else None)
    roofline = {"kernel": "k_decode<W4A16> (persistent decode, all steps)", "bound": "hbm",
                "achieved": weights_gbs, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": weights_gbs / peak, "traffic": traffic, "traffic_unit": "bytes per launch",
                "algorithmic_bytes": wbytes * args.steps,
                "bytes_per_token": wbytes,
                "with_kv_GBps": (wbytes * args.steps + kv_bytes) / (ms_local * 1e-3) / 1e9}
    matvec = isolated_matvecs(local, reps=5) if (rank == 0 and not args.no_matvec) else None

    # End-to-end: the reference-facing call transformer(token, pos) per token
    # with host buffers (token/pos in from pinned memory, logits out to pinned
    # memory, argmax on the host), as the reference's main loop drives it.
    logits = torch.empty(vocab, dtype=torch.float32, pin_memory=True)
    lib = A.lib()
    barrier()
    tok = BOS
    t0 = time.perf_counter()
    for i in range(args.steps):
        p = i % WORKLOAD_TOKENS
        if p == 0:
            tok = BOS
        st = lib.aion_forward(model._h, tok, p, logits.data_ptr())
        if st != 0:
            raise A.AionError(st, lib.aion_last_error(model._h).decode())
        tok = int(np.argmax(logits.numpy()))
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()

    prefill = prefill_leg(model, L, stream, local) if do_prefill else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and args.profile_layers <= 0:
        cb = cpu_reference_decode(path, 2, 1000, budget_s=20.0)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}

    w4a8 = None
    if rank == 0 and world == 1 and not args.no_w4a8 and args.profile_layers <= 0:
        model.close()
        w4a8 = w4a8_leg(path, local, args.steps, args.warmup, cpu=not args.no_cpu)

    # 13B tensor parallelism over every rank of this launch (TP = N).
    tp13b = None
    if not args.no_tp13b and args.profile_layers <= 0:
        model.close()
        barrier()
        tp13b = tp13b_leg(args, world, rank, local, pg, barrier, max_over_ranks)

    if rank == 0:
        line = {
            "metric": "Llama-2-7B int4 decode tok/s (batch 1)",
            "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "s4 weights x s8 activation digits (int32 tensor-core dot), fp32 accumulate",
            "data": "synthetic",
            "config": config_7b(world, args.profile_layers),
            "roofline": roofline, "matvec": matvec,
            "gpu_launches": launches,
            "clocks": clk,
            "e2e": {"value": world * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 32,
                    "d2h_bytes_per_step": vocab * 4},
            "cpu_baseline": cpu,
            "parity": parity,
            "prefill": prefill,
            "w4a8": w4a8,
            "tp13b": tp13b,
        }
        print(json.dumps(line), flush=True)
    model.close()
    if pg:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
