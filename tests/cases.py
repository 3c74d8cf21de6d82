"""Seeded inputs shared by the fixture generator and the tests.

Matrices are N(0, 0.02) from numpy's default_rng(seed) (the distribution of
the workload's random-init weights), quantized with the quantize.c
arithmetic; activations are N(0, 1) as in the isolated-matvec workload.
"""
from __future__ import annotations

import hashlib

import numpy as np

TINY = (288, 768, 6, 6, 6, 32000, 256)          # dim, hidden, layers, heads, kv_heads, vocab, seq_len
LLAMA7B = (4096, 11008, 32, 32, 32, 32000, 2048)
LLAMA13B = (5120, 13824, 40, 40, 40, 32000, 2048)
SEEDS = {"tiny": 0, "7b": 1, "13b": 3}

# Isolated matvec shapes of the 7B workload (rows x cols).
MATVEC_7B = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]
# Small / ragged shapes: one group, odd row counts, tiny-model shapes.
MATVEC_EDGE = [(1, 32), (3, 64), (5, 288), (7, 768), (288, 288), (768, 288), (288, 768), (33, 4096), (17, 11008)]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def matrix(d: int, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((d, n), dtype=np.float32) * np.float32(0.02)).astype(np.float32)


def vector(n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed + 1_000_003)
    return rng.standard_normal(n, dtype=np.float32)


def case_seed(d: int, n: int) -> int:
    return (d * 1_000_003 + n) % (2 ** 31)


def quantizer_kat_inputs() -> dict[str, np.ndarray]:
    """Hand-built edge groups for the quantizer (quantize.c:66-107)."""
    s = np.float32(0.7) / np.float32(7.0)   # a scale
    ties = np.array([7.5, -7.5, 6.5, -6.5, 5.5, -5.5, 4.5, -4.5, 3.5, -3.5, 2.5, -2.5, 1.5, -1.5, 0.5, -0.5] * 2,
                    np.float32)
    cases = {
        "zeros": np.zeros(32, np.float32),                                   # scale -> 1.0
        "one_hot": np.eye(1, 32, 5, dtype=np.float32).ravel() * np.float32(3.0),
        "half_ties": (ties / np.float32(7.5)).astype(np.float32) * np.float32(0.7),
        "scaled_ties": (np.arange(-16, 16, dtype=np.float32) + np.float32(0.5)) * s,
        "clamp": np.linspace(-1.0, 1.0, 32, dtype=np.float32),
        "tiny_values": np.full(32, 1e-30, np.float32),
        "negative_max": -np.abs(np.linspace(0.01, 0.5, 32, dtype=np.float32)),
        "random": matrix(4, 32, 11).ravel(),
    }
    return cases


def actquant_kat_inputs() -> dict[str, np.ndarray]:
    """Edge groups for the activation quantizer (src/kernel_simd.c:186-227)."""
    base = np.linspace(-1, 1, 32, dtype=np.float32)
    return {
        "zeros": np.zeros(32, np.float32),                                    # amax <= 1e-9 -> scale 1
        "below_eps": np.full(32, 5e-10, np.float32),
        "at_eps": np.full(32, 1e-9, np.float32),
        "ramp": base,
        "half_ties": (np.arange(-16, 16, dtype=np.float32) + np.float32(0.5)) / np.float32(127.0) * np.float32(16),
        "large": base * np.float32(1e6),
        "random": vector(64, 5),
    }
