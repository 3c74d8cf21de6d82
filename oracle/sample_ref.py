"""CPU restatement of the device sampler (aion_b200/csrc/sample.cuh), the
checker for its draws.  Test infrastructure only.

The reference has no sampler (src/kernel_simd.c:1236-1243 takes the argmax;
PROB_EPSILON at :37 is unused), so this restates the product's own
definition: integer weights floor(e^((l - max) / T) * 2^32) (float32
subtract and divide, e^x in double rounded to float32), top-k then top-p
thresholds on the order-preserving logit keys, and a SplitMix64 draw of
(seed, stream, position) scanned in index order.  Given the same logits it
returns the same token as the device.
"""
from __future__ import annotations

import math

import numpy as np

M64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M64
    return x ^ (x >> 31)


def uniform(seed: int, stream: int, pos: int) -> float:
    h = splitmix64(splitmix64(seed ^ ((stream * 0xD1B54A32D192ED03) & M64)) ^ pos)
    return (h >> 11) * (1.0 / 9007199254740992.0)


def order_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def weights(logits: np.ndarray, mx: float, temperature: float) -> np.ndarray:
    d = (np.asarray(logits, np.float32) - np.float32(mx)).astype(np.float32)
    q = (d / np.float32(temperature)).astype(np.float32)
    w = np.exp(q.astype(np.float64)).astype(np.float32)
    return (w * np.float32(4294967296.0)).astype(np.uint64)


def _threshold(keys: np.ndarray, vals: np.ndarray, need: int) -> int:
    """Largest key t with sum(vals[keys >= t]) >= need."""
    uk, inv = np.unique(keys, return_inverse=True)          # ascending unique keys
    mass = np.zeros(uk.size, np.uint64)
    np.add.at(mass, inv, vals.astype(np.uint64))
    cum = 0
    for j in range(uk.size - 1, -1, -1):
        cum += int(mass[j])
        if cum >= need:
            return int(uk[j])
    return int(uk[0])


def sample(logits, temperature: float, top_p: float = 1.0, top_k: int = 0, seed: int = 0, stream: int = 0,
           pos: int = 0) -> int:
    lg = np.asarray(logits, np.float32)
    V = lg.size
    mx = float(lg.max()) if lg.max() > np.float32(-1e9) else -1e9
    keys = order_bits(lg)
    w = weights(lg, np.float32(mx), temperature)
    lo = 0
    if 0 < top_k < V:
        lo = _threshold(keys, np.ones(V, np.uint64), top_k)
    if np.float32(top_p) < np.float32(1.0):
        keep = keys >= lo
        mk = int(w[keep].sum(dtype=np.uint64))
        need = max(1, math.ceil(float(np.float32(top_p)) * float(mk)))
        tp = _threshold(keys[keep], w[keep], need)
        lo = max(lo, tp)
    keep = keys >= lo
    wk = np.where(keep, w, np.uint64(0))
    M = int(wk.sum(dtype=np.uint64))
    r = math.floor(uniform(seed, stream, pos) * float(M))
    cs = np.cumsum(wk, dtype=np.uint64)
    return int(np.searchsorted(cs, np.uint64(r), side="right"))
