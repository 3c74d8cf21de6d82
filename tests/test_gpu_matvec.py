"""Kernel-level parity on the GPU, through the C ABI.

Tolerances:
  - re-tile / inverse, activation quantization, W4A8 matvec: bit-exact;
  - W4A16 matvec: the kernel represents the activations as integers
    X = round(x * 2^E) with one exponent per vector (max |x| * 2^E in
    [2^29, 2^30)), computes exact integer group dots and accumulates them in
    fp32.  Per row, against a float64 evaluation of the same int4 matrix:
    |y - y_exact| <= 2^-19 * sum_k |w_k| m_g(k) + 2^-28 * max|x| * sum_k |w_k|
    (+ 1e-30; m_g = the largest magnitude of x's group), a bound the fp32
    sequential oracle meets as well, so |y - y_oracle| is within twice it.
"""
from __future__ import annotations

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu

SHAPES = cases.MATVEC_7B + cases.MATVEC_EDGE


def dequant(packed: np.ndarray, scales: np.ndarray, d: int, n: int) -> np.ndarray:
    lo = (packed & 0xF).astype(np.int8) - 8
    hi = (packed >> 4).astype(np.int8) - 8
    q = np.stack([lo, hi], axis=-1).reshape(d, n).astype(np.float64)
    return q * np.repeat(scales.astype(np.float64).reshape(d, n // 32), 32, axis=1)


@pytest.fixture(scope="module")
def mats():
    import aion_b200 as A
    out = {}
    for d, n in SHAPES:
        seed = cases.case_seed(d, n)
        packed, scales = A.quantize_buffer(cases.matrix(d, n, seed))
        out[(d, n)] = (seed, packed, scales)
    return out


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_retile_roundtrip(cuda, mats, shape):
    import aion_b200 as A
    d, n = shape
    _, packed, scales = mats[shape]
    q = A.QMatrix(scales, packed, d, n)
    s2, p2 = q.download()
    assert (p2 == packed).all() and (s2.view(np.uint32) == scales.view(np.uint32)).all()
    q.free()


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("xscale", [1.0, 1e-3, 1e3])
def test_matvec_w4a16(cuda, oracle, mats, shape, xscale):
    import aion_b200 as A
    torch = cuda
    d, n = shape
    seed, packed, scales = mats[shape]
    x = (cases.vector(n, seed) * np.float32(xscale)).astype(np.float32)
    q = A.QMatrix(scales, packed, d, n)
    xt = torch.from_numpy(x).cuda()
    y = torch.full((d,), float("nan"), device="cuda")
    q.matvec_w4a16(xt, y)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    ref = oracle.matvec_w4a16(x, scales, packed, n, d)
    assert np.isfinite(got).all()
    w = dequant(packed, scales, d, n)
    exact = w @ x.astype(np.float64)
    mg = np.repeat(np.abs(x.astype(np.float64)).reshape(-1, 32).max(axis=1), 32)
    bound = 2.0 ** -19 * (np.abs(w) @ mg) + 2.0 ** -28 * np.abs(x).max() * np.abs(w).sum(axis=1) + 1e-30
    assert (np.abs(got - exact) <= bound).all()
    assert (np.abs(ref - exact) <= bound).all()
    assert (np.abs(got - ref) <= 2 * bound).all()
    q.free()


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_matvec_w4a8_bit_exact(cuda, oracle, mats, shape):
    import aion_b200 as A
    torch = cuda
    d, n = shape
    seed, packed, scales = mats[shape]
    x = cases.vector(n, seed)
    if n >= 64:
        x[32:64] = 0.0          # a group with amax <= 1e-9 (scale 1, all-zero int8)
    q = A.QMatrix(scales, packed, d, n)
    y = torch.empty(d, device="cuda")
    q.matvec_w4a8(torch.from_numpy(x).cuda(), y)
    torch.cuda.synchronize()
    ref = oracle.matvec_w4a8(x, scales, packed, n, d)
    assert (y.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()
    q.free()


@pytest.mark.parametrize("name", sorted(cases.actquant_kat_inputs()))
def test_quantize_activations_bit_exact(cuda, golden_kat, name):
    import aion_b200 as A
    torch = cuda
    x = cases.actquant_kat_inputs()[name]
    qx = torch.empty(x.size, dtype=torch.int8, device="cuda")
    xs = torch.empty(x.size // 32, dtype=torch.float32, device="cuda")
    A.quantize_activations(torch.from_numpy(x).cuda(), qx, xs)
    torch.cuda.synchronize()
    want = golden_kat["actquant"][name]
    assert qx.cpu().numpy().tolist() == want["qx"]
    assert xs.cpu().numpy().view(np.uint32).tolist() == want["xs_hex"]


def test_quantize_activations_large(cuda, oracle):
    import aion_b200 as A
    torch = cuda
    x = cases.vector(11008, 77) * np.float32(4.0)
    qx = torch.empty(x.size, dtype=torch.int8, device="cuda")
    xs = torch.empty(x.size // 32, dtype=torch.float32, device="cuda")
    A.quantize_activations(torch.from_numpy(x).cuda(), qx, xs)
    rq, rs = oracle.quantize_activations(x)
    assert (qx.cpu().numpy() == rq).all() and (xs.cpu().numpy().view(np.uint32) == rs.view(np.uint32)).all()


def test_matvec_on_a_side_stream(cuda, oracle, mats):
    import aion_b200 as A
    torch = cuda
    d, n = 4096, 4096
    seed, packed, scales = mats[(d, n)]
    x = cases.vector(n, seed)
    q = A.QMatrix(scales, packed, d, n)
    s = torch.cuda.Stream()
    xt = torch.from_numpy(x).cuda()
    with torch.cuda.stream(s):
        y = torch.empty(d, device="cuda")
        for _ in range(3):
            q.matvec_w4a16(xt, y, stream=s)
    s.synchronize()
    ref = oracle.matvec_w4a16(x, scales, packed, n, d)
    assert np.abs(y.cpu().numpy() - ref).max() <= 2e-5 * np.abs(ref).max()


def test_matvec_on_the_second_device(cuda, mats):
    """The kernel-level matvec sets its shared-memory opt-in per device: a
    call on device 1 after calls on device 0 gives device 0's result."""
    import aion_b200 as A
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    d, n = 11008, 4096
    seed, packed, scales = mats[(d, n)]
    x = cases.vector(n, seed)
    out = []
    for dev in (0, 1, 0, 1):
        with torch.cuda.device(dev):
            q = A.QMatrix(scales, packed, d, n, device=dev)
            xt = torch.from_numpy(x).to(f"cuda:{dev}")
            y = torch.full((d,), float("nan"), device=f"cuda:{dev}")
            q.matvec_w4a16(xt, y)
            q.status()
            out.append(y.cpu().numpy())
            q.free()
    for y in out[1:]:
        assert (y.view(np.uint32) == out[0].view(np.uint32)).all()


def test_matvec_status_reports_a_timeout(cuda, mats):
    """A matvec whose bounded wait gave up leaves its error word set;
    aion_matvec_status reports it once (AION_ERR_TIMEOUT, y invalid) and
    clears it.  The error is recorded from the host, not provoked on the GPU."""
    import aion_b200 as A
    torch = cuda
    L = A.lib()
    d, n = 4096, 4096
    seed, packed, scales = mats[(d, n)]
    q = A.QMatrix(scales, packed, d, n)
    xt = torch.from_numpy(cases.vector(n, seed)).cuda()
    y = torch.empty(d, device="cuda")
    q.matvec_w4a16(xt, y)
    assert L.aion_matvec_status(q._h, None) == 0
    assert L.aion_matvec_inject_timeout(q._h) == 0
    assert L.aion_matvec_status(q._h, None) == 7          # AION_ERR_TIMEOUT
    assert b"gave up" in L.aion_last_error(None)
    assert L.aion_matvec_status(q._h, None) == 0          # cleared
    q.matvec_w4a16(xt, y)                                 # the matrix stays usable
    assert L.aion_matvec_status(q._h, None) == 0
    q.free()
