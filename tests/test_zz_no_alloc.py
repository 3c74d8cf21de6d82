"""aion_matvec_w4a16_static (the W4A16 matvec on static device scratch, no
allocation) against aion_matvec_w4a16 on the same matrix, through the C ABI.

The static variant runs the same kernel with its scratch in a fixed device
array, so its results equal the handle-based entry point's; the check
allows 1e-6 relative all the same.  Two calls in a row exercise the
per-call tags of the scratch's cut-tile flags, and a loop of calls leaves
the device's free memory unchanged: the call path allocates nothing.  The
file name makes it collect last, so it also runs after every other GPU test
of the session.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu

AION_ERR_SHAPE = 3
STATIC_MAX_ROWS = 32768


def _vp(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("shape", [(4096, 4096), (32000, 4096), (4096, 11008)], ids=lambda s: f"{s[0]}x{s[1]}")
def test_static_scratch_matvec_matches(cuda, shape):
    import aion_b200 as A
    torch = cuda
    L = A.lib()
    d, n = shape
    seed = cases.case_seed(d, n)
    packed, scales = A.quantize_buffer(cases.matrix(d, n, seed))
    q = A.QMatrix(scales, packed, d, n)
    x = torch.from_numpy(cases.vector(n, seed)).cuda()
    want = torch.full((d,), float("nan"), device="cuda")
    assert L.aion_matvec_w4a16(q._h, _vp(x), _vp(want), None) == 0
    torch.cuda.synchronize()
    scale = float(want.abs().max())
    for _ in range(2):
        got = torch.full((d,), float("nan"), device="cuda")
        st = L.aion_matvec_w4a16_static(q._h, _vp(x), _vp(got), None)
        assert st == 0, L.aion_last_error(None)
        torch.cuda.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        assert np.abs(g - w).max() <= 1e-6 * scale
    assert L.aion_matvec_status(q._h, None) == 0, L.aion_last_error(None)
    # No allocation on the call path: free device memory is unchanged by a
    # run of calls (the first call on the device above resolved the array).
    got = torch.empty(d, device="cuda")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(20):
        assert L.aion_matvec_w4a16_static(q._h, _vp(x), _vp(got), None) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    q.free()


def test_static_scratch_rejects_oversize(cuda):
    import aion_b200 as A
    torch = cuda
    L = A.lib()
    d, n = STATIC_MAX_ROWS + 16, 32
    packed, scales = A.quantize_buffer(cases.matrix(d, n, 11))
    q = A.QMatrix(scales, packed, d, n)
    x = torch.ones(n, device="cuda")
    y = torch.empty(d, device="cuda")
    st = L.aion_matvec_w4a16_static(q._h, _vp(x), _vp(y), None)
    assert st == AION_ERR_SHAPE
    assert b"static scratch limit" in L.aion_last_error(None)
    q.free()
