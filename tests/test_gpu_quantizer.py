"""The device quantizer (aion_quantize_buffer_dev) against quantize_buffer
(quantize.c:59-109): bit-exact on the reference's known-answer groups and on
large seeded buffers, through the C ABI."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu


def _quantize_dev(torch, w: np.ndarray):
    import aion_b200 as A
    x = torch.from_numpy(w).cuda()
    packed = torch.empty(w.size // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(w.size // 32, dtype=torch.float32, device="cuda")
    st = A.lib().aion_quantize_buffer_dev(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(packed.data_ptr()),
                                          ctypes.c_void_p(scales.data_ptr()), w.size, None)
    assert st == 0, A.lib().aion_last_error(None)
    torch.cuda.synchronize()
    return packed.cpu().numpy(), scales.cpu().numpy()


@pytest.mark.parametrize("name", sorted(cases.quantizer_kat_inputs()))
def test_device_quantizer_kats(cuda, golden_kat, name):
    w = cases.quantizer_kat_inputs()[name]
    packed, scales = _quantize_dev(cuda, w)
    want = golden_kat["quantizer"].get(name)
    if want is not None:
        assert packed.tolist() == want["packed"]
        assert scales.view(np.uint32).tolist() == want["scales_hex"]
    import aion_b200 as A
    hp, hs = A.quantize_buffer(w)
    assert (packed == hp).all() and (scales.view(np.uint32) == hs.view(np.uint32)).all()


@pytest.mark.parametrize("n,scale", [(32 * 4097, 0.02), (11008 * 4096, 1.0)])
def test_device_quantizer_matches_host(cuda, n, scale):
    import aion_b200 as A
    w = (np.random.default_rng(n).standard_normal(n, dtype=np.float32) * np.float32(scale)).astype(np.float32)
    packed, scales = _quantize_dev(cuda, w)
    hp, hs = A.quantize_buffer(w)
    assert (packed == hp).all() and (scales.view(np.uint32) == hs.view(np.uint32)).all()
