"""The tcgen05 bf16 GEMM (aion_gemm_bf16_tn) against an fp32 product of the
same bf16 operands, through the C ABI.

bf16 x bf16 products are exact in fp32, so the only difference is the order
of the fp32 accumulation: |C - C_ref| <= 1e-5 * sum_k |a_k b_k| per entry.
"""
from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 512), (512, 768, 4096), (1024, 256, 11008)])
def test_gemm_bf16_matches_fp32(cuda, m, n, k):
    import aion_b200 as A
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(n, k, device="cuda", generator=g)).to(torch.bfloat16)
    c = torch.full((m, n), float("nan"), device="cuda")
    st = A.lib().aion_gemm_bf16_tn(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                                   ctypes.c_void_p(c.data_ptr()), m, n, k, None)
    assert st == 0, A.lib().aion_last_error(None)
    torch.cuda.synchronize()
    af, bf = a.float(), b.float()
    want = af @ bf.t()
    bound = 1e-5 * (af.abs() @ bf.abs().t()) + 1e-30
    assert torch.isfinite(c).all()
    assert ((c - want).abs() <= bound).all(), float(((c - want).abs() / bound).max())


def test_gemm_rejects_bad_shape(cuda):
    import aion_b200 as A
    torch = cuda
    a = torch.zeros(100, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(256, 64, device="cuda", dtype=torch.bfloat16)
    c = torch.zeros(100, 256, device="cuda")
    st = A.lib().aion_gemm_bf16_tn(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                                   ctypes.c_void_p(c.data_ptr()), 100, 256, 64, None)
    assert st == 3
