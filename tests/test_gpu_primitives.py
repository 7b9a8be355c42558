"""tcgen05 / TMA building blocks against torch fp32 matmul (GPU)."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D", [64, 32])
def test_umma_selftest(D):
    from lsrm_sparse import _lib

    lib = _lib.lib()
    g = torch.Generator(device="cuda").manual_seed(D)
    a = torch.randn(128, D, device="cuda", generator=g).bfloat16()
    b = torch.randn(128, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(128, D, device="cuda", generator=g).bfloat16()
    p = torch.rand(128, 128, device="cuda", generator=g).bfloat16()
    c1 = torch.full((128, 128), float("nan"), device="cuda")
    c2 = torch.full((128, D), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.lsrm_umma_selftest(D, a.data_ptr(), b.data_ptr(), p.data_ptr(), v.data_ptr(), c1.data_ptr(),
                                c2.data_ptr(), err.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "umma selftest")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref1 = a.float() @ b.float().t()
    ref2 = p.float() @ v.float()
    assert torch.allclose(c1, ref1, atol=1e-3, rtol=1e-4), (c1 - ref1).abs().max()
    assert torch.allclose(c2, ref2, atol=1e-3, rtol=1e-4), (c2 - ref2).abs().max()
