"""CrossAttention's cross/self gate (models_sparse/utils.py:559-570) through
lsrm_sparse.module.CrossSelfGate (fused sigmoid + two-way merge) vs the
reference's formula evaluated in fp32 PyTorch on the same bf16 inputs and
weights: forward and all gradients within 2e-2 max-abs and >= 0.9995 cosine."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cos(a, b):
    a, b = a.detach().double().flatten(), b.detach().double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


@pytest.mark.parametrize("n,dim", [(1000, 64), (4099, 256), (257, 1024)])
def test_cross_self_gate_vs_fp32(n, dim):
    from lsrm_sparse import ops
    from lsrm_sparse.module import CrossSelfGate

    torch.manual_seed(n + dim)
    dev = torch.device("cuda")
    mod = CrossSelfGate(dim).to(dev).to(torch.bfloat16)
    x = torch.randn(n, dim, device=dev, dtype=torch.bfloat16, requires_grad=True)
    xc = torch.randn(n, dim, device=dev, dtype=torch.bfloat16, requires_grad=True)
    xs = torch.randn(n, dim, device=dev, dtype=torch.bfloat16, requires_grad=True)
    out = mod(x, xc, xs)
    go = torch.randn_like(out) * 0.1
    out.backward(go)
    assert ops.read_errors() == 0

    # the reference's formula in fp32 on the same values
    W1, b1 = mod.gate_x[0].weight.float().detach(), mod.gate_x[0].bias.float().detach()
    W2, b2 = mod.proj_x.weight.float().detach(), mod.proj_x.bias.float().detach()
    xr, xcr, xsr = (t.detach().float().requires_grad_() for t in (x, xc, xs))
    g = torch.sigmoid(xr @ W1.t() + b1)
    ref = (xcr * g[:, :dim] + xsr * g[:, dim:]) @ W2.t() + b2
    ref.backward(go.float())
    scale = max(1.0, float(ref.abs().max()))
    assert float((out.float() - ref).abs().max()) <= 2e-2 * scale
    assert _cos(out, ref) >= 0.9995
    for got, want in ((x.grad, xr.grad), (xc.grad, xcr.grad), (xs.grad, xsr.grad)):
        assert float((got.float() - want).abs().max()) <= 2e-2 * max(1.0, float(want.abs().max()))
        assert _cos(got, want) >= 0.9995
