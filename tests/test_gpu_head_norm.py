"""Per-head LayerNorm fused with the Ulysses pack (lsrm_head_layernorm_pack /
_bwd) vs PyTorch's fp32 LayerNorm (the reference's LayerNorm32, non-affine
over head_dim) and vs the unfused pack: forward and backward."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def _ln_ref(x, eps=1e-5):
    return F.layer_norm(x.float(), (x.shape[-1],), eps=eps).to(x.dtype)


@pytest.mark.parametrize("n,H,D,world,dtype", [(1000, 16, 64, 1, torch.bfloat16), (777, 16, 64, 4, torch.bfloat16),
                                               (513, 8, 128, 2, torch.float16), (300, 4, 16, 4, torch.bfloat16),
                                               (64, 2, 256, 2, torch.float16)])
def test_head_layernorm_pack_forward_backward(n, H, D, world, dtype):
    from lsrm_sparse import ops, ulysses

    g = torch.Generator(device="cuda").manual_seed(n + H + D)
    x = (torch.randn(n, H, D, device="cuda", generator=g) * 3 + 1).to(dtype)
    packed = ops.head_layernorm_pack(x, world)
    ref = _ln_ref(x)
    # same values as the unfused LayerNorm then pack (one rounding step of 16-bit apart at most)
    assert torch.equal(packed, ops.ulysses_pack(ulysses.head_layernorm(x).detach(), world))
    got = ops.ulysses_unpack(packed, H).float()
    assert (got - ref.float()).abs().max().item() <= 0.04
    assert _cos(got, ref) >= 0.99999
    # backward vs autograd of the fp32 LayerNorm
    gy = torch.randn(n, H, D, device="cuda", generator=g).to(dtype)
    xr = x.detach().float().requires_grad_()
    F.layer_norm(xr, (D,), eps=1e-5).backward(gy.float())
    dx = ops.head_layernorm_pack_bwd(x, ops.ulysses_pack(gy, world))
    assert (dx.float() - xr.grad).abs().max().item() <= 0.05 * max(1.0, xr.grad.abs().max().item())
    assert _cos(dx, xr.grad) >= 0.9999


def test_head_layernorm_autograd_and_strided_source():
    from lsrm_sparse import ulysses

    big = torch.randn(400, 3, 8, 64, device="cuda").bfloat16()
    x = big[:, 1]  # token stride 3*8*64 elements
    xr = x.detach().clone().requires_grad_()
    y = ulysses.head_layernorm(xr)
    gy = torch.randn_like(y)
    y.backward(gy)
    xf = x.detach().float().requires_grad_()
    F.layer_norm(xf, (64,), eps=1e-5).backward(gy.float())
    assert _cos(y, _ln_ref(x)) >= 0.99999
    assert _cos(xr.grad, xf.grad) >= 0.9999
