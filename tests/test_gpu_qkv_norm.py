"""The projection GEMM with the per-head LayerNorm32 in its epilogue
(lsrm_qkv_norm_fwd / _bwd through ``functional.qkv_norm``) against the
reference's unfused formulation in torch: the q / k / v Linears
(models_sparse/utils.py:114-127), then LayerNorm32 of q and k per head
(non-affine over head_dim, fp32, cast back; :239-270).  Outputs and the
gradients of x and of every weight (and bias) within 2e-2 max-abs (relative
to the tensor's scale) and >= 0.9995 cosine.  Cases: head_dim 64 and 32,
row counts that leave a partial tile, a k / v width that is not a multiple of
the 128-column tile, with and without bias; and one decoder block with the
fused projections against the same block without."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _close(a, b):
    assert a.shape == b.shape
    assert torch.isfinite(a).all()
    a, b = a.detach().float(), b.detach().float()
    scale = max(1.0, float(b.abs().max()))
    assert float((a - b).abs().max()) <= 2e-2 * scale
    a, b = a.double().flatten(), b.double().flatten()
    assert float(a @ b / (a.norm() * b.norm() + 1e-30)) >= 0.9995


def _ln_heads(t, D):
    n = t.shape[0]
    return torch.nn.functional.layer_norm(t.float().view(n, -1, D), (D,), eps=1e-5).to(t.dtype).view(n, -1)


@pytest.mark.parametrize("M,K,dim,kv,D,bias", [(1000, 256, 256, 128, 64, False), (777, 128, 128, 64, 32, True),
                                              (4096, 1024, 1024, 64, 32, False)])
def test_qkv_norm_matches_linears_then_layernorm(M, K, dim, kv, D, bias):
    from lsrm_sparse import functional as F
    from lsrm_sparse import ops

    torch.manual_seed(0)
    lins = [torch.nn.Linear(K, n, bias=bias).to(DEV).bfloat16() for n in (dim, kv, kv)]
    x0 = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    gq, gk, gkn, gv = (torch.randn(M, n, device=DEV, dtype=torch.bfloat16) for n in (dim, kv, kv, kv))
    res = []
    for fused in (True, False):
        for lin in lins:
            lin.zero_grad()
        x = x0.clone().requires_grad_()
        if fused:
            (_, q), (k, kn), (v, _) = F.qkv_norm(x, lins, [(False, True), (True, True), (True, False)], D)
        else:
            q, k, v = (lin(x) for lin in lins)
            q, kn = _ln_heads(q, D), _ln_heads(k, D)
        (q.float() * gq).sum().backward(retain_graph=True)
        ((k.float() * gk).sum() + (kn.float() * gkn).sum() + (v.float() * gv).sum()).backward()
        grads = [x.grad] + [lin.weight.grad.clone() for lin in lins]
        if bias:
            grads += [lin.bias.grad.clone() for lin in lins]
        res.append(([q, k, kn, v], grads))
    assert ops.read_errors() == 0
    for a, b in zip(res[0][0] + res[0][1], res[1][0] + res[1][1]):
        _close(a, b)


def test_blockmix_with_fused_projections_matches_unfused():
    from lsrm_sparse import ops
    from lsrm_sparse.decoder import BlockMix
    from tests.test_gpu_decoder import _scene

    torch.manual_seed(0)
    maps, cu_x, cu_y, nx, ny, M = _scene()
    blocks = [BlockMix(128, num_q_heads=2, num_kv_heads=2, fused_qkv=f).to(DEV).to(torch.bfloat16)
              for f in (False, True)]
    blocks[1].load_state_dict(blocks[0].state_dict())
    x0 = torch.randn(nx, 128, device=DEV, dtype=torch.bfloat16)
    y0 = torch.randn(ny, 128, device=DEV, dtype=torch.bfloat16)
    outs = []
    for blk in blocks:
        x, y = x0.clone().requires_grad_(), y0.clone().requires_grad_()
        ox, oy, _ = blk(x, cu_x, y, cu_y, maps, M)
        g = torch.Generator(device=DEV).manual_seed(1)
        ((ox.float() * torch.randn(ox.shape, device=DEV, generator=g)).sum() +
         (oy.float() * torch.randn(oy.shape, device=DEV, generator=g)).sum()).backward()
        ca = blk.crs_attn
        outs.append([ox, oy, x.grad, y.grad, ca.q_proj_x.weight.grad, ca.k_proj_x.weight.grad,
                     ca.v_proj_y.weight.grad, ca.q_proj_y.weight.grad])
    assert ops.read_errors() == 0
    for a, b in zip(outs[1], outs[0]):
        _close(a, b)
