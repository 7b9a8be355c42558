"""Ulysses pack / unpack kernels vs their torch restatement (bit-exact), and
the single-rank whole-sequence op they wrap."""

import pytest
import torch

from tests.test_ulysses_gloo import pack_ref, unpack_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,H,D,world", [(1000, 16, 64, 8), (333, 16, 64, 2), (77, 8, 32, 4), (5, 2, 64, 8),
                                         (129, 4, 16, 2), (0, 16, 64, 4), (64, 1, 64, 4)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_pack_unpack_match_reference(n, H, D, world, dtype):
    from lsrm_sparse import ops

    g = torch.Generator().manual_seed(n + H + world)
    x = torch.randn(n, H, D, generator=g).to(dtype)
    y = ops.ulysses_pack(x.cuda(), world)
    ref = pack_ref(x, world)
    assert y.shape == ref.shape
    assert torch.equal(y.cpu(), ref)
    back = ops.ulysses_unpack(y, H)
    assert torch.equal(back.cpu(), unpack_ref(ref, H))
    if H >= world:
        assert torch.equal(back.cpu(), x)


def test_pack_strided_source():
    from lsrm_sparse import ops

    x = torch.randn(300, 24, 64, dtype=torch.bfloat16, device="cuda")
    view = x[:, 4:20]  # token stride 24*64, 16 heads
    y = ops.ulysses_pack(view, 4)
    assert torch.equal(y.cpu(), pack_ref(view.cpu().contiguous(), 4))
