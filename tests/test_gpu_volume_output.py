"""prepare_volume_output on the GPU (lsrm_prepare_volume_output) vs the
reference fixture and the oracle: every output bit-exact (a feature
transpose, integer boundaries and an integer index volume)."""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _run(volume, vidx, C, u, res, batch_size=None):
    from lsrm_sparse import volume as V

    out = V.prepare_volume_output(volume.cuda(), vidx.cuda(), torch.zeros(1, device="cuda"), C, u, res,
                                  batch_size=batch_size)
    torch.cuda.synchronize()
    return out


def _case(seed, counts, res, u, C, dtype):
    g = torch.Generator().manual_seed(seed)
    parts = []
    for b, n in enumerate(counts):
        flat = torch.randperm(res ** 3, generator=g)[:n]
        z, y, x = flat // (res * res), (flat // res) % res, flat % res
        parts.append(torch.stack([torch.full_like(z, b), z, y, x], 1))
    vidx = torch.cat(parts).to(torch.int32)
    volume = torch.randn(vidx.shape[0], C * u ** 3, generator=g).to(dtype)
    return volume, vidx


def _check(out, volume, vidx, C, u, res, B=None):
    from lsrm_sparse import ops

    assert ops.read_errors() == 0
    feat, cu, seqlens, iv = oracle.prepare_volume_output(volume.float().numpy() if volume.dtype == torch.bfloat16
                                                         else volume.numpy(), vidx.numpy(), C, u, res, batch_size=B)
    got = out["sparse_feat"].cpu()
    if volume.dtype == torch.bfloat16:
        assert torch.equal(got.float(), torch.from_numpy(feat))
    else:
        assert np.array_equal(got.numpy(), feat)
    assert np.array_equal(out["cu_seqlens"].cpu().numpy(), cu)
    assert np.array_equal(out["seqlens"].cpu().numpy(), seqlens)
    assert np.array_equal(out["index_volume"].cpu().numpy(), iv)


def test_volume_output_matches_reference_fixture(golden):
    g = golden("volume_output")
    C, u, res = int(g["output_dim"]), int(g["upsample_scale"]), int(g["vol_res"])
    out = _run(torch.from_numpy(g["volume"]), torch.from_numpy(g["volume_index"]), C, u, res)
    from lsrm_sparse import ops

    assert ops.read_errors() == 0
    assert np.array_equal(out["sparse_feat"].cpu().numpy(), g["sparse_feat"])
    assert np.array_equal(out["cu_seqlens"].cpu().numpy(), g["cu_seqlens"])
    assert np.array_equal(out["seqlens"].cpu().numpy(), g["seqlens"])
    assert np.array_equal(out["index_volume"].cpu().numpy(), g["index_volume"])


@pytest.mark.parametrize("u,C,dtype", [(1, 32, torch.float32), (2, 32, torch.bfloat16), (2, 8, torch.float32),
                                       (3, 16, torch.bfloat16), (4, 32, torch.float32)])
def test_volume_output_vs_oracle(u, C, dtype):
    res = 20
    volume, vidx = _case(7 + u + C, [900, 3, 1500], res, u, C, dtype)
    out = _run(volume, vidx, C, u, res)
    _check(out, volume, vidx, C, u, res)


def test_volume_output_given_batch_size_and_empty():
    # batch size passed explicitly; an empty input gives empty ranges and an all -1 volume
    volume, vidx = _case(3, [50, 60], 8, 2, 4, torch.float32)
    _check(_run(volume, vidx, 4, 2, 8, batch_size=2), volume, vidx, 4, 2, 8, B=2)
    out = _run(torch.zeros(0, 32), torch.zeros(0, 4, dtype=torch.int32), 4, 2, 8, batch_size=2)
    assert out["sparse_feat"].shape == (0, 4)
    assert out["cu_seqlens"].cpu().tolist() == [0, 0, 0]
    assert out["seqlens"].cpu().tolist() == [0, 0]
    assert bool((out["index_volume"] == -1).all())


def test_volume_output_flags_bad_index():
    from lsrm_sparse import ops

    ops.read_errors()
    volume, vidx = _case(5, [40, 40], 8, 2, 4, torch.float32)
    vidx[10, 1] = 8  # outside the 8^3 token grid
    _run(volume, vidx, 4, 2, 8)
    assert ops.read_errors() & 0x8  # LSRM_ERR_BAD_INDEX


def test_volume_output_gradient_is_the_inverse_transpose():
    """``sparse_feat`` is differentiable with respect to ``volume``: its
    gradient is the reference's reshape / permute (voldecoder.py:200-207)
    taken backward, bit for bit."""
    volume, vidx = _case(7, [300, 200], 16, 2, 8, torch.float32)
    a = volume.cuda().requires_grad_()
    out = _run(a, vidx, 8, 2, 16)
    g = torch.randn(out["sparse_feat"].shape, device="cuda")
    out["sparse_feat"].backward(g)
    b = volume.cuda().requires_grad_()
    ref = b.reshape(-1, 8, 2, 2, 2).permute(0, 2, 3, 4, 1).reshape(-1, 8)
    assert torch.equal(ref.detach(), out["sparse_feat"].detach())
    ref.backward(g)
    assert torch.equal(a.grad, b.grad)
