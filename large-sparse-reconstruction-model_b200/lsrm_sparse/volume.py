"""Output formatting of the upsampled volume decoder on the device.

Mirrors ``VolTransformer.prepare_volume_output``
(models_sparse/voldecoder.py:196-268): same arguments (the module's
``output_dim``, ``upsample_scale`` and ``vol_res`` passed explicitly), same
output dict.  The reference builds the index volume with one Python loop step
per batch element and reads the batch boundaries back with ``.item()``; here
one library call (``lsrm_prepare_volume_output``) writes everything on the
current stream.  ``batch_size`` may be given to avoid the one host read of
``volume_index[:, 0].max()`` that the reference also does.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib, ops
from ._lib import check


def prepare_volume_output(volume: torch.Tensor, volume_index: torch.Tensor, prior_volume: torch.Tensor,
                          output_dim: int, upsample_scale: int, vol_res: int,
                          batch_size: Optional[int] = None) -> dict:
    """volume [N, output_dim * u^3] (channel-major per token), volume_index
    [N, 4] int (batch, z, y, x), grouped by ascending batch id.  Returns
    sparse_feat [N * u^3, output_dim], dense_feat (= prior_volume),
    cu_seqlens / seqlens (int32, in sub-voxels) and index_volume
    [B, R*u, R*u, R*u] int32 (-1 where no sub-voxel lies).  ``sparse_feat``
    is differentiable with respect to ``volume``."""
    u = int(upsample_scale)
    S = u ** 3
    if volume.dim() != 2 or volume.shape[1] != output_dim * S:
        raise ValueError(f"volume must be [N, output_dim * upsample_scale^3] = [N, {output_dim * S}]")
    if volume.element_size() not in (2, 4):
        raise TypeError(f"volume elements must be 2 or 4 bytes, got {volume.dtype}")
    vidx = volume_index.to(torch.int32).contiguous()
    if vidx.dim() != 2 or vidx.shape[1] != 4 or vidx.shape[0] != volume.shape[0]:
        raise ValueError("volume_index must be [N, 4] (batch, z, y, x)")
    if batch_size is None:
        batch_size = int(vidx[:, 0].max().item()) + 1 if vidx.shape[0] else 1
    sparse_feat, cu, seqlens, index_volume = _PrepareVolumeOutput.apply(volume, vidx, int(output_dim), u,
                                                                        int(vol_res), int(batch_size))
    return {"sparse_feat": sparse_feat, "dense_feat": prior_volume, "cu_seqlens": cu, "seqlens": seqlens,
            "index_volume": index_volume}


class _PrepareVolumeOutput(torch.autograd.Function):
    """The library call as an autograd node: ``sparse_feat`` row (n, s)
    channel c is ``volume[n, c * u^3 + s]``, so its gradient flows back to
    ``volume`` by the inverse transpose (the reference's reshape / permute is
    differentiable the same way); the offsets and the index volume are
    integer outputs."""

    @staticmethod
    def forward(ctx, volume, vidx, output_dim, u, vol_res, batch_size):
        L = _lib.lib()
        S = u ** 3
        volume = volume.contiguous()
        dev = volume.device
        n, R = volume.shape[0], vol_res * u
        sparse_feat = torch.empty(n * S, output_dim, dtype=volume.dtype, device=dev)
        cu = torch.empty(batch_size + 1, dtype=torch.int32, device=dev)
        seqlens = torch.empty(batch_size, dtype=torch.int32, device=dev)
        index_volume = torch.empty(batch_size, R, R, R, dtype=torch.int32, device=dev)
        rc = L.lsrm_prepare_volume_output(ops._ptr(volume), volume.element_size(), ops._ptr(vidx), n, output_dim,
                                          u, vol_res, batch_size, ops._ptr(sparse_feat), ops._ptr(cu),
                                          ops._ptr(seqlens), ops._ptr(index_volume), ops._ptr(ops._err_word(dev)),
                                          ops._stream())
        check(rc, "lsrm_prepare_volume_output")
        ctx.od, ctx.S = output_dim, S
        ctx.mark_non_differentiable(cu, seqlens, index_volume)
        return sparse_feat, cu, seqlens, index_volume

    @staticmethod
    def backward(ctx, g, *_):
        if g is None:
            return None, None, None, None, None, None
        dv = g.reshape(-1, ctx.S, ctx.od).transpose(1, 2).reshape(-1, ctx.od * ctx.S)
        return dv, None, None, None, None, None
