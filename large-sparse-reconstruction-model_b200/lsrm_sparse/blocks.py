"""Block metadata of sparse voxel sequences on the device.

Mirrors ``sort_volume_blocks`` (misc/sparse_utils.py:126-152) and
``compute_block_separation`` (misc/sparse_utils.py:592-641): same arguments,
same results.  The keys and the per-cell histogram are CUDA kernels of
liblsrm_sparse.so; the sort itself is torch's (a library radix sort).
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib, ops
from ._lib import check


def volume_sort_keys(coords: torch.Tensor, volume_res: int, block_size: int) -> torch.Tensor:
    """int64 key per voxel: batch, block cell (z, y, x), position in the cell."""
    L = _lib.lib()
    coords = coords.to(torch.int32).contiguous()
    if coords.dim() != 2 or coords.shape[1] != 4:
        raise ValueError("coords must be [n, 4] (batch, z, y, x)")
    keys = torch.empty(coords.shape[0], dtype=torch.int64, device=coords.device)
    rc = L.lsrm_volume_sort_keys(coords.shape[0], ops._ptr(coords), int(volume_res), int(block_size), ops._ptr(keys),
                                 ops._stream())
    check(rc, "lsrm_volume_sort_keys")
    return keys


def sort_volume_blocks(feats, coords, args, coords_idx=None):
    """Reorders voxels block-major; returns ``(feats, coords, coords_idx)``.
    ``args`` needs ``block_size`` and ``volume_res`` (the reference reads
    them from its run arguments)."""
    if coords_idx is None:
        keys = volume_sort_keys(coords, args.volume_res, args.block_size)
        coords_idx = torch.argsort(keys)
    return feats[coords_idx, :], coords[coords_idx, :], coords_idx


def compute_block_separation(k_coords: torch.Tensor, DIM: int, block_size: Sequence[int], batch_size: int,
                             resolution: Sequence[int]):
    """``(cu_seqblocks, cu_block_include_tokens)`` int32 on the coordinates'
    device.  Unlike the reference, ``k_coords`` is not modified.  One host
    synchronisation (the number of blocks sizes the result)."""
    cu_seqblocks, cu_blk, _ = block_separation(k_coords, DIM, block_size, int(batch_size), resolution)
    return cu_seqblocks, cu_blk


def block_separation(k_coords: torch.Tensor, DIM: int, block_size: Sequence[int], batch_size: int,
                     resolution: Sequence[int]):
    """Returns ``(cu_seqblocks, cu_block_include_tokens, cu_seqlens)``."""
    L = _lib.lib()
    dev = k_coords.device
    coords = k_coords.to(torch.int32).contiguous()
    n = coords.shape[0]
    if coords.dim() != 2 or coords.shape[1] != DIM + 1:
        raise ValueError(f"k_coords must be [n, {DIM + 1}]")
    bs = (ctypes.c_int32 * DIM)(*[int(x) for x in block_size[:DIM]])
    res = (ctypes.c_int32 * DIM)(*[int(x) for x in resolution[:DIM]])
    nbytes = L.lsrm_block_separation_workspace_bytes(DIM, bs, res, int(batch_size))
    if nbytes == 0:
        raise ValueError("bad block separation arguments")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    cu_seqlens = torch.empty(batch_size + 1, dtype=torch.int32, device=dev)
    cu_seqblocks = torch.empty(batch_size + 1, dtype=torch.int32, device=dev)
    cu_blk = torch.empty(n + 1, dtype=torch.int32, device=dev)
    nblk = torch.empty(1, dtype=torch.int32, device=dev)
    rc = L.lsrm_block_separation(n, ops._ptr(coords), DIM, bs, res, int(batch_size), ops._ptr(cu_seqlens),
                                 ops._ptr(cu_seqblocks), ops._ptr(cu_blk), ops._ptr(nblk), ops._ptr(ws), nbytes,
                                 ops._ptr(ops._err_word(dev)), ops._stream())
    check(rc, "lsrm_block_separation")
    nb = int(nblk.item())
    return cu_seqblocks, cu_blk[: nb + 1], cu_seqlens


def volume_block_topk(coords: torch.Tensor, cu_seqblocks: torch.Tensor, cu_block_include_tokens: torch.Tensor,
                      batch_size: int, volume_res: int, bbox_radius: float, topk: int) -> torch.Tensor:
    """[n, topk] int32: per voxel token the topk blocks of its batch element
    nearest to it (block centre = mean of its voxels' points), sorted ids,
    -1 padding.  No host synchronisation."""
    L = _lib.lib()
    coords = coords.to(torch.int32).contiguous()
    if coords.dim() != 2 or coords.shape[1] != 4:
        raise ValueError("coords must be [n, 4] (batch, z, y, x)")
    n = coords.shape[0]
    out = torch.empty(n, int(topk), dtype=torch.int32, device=coords.device)
    cent = torch.empty(max(n, 1), 3, dtype=torch.float32, device=coords.device)
    radius = float(bbox_radius) * 1.05  # as from_volcoords_to_points (misc/sparse_utils.py:645)
    rc = L.lsrm_volume_block_topk(ops._ptr(coords), n, ops._ptr(ops._i32(cu_seqblocks)),
                                  ops._ptr(ops._i32(cu_block_include_tokens)), int(batch_size), int(volume_res),
                                  radius, int(topk), ops._ptr(cent), ops._ptr(out),
                                  ops._ptr(ops._err_word(coords.device)), ops._stream())
    check(rc, "lsrm_volume_block_topk")
    return out


def build_volume_to_volume_attn(volfeat_coords: torch.Tensor, args):
    """``build_volume_to_volume_attn`` (misc/sparse_utils.py:1203-1279): the
    block separation of the (block-sorted) voxel tokens and, with
    ``args.use_3d_aware_attn``, the geometric top-``args.topk_volume`` block
    selection, stacked twice as the reference does.  Same arguments and dict
    keys; ``volfeat_coords`` is not modified.  One host synchronisation for the
    batch size (as the reference) and one inside the separation."""
    bs = int(args.block_size)
    res = int(args.volume_res)
    batch_size = int(volfeat_coords[:, 0].max().item()) + 1
    cu_seqblocks, cu_blk, _ = block_separation(volfeat_coords, 3, [bs, bs, bs], batch_size, [res, res, res])
    block_topk = None
    if getattr(args, "use_3d_aware_attn", False):
        bt = volume_block_topk(volfeat_coords, cu_seqblocks, cu_blk, batch_size, res, args.bbox_radius,
                               args.topk_volume)
        block_topk = torch.stack([bt, bt], dim=0)
    return {"block_topk": block_topk, "cu_seqblocks": cu_seqblocks.to(torch.int32),
            "cu_block_include_tokens": cu_blk.to(torch.int32)}
