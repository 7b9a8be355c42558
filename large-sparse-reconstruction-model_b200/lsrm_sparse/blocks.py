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
