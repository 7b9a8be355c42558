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


def image_sort_keys(coords: torch.Tensor, views: int, patch_res: int, block_size: int) -> torch.Tensor:
    """int64 key per image token: batch, view, block row, block column,
    position in the block (misc/sparse_utils.py:97-116)."""
    L = _lib.lib()
    coords = coords.to(torch.int32).contiguous()
    if coords.dim() != 2 or coords.shape[1] != 4:
        raise ValueError("coords must be [n, 4] (batch, view, patch row, patch column)")
    keys = torch.empty(coords.shape[0], dtype=torch.int64, device=coords.device)
    rc = L.lsrm_image_sort_keys(coords.shape[0], ops._ptr(coords), int(views), int(patch_res), int(block_size),
                                ops._ptr(keys), ops._stream())
    check(rc, "lsrm_image_sort_keys")
    return keys


def sort_image_blocks(feats, coords, args, coords_idx=None):
    """``sort_image_blocks`` (misc/sparse_utils.py:95-124): reorders image
    tokens block-major; returns ``(feats, coords, coords_idx)``.  ``args``
    needs ``block_size``, ``patch_size`` and ``input_image_res``.  One host
    synchronisation for the view count, as the reference."""
    if coords_idx is None:
        views = int(coords[:, 1].max().item()) + 1
        keys = image_sort_keys(coords, views, int(args.input_image_res[1]) // int(args.patch_size),
                               int(args.block_size))
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


# ---------------------------------------------------------------------------
# Image-side 3D-aware attention maps (misc/sparse_utils.py:644-1300)
# ---------------------------------------------------------------------------

def _f32(t: torch.Tensor, device) -> torch.Tensor:
    return t.to(device=device, dtype=torch.float32).contiguous()


def voxel_points(coords: torch.Tensor, volume_res: int, bbox_radius: float) -> torch.Tensor:
    """``from_volcoords_to_points`` (misc/sparse_utils.py:644-650): [n, 3]
    float32 points of voxel coords (batch, z, y, x)."""
    L = _lib.lib()
    coords = coords.to(torch.int32).contiguous()
    out = torch.empty(coords.shape[0], 3, dtype=torch.float32, device=coords.device)
    rc = L.lsrm_voxel_points(ops._ptr(coords), coords.shape[0], int(volume_res), float(bbox_radius) * 1.05,
                             ops._ptr(out), ops._stream())
    check(rc, "lsrm_voxel_points")
    return out


def from_volcoords_to_points(volcoords: torch.Tensor, args) -> torch.Tensor:
    """Same arguments as the reference function (misc/sparse_utils.py:644)."""
    return voxel_points(volcoords, args.volume_res, args.bbox_radius)


def from_imcoords_to_points(imcoords: torch.Tensor, dense_points, args) -> torch.Tensor:
    """``from_imcoords_to_points`` (misc/sparse_utils.py:653-687): per image
    token (batch, view, patch row, patch column) the surface point of its
    patch whose mask value is largest (the first on ties).  [n, 3] float32."""
    L = _lib.lib()
    dev = imcoords.device
    coords = imcoords.to(torch.int32).contiguous()
    sp = _f32(dense_points["surface_points_input"], dev)
    B, M, S = sp.shape[0], sp.shape[1], sp.shape[2]
    sm = _f32(dense_points["masks_input"], dev).reshape(B, M, S, S)
    pr = int(args.input_image_res[1]) // int(args.patch_size)
    out = torch.empty(coords.shape[0], 3, dtype=torch.float32, device=dev)
    rc = L.lsrm_image_token_points(ops._ptr(coords), coords.shape[0], ops._ptr(sp), ops._ptr(sm), B, M, S, pr,
                                   ops._ptr(out), ops._ptr(ops._err_word(dev)), ops._stream())
    check(rc, "lsrm_image_token_points")
    return out


def camera_terms(batch, device):
    """The per-view values of misc/sparse_utils.py:1097-1135 with the
    reference's own torch calls (batched over views, on ``device``):
    world_to_cam = inverse(camera[:16] as 4x4) [B, M, 4, 4], tan(fov / 2)
    [B, M], and with ``crop_input`` / ``origin_size`` in ``batch``
    (origin - 1, rows start, columns start, crop size - 1) [B, M, 4]."""
    cams = batch["cameras_input"].to(device)
    B, M = cams.shape[:2]
    w2c = torch.inverse(cams[..., :16].reshape(B, M, 4, 4))
    th = torch.tan(cams[..., 16] / 2.0)
    crop = None
    if "crop_input" in batch:
        ci = batch["crop_input"].to(device)
        osz = batch["origin_size"].to(device)[:, 0]
        o1 = (osz - 1)[:, None].expand(B, M)
        crop = torch.stack([o1.to(torch.float32), ci[..., 0].to(torch.float32), ci[..., 2].to(torch.float32),
                            (ci[..., 1] - ci[..., 0] - 1).to(torch.float32)], -1)
    return _f32(w2c, device), _f32(th, device), (None if crop is None else _f32(crop, device))


def view_block_topk(points: torch.Tensor, point_coords: torch.Tensor, batch, dense_points, args) -> torch.Tensor:
    """The view-block selection shared by build_volume_to_image_attn and
    build_image_to_image_attn (misc/sparse_utils.py:1019-1187, :717-885):
    [n, topk_multiimage * image_num_per_batch] int32 per query point.  No host
    synchronisation."""
    dev = points.device
    mi = batch["mask_input"].to(device=dev)[:, :, 0]
    w2c, th, crop = camera_terms(batch, dev)
    return view_block_topk_raw(points, point_coords, mi, dense_points["surface_points_input"],
                               dense_points["masks_input"], w2c, th, crop, int(args.patch_size), int(args.block_size),
                               int(args.attn_winsize) ** 2, int(args.topk_multiimage) * int(args.image_num_per_batch),
                               float(args.bbox_radius) * 2)


def view_block_topk_raw(points, point_coords, mask_input, surface_points, surface_masks, world_to_cam, tan_half,
                        crop, patch_size: int, block_size: int, win: int, topk: int, max_dist: float):
    """``lsrm_view_block_topk`` on tensors: ``mask_input`` [B, M, H, W],
    ``surface_points`` [B, M, S, S, 3], ``surface_masks`` [B, M, S, S(, 1)],
    ``world_to_cam`` [B, M, 4, 4], ``tan_half`` [B, M], ``crop`` [B, M, 4] or
    None (see ``camera_terms``)."""
    L = _lib.lib()
    dev = points.device
    pts = _f32(points, dev)
    qc = point_coords.to(torch.int32).contiguous()
    sp = _f32(surface_points, dev)
    B, M, S = sp.shape[0], sp.shape[1], sp.shape[2]
    sm = _f32(surface_masks, dev).reshape(B, M, S, S)
    mi = mask_input.to(device=dev)
    if mi.dtype != torch.float32:
        mi = mi.to(torch.float32)
    H, W = mi.shape[-2:]
    if mi.stride(-1) != 1 or mi.stride(-2) != W or mi.stride(0) != M * mi.stride(1):
        mi = mi.contiguous()
    w2c, th = _f32(world_to_cam, dev), _f32(tan_half, dev)
    crop = None if crop is None else _f32(crop, dev)
    n = pts.shape[0]
    ps, bs = int(patch_size), int(block_size)
    nbytes = L.lsrm_view_block_topk_workspace_bytes(B, M, H, W, S, ps, bs, win, n)
    if nbytes == 0:
        raise ValueError("unsupported view geometry (blocks per side must agree and divide the surface grid; "
                         "views * attn_winsize^2 <= 512, attn_winsize <= 5)")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = torch.empty(n, topk, dtype=torch.int32, device=dev)
    rc = L.lsrm_view_block_topk(ops._ptr(pts), ops._ptr(qc), n, B, M, ops._ptr(mi), mi.stride(1), H, W,
                                ops._ptr(sp), ops._ptr(sm), S, ps, bs, ops._ptr(w2c), ops._ptr(th), ops._ptr(crop),
                                int(win), int(topk), float(max_dist), ops._ptr(out), ops._ptr(ws), nbytes,
                                ops._ptr(ops._err_word(dev)), ops._stream())
    check(rc, "lsrm_view_block_topk")
    return out


def _image_separation(imfeat_coords, dense_points, args):
    bs = int(args.block_size)
    batch_size = int(imfeat_coords[:, 0].max().item()) + 1
    r = int(args.input_image_res[-1]) // bs
    M = dense_points["surface_points_input"].shape[1]
    cu_sb, cu_blk, _ = block_separation(imfeat_coords, 3, [1, bs, bs], batch_size, [M, r, r])
    return cu_sb, cu_blk


def build_image_to_image_attn(imfeat_coords: torch.Tensor, batch, dense_points, args):
    """``build_image_to_image_attn`` (misc/sparse_utils.py:690-898): same
    arguments and dict keys; ``imfeat_coords`` is not modified."""
    cu_sb, cu_blk = _image_separation(imfeat_coords, dense_points, args)
    block_topk = None
    if getattr(args, "use_3d_aware_attn", False):
        pts = from_imcoords_to_points(imfeat_coords, dense_points, args)
        bt = view_block_topk(pts, imfeat_coords, batch, dense_points, args)
        block_topk = torch.stack([bt, bt], dim=0)
    return {"block_topk": block_topk, "cu_seqblocks": cu_sb.to(torch.int32),
            "cu_block_include_tokens": cu_blk.to(torch.int32)}


def build_volume_to_image_attn(imfeat_coords: torch.Tensor, volfeat_coords: torch.Tensor, batch, dense_points, args):
    """``build_volume_to_image_attn`` (misc/sparse_utils.py:991-1200): same
    arguments and dict keys (image blocks as keys, voxels as queries)."""
    cu_sb, cu_blk = _image_separation(imfeat_coords, dense_points, args)
    block_topk = None
    if getattr(args, "use_3d_aware_attn", False):
        pts = from_volcoords_to_points(volfeat_coords, args)
        bt = view_block_topk(pts, volfeat_coords, batch, dense_points, args)
        block_topk = torch.stack([bt, bt], dim=0)
    return {"block_topk": block_topk, "cu_seqblocks": cu_sb.to(torch.int32),
            "cu_block_include_tokens": cu_blk.to(torch.int32)}


def build_image_to_volume_attn(imfeat_coords: torch.Tensor, volfeat_coords: torch.Tensor, dense_points, args):
    """``build_image_to_volume_attn`` (misc/sparse_utils.py:901-988): same
    arguments and dict keys (volume blocks as keys, image tokens as
    queries)."""
    bs = int(args.block_size)
    res = int(args.volume_res)
    batch_size = int(volfeat_coords[:, 0].max().item()) + 1
    cu_sb, cu_blk, _ = block_separation(volfeat_coords, 3, [bs, bs, bs], batch_size, [res, res, res])
    block_topk = None
    if getattr(args, "use_3d_aware_attn", False):
        L = _lib.lib()
        dev = volfeat_coords.device
        pts = from_imcoords_to_points(imfeat_coords, dense_points, args)
        qc = imfeat_coords.to(torch.int32).contiguous()
        vc = volfeat_coords.to(torch.int32).contiguous()
        topk = int(args.topk_volume)
        bt = torch.empty(qc.shape[0], topk, dtype=torch.int32, device=dev)
        cent = torch.empty(max(vc.shape[0], 1), 3, dtype=torch.float32, device=dev)
        rc = L.lsrm_points_volume_block_topk(ops._ptr(pts), ops._ptr(qc), qc.shape[0], ops._ptr(vc), vc.shape[0],
                                             ops._ptr(cu_sb), ops._ptr(cu_blk), batch_size, res,
                                             float(args.bbox_radius) * 1.05, topk, ops._ptr(cent), ops._ptr(bt),
                                             ops._ptr(ops._err_word(dev)), ops._stream())
        check(rc, "lsrm_points_volume_block_topk")
        block_topk = torch.stack([bt, bt], dim=0)
    return {"block_topk": block_topk, "cu_seqblocks": cu_sb.to(torch.int32),
            "cu_block_include_tokens": cu_blk.to(torch.int32)}


def build_3D_aware_attn(imfeat_coords: torch.Tensor, volfeat_coords: torch.Tensor, batch, dense_points, args):
    """``build_3D_aware_attn`` (misc/sparse_utils.py:1283-1298): the four maps
    under the reference's keys."""
    return {"img_to_img_attn": build_image_to_image_attn(imfeat_coords, batch, dense_points, args),
            "img_to_vol_attn": build_image_to_volume_attn(imfeat_coords, volfeat_coords, dense_points, args),
            "vol_to_img_attn": build_volume_to_image_attn(imfeat_coords, volfeat_coords, batch, dense_points, args),
            "vol_to_vol_attn": build_volume_to_volume_attn(volfeat_coords, args)}
