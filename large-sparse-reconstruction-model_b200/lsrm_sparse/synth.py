"""Seeded synthetic voxel workloads standing in for the reference's datasets
(GSO / ORB / DTC are not available here): surface voxels of a random-sphere
SDF shell, sorted in Morton order and grouped into octree-cell blocks."""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import numpy as np


def morton3(x: np.ndarray, y: np.ndarray, z: np.ndarray, bits: int) -> np.ndarray:
    """Interleave the bits of (x, y, z) (z lowest) into a Morton code."""
    x = x.astype(np.uint64)
    y = y.astype(np.uint64)
    z = z.astype(np.uint64)
    code = np.zeros(x.shape, dtype=np.uint64)
    for b in range(bits):
        ub = np.uint64(b)
        code |= ((x >> ub) & np.uint64(1)) << np.uint64(3 * b + 2)
        code |= ((y >> ub) & np.uint64(1)) << np.uint64(3 * b + 1)
        code |= ((z >> ub) & np.uint64(1)) << np.uint64(3 * b)
    return code


def _spheres(rng, n_spheres, radius):
    ns = int(rng.integers(n_spheres[0], n_spheres[1] + 1))
    centres = rng.uniform(-0.5, 0.5, (ns, 3))
    radii = rng.uniform(radius[0], radius[1], ns)
    return centres, radii


def scene_spheres(seed: int, n_spheres=(6, 12), radius=(0.08, 0.2)) -> Tuple[np.ndarray, np.ndarray]:
    """The spheres (centres [k, 3] in [-0.5, 0.5]^3, radii [k]) whose shell
    ``sdf_shell_voxels`` with the same seed and ranges voxelises."""
    return _spheres(np.random.default_rng(seed), n_spheres, radius)


def sdf_shell_voxels(res: int, n_target: int, seed: int, n_spheres=(6, 12), radius=(0.08, 0.2),
                     thickness_vox: float = 1.5) -> Tuple[np.ndarray, int]:
    """Voxels (int32 [n, 3], x/y/z) with |sdf| < thickness of the union of
    random spheres (centres in [-0.5, 0.5]^3), Morton sorted, subsampled to
    ``n_target`` with the seed.  Returns (voxels, shell size before
    subsampling)."""
    rng = np.random.default_rng(seed)
    centres, radii = _spheres(rng, n_spheres, radius)
    thr = thickness_vox / res
    cand = []
    for c, r in zip(centres, radii):
        lo = np.clip(np.floor((c - r - thr + 0.5) * res).astype(int), 0, res - 1)
        hi = np.clip(np.ceil((c + r + thr + 0.5) * res).astype(int), 0, res - 1)
        xs = np.arange(lo[0], hi[0] + 1)
        ys = np.arange(lo[1], hi[1] + 1)
        px = (xs + 0.5) / res - 0.5 - c[0]
        py = (ys + 0.5) / res - 0.5 - c[1]
        d2xy = px[:, None] ** 2 + py[None, :] ** 2
        for zi in range(lo[2], hi[2] + 1):
            pz = (zi + 0.5) / res - 0.5 - c[2]
            d = np.sqrt(d2xy + pz * pz) - r
            ix, iy = np.nonzero(np.abs(d) < thr)
            if ix.size:
                cand.append(np.stack([xs[ix], ys[iy], np.full(ix.size, zi)], 1))
    vox = np.concatenate(cand, 0).astype(np.int64)
    lin = np.unique(vox[:, 0] * res * res + vox[:, 1] * res + vox[:, 2])
    vox = np.stack([lin // (res * res), (lin // res) % res, lin % res], 1)
    p = (vox + 0.5) / res - 0.5
    sdf = np.full(len(vox), np.inf)
    for c, r in zip(centres, radii):
        sdf = np.minimum(sdf, np.sqrt(((p - c) ** 2).sum(1)) - r)
    vox = vox[np.abs(sdf) < thr]
    shell = len(vox)
    if shell > n_target:
        keep = np.sort(rng.choice(shell, n_target, replace=False))
        vox = vox[keep]
    bits = int(np.ceil(np.log2(res)))
    code = morton3(vox[:, 0], vox[:, 1], vox[:, 2], bits)
    order = np.argsort(code, kind="stable")
    return vox[order].astype(np.int32), shell


def octree_blocks(vox_sorted: np.ndarray, res: int, min_len: int, max_len: int) -> List[int]:
    """Block lengths of Morton-sorted voxels: split Morton-aligned octree
    cells until they hold <= max_len voxels, then merge runs of consecutive
    cells shorter than min_len while the merged block stays <= max_len."""
    bits = int(np.ceil(np.log2(res)))
    code = morton3(vox_sorted[:, 0], vox_sorted[:, 1], vox_sorted[:, 2], bits)
    out = []
    stack = [(0, len(code), 0)]
    while stack:
        s, e, lvl = stack.pop()
        if e - s <= max_len or lvl >= bits:
            if e > s:
                out.append((s, e))
            continue
        shift = np.uint64(3 * (bits - lvl - 1))
        child = ((code[s:e] >> shift) & np.uint64(7)).astype(np.int64)
        bounds = np.searchsorted(child, np.arange(9))
        for c in range(7, -1, -1):  # pushed in reverse so cells pop in order
            a, b = s + bounds[c], s + bounds[c + 1]
            if b > a:
                stack.append((a, b, lvl + 1))
    out.sort()
    lens = [int(e - s) for s, e in out]
    merged = []
    cur = 0
    for l in lens:
        if cur == 0:
            cur = l
        elif cur < min_len and cur + l <= max_len:
            cur += l
        else:
            merged.append(cur)
            cur = l
    if cur:
        if cur < min_len and merged and merged[-1] + cur <= max_len:
            merged[-1] += cur
        else:
            merged.append(cur)
    assert sum(merged) == len(code)
    return merged


def uniform_blocks(n_tokens: int, n_blocks: int, lo: int, hi: int, seed: int) -> List[int]:
    """Block lengths drawn uniform in [lo, hi], rescaled to sum to n_tokens
    (the rounding remainder goes to the last block)."""
    rng = np.random.default_rng(seed)
    raw = rng.integers(lo, hi + 1, n_blocks).astype(np.float64)
    lens = np.floor(raw * n_tokens / raw.sum()).astype(np.int64)
    lens[-1] += n_tokens - lens.sum()
    return [int(x) for x in lens]


@dataclass
class VoxelWorkload:
    n_tokens: int
    block_lens: List[int]
    shell_size: int
    res: int


def voxel_workload(n_tokens: int, res: int, min_len: int, max_len: int, seed: int) -> VoxelWorkload:
    vox, shell = sdf_shell_voxels(res, n_tokens, seed)
    tries = 0
    while len(vox) < n_tokens and tries < 8:  # too few shell voxels: draw again
        tries += 1
        vox, shell = sdf_shell_voxels(res, n_tokens, seed + 1000 * tries)
    if len(vox) < n_tokens:
        raise ValueError(f"shell has {len(vox)} voxels < {n_tokens}")
    lens = octree_blocks(vox, res, min_len, max_len)
    return VoxelWorkload(n_tokens, lens, shell, res)


def _look_at(pos: np.ndarray, target: np.ndarray) -> np.ndarray:
    """Camera-to-world 4x4 (OpenGL axes: the camera looks down -z, y up)."""
    f = target - pos
    f /= np.linalg.norm(f)
    up = np.array([0.0, 0.0, 1.0]) if abs(f[2]) < 0.9 else np.array([0.0, 1.0, 0.0])
    r = np.cross(f, up)
    r /= np.linalg.norm(r)
    u = np.cross(r, f)
    m = np.eye(4)
    m[:3, 0], m[:3, 1], m[:3, 2], m[:3, 3] = r, u, -f, pos
    return m


def _cast(o: np.ndarray, d: np.ndarray, centres: np.ndarray, radii: np.ndarray):
    """Nearest hit of rays (o, d [n, 3], d unit) with a union of spheres:
    (hit, point, closest approach to any sphere surface)."""
    t_best = np.full(d.shape[0], np.inf)
    gap = np.full(d.shape[0], np.inf)
    for c, r in zip(centres, radii):
        oc = o - c
        b = (oc * d).sum(1)
        cc = (oc * oc).sum(1) - r * r
        disc = b * b - cc
        hit = disc >= 0
        t = -b - np.sqrt(np.where(hit, disc, 0.0))
        t_best = np.where(hit & (t > 0) & (t < t_best), t, t_best)
        closest = np.sqrt(np.maximum((oc * oc).sum(1) - b * b, 0.0)) - r
        gap = np.minimum(gap, closest)
    hit = np.isfinite(t_best)
    t_pt = np.where(hit, t_best, np.maximum(-(o * d).sum(1), 0.0))
    return hit, o + t_pt[:, None] * d, gap


def _pixel_ndc(n_pix: int, crop=None, origin=None):
    """Normalised device coordinate of pixel centres 0..n-1 along one axis,
    inverting the reference's pixel mapping (misc/sparse_utils.py:1129-1146):
    u = i / (n - 1), or with a crop (start, size) of an image of ``origin``
    pixels u = (i / (n - 1) * (size - 1) + start) / (origin - 1)."""
    i = np.arange(n_pix, dtype=np.float64) / (n_pix - 1)
    if crop is not None:
        i = (i * (crop[1] - 1) + crop[0]) / (origin - 1)
    return 2.0 * i - 1.0


def view_scene(centres: np.ndarray, radii: np.ndarray, batch: int, views: int, image_res: int,
               surface_res: int, seed: int, world_scale: float = 1.05, crop: bool = False,
               cam_dist=(1.8, 2.4), fov=(0.6, 0.9)):
    """Posed views of a union of spheres, in the reference's input layout
    (misc/sparse_utils.py:653-1200):

    * ``cameras`` [B, M, 18] float32: row-major camera-to-world 4x4, the field
      of view (radians), one unused entry;
    * ``mask_input`` [B, M, 1, H, H] float32: 1 where a pixel's ray hits;
    * ``surface_points`` [B, M, S, S, 3] float32: the hit point per ray at the
      surface resolution (closest approach where it misses);
    * ``surface_masks`` [B, M, S, S] float32: 1 on hits, 0.3 / 0.15 on rays
      passing within 1 / 3 % of the scene of a sphere (either side of the
      reference's 0.2 threshold), else 0;
    * with ``crop``: ``crop_input`` [B, M, 4] (rows start, end, columns start,
      end) and ``origin_size`` [B, 2], the images being crops of larger ones.

    Sphere centres and radii are given in [-0.5, 0.5] units and scaled by
    ``world_scale`` (voxel points of the reference span the bounding radius
    times 1.05)."""
    rng = np.random.default_rng(seed)
    c = np.asarray(centres, np.float64) * world_scale
    r = np.asarray(radii, np.float64) * world_scale
    cams = np.zeros((batch, views, 18), np.float32)
    mask_input = np.zeros((batch, views, 1, image_res, image_res), np.float32)
    sp = np.zeros((batch, views, surface_res, surface_res, 3), np.float32)
    sm = np.zeros((batch, views, surface_res, surface_res), np.float32)
    crop_input = np.zeros((batch, views, 4), np.float32)
    origin_size = np.zeros((batch, 2), np.float32)
    for b in range(batch):
        origin = float(int(image_res * rng.uniform(1.2, 1.6))) if crop else None
        if crop:
            origin_size[b] = origin
        for m in range(views):
            d = rng.normal(size=3)
            d /= np.linalg.norm(d)
            pos = d * rng.uniform(*cam_dist)
            c2w = _look_at(pos, rng.uniform(-0.05, 0.05, 3))
            fv = rng.uniform(*fov)
            cams[b, m, :16] = c2w.reshape(-1)
            cams[b, m, 16] = fv
            t = np.tan(fv / 2.0)
            cr = None
            if crop:
                size = float(int(origin * rng.uniform(0.6, 0.8)))
                hs = float(int(rng.uniform(0, origin - size)))
                ws = float(int(rng.uniform(0, origin - size)))
                crop_input[b, m] = (hs, hs + size, ws, ws + size)
                cr = ((ws, size), (hs, size))
            for res, is_surface in ((image_res, False), (surface_res, True)):
                nx = _pixel_ndc(res, None if cr is None else cr[0], origin)
                ny = _pixel_ndc(res, None if cr is None else cr[1], origin)
                gy, gx = np.meshgrid(ny, nx, indexing="ij")
                dc = np.stack([gx * t, -gy * t, -np.ones_like(gx)], -1).reshape(-1, 3)
                dw = dc @ c2w[:3, :3].T
                dw /= np.linalg.norm(dw, axis=1, keepdims=True)
                hit, pt, gap = _cast(np.broadcast_to(pos, dw.shape), dw, c, r)
                if is_surface:
                    sp[b, m] = pt.reshape(res, res, 3)
                    soft = np.where(gap < 0.01, 0.3, np.where(gap < 0.03, 0.15, 0.0))
                    sm[b, m] = np.where(hit, 1.0, soft).reshape(res, res)
                else:
                    mask_input[b, m, 0] = hit.reshape(res, res)
    out = dict(cameras=cams, mask_input=mask_input, surface_points=sp, surface_masks=sm)
    if crop:
        out["crop_input"] = crop_input
        out["origin_size"] = origin_size
    return out


def image_tokens(mask_input: np.ndarray, patch_size: int, block_size: int) -> np.ndarray:
    """Image tokens (int32 [n, 4]: batch, image, patch row, patch column) of
    the patches whose pixel mask is non-zero (sparsify_imfeat,
    misc/sparse_utils.py:251-262), in sort_image_blocks order (batch, image,
    block row, block column, row and column in the block; :95-118)."""
    B, M, _, H, W = mask_input.shape
    ph, pw = H // patch_size, W // patch_size
    pm = mask_input[:, :, 0].reshape(B, M, ph, patch_size, pw, patch_size).sum((3, 5))
    b, m, y, x = np.nonzero(pm)
    key = np.lexsort((x % block_size, y % block_size, x // block_size, y // block_size, m, b))
    return np.stack([b, m, y, x], 1)[key].astype(np.int32)
