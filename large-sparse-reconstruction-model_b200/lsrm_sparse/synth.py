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


def sdf_shell_voxels(res: int, n_target: int, seed: int, n_spheres=(6, 12), radius=(0.08, 0.2),
                     thickness_vox: float = 1.5) -> Tuple[np.ndarray, int]:
    """Voxels (int32 [n, 3], x/y/z) with |sdf| < thickness of the union of
    random spheres (centres in [-0.5, 0.5]^3), Morton sorted, subsampled to
    ``n_target`` with the seed.  Returns (voxels, shell size before
    subsampling)."""
    rng = np.random.default_rng(seed)
    ns = int(rng.integers(n_spheres[0], n_spheres[1] + 1))
    centres = rng.uniform(-0.5, 0.5, (ns, 3))
    radii = rng.uniform(radius[0], radius[1], ns)
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
