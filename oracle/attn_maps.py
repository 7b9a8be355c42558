"""CPU restatement of the reference's image-side attention maps.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): never imported by the
shipped package.  numpy float32 with the reference's operation order, so that
the CUDA kernels can be compared bit for bit; ties are broken by the lower
position (the reference leaves them to ``torch.topk``).

Restated functions (paths relative to the root of
chenxiex/Large-Sparse-Reconstruction-Model):

* ``image_token_points``      from_imcoords_to_points, misc/sparse_utils.py:653-687
* ``image_volume_block_topk`` the geometric part of build_image_to_volume_attn,
                              misc/sparse_utils.py:901-988
* ``view_block_topk``         the geometric part of build_volume_to_image_attn
                              (:991-1200) and build_image_to_image_attn
                              (:690-898), with compute_block_topk_dist_chunked
                              (:16-56)
"""

from __future__ import annotations

from fractions import Fraction

import numpy as np

from .nsa_oracle import volume_block_topk

f32 = np.float32


def fma32(a, b, c):
    """Correctly rounded float32 a*b + c, elementwise.  The float64 sum of the
    exact product is rounded once more to float32; where that float64 value is
    exactly halfway between two float32 numbers the double rounding may be
    wrong, and those entries are recomputed exactly."""
    a = np.asarray(a, f32)
    b = np.asarray(b, f32)
    c = np.asarray(c, f32)
    a, b, c = np.broadcast_arrays(a, b, c)
    r64 = a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)
    out = r64.astype(f32)
    bits = r64.view(np.uint64)
    mid = (bits & np.uint64((1 << 29) - 1)) == np.uint64(1 << 28)
    for idx in zip(*np.nonzero(mid)):
        exact = Fraction(float(a[idx])) * Fraction(float(b[idx])) + Fraction(float(c[idx]))
        lo = f32(float(exact))
        # nearest float32 to the exact value, ties to even
        cand = [lo, np.nextafter(lo, f32(np.inf)), np.nextafter(lo, f32(-np.inf))]
        best = min(cand, key=lambda v: (abs(Fraction(float(v)) - exact), int(np.array(v, f32).view(np.uint32)) & 1))
        out[idx] = best
    return out


def image_token_points(imcoords, surface_points, masks, patch_res: int):
    """from_imcoords_to_points (misc/sparse_utils.py:653-687): per image token
    (batch, image, patch row, patch column) the surface point of its patch
    whose mask value is largest (first one in row-major order on ties).
    ``surface_points`` [B, M, S, S, 3], ``masks`` [B, M, S, S] (or with a
    trailing 1)."""
    c = np.asarray(imcoords).astype(np.int64)
    sp = np.asarray(surface_points, f32)
    B, M, S = sp.shape[0], sp.shape[1], sp.shape[2]
    mk = np.asarray(masks, f32).reshape(B, M, S, S)
    ps = S // patch_res
    out = np.zeros((c.shape[0], 3), f32)
    for i, (b, m, py, px) in enumerate(c[:, :4]):
        patch = mk[b, m, py * ps:(py + 1) * ps, px * ps:(px + 1) * ps].reshape(-1)
        j = int(np.argmax(patch))  # first maximum
        out[i] = sp[b, m, py * ps + j // ps, px * ps + j % ps]
    return out


def image_volume_block_topk(points, batch_ids, volcoords, cu_seqblocks, cu_block_include_tokens, batch: int,
                            volume_res: int, bbox_radius: float, topk: int):
    """The block selection of build_image_to_volume_attn with use_3d_aware_attn
    (misc/sparse_utils.py:939-983): per image-token point the ``topk`` volume
    blocks of its batch element whose centre is nearest, ranked by
    d^2 = (dx^2 + dy^2) + dz^2 (ties to the lower id; the reference ranks
    sqrt(d^2)), sorted ids, -1 padding.  Block centres as in the
    volume-to-volume map."""
    _, _, cent = volume_block_topk(volcoords, cu_seqblocks, cu_block_include_tokens, batch, volume_res,
                                   bbox_radius, topk, return_geometry=True, rows=[])
    cu_sb = np.asarray(cu_seqblocks).astype(np.int64)
    p = np.asarray(points, f32)
    bid = np.asarray(batch_ids).astype(np.int64)
    out = np.full((p.shape[0], topk), -1, np.int32)
    for t in range(p.shape[0]):
        b0, b1 = int(cu_sb[bid[t]]), int(cu_sb[bid[t] + 1])
        d = (p[t][None, :] - cent[b0:b1]).astype(f32)
        sq = (d * d).astype(f32)
        d2 = ((sq[:, 0] + sq[:, 1]).astype(f32) + sq[:, 2]).astype(f32)
        sel = np.sort(np.lexsort((np.arange(b1 - b0), d2))[:topk])
        out[t, : sel.size] = sel
    return out


def camera_terms(cameras, crop_input=None, origin_size=None):
    """The per-camera values of misc/sparse_utils.py:1097-1135, with the
    reference's own torch calls, one camera at a time on the CPU:
    world_to_cam = inverse(camera[:16] as 4x4), tan(fov / 2), and with a crop
    (origin - 1, rows start, columns start, crop size - 1).  Returns numpy
    float32 ([B, M, 4, 4], [B, M], [B, M, 4] or None)."""
    import torch

    cams = torch.as_tensor(np.asarray(cameras, f32))
    B, M = cams.shape[:2]
    w2c = np.zeros((B, M, 4, 4), f32)
    th = np.zeros((B, M), f32)
    crop = None if crop_input is None else np.zeros((B, M, 4), f32)
    for b in range(B):
        for m in range(M):
            w2c[b, m] = torch.inverse(cams[b, m, :16].reshape(4, 4)).numpy()
            th[b, m] = torch.tan(cams[b, m, 16] / 2.0).item()
            if crop is not None:
                ci = torch.as_tensor(np.asarray(crop_input))[b, m]
                o = torch.as_tensor(np.asarray(origin_size))[b, 0]
                crop[b, m] = [(o - 1).item(), ci[0].item(), ci[2].item(), (ci[1] - ci[0] - 1).item()]
    return w2c, th, crop


def voxel_points(coords, volume_res: int, bbox_radius: float):
    """from_volcoords_to_points (misc/sparse_utils.py:644-650) in float32:
    2 * (c / (res - 1) - 0.5) * (bbox_radius * 1.05), (x, y, z) from columns
    3, 2, 1."""
    c = np.asarray(coords).astype(np.int64)
    r = f32(bbox_radius * 1.05)
    den = f32(volume_res - 1)

    def pt(v):
        return (f32(2.0) * ((v.astype(f32) / den).astype(f32) - f32(0.5))).astype(f32) * r

    return np.stack([pt(c[:, 3]), pt(c[:, 2]), pt(c[:, 1])], 1).astype(f32)


def view_block_geometry(mask_img, surface, smask, patch_size: int, block_size: int):
    """Per image: the selected blocks (pixel mask non-zero somewhere in the
    block, row-major), their centres in block units, and per selected block its
    surface points and validity (mask > 0.2 in float32) — the per-image part of
    misc/sparse_utils.py:1037-1095.  The reference tests ``sum != 0``; for
    non-negative masks that is "some value non-zero"."""
    H, W = mask_img.shape
    bp = patch_size * block_size
    bh, bw = H // bp, W // bp
    S = surface.shape[0]
    ib = S // bh
    mb = mask_img.reshape(bh, bp, bw, bp).transpose(0, 2, 1, 3).reshape(bh * bw, -1)
    sel = np.nonzero((mb != 0).any(1))[0]
    pts = surface.reshape(bh, ib, bw, ib, 3).transpose(0, 2, 1, 3, 4).reshape(bh * bw, ib * ib, 3)[sel]
    val = (smask.reshape(bh, ib, bw, ib).transpose(0, 2, 1, 3).reshape(bh * bw, ib * ib) > f32(0.2))[sel]
    cx = ((sel % bw).astype(f32) + f32(0.5)).astype(f32)
    cy = ((sel // bw).astype(f32) + f32(0.5)).astype(f32)
    return sel, cx, cy, pts.astype(f32), val, ib


def project_to_blocks(points, w2c, tan_half, S: int, ib: int, crop=None):
    """Block-unit image coordinates of world points (misc/sparse_utils.py:
    1097-1146): [p, 1] @ world_to_cam^T as a fused multiply-add chain over
    k = 0..3 (torch's CPU matmul order), x / max(-z, 1e-6), -y / max(-z, 1e-6),
    0.5 * (v / tan(fov/2) + 1), then either v * (S - 1) or the crop mapping
    ((v * (origin - 1) - offset) / (crop - 1)) * (S - 1), divided by the
    block's point count per side.  ``crop`` = (origin - 1, rows start,
    columns start, crop size - 1) as float32."""
    p = np.asarray(points, f32)
    w = np.asarray(w2c, f32).reshape(4, 4)
    proj = []
    for j in range(3):
        s = (p[:, 0] * w[j, 0]).astype(f32)
        s = fma32(p[:, 1], w[j, 1], s)
        s = fma32(p[:, 2], w[j, 2], s)
        s = (s + w[j, 3]).astype(f32)
        proj.append(s)
    x, y, z = proj
    den = np.maximum((-z).astype(f32), f32(1e-6))
    px = (x / den).astype(f32)
    py = ((-y).astype(f32) / den).astype(f32)
    th = f32(tan_half)
    px = (f32(0.5) * ((px / th).astype(f32) + f32(1))).astype(f32)
    py = (f32(0.5) * ((py / th).astype(f32) + f32(1))).astype(f32)
    if crop is None:
        gx = (px * f32(S - 1)).astype(f32)
        gy = (py * f32(S - 1)).astype(f32)
    else:
        o1, hs, ws, cs1 = (f32(v) for v in crop)
        gx = ((((px * o1).astype(f32) - ws).astype(f32) / cs1).astype(f32) * f32(S - 1)).astype(f32)
        gy = ((((py * o1).astype(f32) - hs).astype(f32) / cs1).astype(f32) * f32(S - 1)).astype(f32)
    return (gx / f32(ib)).astype(f32), (gy / f32(ib)).astype(f32)


def view_block_topk(points, batch_ids, mask_input, surface_points, surface_masks, world_to_cam, tan_half,
                    patch_size: int, block_size: int, win: int, topk: int, max_dist: float, crop=None,
                    return_values: bool = False):
    """Per query point (a voxel's or an image token's) the ``topk`` image blocks
    of its batch element chosen by build_volume_to_image_attn /
    build_image_to_image_attn with use_3d_aware_attn
    (misc/sparse_utils.py:1019-1187 and :717-885):

    1. per image with selected blocks: project the point, take the ``win``
       selected blocks whose centres are nearest in block units
       (d = (dx^2) + (dy^2)), in ascending order, ties to the lower position;
    2. each candidate's value = min over the block's surface points of
       sqrt((dx^2 + dy^2) + dz^2) where the point is valid and ``max_dist``
       where it is not (misc/sparse_utils.py:16-56);
    3. candidates in image order, then rank order; the ``topk`` smallest
       values (ties to the lower position) are kept in position order, as
       block ids offset by the selected-block count of the earlier images;
       -1 padding.

    ``mask_input`` [B, M, H, W]; ``surface_points`` [B, M, S, S, 3];
    ``surface_masks`` [B, M, S, S]; ``world_to_cam`` [B, M, 4, 4]; ``tan_half``
    [B, M]; ``crop`` None or [B, M, 4] as in ``project_to_blocks``."""
    p = np.asarray(points, f32)
    bid = np.asarray(batch_ids).astype(np.int64)
    mi = np.asarray(mask_input, f32)
    sp = np.asarray(surface_points, f32)
    B, M = sp.shape[0], sp.shape[1]
    S = sp.shape[2]
    sm = np.asarray(surface_masks, f32).reshape(B, M, S, S)
    w2c = np.asarray(world_to_cam, f32).reshape(B, M, 4, 4)
    th = np.asarray(tan_half, f32).reshape(B, M)
    md = f32(max_dist)
    n = p.shape[0]
    out = np.full((n, topk), -1, np.int32)
    detail = []
    for b in range(B):
        rows = np.nonzero(bid == b)[0]
        if rows.size == 0:
            continue
        q = p[rows]
        cand_val, cand_id = [], []
        offset = 0
        for m in range(M):
            sel, cx, cy, pts, val, ib = view_block_geometry(mi[b, m], sp[b, m], sm[b, m], patch_size, block_size)
            if sel.size == 0:
                continue
            bx, by = project_to_blocks(q, w2c[b, m], th[b, m], S, ib, None if crop is None else np.asarray(crop)[b, m])
            dx = (bx[:, None] - cx[None, :]).astype(f32)
            dy = (by[:, None] - cy[None, :]).astype(f32)
            d2d = ((dx * dx).astype(f32) + (dy * dy).astype(f32)).astype(f32)
            wm = min(win, sel.size)
            order = np.lexsort((np.broadcast_to(np.arange(sel.size), d2d.shape), d2d), axis=1)[:, :wm]

            def block_value(blk):
                d = (q[:, None, :] - pts[blk]).astype(f32)  # [nq, P, 3]
                sq = (d * d).astype(f32)
                dd = ((sq[..., 0] + sq[..., 1]).astype(f32) + sq[..., 2]).astype(f32)
                vv = val[blk]
                dist = np.sqrt(np.where(vv, dd, f32(np.inf)).min(1)).astype(f32)
                return np.where(~vv.all(1), np.minimum(dist, md), dist)

            v = np.stack([block_value(order[:, r]) for r in range(wm)], 1)
            if return_values:  # every selected block, for tie-aware comparisons
                full = np.stack([block_value(np.full(q.shape[0], j)) for j in range(sel.size)], 1)
                detail.append((b, m, offset, rows, d2d, full))
            cand_val.append(v)
            cand_id.append((order + offset).astype(np.int32))
            offset += sel.size
        if not cand_val:
            continue
        cv = np.concatenate(cand_val, 1)
        ci = np.concatenate(cand_id, 1)
        C = cv.shape[1]
        k = min(C, topk)
        for i, t in enumerate(rows):
            pick = np.sort(np.lexsort((np.arange(C), cv[i]))[:k])
            out[t, :k] = ci[i, pick]
    return (out, detail) if return_values else out


def view_rows_equivalent(ours, ref, detail, win: int):
    """Rows of two view_block_topk results that agree up to the resolution of
    ties (the reference leaves ties to torch.topk, whose order follows no
    rule).  ``detail`` comes from ``view_block_topk(..., return_values=True)``.
    A reference row passes when it is a valid result for SOME resolution of
    ties: the same length as ours; per image, the listed blocks lie in the
    window (2D distance below the window's last distance, or equal to it,
    at most as many of those as the window has room for); the listed values
    are all <= the values of every window candidate left out (the window's
    tied places filled with the largest values); and the row lists blocks
    in (image, 2D distance) order.  Returns the rows that fail."""
    info = {}
    for b, m, off, rows, d2d, full in detail:
        for i, t in enumerate(rows):
            info.setdefault(int(t), []).append((m, off, d2d[i], full[i]))
    bad = []
    for t in range(ours.shape[0]):
        a, r = ours[t], ref[t]
        if np.array_equal(a, r):
            continue
        rr = [int(x) for x in r[r >= 0]]
        if (a >= 0).sum() != len(rr) or t not in info:
            bad.append(t)
            continue
        ok = True
        chosen_vals, left_vals, keys = [], [], {}
        for m, off, d2d, full in info[t]:
            mine = [x - off for x in rr if off <= x < off + d2d.size]
            for j in mine:
                keys[j + off] = (m, d2d[j])
            wm = min(win, d2d.size)
            kth = np.sort(d2d)[wm - 1]
            must = set(np.nonzero(d2d < kth)[0].tolist())
            tie = set(np.nonzero(d2d == kth)[0].tolist())
            slots = wm - len(must)
            got_tie = [j for j in mine if j in tie]
            if any(j not in must and j not in tie for j in mine) or len(got_tie) > slots:
                ok = False
                break
            chosen_vals += [full[j] for j in mine]
            left_vals += [full[j] for j in must if j not in mine]
            rest = sorted((full[j] for j in tie if j not in mine), reverse=True)
            left_vals += rest[: slots - len(got_tie)]
        if ok and chosen_vals and left_vals:
            ok = max(chosen_vals) <= min(left_vals)
        order = [keys.get(x) for x in rr]
        ok = ok and all(k is not None for k in order)
        ok = ok and all(p <= q for p, q in zip(order, order[1:]))
        if not ok:
            bad.append(t)
    return bad


def image_sort_keys(coords, views: int, patch_res: int, block_size: int):
    """sort_image_blocks' key (misc/sparse_utils.py:97-116) in int64:
    batch, view, block row, block column, row and column in the block."""
    c = np.asarray(coords).astype(np.int64)
    bs = int(block_size)
    o1, o2, o3, o4 = views * patch_res * patch_res, patch_res * patch_res, patch_res * bs, bs * bs
    return (o1 * c[:, 0] + o2 * c[:, 1] + o3 * (c[:, 2] // bs) + o4 * (c[:, 3] // bs) + bs * (c[:, 2] % bs)
            + c[:, 3] % bs)
