"""Image-side 3D-aware attention maps on the GPU (lsrm_image_token_points,
lsrm_points_volume_block_topk, lsrm_view_block_topk via lsrm_sparse.blocks):
bit for bit against the oracle given the same per-view camera terms, and
against the reference fixtures (exact where the reference's result is a
rule; for the view maps through the oracle, whose rows match the
reference's up to the resolution of ties)."""

import types

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _args(g):
    M = g["scene_cameras"].shape[1]
    H = int(g["image_res"])
    return types.SimpleNamespace(block_size=int(g["block_size"]), volume_res=int(g["volume_res"]),
                                 use_3d_aware_attn=True, topk_volume=int(g["topk_volume"]),
                                 bbox_radius=float(g["bbox_radius"]), attn_winsize=int(g["attn_winsize"]),
                                 topk_multiimage=int(g["topk_multiimage"]), image_num_per_batch=M,
                                 input_image_res=[H // 2, H], patch_size=int(g["patch_size"]))


def _inputs(sc, prefix=""):
    batch = {"mask_input": torch.from_numpy(sc[prefix + "mask_input"]).to(DEV),
             "cameras_input": torch.from_numpy(sc[prefix + "cameras"]).to(DEV)}
    if prefix + "crop_input" in sc:
        batch["crop_input"] = torch.from_numpy(sc[prefix + "crop_input"]).to(DEV)
        batch["origin_size"] = torch.from_numpy(sc[prefix + "origin_size"]).to(DEV)
    dense = {"surface_points_input": torch.from_numpy(sc[prefix + "surface_points"]).to(DEV),
             "masks_input": torch.from_numpy(sc[prefix + "surface_masks"]).to(DEV)}
    return batch, dense


def _gpu_view(pts, coords, sc, w2c, th, crop, ps, bs, win, topk, max_dist, prefix=""):
    from lsrm_sparse import blocks

    out = blocks.view_block_topk_raw(torch.from_numpy(np.ascontiguousarray(pts)).to(DEV),
                                     torch.from_numpy(np.ascontiguousarray(coords)).to(DEV),
                                     torch.from_numpy(sc[prefix + "mask_input"][:, :, 0]).to(DEV),
                                     torch.from_numpy(sc[prefix + "surface_points"]).to(DEV),
                                     torch.from_numpy(sc[prefix + "surface_masks"]).to(DEV),
                                     torch.from_numpy(w2c), torch.from_numpy(th),
                                     None if crop is None else torch.from_numpy(crop), ps, bs, win, topk, max_dist)
    return out.cpu().numpy()


@pytest.mark.parametrize("name", ["image_maps", "image_maps_crop"])
def test_image_maps_vs_reference_fixture(golden, name):
    from lsrm_sparse import blocks, ops

    g = golden(name)
    args = _args(g)
    batch, dense = _inputs(g, "scene_")
    imc = torch.from_numpy(g["imcoords"]).to(DEV)
    volc = torch.from_numpy(g["volcoords"]).to(DEV)
    maps = blocks.build_3D_aware_attn(imc, volc, batch, dense, args)
    pts = blocks.from_imcoords_to_points(imc, dense, args).cpu().numpy()
    assert ops.read_errors() == 0
    assert np.array_equal(pts, g["impoints"])
    for key, ref in (("img_to_img_attn", "i2i"), ("img_to_vol_attn", "i2v"), ("vol_to_img_attn", "v2i")):
        for k in ("cu_seqblocks", "cu_block_include_tokens"):
            assert np.array_equal(maps[key][k].cpu().numpy(), g[f"{ref}_{k}"]), (key, k)
    assert np.array_equal(maps["img_to_vol_attn"]["block_topk"].cpu().numpy(), g["i2v_block_topk"])

    B, M = g["scene_cameras"].shape[:2]
    ps, bs = args.patch_size, args.block_size
    win, topk, md = args.attn_winsize ** 2, args.topk_multiimage * M, 2 * args.bbox_radius
    volpts = oracle.voxel_points(g["volcoords"], args.volume_res, args.bbox_radius)
    assert np.array_equal(blocks.voxel_points(volc, args.volume_res, args.bbox_radius).cpu().numpy(), volpts)
    mi = g["scene_mask_input"][:, :, 0]
    sp, sm = g["scene_surface_points"], g["scene_surface_masks"]
    # the reference's per-view terms (CPU torch.inverse / tan): GPU == oracle, oracle == reference up to ties
    w2c, th, crop = oracle.camera_terms(g["scene_cameras"], g.get("scene_crop_input"), g.get("scene_origin_size"))
    for key, q, qc in (("i2i", g["impoints"], g["imcoords"]), ("v2i", volpts, g["volcoords"])):
        gpu = _gpu_view(q, qc, g, w2c, th, crop, ps, bs, win, topk, md, "scene_")
        ora, det = oracle.view_block_topk(q, qc[:, 0], mi, sp, sm, w2c, th, ps, bs, win, topk, md, crop=crop,
                                          return_values=True)
        assert np.array_equal(gpu, ora), key
        assert oracle.view_rows_equivalent(ora, g[f"{key}_block_topk"][0], det, win) == [], key
    # the builders' own device-side terms: GPU == oracle on those terms
    tw, tt, tc = (None if x is None else x.cpu().numpy() for x in blocks.camera_terms(batch, DEV))
    for key, q, qc in (("img_to_img_attn", g["impoints"], g["imcoords"]), ("vol_to_img_attn", volpts, g["volcoords"])):
        ora = oracle.view_block_topk(q, qc[:, 0], mi, sp, sm, tw, tt, ps, bs, win, topk, md, crop=tc)
        bt = maps[key]["block_topk"].cpu().numpy()
        assert np.array_equal(bt[0], bt[1])
        assert np.array_equal(bt[0], ora), key


def _synthetic(crop, seed=3):
    from lsrm_sparse import synth

    spheres = ((3, 5), (0.15, 0.3))
    centres, radii = synth.scene_spheres(seed, *spheres)
    B, M, H, S = 2, 6, 256, 128
    sc = synth.view_scene(centres, radii, B, M, H, S, seed + 8, crop=crop)
    sc["mask_input"][1, 2] = 0  # a view without selected blocks
    sc["mask_input"][1, 3] = 0
    sc["mask_input"][1, 3, 0, 100:105, 200:203] = 1  # one selected block: the window is cut to it
    parts = []
    for b, n in enumerate((3001, 2500)):
        vox, _ = synth.sdf_shell_voxels(64, n, seed + b, *spheres)
        parts.append(np.stack([np.full(len(vox), b), vox[:, 2], vox[:, 1], vox[:, 0]], 1))
    coords = np.concatenate(parts).astype(np.int32)
    return sc, coords


@pytest.mark.parametrize("crop", [False, True])
@pytest.mark.parametrize("winsize", [2, 3])
def test_view_block_topk_vs_oracle_synthetic(crop, winsize):
    """Voxel queries of two batch elements (a batch boundary inside a warp,
    a count that is not a multiple of 32) against six 256x256 views (8x8
    blocks of 16x16 surface points), one view empty and one with a single
    selected block."""
    from lsrm_sparse import ops

    sc, coords = _synthetic(crop)
    pts = oracle.voxel_points(coords, 64, 0.5)
    w2c, th, cr = oracle.camera_terms(sc["cameras"], sc.get("crop_input"), sc.get("origin_size"))
    M = sc["cameras"].shape[1]
    win, topk = winsize * winsize, 3 * M
    gpu = _gpu_view(pts, coords, sc, w2c, th, cr, 8, 4, win, topk, 1.0)
    assert ops.read_errors() == 0
    ora = oracle.view_block_topk(pts, coords[:, 0], sc["mask_input"][:, :, 0], sc["surface_points"],
                                 sc["surface_masks"], w2c, th, 8, 4, win, topk, 1.0, crop=cr)
    assert np.array_equal(gpu, ora)
    assert (gpu >= 0).sum(1).min() > 0


def test_view_block_topk_edges():
    """A batch element whose views have no selected block gets -1 rows; a
    query with an out-of-range batch id sets LSRM_ERR_BAD_INDEX and gets a
    -1 row; the others are unaffected."""
    from lsrm_sparse import ops

    sc, coords = _synthetic(False)
    sc["mask_input"][1] = 0
    coords = coords.copy()
    coords[7, 0] = 9
    pts = oracle.voxel_points(coords, 64, 0.5)
    w2c, th, _ = oracle.camera_terms(sc["cameras"])
    gpu = _gpu_view(pts, coords, sc, w2c, th, None, 8, 4, 4, 12, 1.0)
    assert ops.read_errors() & 0x8
    assert (gpu[coords[:, 0] == 1] == -1).all()
    assert (gpu[7] == -1).all()
    keep = coords[:, 0] == 0
    ora = oracle.view_block_topk(pts[keep], coords[keep, 0], sc["mask_input"][:, :, 0], sc["surface_points"],
                                 sc["surface_masks"], w2c, th, 8, 4, 4, 12, 1.0)
    assert np.array_equal(gpu[keep], ora)
