"""Decoder blocks (lsrm_sparse.decoder: CrossAttention, BlockMix) on a small
voxel + posed-view scene with the 3D-aware maps: forward and backward run,
and the fused glue (per-head LayerNorm32 of q / k / compressed k, the
cross/self gates) agrees with the reference's unfused formulation
(models_sparse/utils.py:239-270, 272-574, 575-640) restated below with torch
ops over the same sparse-attention modules: outputs and gradients within
2e-2 max-abs (relative to the tensor's scale) and >= 0.9995 cosine."""

import types

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _cos(a, b):
    a, b = a.detach().double().flatten(), b.detach().double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def _scene_coords():
    """Voxel tokens (batch, z, y, x) of a two-sphere shell in a 32^3 volume,
    Morton-block order, and the image tokens (batch, view, row, column) of 4
    posed 64^2 views; returns (volc, imc, view scene)."""
    from lsrm_sparse import blocks, synth

    spheres = ((2, 3), (0.2, 0.3))
    centres, radii = synth.scene_spheres(5, *spheres)
    sc = synth.view_scene(centres, radii, 1, 4, 64, 32, 6)
    im = synth.image_tokens(sc["mask_input"], 4, 4)
    vox, _ = synth.sdf_shell_voxels(32, 1800, 5, *spheres)
    vol = np.stack([np.zeros(len(vox)), vox[:, 2], vox[:, 1], vox[:, 0]], 1).astype(np.int32)
    volc = torch.from_numpy(vol).to(DEV)
    volc = volc[torch.argsort(blocks.volume_sort_keys(volc, 32, 4), stable=True)].contiguous()
    return volc, torch.from_numpy(im).to(DEV), sc


def _scene():
    from lsrm_sparse import blocks

    M, H, ps, bs = 4, 64, 4, 4
    volc, imc, sc = _scene_coords()
    args = types.SimpleNamespace(block_size=bs, volume_res=32, use_3d_aware_attn=True, topk_volume=8,
                                 bbox_radius=0.5, attn_winsize=2, topk_multiimage=2, image_num_per_batch=M,
                                 input_image_res=[H // 2, H], patch_size=ps)
    batch = {"mask_input": torch.from_numpy(sc["mask_input"]).to(DEV),
             "cameras_input": torch.from_numpy(sc["cameras"]).to(DEV)}
    dense = {"surface_points_input": torch.from_numpy(sc["surface_points"]).to(DEV),
             "masks_input": torch.from_numpy(sc["surface_masks"]).to(DEV)}
    maps = blocks.build_3D_aware_attn(imc, volc, batch, dense, args)
    cu_x = torch.tensor([0, volc.shape[0]], dtype=torch.int32, device=DEV)
    cu_y = torch.tensor([0, imc.shape[0]], dtype=torch.int32, device=DEV)
    return maps, cu_x, cu_y, volc.shape[0], imc.shape[0], M


def _reference_block(blk, x, cu_x, y, cu_y, maps, im_num):
    """BlockMix.forward / CrossAttention.forward as the reference writes them
    (torch LayerNorm32 per head, sigmoid gates as separate ops), over the
    same submodules and weights."""
    ca = blk.crs_attn
    D = ca.head_dim

    def ln_heads(t, heads):
        return torch.nn.functional.layer_norm(t.view(-1, heads, D).float(), (D,), eps=1e-5).to(t.dtype).view(
            t.shape[0], -1)

    x = blk.norm(x)
    y = blk.norm(y)
    q_x, k_x, v_x = ca.q_proj_x(x), ca.k_proj_x(x), ca.v_proj_x(x)
    k_y, v_y, q_y = ca.k_proj_y(y), ca.v_proj_y(y), ca.q_proj_y(y)
    ck_x2x, cv_x2x = ca.x_2_x_attn_in(k_x, v_x, maps["vol_to_vol_attn"])
    ck_x2y, cv_x2y = ca.x_2_y_attn_in(k_y, v_y, maps["vol_to_img_attn"])
    ck_y2y, cv_y2y = ca.y_2_y_attn_in(k_y, v_y, maps["img_to_img_attn"])
    ck_y2x, cv_y2x = ca.y_2_x_attn_in(k_x, v_x, maps["img_to_vol_attn"])
    Hq, Hkv = ca.num_q_heads, ca.num_kv_heads
    q_x, k_x, ck_x2x = ln_heads(q_x, Hq), ln_heads(k_x, Hkv), ln_heads(ck_x2x, Hkv)
    k_y, ck_x2y = ln_heads(k_y, Hkv), ln_heads(ck_x2y, Hkv)
    q_y, ck_y2y, ck_y2x = ln_heads(q_y, Hq), ln_heads(ck_y2y, Hkv), ln_heads(ck_y2x, Hkv)
    xc, _ = ca.x_2_y_attn_mid(q_x, cu_x, k_y, ck_x2y, v_y, cv_x2y, ca.topk_multiimage * im_num,
                              maps["vol_to_img_attn"])
    xs, _ = ca.x_2_x_attn_mid(q_x, cu_x, k_x, ck_x2x, v_x, cv_x2x, ca.topk_volume, maps["vol_to_vol_attn"])
    yc, _ = ca.y_2_x_attn_mid(q_y, cu_y, k_x, ck_y2x, v_x, cv_y2x, ca.topk_volume, maps["img_to_vol_attn"])
    ys, _ = ca.y_2_y_attn_mid(q_y, cu_y, k_y, ck_y2y, v_y, cv_y2y, ca.topk_multiimage * im_num,
                              maps["img_to_img_attn"])
    x_cross = ca.x_2_y_attn_out(x, q_x, k_y, v_y, maps["vol_to_img_attn"], xc)
    x_self = ca.x_2_x_attn_out(x, q_x, k_x, v_x, maps["vol_to_vol_attn"], xs)
    y_cross = ca.y_2_x_attn_out(y, q_y, k_x, v_x, maps["img_to_vol_attn"], yc)
    y_self = ca.y_2_y_attn_out(y, q_y, k_y, v_y, maps["img_to_img_attn"], ys)
    dim = ca.dim
    gx = ca.gate_x(x)
    x_res = ca.proj_x(x_cross * gx[:, :dim] + x_self * gx[:, dim:])
    gy = ca.gate_y(y)
    y_res = ca.proj_y(y_cross * gy[:, :dim] + y_self * gy[:, dim:])
    x = blk.norm(x + x_res)
    x = x + blk.mlp_x_1(x)
    y = blk.norm(y + y_res)
    y = y + blk.mlp_y_1(y)
    return x, y


def test_blockmix_matches_unfused_reference_glue():
    from lsrm_sparse import ops
    from lsrm_sparse.decoder import BlockMix

    torch.manual_seed(0)
    maps, cu_x, cu_y, nx, ny, M = _scene()
    blk = BlockMix(128, num_q_heads=2, num_kv_heads=2, topk_volume=8, topk_multiimage=2).to(DEV).to(torch.bfloat16)
    x0 = torch.randn(nx, 128, device=DEV, dtype=torch.bfloat16)
    y0 = torch.randn(ny, 128, device=DEV, dtype=torch.bfloat16)
    outs, grads = [], []
    for fn in (lambda x, y: blk(x, cu_x, y, cu_y, maps, M)[:2],
               lambda x, y: _reference_block(blk, x, cu_x, y, cu_y, maps, M)):
        blk.zero_grad()
        x = x0.clone().requires_grad_()
        y = y0.clone().requires_grad_()
        ox, oy = fn(x, y)
        g = torch.Generator(device=DEV).manual_seed(1)
        (ox.float() * torch.randn(ox.shape, device=DEV, generator=g)).sum().backward(retain_graph=True)
        (oy.float() * torch.randn(oy.shape, device=DEV, generator=g)).sum().backward()
        outs.append((ox.detach(), oy.detach()))
        grads.append((x.grad, y.grad, blk.crs_attn.q_proj_x.weight.grad.clone(),
                      blk.crs_attn.gate_y[0].weight.grad.clone()))
    assert ops.read_errors() == 0
    for a, b in list(zip(outs[0], outs[1])) + list(zip(grads[0], grads[1])):
        assert torch.isfinite(a).all()
        scale = max(1.0, float(b.float().abs().max()))
        assert float((a.float() - b.float()).abs().max()) <= 2e-2 * scale
        assert _cos(a, b) >= 0.9995
