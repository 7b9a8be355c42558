"""The whole volume decoder (lsrm_sparse.decoder.VolTransformer) on a small
voxel + posed-view scene with the 3D-aware maps: its forward — position
embedding, the layer loop with skip links and skip blocks, the optional
per-layer prior fusion and output gate, the final norm, the upsampler and the
output formatting — against the reference's forward
(models_sparse/voldecoder.py:196-424) restated below with torch ops over the
same submodules and weights.  Outputs and gradients within 2e-2 max-abs
(relative to the tensor's scale) and >= 0.9995 cosine; the index volume and
the offsets bit for bit."""

import pytest
import torch

from tests.test_gpu_decoder import _cos, _scene, _scene_coords

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _reference_prepare(m, volume, volume_index, prior_volume):
    """VolTransformer.prepare_volume_output as voldecoder.py:196-268 writes it."""
    u, od = m.upsample_scale, m.output_dim
    B = int(volume_index[:, 0].max()) + 1
    sparse = volume.reshape(-1, od, u, u, u).permute(0, 2, 3, 4, 1).reshape(-1, od)
    c = volume_index.clone().reshape(-1, 4, 1, 1, 1).repeat(1, 1, u, u, u).permute(0, 2, 3, 4, 1) * u
    zo, yo, xo = torch.meshgrid(*(torch.arange(u, dtype=torch.int32, device=DEV),) * 3, indexing="ij")
    c[..., 1] += zo[None]
    c[..., 2] += yo[None]
    c[..., 3] += xo[None]
    c = c.reshape(-1, 4)
    gap = volume_index[1:, 0] - volume_index[:-1, 0]
    seq = torch.nonzero(gap) + 1
    cu = torch.tensor([0] + [int(seq[n]) for n in range(B - 1)] + [volume_index.shape[0]], dtype=torch.int32,
                      device=DEV) * u ** 3
    R = m.vol_res * u
    iv = -torch.ones(B, R, R, R, dtype=torch.int32, device=DEV)
    for n in range(B):
        s, e = int(cu[n]), int(cu[n + 1])
        cc = c[s:e, 1:4]
        iv[n, cc[:, 0], cc[:, 1], cc[:, 2]] = torch.arange(e - s, dtype=torch.int32, device=DEV)
    return {"sparse_feat": sparse, "cu_seqlens": cu, "index_volume": iv}


def _reference_forward(m, y, prior_imfeat_list, image_index, prior_volfeat, mask_volume, volume_index,
                       prior_volume, volume_coords_idx, maps, im_num):
    """VolTransformer.forward (voldecoder.py:270-424), one GPU, no checkpoints.
    The position tables are indexed as fp32 copies (the same values): in
    bf16 the gradient's scatter-add over ~60 tokens per table row rounds
    differently for every summation order, by up to a few percent."""
    B = int(image_index[:, 0].max()) + 1
    C = m.embed_dim
    if m.use_decomposed_embed:
        x = torch.cat([m.pos_embed_z.float().reshape(-1, m.embed_dim_z)[volume_index[:, 1].long()],
                       m.pos_embed_y.float().reshape(-1, m.embed_dim_y)[volume_index[:, 2].long()],
                       m.pos_embed_x.float().reshape(-1, m.embed_dim_x)[volume_index[:, 3].long()]],
                      dim=-1).to(y.dtype)
    else:
        x = m.pos_embed.float().repeat(B, 1, 1).reshape(-1, C)
        x = x[mask_volume, :]
        x = x[volume_coords_idx, :].to(y.dtype)
    prior_imfeat = torch.cat(prior_imfeat_list, dim=1)

    def cu_of(ids):
        seq = torch.nonzero(ids[1:] - ids[:-1]) + 1
        return torch.tensor([0] + [int(seq[n]) for n in range(B - 1)] + [ids.shape[0]], dtype=torch.int32,
                            device=DEV)

    cu_v, cu_i = cu_of(volume_index[:, 0]), cu_of(image_index[:, 0])
    y_list = []
    for idx, blk in enumerate(m.cross_blocks):
        if m.fuse_all_layers:
            x = x + m.fuse_prior_volfeats[idx](prior_volfeat)
            y = y + m.fuse_prior_imfeats[idx](prior_imfeat)
        x, y, _ = blk(x, cu_v, y, cu_i, maps, im_num)
        if idx in m.skip_links:
            y_list.insert(0, y)
    y_list.insert(0, y)
    for n, blk in enumerate(m.skip_blocks):
        if m.fuse_all_layers:
            x = x + m.skip_fuse_prior_volfeats[n](prior_volfeat)
            y = y_list[n + 1] + m.skip_fuse_prior_imfeats[n](torch.cat([y_list[0], prior_imfeat], dim=1))
        elif n == 0:
            y = y_list[n + 1] + m.skip_fuse_prior_imfeats[n](y_list[0])
        else:
            y = y_list[n + 1]
        x, _ = blk(x, cu_v, y, cu_i, maps, im_num)
    if m.fuse_all_layers:
        g = torch.sigmoid(m.fuse_pred_volfeat(x))
        x = m.norm(x * g[:, :C] + prior_volfeat * g[:, C:])
    else:
        x = m.norm(x)
    return _reference_prepare(m, m.upsampler(x), volume_index, prior_volume)


@pytest.mark.parametrize("variant", ["decomposed", "full_embed_fuse_all"])
def test_voltransformer_matches_reference_forward(variant):
    from lsrm_sparse import ops
    from lsrm_sparse.decoder import VolTransformer

    torch.manual_seed(0)
    maps, cu_x, cu_y, nx, ny, M = _scene()
    vol_res, C = 32, 128
    fuse = variant == "full_embed_fuse_all"
    m = VolTransformer(vol_res=vol_res, upsample_scale=2, embed_dim=C, output_dim=8, depth=3, num_q_heads=2,
                       num_kv_heads=2, skip_links=(1, 0), use_decomposed_embed=not fuse, fuse_all_layers=fuse,
                       topk_volume=8, topk_multiimage=2).to(DEV).to(torch.bfloat16)
    vi, ii, _ = _scene_coords()
    assert vi.shape[0] == nx and ii.shape[0] == ny
    # the full table's rows: a flat mask over the volume, reordered to the token order
    flat = (vi[:, 1].long() * vol_res + vi[:, 2].long()) * vol_res + vi[:, 3].long()
    mask = torch.zeros(vol_res ** 3, dtype=torch.bool, device=DEV)
    mask[flat] = True
    vci = torch.searchsorted(torch.nonzero(mask).squeeze(1), flat)
    fuse_ratio = len(m.skip_links) + 1
    g = torch.Generator(device=DEV).manual_seed(2)
    y0 = torch.randn(ny, C, device=DEV, dtype=torch.bfloat16, generator=g)
    prior_im = [torch.randn(ny, C, device=DEV, dtype=torch.bfloat16, generator=g) for _ in range(fuse_ratio)]
    prior_vol = torch.randn(nx, C, device=DEV, dtype=torch.bfloat16, generator=g)
    prior_volume = torch.randn(1, 8, 4, 4, 4, device=DEV)
    outs, grads = [], []
    for fn in (lambda y: m(y, prior_im, ii, prior_vol, mask, vi, prior_volume, vci, maps, M)[0],
               lambda y: _reference_forward(m, y, prior_im, ii, prior_vol, mask, vi, prior_volume, vci, maps, M)):
        m.zero_grad()
        y = y0.clone().requires_grad_()
        o = fn(y)
        w = torch.randn(o["sparse_feat"].shape, device=DEV, generator=torch.Generator(device=DEV).manual_seed(3))
        (o["sparse_feat"].float() * w).sum().backward()
        outs.append(o)
        emb = [m.pos_embed] if fuse else [m.pos_embed_z, m.pos_embed_y, m.pos_embed_x]
        grads.append([y.grad] + [t.grad.clone() for t in emb] +
                     [m.cross_blocks[0].crs_attn.q_proj_x.weight.grad.clone(),
                      m.skip_blocks[1].mlp_x_1.fc2.weight.grad.clone(),
                      m.upsampler.dconv3d.weight.grad.clone()] +
                     ([m.fuse_pred_volfeat.weight.grad.clone(), m.fuse_prior_imfeats[2].weight.grad.clone()]
                      if fuse else [m.skip_fuse_prior_imfeats[0].weight.grad.clone()]))
    assert ops.read_errors() == 0
    assert torch.equal(outs[0]["index_volume"], outs[1]["index_volume"])
    assert torch.equal(outs[0]["cu_seqlens"], outs[1]["cu_seqlens"])
    assert outs[0]["dense_feat"] is prior_volume
    for a, b in [(outs[0]["sparse_feat"], outs[1]["sparse_feat"])] + list(zip(grads[0], grads[1])):
        assert a.shape == b.shape
        assert torch.isfinite(a).all()
        scale = max(1.0, float(b.detach().float().abs().max()))
        assert float((a.float() - b.float()).abs().max()) <= 2e-2 * scale
        assert _cos(a, b) >= 0.9995

