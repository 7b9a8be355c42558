"""Generate golden fixtures by running the REFERENCE implementation on the CPU.

Run once in a container that holds the reference checkout (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --ref /path/to/reference

What runs, all unmodified reference code:

* ``native_sparse_attend`` (sparse/ops/triton_native_sparse_attention_impl_kvcentric.py
  :1382-1435) through ``TRITON_INTERPRET=1``, forward (output, log2 LSE) and
  backward (dQ, dK, dV).  fp16 only: the interpreter mis-computes bf16.
* ``get_block_score`` (sparse/ops/block_score.py:16-98), fp32.
* ``SpatialSparseAttentionIn`` (ResBlock compression + segment mean,
  sparse/module/spatial_sparse_attention.py:16-67) with its own random init.
* ``sort_volume_blocks`` / ``compute_block_separation``
  (misc/sparse_utils.py:126-152, 592-641): block metadata of voxel and
  image-patch coordinates.
* ``sort_image_blocks`` (misc/sparse_utils.py:95-124, ``--only imsort``).
* ``build_image_to_image_attn``, ``build_image_to_volume_attn``,
  ``build_volume_to_image_attn`` and ``from_imcoords_to_points``
  (misc/sparse_utils.py:653-1200) on posed views of a sphere scene from
  ``lsrm_sparse.synth.view_scene`` (``--only image``).
* the state-dict layout of ``BlockMix`` / ``BlockMixOneside``
  (models_sparse/utils.py:575-705) with and without weight norm, and of
  ``VolTransformer`` (models_sparse/voldecoder.py:39-194) with the decomposed
  and the full position embedding (``--only modules``, ``module_keys.json``).
* ``VolTransformer.forward`` with its decoder blocks replaced by seeded stubs
  (``StubDecoderBlock``; the real blocks need the GPU): embedding, skip links,
  final norm, upsampler and ``prepare_volume_output``, outputs and gradients
  (``--only voltransformer``).
* ``SpatialSparseAttentionOut`` (sigmoid-gated merge, :196-270) with and
  without the window branch.  ``flash_attn_varlen_func`` has no CPU kernel, so
  for the window branch it is replaced by ``_cpu_varlen_attention`` below (a
  plain restatement of flash-attn's varlen contract); the gate math that the
  fixture pins is the reference's.

Fixtures are small ``.npz`` files next to this script.  Nothing at test time
reads the reference checkout.
"""

from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _cpu_varlen_attention(q, k, v, cu_q, cu_k, max_q, max_k, dropout_p=0.0, softmax_scale=None,
                          causal=False, return_attn_probs=False, **_):
    """flash_attn_varlen_func contract on the CPU: per-sequence softmax
    attention, GQA by head grouping, natural-log LSE ``[Hq, total_q]``."""
    assert not causal
    Hq, Hkv, D = q.shape[1], k.shape[1], q.shape[2]
    G = Hq // Hkv
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    out = torch.zeros_like(q, dtype=torch.float32)
    lse = torch.zeros(Hq, q.shape[0], dtype=torch.float32)
    cq, ck = cu_q.tolist(), cu_k.tolist()
    for b in range(len(cq) - 1):
        qs, qe, ks, ke = cq[b], cq[b + 1], ck[b], ck[b + 1]
        for h in range(Hq):
            s = (q[qs:qe, h].float() @ k[ks:ke, h // G].float().t()) * scale
            lse[h, qs:qe] = torch.logsumexp(s, -1)
            out[qs:qe, h] = torch.softmax(s, -1) @ v[ks:ke, h // G].float()
    out = out.to(q.dtype)
    if return_attn_probs:
        return out, lse, None
    return out


def _blocks(lengths):
    return torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32)


def _unique_topk(gen, n, nb, k, pad_tail=0):
    """[n, k] ascending unique ids in [0, nb); the last ``pad_tail`` of every
    row replaced by -1 (the reference's tail padding)."""
    rows = []
    kk = min(k, nb)
    for _ in range(n):
        sel = torch.randperm(nb, generator=gen)[:kk].sort().values
        row = torch.full((k,), -1, dtype=torch.int32)
        row[:kk] = sel.to(torch.int32)
        if pad_tail:
            row[kk - pad_tail:kk] = -1
        rows.append(row)
    return torch.stack(rows)


def selection_cases():
    """(name, seq_block_lengths, Hq, Hkv, D, k, special)."""
    return [
        ("sel_g2_d32", [[7, 8, 5, 13, 7]], 4, 2, 32, 3, None),
        ("sel_mha_d64_2seq_pad", [[20, 33, 12, 9], [40, 16]], 2, 2, 64, 3, "pad"),
        ("sel_g2_long_blocks", [[150, 70, 5]], 2, 1, 32, 2, None),
        ("sel_dup_and_empty", [[10, 0, 12, 9, 17]], 2, 1, 32, 3, "dup_empty"),
        ("sel_g4_d64", [[16, 24, 8, 40, 12, 28]], 8, 2, 64, 4, None),
    ]


def make_selection(native_sparse_attend, name, seq_blocks, Hq, Hkv, D, k, special, seed):
    gen = torch.Generator().manual_seed(seed)
    lens = [l for s in seq_blocks for l in s]
    cu_blk = _blocks(lens)
    cu_seqblocks = _blocks([len(s) for s in seq_blocks])
    cu_seqlens = _blocks([sum(s) for s in seq_blocks])
    N = int(cu_seqlens[-1])
    q = (torch.randn(N, Hq, D, generator=gen) * 0.5).half()
    kk = (torch.randn(N, Hkv, D, generator=gen) * 0.5).half()
    v = (torch.randn(N, Hkv, D, generator=gen) * 0.5).half()
    do = (torch.randn(N, Hq, D, generator=gen) * 0.1).half()
    topk = torch.full((Hkv, N, k), -1, dtype=torch.int32)
    for b, blocks in enumerate(seq_blocks):
        qs, qe = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        for h in range(Hkv):
            topk[h, qs:qe] = _unique_topk(gen, qe - qs, len(blocks), k, pad_tail=1 if special == "pad" and b == 1 else 0)
    if special == "dup_empty":
        # a duplicated block id (attended twice) and a row with no selection
        topk[0, 3] = torch.tensor([2, 2, 4], dtype=torch.int32)
        topk[0, 5] = torch.tensor([1, 1, -1], dtype=torch.int32)  # block 1 is empty
        topk[0, 7] = torch.tensor([-1, -1, -1], dtype=torch.int32)
    qr, kr, vr = (t.clone().requires_grad_() for t in (q, kk, v))
    o, lse = native_sparse_attend(qr, kr, vr, topk, cu_seqblocks, cu_blk, cu_seqlens, cu_seqlens, return_lse=True)
    o.backward(do)
    return dict(
        q=q.float().numpy(), k=kk.float().numpy(), v=v.float().numpy(), do=do.float().numpy(),
        block_topk=topk.numpy(), cu_seqblocks=cu_seqblocks.numpy(), cu_block_include_tokens=cu_blk.numpy(),
        cu_seqlens=cu_seqlens.numpy(), o=o.detach().float().numpy(), lse_log2=lse.detach().float().numpy(),
        dq=qr.grad.float().numpy(), dk=kr.grad.float().numpy(), dv=vr.grad.float().numpy(),
        dtype=np.array("float16"),
    )


def make_block_score(get_block_score, seed, seq_q, seq_nb, Hq, Hkv, D, topk):
    gen = torch.Generator().manual_seed(seed)
    cu_q = _blocks(seq_q)
    cu_c = _blocks(seq_nb)
    N, NB = int(cu_q[-1]), int(cu_c[-1])
    q = torch.randn(N, Hq, D, generator=gen).bfloat16().float()
    ck = torch.randn(NB, Hkv, D, generator=gen).bfloat16().float()
    # a consistent LSE: the compressed attention's own natural-log LSE
    _, lse, _ = _cpu_varlen_attention(q, ck, ck, cu_q, cu_c, 0, 0, return_attn_probs=True)
    out = get_block_score(q, ck, lse, topk, cu_q, cu_c, cu_q[1:] - cu_q[:-1], cu_c[1:] - cu_c[:-1], None)
    return dict(q=q.numpy(), ck=ck.numpy(), lse=lse.numpy(), cu_seqlens_q=cu_q.numpy(),
                compressed_cu_seqlens=cu_c.numpy(), topk=np.array(topk), block_topk=out.numpy())


def make_compress(SpatialSparseAttentionIn, seed):
    torch.manual_seed(seed)
    D, Hkv = 32, 2
    mod = SpatialSparseAttentionIn(head_dim=D, num_kv_heads=Hkv)
    lens = [5, 9, 1, 14, 3, 8]
    cu = _blocks(lens)
    N = int(cu[-1])
    k = torch.randn(N, Hkv * D)
    v = torch.randn(N, Hkv * D)
    with torch.no_grad():
        ck, cv = mod(k, v, {"cu_block_include_tokens": cu})
    sd = {n: p.detach().numpy() for n, p in mod.state_dict().items()}
    out = dict(k=k.numpy(), v=v.numpy(), cu_block_include_tokens=cu.numpy(), ck=ck.numpy(), cv=cv.numpy())
    out.update({"w:" + n: a for n, a in sd.items()})
    return out


def make_gate(SpatialSparseAttentionOut, ssa_module, seed, window):
    torch.manual_seed(seed)
    hidden, Hq, Hkv = 64, 4, 2
    D = hidden // Hq
    mod = SpatialSparseAttentionOut(hidden_dim=hidden, num_q_heads=Hq, num_kv_heads=Hkv, is_window_attn=window)
    lens = [6, 10, 4, 12]
    cu = _blocks(lens)
    N = int(cu[-1])
    x = torch.randn(N, hidden)
    q = torch.randn(N, Hq * D)
    k = torch.randn(N, Hkv * D)
    v = torch.randn(N, Hkv * D)
    sel = torch.randn(N, hidden)
    comp = torch.randn(N, hidden)
    with torch.no_grad():
        out = mod(x, q, k, v, {"cu_block_include_tokens": cu}, {"selection_attn": sel, "compressed_attn": comp})
    return dict(x=x.numpy(), q=q.numpy(), k=k.numpy(), v=v.numpy(), selection=sel.numpy(),
                compressed=comp.numpy(), cu_block_include_tokens=cu.numpy(), out=out.numpy(),
                gate_weight=mod.gate[0].weight.detach().numpy(), window=np.array(window))


def _unique_coords(gen, n, batch, res):
    """n distinct voxels per batch element of a res^3 grid, grouped by batch."""
    out = []
    for b in range(batch):
        flat = torch.randperm(res ** 3, generator=gen)[:n]
        z, y, x = flat // (res * res), (flat // res) % res, flat % res
        out.append(torch.stack([torch.full_like(z, b), z, y, x], 1))
    return torch.cat(out).to(torch.int32)


def make_block_metadata(sparse_utils, seed):
    """sort_volume_blocks (misc/sparse_utils.py:126-152) and
    compute_block_separation (:592-641) on a volume case and an image-patch
    case.  compute_block_separation runs on float coordinates (integral
    values): its torch.histc has no CPU kernel for integer tensors; the
    arithmetic is the same."""
    import types

    gen = torch.Generator().manual_seed(seed)
    res, bs, batch = 32, 8, 3
    coords = _unique_coords(gen, 700, batch, res)
    coords = coords[torch.randperm(coords.shape[0], generator=gen)]
    coords = coords[torch.argsort(coords[:, 0], stable=True)]  # grouped by batch, voxel order shuffled
    feats = torch.arange(coords.shape[0], dtype=torch.float32)[:, None]
    args = types.SimpleNamespace(block_size=bs, volume_res=res)
    _, sorted_coords, idx = sparse_utils.sort_volume_blocks(feats, coords.clone(), args)
    cu_sb, cu_blk = sparse_utils.compute_block_separation(sorted_coords.clone().float(), 3, [bs, bs, bs], batch,
                                                          [res, res, res])
    # image patches: [view, row, col], blocks of 1 x 4 x 4 over a (views, 8, 8) grid
    img = []
    for b in range(2):
        v, r, c = torch.meshgrid(torch.arange(3), torch.arange(8), torch.arange(8), indexing="ij")
        keep = torch.rand(v.numel(), generator=gen) < 0.7
        img.append(torch.stack([torch.full((int(keep.sum()),), b), v.flatten()[keep], r.flatten()[keep],
                                c.flatten()[keep]], 1))
    img = torch.cat(img).to(torch.int32)
    img_sb, img_blk = sparse_utils.compute_block_separation(img.clone().float(), 3, [1, 4, 4], 2, [3, 8, 8])
    return dict(coords=coords.numpy(), volume_res=np.int32(res), block_size=np.int32(bs), batch=np.int32(batch),
                sort_idx=idx.numpy().astype(np.int64), cu_seqblocks=cu_sb.numpy().astype(np.int32),
                cu_block_include_tokens=cu_blk.numpy().astype(np.int32), img_coords=img.numpy(),
                img_cu_seqblocks=img_sb.numpy().astype(np.int32),
                img_cu_block_include_tokens=img_blk.numpy().astype(np.int32))


def make_volume_output(voldecoder, seed):
    """VolTransformer.prepare_volume_output (models_sparse/voldecoder.py:196-268)
    run on the CPU through the reference method itself (a stand-in `self`
    carrying output_dim / upsample_scale / vol_res): three batch elements of
    unique voxels in shuffled order (grouped by batch), u = 2, 8 channels, a
    16^3 token grid."""
    import types

    gen = torch.Generator().manual_seed(seed)
    res, u, C = 16, 2, 8
    parts = []
    for b, n in enumerate((150, 37, 200)):
        flat = torch.randperm(res ** 3, generator=gen)[:n]
        z, y, x = flat // (res * res), (flat // res) % res, flat % res
        parts.append(torch.stack([torch.full_like(z, b), z, y, x], 1))
    vidx = torch.cat(parts).to(torch.int32)
    volume = torch.randn(vidx.shape[0], C * u ** 3, generator=gen)
    prior = torch.zeros(1)
    me = types.SimpleNamespace(output_dim=C, upsample_scale=u, vol_res=res)
    out = voldecoder.VolTransformer.prepare_volume_output(me, volume, vidx, prior)
    return dict(volume=volume.numpy(), volume_index=vidx.numpy(), output_dim=np.int32(C), upsample_scale=np.int32(u),
                vol_res=np.int32(res), sparse_feat=out["sparse_feat"].numpy(),
                cu_seqlens=out["cu_seqlens"].numpy().astype(np.int32), seqlens=out["seqlens"].numpy().astype(np.int32),
                index_volume=out["index_volume"].numpy().astype(np.int32))


def make_volume_geo_topk(sparse_utils, seed):
    """build_volume_to_volume_attn with use_3d_aware_attn (misc/sparse_utils.py:
    1203-1279) on two batch elements of an SDF-shell-like voxel set, sorted
    into blocks by sort_volume_blocks first (the reference's order).  The
    separation's torch.histc has no CPU kernel for integer tensors: it is
    called here on a float copy of the (integral) input, same counts."""
    import types

    gen = torch.Generator().manual_seed(seed)
    res, bs, k = 32, 8, 8
    parts = []
    for b, n in enumerate((900, 400)):
        flat = torch.randperm(res ** 3, generator=gen)[:n]
        z, y, x = flat // (res * res), (flat // res) % res, flat % res
        parts.append(torch.stack([torch.full_like(z, b), z, y, x], 1))
    coords = torch.cat(parts).to(torch.int32)
    args = types.SimpleNamespace(block_size=bs, volume_res=res, use_3d_aware_attn=True, topk_volume=k,
                                 bbox_radius=0.5)
    feats = torch.zeros(coords.shape[0], 1)
    _, coords_sorted, _ = sparse_utils.sort_volume_blocks(feats, coords.clone(), args)
    histc = torch.histc
    torch.histc = lambda x, *a, **kw: histc(x.float(), *a, **kw)
    try:
        out = sparse_utils.build_volume_to_volume_attn(coords_sorted.clone(), args)
    finally:
        torch.histc = histc
    return dict(coords=coords_sorted.numpy().astype(np.int32), volume_res=np.int32(res), block_size=np.int32(bs),
                topk=np.int32(k), bbox_radius=np.float64(0.5), batch=np.int32(2),
                block_topk=out["block_topk"].numpy(), cu_seqblocks=out["cu_seqblocks"].numpy(),
                cu_block_include_tokens=out["cu_block_include_tokens"].numpy())


def make_image_maps(sparse_utils, seed, crop):
    """The image-side attention maps with use_3d_aware_attn on two batch
    elements of three 64x64 views (patch 4, block 4: 4x4 blocks per view,
    32x32 surface points) of a two-to-three-sphere scene, and the voxels of
    the same scene's shell (32^3 grid).  Cameras, masks and surface points come
    from ``lsrm_sparse.synth.view_scene``; image tokens are the patches with
    mask, in sort_image_blocks order; voxels are sorted by sort_volume_blocks.
    The separation's torch.histc gets a float copy (see
    ``make_volume_geo_topk``)."""
    import types

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "large-sparse-reconstruction-model_b200"))
    from lsrm_sparse import synth

    res, bs, ps, H, S, B, M = 32, 4, 4, 64, 32, 2, 3
    centres, radii = synth.scene_spheres(seed, (2, 3), (0.2, 0.3))
    scene = synth.view_scene(centres, radii, B, M, H, S, seed + 1, crop=crop)
    imcoords = torch.from_numpy(synth.image_tokens(scene["mask_input"], ps, bs))
    parts = []
    for b, n in enumerate((1500, 1100)):
        vox, _ = synth.sdf_shell_voxels(res, n, seed, (2, 3), (0.2, 0.3))
        parts.append(np.stack([np.full(len(vox), b), vox[:, 2], vox[:, 1], vox[:, 0]], 1))
    volcoords = torch.from_numpy(np.concatenate(parts).astype(np.int32))
    args = types.SimpleNamespace(block_size=bs, volume_res=res, use_3d_aware_attn=True, topk_volume=8,
                                 bbox_radius=0.5, attn_winsize=2, topk_multiimage=2, image_num_per_batch=M,
                                 input_image_res=[H // 2, H], patch_size=ps)
    _, volcoords, _ = sparse_utils.sort_volume_blocks(torch.zeros(volcoords.shape[0], 1), volcoords.clone(), args)
    batch = {"mask_input": torch.from_numpy(scene["mask_input"]),
             "cameras_input": torch.from_numpy(scene["cameras"])}
    if crop:
        batch["crop_input"] = torch.from_numpy(scene["crop_input"])
        batch["origin_size"] = torch.from_numpy(scene["origin_size"])
    dense = {"surface_points_input": torch.from_numpy(scene["surface_points"]),
             "masks_input": torch.from_numpy(scene["surface_masks"])}
    histc = torch.histc
    torch.histc = lambda x, *a, **kw: histc(x.float(), *a, **kw)
    try:
        i2i = sparse_utils.build_image_to_image_attn(imcoords.clone(), batch, dense, args)
        i2v = sparse_utils.build_image_to_volume_attn(imcoords.clone(), volcoords.clone(), dense, args)
        v2i = sparse_utils.build_volume_to_image_attn(imcoords.clone(), volcoords.clone(), batch, dense, args)
    finally:
        torch.histc = histc
    impoints = sparse_utils.from_imcoords_to_points(imcoords.clone(), dense, args)
    out = dict(imcoords=imcoords.numpy(), volcoords=volcoords.numpy().astype(np.int32),
               impoints=impoints.numpy(), volume_res=np.int32(res), block_size=np.int32(bs),
               patch_size=np.int32(ps), image_res=np.int32(H), topk_volume=np.int32(8), attn_winsize=np.int32(2),
               topk_multiimage=np.int32(2), bbox_radius=np.float64(0.5), batch=np.int32(B))
    for k, v in scene.items():
        out["scene_" + k] = v
    for name, r in (("i2i", i2i), ("i2v", i2v), ("v2i", v2i)):
        for k, v in r.items():
            out[f"{name}_{k}"] = v.numpy()
    return out


def make_image_sort(sparse_utils, seed):
    """sort_image_blocks (misc/sparse_utils.py:95-124) on shuffled image
    tokens of two batch elements, three views of 16 x 16 patches, blocks of
    4 x 4 patches."""
    import types

    gen = torch.Generator().manual_seed(seed)
    parts = []
    for b in range(2):
        v, r, c = torch.meshgrid(torch.arange(3), torch.arange(16), torch.arange(16), indexing="ij")
        keep = torch.rand(v.numel(), generator=gen) < 0.5
        parts.append(torch.stack([torch.full((int(keep.sum()),), b), v.flatten()[keep], r.flatten()[keep],
                                  c.flatten()[keep]], 1))
    coords = torch.cat(parts).to(torch.int32)
    coords = coords[torch.randperm(coords.shape[0], generator=gen)]
    args = types.SimpleNamespace(block_size=4, patch_size=8, input_image_res=[64, 128])
    feats = torch.arange(coords.shape[0], dtype=torch.float32)[:, None]
    _, sorted_coords, idx = sparse_utils.sort_image_blocks(feats, coords.clone(), args)
    return dict(coords=coords.numpy(), sorted_coords=sorted_coords.numpy(), sort_idx=idx.numpy().astype(np.int64),
                block_size=np.int32(4), patch_size=np.int32(8), image_res=np.int32(128))


MODULE_CASES = [  # (name, BlockMix kwargs): small dims, the reference's layer layout
    ("blockmix", dict(dim=64, num_q_heads=4, num_kv_heads=2)),
    ("blockmix_weight_norm", dict(dim=64, num_q_heads=4, num_kv_heads=2, use_weight_norm=True, qkv_bias=True)),
    ("blockmix_oneside_weight_norm", dict(dim=64, num_q_heads=4, num_kv_heads=4, use_weight_norm=True,
                                          oneside=True)),
]


VOLT_CASES = [  # (name, VolTransformer kwargs): small dims, the reference's decoder layout
    ("voltransformer_decomposed", dict(vol_res=8, upsample_scale=2, embed_dim=64, output_dim=8, depth=3,
                                       num_q_heads=4, num_kv_heads=2, skip_links=(1,), use_decomposed_embed=True)),
    ("voltransformer_fuse_all_weight_norm", dict(vol_res=4, upsample_scale=2, embed_dim=64, output_dim=4, depth=3,
                                                 num_q_heads=4, num_kv_heads=4, skip_links=(2, 0),
                                                 fuse_all_layers=True, use_weight_norm=True, qkv_bias=True)),
]


def make_module_keys(utils, voldecoder=None):
    """State-dict layout (parameter name -> shape) of the reference's
    ``BlockMix`` / ``BlockMixOneside`` (models_sparse/utils.py:575-705), which
    holds ``CrossAttention`` (:80-240, weight norm at :228-236) and ``Mlp``,
    and of ``VolTransformer`` (models_sparse/voldecoder.py:39-194)."""
    out = {}
    for name, kw in MODULE_CASES:
        kw = dict(kw)
        cls = utils.BlockMixOneside if kw.pop("oneside", False) else utils.BlockMix
        m = cls(**kw)
        out[name] = {k: list(v.shape) for k, v in m.state_dict().items()}
    if voldecoder is not None:
        for name, kw in VOLT_CASES:
            m = voldecoder.VolTransformer(**kw)
            out[name] = {k: list(v.shape) for k, v in m.state_dict().items()}
    return out


class StubDecoderBlock(torch.nn.Module):
    """A deterministic stand-in for BlockMix / BlockMixOneside with their call
    signature (x, cu_seqlens_x, y, cu_seqlens_y, attn_map, im_num) and return
    shape: x gains tanh(x Wx) and a share of the image tokens' mean, so the y
    that the skip links route reaches the output.  It lets the reference's
    VolTransformer run on the CPU (its attention needs the GPU) and pins the
    orchestration around the blocks: embedding, skip links, final norm,
    upsampler, output formatting."""

    def __init__(self, dim, seed, oneside):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.wx = torch.nn.Parameter(torch.randn(dim, dim, generator=g) / math.sqrt(dim))
        self.wy = torch.nn.Parameter(torch.randn(dim, dim, generator=g) / math.sqrt(dim))
        self.oneside = oneside

    def forward(self, x, cu_seqlens_x, y, cu_seqlens_y, attn_map, im_num):
        x = x + torch.tanh(x @ self.wx) + 0.1 * y.mean(0, keepdim=True)
        if self.oneside:
            return x, {}
        return x, y + torch.tanh(y @ self.wy), {}


def stub_blocks(model, dim):
    """Replaces a VolTransformer's decoder blocks by StubDecoderBlocks (seeded
    by position)."""
    model.cross_blocks = torch.nn.ModuleList(StubDecoderBlock(dim, 1000 + i, False)
                                             for i in range(len(model.cross_blocks)))
    model.skip_blocks = torch.nn.ModuleList(StubDecoderBlock(dim, 2000 + i, True)
                                            for i in range(len(model.skip_blocks)))
    return model


VOLT_FWD_CASES = [  # (name, VolTransformer kwargs) for the orchestration fixtures
    ("voltransformer_fwd_decomposed", dict(vol_res=8, upsample_scale=2, embed_dim=32, output_dim=4, depth=3,
                                           num_q_heads=2, num_kv_heads=2, skip_links=(1, 0),
                                           use_decomposed_embed=True)),
    ("voltransformer_fwd_full_embed", dict(vol_res=4, upsample_scale=2, embed_dim=32, output_dim=4, depth=2,
                                           num_q_heads=2, num_kv_heads=2, skip_links=(0,))),
]


def volt_inputs(kw, seed):
    """Two batch elements of voxels (unique coordinates, grouped by batch) and
    image tokens, the flat voxel mask and its token order, random features."""
    g = torch.Generator().manual_seed(seed)
    R, C = kw["vol_res"], kw["embed_dim"]
    parts, flats = [], []
    for b, n in enumerate((37, 29)):
        flat = torch.randperm(R ** 3, generator=g)[:n]
        parts.append(torch.stack([torch.full_like(flat, b), flat // (R * R), (flat // R) % R, flat % R], 1))
        flats.append(flat + b * R ** 3)
    volume_index = torch.cat(parts).long()
    flat = torch.cat(flats)
    mask = torch.zeros(2 * R ** 3, dtype=torch.bool)
    mask[flat] = True
    coords_idx = torch.searchsorted(torch.nonzero(mask).squeeze(1), flat)
    image_index = torch.cat([torch.zeros(10, 4), torch.ones(8, 4)]).long()
    ny, n = image_index.shape[0], volume_index.shape[0]
    return dict(y=torch.randn(ny, C, generator=g), prior_imfeat=torch.randn(ny, C, generator=g),
                image_index=image_index, prior_volfeat=torch.randn(n, C, generator=g), mask_volume=mask,
                volume_index=volume_index, volume_coords_idx=coords_idx,
                grad_w=torch.randn(n * kw["upsample_scale"] ** 3, kw["output_dim"], generator=g))


def make_volt_forward(voldecoder, name, kw, seed):
    """The reference's VolTransformer.forward (models_sparse/voldecoder.py:
    270-424, prepare_volume_output :196-268) with stub blocks, fp32 on the
    CPU: inputs, the state dict, the output dict and the gradients of a
    seeded weighted sum of sparse_feat with respect to y and the model's
    parameters."""
    torch.manual_seed(seed)
    m = stub_blocks(voldecoder.VolTransformer(**kw), kw["embed_dim"])
    inp = volt_inputs(kw, seed + 1)
    y = inp["y"].clone().requires_grad_()
    out, _ = m(y, [inp["prior_imfeat"]], inp["image_index"], inp["prior_volfeat"], inp["mask_volume"],
               inp["volume_index"], torch.zeros(1), inp["volume_coords_idx"], {}, 4)
    (out["sparse_feat"] * inp["grad_w"]).sum().backward()
    res = {"in_" + k: v.numpy() for k, v in inp.items()}
    res.update({"sd_" + k: v.detach().numpy() for k, v in m.state_dict().items()})
    res.update({"grad_" + k: p.grad.numpy() for k, p in m.named_parameters() if p.grad is not None})
    res.update(out_sparse_feat=out["sparse_feat"].detach().numpy(), out_cu_seqlens=out["cu_seqlens"].numpy(),
               out_index_volume=out["index_volume"].numpy(), grad_y=y.grad.numpy())
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    ap.add_argument("--only", choices=["blocks", "volume", "geo", "image", "imsort", "modules", "voltransformer"],
                    default=None,
                    help="regenerate one group of fixtures")
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.ref)
    from misc import sparse_utils

    if args.only == "modules":
        import json

        from models_sparse import utils, voldecoder

        with open(os.path.join(HERE, "module_keys.json"), "w") as f:
            json.dump(make_module_keys(utils, voldecoder), f, indent=1, sort_keys=True)
        print("wrote module_keys.json")
        return
    if args.only == "voltransformer":
        from models_sparse import voldecoder

        for i, (name, kw) in enumerate(VOLT_FWD_CASES):
            np.savez_compressed(os.path.join(HERE, name + ".npz"), **make_volt_forward(voldecoder, name, kw, 300 + i))
            print("wrote", name)
        return
    if args.only == "imsort":
        np.savez_compressed(os.path.join(HERE, "image_sort.npz"), **make_image_sort(sparse_utils, 81))
        print("wrote image_sort")
        return
    if args.only == "image":
        for crop in (False, True):
            name = "image_maps_crop" if crop else "image_maps"
            np.savez_compressed(os.path.join(HERE, name + ".npz"), **make_image_maps(sparse_utils, 71, crop))
            print("wrote", name)
        return
    if args.only == "geo":
        np.savez_compressed(os.path.join(HERE, "volume_geo_topk.npz"), **make_volume_geo_topk(sparse_utils, 61))
        print("wrote volume_geo_topk")
        return
    if args.only == "volume":
        from models_sparse import voldecoder

        np.savez_compressed(os.path.join(HERE, "volume_output.npz"), **make_volume_output(voldecoder, 51))
        print("wrote volume_output")
        return
    np.savez_compressed(os.path.join(HERE, "block_metadata.npz"), **make_block_metadata(sparse_utils, 41))
    print("wrote block_metadata")
    if args.only == "blocks":
        return
    import flash_attn  # noqa: F401  (import check only; no CPU kernel)

    from sparse.ops import block_window_attention as bwa
    from sparse.ops.block_score import get_block_score
    from sparse.ops.triton_native_sparse_attention_impl_kvcentric import native_sparse_attend
    from sparse.module import spatial_sparse_attention as ssa

    bwa.flash_attn_varlen_func = _cpu_varlen_attention
    ssa.flash_attn_varlen_func = _cpu_varlen_attention

    for i, (name, seq_blocks, Hq, Hkv, D, k, special) in enumerate(selection_cases()):
        data = make_selection(native_sparse_attend, name, seq_blocks, Hq, Hkv, D, k, special, seed=100 + i)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **data)
        print("wrote", name)
    bs_cases = [
        ("score_g1", 11, [37, 21], [9, 5], 4, 4, 32, 4),
        ("score_g4", 12, [50], [12], 8, 2, 64, 5),
        ("score_few_blocks", 13, [19, 23], [3, 7], 2, 1, 16, 4),
    ]
    for name, seed, sq, snb, Hq, Hkv, D, topk in bs_cases:
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"),
                            **make_block_score(get_block_score, seed, sq, snb, Hq, Hkv, D, topk))
        print("wrote", name)
    np.savez_compressed(os.path.join(HERE, "compress_resblock.npz"), **make_compress(ssa.SpatialSparseAttentionIn, 21))
    print("wrote compress_resblock")
    for window in (False, True):
        nm = "gate_window" if window else "gate_nowindow"
        np.savez_compressed(os.path.join(HERE, f"{nm}.npz"), **make_gate(ssa.SpatialSparseAttentionOut, ssa, 31, window))
        print("wrote", nm)


if __name__ == "__main__":
    main()
