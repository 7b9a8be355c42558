"""The sparse decoder's building blocks (models_sparse/utils.py), assembled
from this package's modules on one GPU (the reference's non-sequence-parallel
path):

* ``Mlp``             — models_sparse/utils.py:80-106
* ``CrossAttention``  — :108-574: volume tokens x and image tokens y, each
  attending to both sets through SpatialSparseAttentionIn / Mid / Out
* ``BlockMix``        — :575-640, ``BlockMixOneside`` — :643-705
* ``VolUpsampler``    — models_sparse/voldecoder.py:18-36
* ``VolTransformer``  — models_sparse/voldecoder.py:39-424: position
  embedding, the layer loop with skip links and one-sided skip blocks, the
  final norm, the upsampler and the output formatting

Constructor arguments, forward signatures, return values and parameter names
are the reference's, so its state dicts load (weight-normed Linears keep the
reference's parametrization).  Differences inside: the per-head LayerNorm32
of q / k / compressed k is the fused ``lsrm_head_layernorm_pack`` (one pass
each way), and the cross/self gate's sigmoid and merge are the fused
two-branch ``lsrm_gate_merge``; the Linears are library GEMMs.  With
``use_sequence_parallel=True`` the inputs are one rank's whole blocks as
``ulysses.seq_parallel_token_blocks`` distributed them, and the attention
cores exchange heads and sequence through ``lsrm_sparse.ulysses`` (Ulysses)
instead of the reference's K/V all-gathers.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import functional as F
from .module import LayerNorm32, SpatialSparseAttentionIn, SpatialSparseAttentionMid, SpatialSparseAttentionOut
from .ulysses import head_layernorm


class Mlp(nn.Module):
    def __init__(self, in_features, hidden_features=None, out_features=None, act_layer=nn.GELU, bias=True,
                 use_weight_norm=False):
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        self.fc1 = nn.Linear(in_features, hidden_features, bias=bias)
        self.act = act_layer()
        self.fc2 = nn.Linear(hidden_features, out_features, bias=bias)
        if use_weight_norm:
            self.fc1 = nn.utils.parametrizations.weight_norm(self.fc1)
            self.fc2 = nn.utils.parametrizations.weight_norm(self.fc2)

    def forward(self, x):
        return self.fc2(self.act(self.fc1(x)))


def _attn_triple(dim, num_q_heads, num_kv_heads, window):
    return (SpatialSparseAttentionIn(head_dim=dim // num_q_heads, num_kv_heads=num_kv_heads),
            SpatialSparseAttentionMid(hidden_dim=dim, num_q_heads=num_q_heads, num_kv_heads=num_kv_heads,
                                      is_window_attn=window),
            SpatialSparseAttentionOut(hidden_dim=dim, num_q_heads=num_q_heads, num_kv_heads=num_kv_heads,
                                      is_window_attn=window))


class CrossAttention(nn.Module):
    def __init__(self, dim, num_q_heads=32, num_kv_heads=2, qkv_bias=False, use_weight_norm=False, oneside=False,
                 topk_volume=8, topk_multiimage=2, use_sequence_parallel=False, no_checkpoint_all_gather=False, *,
                 fused_qkv=None):
        super().__init__()
        # fused_qkv: each token set's q / k / v projections run as one GEMM with the per-head LayerNorm32 of
        # q and k in its epilogue (lsrm_qkv_norm_fwd; bf16 on the GPU, head_dim 32 or 64, width a multiple
        # of 64); None: wherever those hold; False: the Linears, then the fused per-head LayerNorm
        self.fused_qkv = fused_qkv
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.dim = dim
        self.head_dim = dim // num_q_heads
        kv_dim = self.head_dim * num_kv_heads
        self.q_proj_x = nn.Linear(dim, dim, bias=qkv_bias)
        self.k_proj_x = nn.Linear(dim, kv_dim, bias=qkv_bias)
        self.v_proj_x = nn.Linear(dim, kv_dim, bias=qkv_bias)
        self.gate_x = nn.Sequential(nn.Linear(dim, 2 * dim), nn.Sigmoid())
        self.proj_x = nn.Linear(dim, dim)
        self.norm_layer_q = LayerNorm32(self.head_dim, elementwise_affine=False)
        self.norm_layer_kv = LayerNorm32(self.head_dim, elementwise_affine=False)
        self.use_sequence_parallel = use_sequence_parallel
        self.no_checkpoint_all_gather = no_checkpoint_all_gather
        self.topk_volume = topk_volume
        self.topk_multiimage = topk_multiimage
        self.x_2_x_attn_in, self.x_2_x_attn_mid, self.x_2_x_attn_out = _attn_triple(dim, num_q_heads, num_kv_heads,
                                                                                   True)
        self.x_2_y_attn_in, self.x_2_y_attn_mid, self.x_2_y_attn_out = _attn_triple(dim, num_q_heads, num_kv_heads,
                                                                                   False)
        self.oneside = oneside
        self.k_proj_y = nn.Linear(dim, kv_dim, bias=qkv_bias)
        self.v_proj_y = nn.Linear(dim, kv_dim, bias=qkv_bias)
        if not oneside:
            self.q_proj_y = nn.Linear(dim, dim, bias=qkv_bias)
            self.gate_y = nn.Sequential(nn.Linear(dim, 2 * dim, bias=False), nn.Sigmoid())
            self.proj_y = nn.Linear(dim, dim)
            self.y_2_y_attn_in, self.y_2_y_attn_mid, self.y_2_y_attn_out = _attn_triple(
                dim, num_q_heads, num_kv_heads, True)
            self.y_2_x_attn_in, self.y_2_x_attn_mid, self.y_2_x_attn_out = _attn_triple(
                dim, num_q_heads, num_kv_heads, False)
        if use_weight_norm:  # the same projections as models_sparse/utils.py:228-236
            wn = nn.utils.parametrizations.weight_norm
            self.q_proj_x, self.k_proj_x, self.v_proj_x = wn(self.q_proj_x), wn(self.k_proj_x), wn(self.v_proj_x)
            self.proj_x = wn(self.proj_x)
            self.k_proj_y, self.v_proj_y = wn(self.k_proj_y), wn(self.v_proj_y)
            if not oneside:
                self.q_proj_y, self.proj_y = wn(self.q_proj_y), wn(self.proj_y)

    def _projections(self, x, y):
        """q (normalised), k (raw and normalised) and v of both token sets:
        q_x, k_x, kn_x, v_x, q_y (None one-sided), k_y, kn_y, v_y.  With
        ``fused_qkv`` every set is one GEMM with the norms in its epilogue;
        otherwise the Linears, then the fused per-head LayerNorm32
        (models_sparse/utils.py:114-127, 239-270)."""
        Hq, Hkv = self.num_q_heads, self.num_kv_heads
        fused = self.fused_qkv
        if fused is None:
            fused = x.is_cuda and x.dtype == torch.bfloat16 and self.head_dim in (32, 64) and self.dim % 64 == 0
        if fused:
            D, eps = self.head_dim, self.norm_layer_q.eps
            (_, q_x), (k_x, kn_x), (v_x, _) = F.qkv_norm(
                x, [self.q_proj_x, self.k_proj_x, self.v_proj_x], [(False, True), (True, True), (True, False)], D, eps)
            if self.oneside:
                (k_y, kn_y), (v_y, _) = F.qkv_norm(y, [self.k_proj_y, self.v_proj_y], [(True, True), (True, False)],
                                                  D, eps)
                q_y = None
            else:
                (_, q_y), (k_y, kn_y), (v_y, _) = F.qkv_norm(
                    y, [self.q_proj_y, self.k_proj_y, self.v_proj_y], [(False, True), (True, True), (True, False)],
                    D, eps)
            return q_x, k_x, kn_x, v_x, q_y, k_y, kn_y, v_y
        q_x, k_x, v_x = self.q_proj_x(x), self.k_proj_x(x), self.v_proj_x(x)
        k_y, v_y = self.k_proj_y(y), self.v_proj_y(y)
        q_y = None if self.oneside else self._norm(self.q_proj_y(y), Hq)
        return self._norm(q_x, Hq), k_x, self._norm(k_x, Hkv), v_x, q_y, k_y, self._norm(k_y, Hkv), v_y

    def _norm(self, t, heads):
        """LayerNorm32 over head_dim of [n, heads * head_dim] (norm_layer_q /
        norm_layer_kv, models_sparse/utils.py:239-270), fused."""
        n = t.shape[0]
        return head_layernorm(t.reshape(n, heads, self.head_dim), self.norm_layer_q.eps).reshape(n, -1)

    @staticmethod
    def _gate(x, gate, x_cross, x_self):
        lin = gate[0]
        return F.gate_merge(nn.functional.linear(x, lin.weight, lin.bias), [x_cross, x_self])

    def forward(self, x, cu_seqlens_x, y, cu_seqlens_y, im_num, attn_map):
        if self.use_sequence_parallel:
            return self._forward_sequence_parallel(x, y, im_num, attn_map)
        q_x, k_x_raw, k_x, v_x, q_y, k_y_raw, k_y, v_y = self._projections(x, y)
        # the compression reads the raw keys / values (the In modules run before the norms)
        ck_x2x, cv_x2x = self.x_2_x_attn_in(k_x_raw, v_x, attn_map["vol_to_vol_attn"])
        ck_x2y, cv_x2y = self.x_2_y_attn_in(k_y_raw, v_y, attn_map["vol_to_img_attn"])
        if not self.oneside:
            ck_y2y, cv_y2y = self.y_2_y_attn_in(k_y_raw, v_y, attn_map["img_to_img_attn"])
            ck_y2x, cv_y2x = self.y_2_x_attn_in(k_x_raw, v_x, attn_map["img_to_vol_attn"])
        Hkv = self.num_kv_heads
        ck_x2x, ck_x2y = self._norm(ck_x2x, Hkv), self._norm(ck_x2y, Hkv)
        if not self.oneside:
            ck_y2y, ck_y2x = self._norm(ck_y2y, Hkv), self._norm(ck_y2x, Hkv)

        sparse_info = {}
        x_cross_out, sparse_info["v_2_i"] = self.x_2_y_attn_mid(
            q_x, cu_seqlens_x, k_y, ck_x2y, v_y, cv_x2y, self.topk_multiimage * im_num, attn_map["vol_to_img_attn"])
        x_self_out, sparse_info["v_2_v"] = self.x_2_x_attn_mid(
            q_x, cu_seqlens_x, k_x, ck_x2x, v_x, cv_x2x, self.topk_volume, attn_map["vol_to_vol_attn"])
        if not self.oneside:
            y_cross_out, sparse_info["i_2_v"] = self.y_2_x_attn_mid(
                q_y, cu_seqlens_y, k_x, ck_y2x, v_x, cv_y2x, self.topk_volume, attn_map["img_to_vol_attn"])
            y_self_out, sparse_info["i_2_i"] = self.y_2_y_attn_mid(
                q_y, cu_seqlens_y, k_y, ck_y2y, v_y, cv_y2y, self.topk_multiimage * im_num,
                attn_map["img_to_img_attn"])

        x_cross = self.x_2_y_attn_out(x, q_x, k_y, v_y, attn_map["vol_to_img_attn"], x_cross_out)
        x_self = self.x_2_x_attn_out(x, q_x, k_x, v_x, attn_map["vol_to_vol_attn"], x_self_out)
        x_new = self.proj_x(self._gate(x, self.gate_x, x_cross, x_self))
        if self.oneside:
            return x_new, sparse_info
        y_cross = self.y_2_x_attn_out(y, q_y, k_x, v_x, attn_map["img_to_vol_attn"], y_cross_out)
        y_self = self.y_2_y_attn_out(y, q_y, k_y, v_y, attn_map["img_to_img_attn"], y_self_out)
        y_new = self.proj_y(self._gate(y, self.gate_y, y_cross, y_self))
        return x_new, y_new, sparse_info


    def _forward_sequence_parallel(self, x, y, im_num, attn_map):
        """This rank's volume tokens ``x`` and image tokens ``y`` (whole blocks,
        as ``ulysses.seq_parallel_token_blocks`` distributed them, with
        ``attn_map["sp"]`` set).  Everything token-local runs on the local
        tokens with all heads: projections, the ResBlock compression of each
        local block (``local_cu_block_include_tokens``), the per-head norms,
        the intra-block window branch and the gates.  The compressed and
        selected branches, which attend across blocks, run on the whole
        sequences for this rank's heads: q / k / v and the compressed keys go
        sequence -> head by one all-to-all each, the branch outputs come back
        head -> sequence (the Ulysses scheme; the reference all-gathers K/V
        instead, models_sparse/utils.py:326-474)."""
        from . import ulysses

        sp = attn_map["sp"]
        W, rank, group = sp.world, sp.rank, sp.group
        Hq, Hkv, D = self.num_q_heads, self.num_kv_heads, self.head_dim
        if Hkv % W:
            raise ValueError(f"sequence parallelism needs the kv heads ({Hkv}) to split evenly over {W} ranks")
        hp, hkp = Hq // W, Hkv // W
        k0, k1 = rank * hkp, (rank + 1) * hkp
        m_vv, m_vi = attn_map["vol_to_vol_attn"], attn_map["vol_to_img_attn"]
        q_x, k_x_raw, k_x, v_x, q_y, k_y_raw, k_y, v_y = self._projections(x, y)
        # compression of the raw keys / values on local whole blocks, then the per-head norms (the
        # reference's order: In modules first, _normalize_qkv after)
        ck_x2x, cv_x2x = self.x_2_x_attn_in(k_x_raw, v_x, m_vv)
        ck_x2y, cv_x2y = self.x_2_y_attn_in(k_y_raw, v_y, m_vi)
        if not self.oneside:
            m_ii, m_iv = attn_map["img_to_img_attn"], attn_map["img_to_vol_attn"]
            ck_y2y, cv_y2y = self.y_2_y_attn_in(k_y_raw, v_y, m_ii)
            ck_y2x, cv_y2x = self.y_2_x_attn_in(k_x_raw, v_x, m_iv)
            ck_y2y, ck_y2x = self._norm(ck_y2y, Hkv), self._norm(ck_y2x, Hkv)
        ck_x2x, ck_x2y = self._norm(ck_x2x, Hkv), self._norm(ck_x2y, Hkv)

        def to_heads(t, plan, heads):  # [n_local, heads*D] -> [N, heads/W * D]
            h = ulysses.seq_to_head(t.reshape(t.shape[0], heads, D), plan, group)
            return h.reshape(h.shape[0], -1)

        def to_tokens(t, plan):  # [N, hp*D] -> [n_local, Hq*D]
            return ulysses.head_to_seq(t.reshape(t.shape[0], hp, D), plan, Hq, group).reshape(-1, Hq * D)

        def heads_of(m):  # this rank's kv heads of a map, the whole sequence's block tables
            return {"block_topk": m["block_topk"][k0:k1], "cu_seqblocks": m["cu_seqblocks"],
                    "cu_block_include_tokens": m["cu_block_include_tokens"]}

        mid = SpatialSparseAttentionMid(hidden_dim=hp * D, num_q_heads=hp, num_kv_heads=hkp)
        Nx, Ny = sp.vol.total, sp.img.total
        cu_nx = torch.tensor([0, Nx], dtype=torch.int32, device=x.device)
        cu_ny = torch.tensor([0, Ny], dtype=torch.int32, device=x.device)
        qh_x, kh_x, vh_x = to_heads(q_x, sp.vol, Hq), to_heads(k_x, sp.vol, Hkv), to_heads(v_x, sp.vol, Hkv)
        kh_y, vh_y = to_heads(k_y, sp.img, Hkv), to_heads(v_y, sp.img, Hkv)
        sparse_info = {}
        o, sparse_info["v_2_i"] = mid(qh_x, cu_nx, kh_y, to_heads(ck_x2y, sp.img_blocks, Hkv), vh_y,
                                      to_heads(cv_x2y, sp.img_blocks, Hkv), self.topk_multiimage * im_num,
                                      heads_of(m_vi))
        x_cross_out = {k: to_tokens(t, sp.vol) for k, t in o.items()}
        o, sparse_info["v_2_v"] = mid(qh_x, cu_nx, kh_x, to_heads(ck_x2x, sp.vol_blocks, Hkv), vh_x,
                                      to_heads(cv_x2x, sp.vol_blocks, Hkv), self.topk_volume, heads_of(m_vv))
        x_self_out = {k: to_tokens(t, sp.vol) for k, t in o.items()}
        x_cross = self.x_2_y_attn_out(x, q_x, k_y, v_y, m_vi, x_cross_out)
        x_self = self.x_2_x_attn_out(x, q_x, k_x, v_x, m_vv, x_self_out)  # window: local blocks
        x_new = self.proj_x(self._gate(x, self.gate_x, x_cross, x_self))
        if self.oneside:
            return x_new, sparse_info
        qh_y = to_heads(q_y, sp.img, Hq)
        o, sparse_info["i_2_v"] = mid(qh_y, cu_ny, kh_x, to_heads(ck_y2x, sp.vol_blocks, Hkv), vh_x,
                                      to_heads(cv_y2x, sp.vol_blocks, Hkv), self.topk_volume, heads_of(m_iv))
        y_cross_out = {k: to_tokens(t, sp.img) for k, t in o.items()}
        o, sparse_info["i_2_i"] = mid(qh_y, cu_ny, kh_y, to_heads(ck_y2y, sp.img_blocks, Hkv), vh_y,
                                      to_heads(cv_y2y, sp.img_blocks, Hkv), self.topk_multiimage * im_num,
                                      heads_of(m_ii))
        y_self_out = {k: to_tokens(t, sp.img) for k, t in o.items()}
        y_cross = self.y_2_x_attn_out(y, q_y, k_x, v_x, m_iv, y_cross_out)
        y_self = self.y_2_y_attn_out(y, q_y, k_y, v_y, m_ii, y_self_out)
        y_new = self.proj_y(self._gate(y, self.gate_y, y_cross, y_self))
        return x_new, y_new, sparse_info


class BlockMix(nn.Module):
    def __init__(self, dim, num_q_heads=32, num_kv_heads=2, mlp_ratio=4.0, qkv_bias=False, act_layer=nn.GELU,
                 norm_layer=LayerNorm32, use_weight_norm=False, topk_volume=8, topk_multiimage=2,
                 use_sequence_parallel=False, no_checkpoint_all_gather=False, *, oneside=False, fused_qkv=None):
        super().__init__()
        hidden = int(dim * mlp_ratio)
        self.oneside = oneside
        self.norm = norm_layer(dim, elementwise_affine=False)
        self.crs_attn = CrossAttention(dim, num_q_heads=num_q_heads, num_kv_heads=num_kv_heads, qkv_bias=qkv_bias,
                                       use_weight_norm=use_weight_norm, oneside=oneside, topk_volume=topk_volume,
                                       topk_multiimage=topk_multiimage, use_sequence_parallel=use_sequence_parallel,
                                       no_checkpoint_all_gather=no_checkpoint_all_gather, fused_qkv=fused_qkv)
        self.mlp_x_1 = Mlp(in_features=dim, hidden_features=hidden, act_layer=act_layer,
                           use_weight_norm=use_weight_norm)
        if not oneside:
            self.mlp_y_1 = Mlp(in_features=dim, hidden_features=hidden, act_layer=act_layer,
                               use_weight_norm=use_weight_norm)

    def forward(self, x, cu_seqlens_x, y, cu_seqlens_y, attn_map, im_num):
        x = self.norm(x)
        y = self.norm(y)
        res = self.crs_attn(x, cu_seqlens_x, y, cu_seqlens_y, im_num, attn_map)
        x = self.norm(x + res[0])
        x = x + self.mlp_x_1(x)
        if self.oneside:
            return x, res[1]
        y = self.norm(y + res[1])
        y = y + self.mlp_y_1(y)
        return x, y, res[2]


class BlockMixOneside(BlockMix):
    def __init__(self, dim, num_q_heads=32, num_kv_heads=2, mlp_ratio=4.0, qkv_bias=False, act_layer=nn.GELU,
                 norm_layer=LayerNorm32, use_weight_norm=False, topk_volume=8, topk_multiimage=2,
                 use_sequence_parallel=False, no_checkpoint_all_gather=False, *, fused_qkv=None):
        super().__init__(dim, num_q_heads, num_kv_heads, mlp_ratio, qkv_bias, act_layer, norm_layer, use_weight_norm,
                         topk_volume, topk_multiimage, use_sequence_parallel, no_checkpoint_all_gather,
                         oneside=True, fused_qkv=fused_qkv)


# ---------------------------------------------------------------------------
# The whole volume decoder: embedding, layer loop with skip blocks, upsampler,
# output formatting (models_sparse/voldecoder.py)
# ---------------------------------------------------------------------------


class VolUpsampler(nn.Module):
    """models_sparse/voldecoder.py:18-36: one Linear from the token width to
    ``output_dim * upsample_scale**3`` sub-voxel features (channel-major per
    token, the layout ``prepare_volume_output`` reads)."""

    def __init__(self, upsample_scale, embed_dim=1024, output_dim=32, use_weight_norm=False):
        super().__init__()
        self.output_dim = output_dim
        self.upsample_scale = upsample_scale
        self.dconv3d = nn.Linear(embed_dim, output_dim * (upsample_scale ** 3))
        if use_weight_norm:
            self.dconv3d = nn.utils.parametrizations.weight_norm(self.dconv3d)

    def forward(self, volume):
        return self.dconv3d(volume)


def batch_cu_seqlens(batch_ids: torch.Tensor, batch_size: int) -> torch.Tensor:
    """int32 [batch_size + 1] offsets of the runs of equal ids in ``batch_ids``
    (grouped by ascending batch id, as the reference assumes), found on the
    device; the reference walks the id gaps with one ``.item()`` per batch
    element (models_sparse/voldecoder.py:318-337)."""
    b = batch_ids.to(torch.int64).contiguous()
    probe = torch.arange(batch_size + 1, device=b.device, dtype=torch.int64)
    return torch.searchsorted(b, probe).to(torch.int32)


class VolTransformer(nn.Module):
    """models_sparse/voldecoder.py:39-424 over this package's decoder blocks.

    Same constructor arguments, parameter names (``pos_embed`` or
    ``pos_embed_{x,y,z}``, ``cross_blocks``, ``skip_blocks``,
    ``skip_fuse_prior_imfeats``, ``fuse_prior_*``, ``fuse_pred_volfeat``,
    ``norm``, ``upsampler.dconv3d``), initialisation rule and forward
    signature, so the reference's checkpoints load and its callers run
    unchanged.  Differences inside: the batch offsets are found on the device
    (``batch_cu_seqlens``) instead of one host read per batch element; the
    ``fuse_all_layers`` output gate ``x * g[:, :C] + prior * g[:, C:]`` is the
    fused two-branch ``gate_merge``; ``prepare_volume_output`` is the one-call
    ``lsrm_prepare_volume_output``; under ``use_sequence_parallel`` the token
    distribution and the final collect are ``ulysses.seq_parallel_token_blocks``
    and the blocks exchange heads (Ulysses) instead of all-gathering K/V."""

    def __init__(self, vol_res=64, upsample_scale=4, embed_dim=1024, output_dim=32, depth=24, num_q_heads=32,
                 num_kv_heads=2, mlp_ratio=4.0, qkv_bias=False, cp_freq=1, use_weight_norm=False,
                 skip_links=(17, 11, 4), topk_volume=8, topk_multiimage=2, use_decomposed_embed=False,
                 use_sequence_parallel=False, no_checkpoint_all_gather=False, fuse_all_layers=False, *,
                 fused_qkv=None):
        super().__init__()
        import math

        self.topk_multiimage = topk_multiimage
        self.topk_volume = topk_volume
        self.depth = depth
        self.embed_dim = embed_dim
        self.vol_res = vol_res
        self.upsample_scale = upsample_scale
        self.output_dim = output_dim
        self.num_token = vol_res * vol_res * vol_res
        self.fuse_all_layers = fuse_all_layers
        self.use_decomposed_embed = use_decomposed_embed
        self.use_sequence_parallel = use_sequence_parallel
        self.no_checkpoint_all_gather = no_checkpoint_all_gather
        scale = 1.0 / math.sqrt(float(embed_dim))
        if use_decomposed_embed:  # one table per axis, concatenated z | y | x
            self.embed_dim_z = embed_dim // 3
            self.embed_dim_x = (embed_dim - self.embed_dim_z) // 2
            self.embed_dim_y = embed_dim - self.embed_dim_z - self.embed_dim_x
            self.pos_embed_x = nn.Parameter(torch.randn(1, vol_res, self.embed_dim_x) * scale)
            self.pos_embed_y = nn.Parameter(torch.randn(1, vol_res, self.embed_dim_y) * scale)
            self.pos_embed_z = nn.Parameter(torch.randn(1, vol_res, self.embed_dim_z) * scale)
        else:
            self.pos_embed = nn.Parameter(torch.randn(1, self.num_token, embed_dim) * scale)
        blk_kw = dict(num_q_heads=num_q_heads, num_kv_heads=num_kv_heads, mlp_ratio=mlp_ratio, qkv_bias=qkv_bias,
                      norm_layer=LayerNorm32, use_weight_norm=use_weight_norm, topk_volume=topk_volume,
                      topk_multiimage=topk_multiimage, use_sequence_parallel=use_sequence_parallel,
                      no_checkpoint_all_gather=no_checkpoint_all_gather, fused_qkv=fused_qkv)
        fuse_imfeat_ratio = len(skip_links) + 1
        self.fuse_prior_volfeats = nn.ModuleList(
            [nn.Linear(embed_dim, embed_dim, bias=False) for _ in range(depth)] if fuse_all_layers else [])
        self.fuse_prior_imfeats = nn.ModuleList(
            [nn.Linear(embed_dim * fuse_imfeat_ratio, embed_dim, bias=False) for _ in range(depth)]
            if fuse_all_layers else [])
        self.cross_blocks = nn.ModuleList([BlockMix(dim=embed_dim, **blk_kw) for _ in range(depth)])
        self.skip_links = skip_links
        skip_vol, skip_im = [], []
        for n in range(len(skip_links)):
            if fuse_all_layers:
                skip_vol.append(nn.Linear(embed_dim, embed_dim, bias=False))
                skip_im.append(nn.Linear(embed_dim * (fuse_imfeat_ratio + 1), embed_dim, bias=False))
            elif n == 0:
                skip_im.append(nn.Linear(embed_dim, embed_dim, bias=False))
        self.skip_fuse_prior_volfeats = nn.ModuleList(skip_vol)
        self.skip_fuse_prior_imfeats = nn.ModuleList(skip_im)
        self.skip_blocks = nn.ModuleList([BlockMixOneside(dim=embed_dim, **blk_kw) for _ in skip_links])
        if fuse_all_layers:
            self.fuse_pred_volfeat = nn.Linear(embed_dim, 2 * embed_dim, bias=False)
        self.norm = LayerNorm32(embed_dim)
        self.upsampler = VolUpsampler(upsample_scale=upsample_scale, embed_dim=embed_dim, output_dim=output_dim,
                                      use_weight_norm=use_weight_norm)
        self.apply(self._init_weights)
        self.cp_freq = int(cp_freq)

    @staticmethod
    def _init_weights(m):
        """The reference's rule (voldecoder.py:183-193): Linear weights from a
        normal of std 0.02 truncated to [-2, 2], biases 0; LayerNorm weight 1,
        bias 0."""
        if isinstance(m, nn.Linear):
            nn.init.trunc_normal_(m.weight, std=0.02, a=-2.0, b=2.0)
            if m.bias is not None:
                nn.init.constant_(m.bias, 0)
        elif isinstance(m, nn.LayerNorm):
            if m.bias is not None:
                nn.init.constant_(m.bias, 0)
            if m.weight is not None:
                nn.init.constant_(m.weight, 1.0)

    def prepare_volume_output(self, volume, volume_index, prior_volume):
        from .volume import prepare_volume_output

        return prepare_volume_output(volume, volume_index, prior_volume, self.output_dim, self.upsample_scale,
                                     self.vol_res)

    def embed(self, volume_index, mask_volume, volume_coords_idx, batch_size, dtype):
        """Position embedding of the voxel tokens (voldecoder.py:285-299):
        three per-axis tables gathered by the (z, y, x) columns of
        ``volume_index`` and concatenated, or the full table's rows of the
        voxels ``mask_volume`` keeps (a flat mask over ``batch_size`` copies
        of the volume), reordered by ``volume_coords_idx``.  The gathers read
        fp32 copies of the tables, so the backward's scatter-add (many tokens
        per table row) accumulates in fp32 whatever the parameters' dtype; the
        values are the tables' own."""
        if self.use_decomposed_embed:
            vi = volume_index.long()
            return torch.cat([self.pos_embed_z[0].float().index_select(0, vi[:, 1]),
                              self.pos_embed_y[0].float().index_select(0, vi[:, 2]),
                              self.pos_embed_x[0].float().index_select(0, vi[:, 3])], dim=-1).to(dtype)
        rows = torch.nonzero(mask_volume.reshape(-1)).squeeze(1)
        rows = rows.index_select(0, volume_coords_idx.reshape(-1).long()) % self.num_token
        return self.pos_embed[0].float().index_select(0, rows).to(dtype)

    def _run(self, blk, *args):
        import torch.utils.checkpoint as cp

        return cp.checkpoint(blk, *args, use_reentrant=False)

    def forward(self, y, prior_imfeat_list, image_index, prior_volfeat, mask_volume, volume_index, prior_volume,
                volume_coords_idx, attn_map, im_num):
        batch_size = int(image_index[:, 0].max().item()) + 1
        x = self.embed(volume_index, mask_volume, volume_coords_idx, batch_size, y.dtype)
        prior_imfeat = torch.cat(prior_imfeat_list, dim=1)
        if self.use_sequence_parallel:
            from .ulysses import seq_parallel_token_blocks

            vol = [x] if prior_volfeat is None else [x, prior_volfeat]
            vol, (y, prior_imfeat), cu_vol, cu_img, attn_map = seq_parallel_token_blocks(
                vol, [y, prior_imfeat], attn_map, mode="distribute")
            x, prior_volfeat = vol[0], (vol[1] if len(vol) > 1 else None)
        else:
            cu_vol = batch_cu_seqlens(volume_index[:, 0], batch_size)
            cu_img = batch_cu_seqlens(image_index[:, 0], batch_size)
        y_list, sparse_info_arr = [], []
        for idx, blk in enumerate(self.cross_blocks):
            if self.fuse_all_layers:
                x = x + self.fuse_prior_volfeats[idx](prior_volfeat)
                y = y + self.fuse_prior_imfeats[idx](prior_imfeat)
            args = (x, cu_vol, y, cu_img, attn_map, im_num)
            if self.cp_freq > 0 and idx % self.cp_freq == 0:
                x, y, sparse_info = self._run(blk, *args)
            else:
                x, y, sparse_info = blk(*args)
            if idx in self.skip_links:
                y_list.insert(0, y)
            sparse_info_arr.append(sparse_info)
        y_list.insert(0, y)
        for n, blk in enumerate(self.skip_blocks):
            if self.fuse_all_layers:
                x = x + self.skip_fuse_prior_volfeats[n](prior_volfeat)
                y = y_list[n + 1] + self.skip_fuse_prior_imfeats[n](torch.cat([y_list[0], prior_imfeat], dim=1))
            elif n == 0:
                y = y_list[n + 1] + self.skip_fuse_prior_imfeats[n](y_list[0])
            else:
                y = y_list[n + 1]
            args = (x, cu_vol, y, cu_img, attn_map, im_num)
            if self.cp_freq > 0 and n % self.cp_freq == 0:
                x, sparse_info = self._run(blk, *args)
            else:
                x, sparse_info = blk(*args)
            sparse_info_arr.append(sparse_info)
        if self.fuse_all_layers:  # x * g[:, :C] + prior * g[:, C:], g = sigmoid(fuse_pred_volfeat(x)), fused
            x = F.gate_merge(self.fuse_pred_volfeat(x), [x, prior_volfeat.to(x.dtype)])
        x = self.norm(x)
        volume = self.upsampler(x)
        if self.use_sequence_parallel:
            from .ulysses import seq_parallel_token_blocks

            (volume,), _, _, _, _ = seq_parallel_token_blocks([volume], [], attn_map, mode="collect")
        return self.prepare_volume_output(volume, volume_index, prior_volume), sparse_info_arr
