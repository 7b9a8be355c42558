"""The sparse decoder's building blocks (models_sparse/utils.py), assembled
from this package's modules on one GPU (the reference's non-sequence-parallel
path):

* ``Mlp``             — models_sparse/utils.py:80-106
* ``CrossAttention``  — :108-574: volume tokens x and image tokens y, each
  attending to both sets through SpatialSparseAttentionIn / Mid / Out
* ``BlockMix``        — :575-640, ``BlockMixOneside`` — :643-705

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
                 topk_volume=8, topk_multiimage=2, use_sequence_parallel=False, no_checkpoint_all_gather=False):
        super().__init__()
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
        q_x, k_x, v_x = self.q_proj_x(x), self.k_proj_x(x), self.v_proj_x(x)
        k_y, v_y = self.k_proj_y(y), self.v_proj_y(y)
        if not self.oneside:
            q_y = self.q_proj_y(y)
        ck_x2x, cv_x2x = self.x_2_x_attn_in(k_x, v_x, attn_map["vol_to_vol_attn"])
        ck_x2y, cv_x2y = self.x_2_y_attn_in(k_y, v_y, attn_map["vol_to_img_attn"])
        if not self.oneside:
            ck_y2y, cv_y2y = self.y_2_y_attn_in(k_y, v_y, attn_map["img_to_img_attn"])
            ck_y2x, cv_y2x = self.y_2_x_attn_in(k_x, v_x, attn_map["img_to_vol_attn"])
        Hq, Hkv = self.num_q_heads, self.num_kv_heads
        q_x, k_x, ck_x2x = self._norm(q_x, Hq), self._norm(k_x, Hkv), self._norm(ck_x2x, Hkv)
        k_y, ck_x2y = self._norm(k_y, Hkv), self._norm(ck_x2y, Hkv)
        if not self.oneside:
            q_y, ck_y2y, ck_y2x = self._norm(q_y, Hq), self._norm(ck_y2y, Hkv), self._norm(ck_y2x, Hkv)

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
        q_x, k_x, v_x = self.q_proj_x(x), self.k_proj_x(x), self.v_proj_x(x)
        k_y, v_y = self.k_proj_y(y), self.v_proj_y(y)
        # compression of the raw keys / values on local whole blocks, then the per-head norms (the
        # reference's order: In modules first, _normalize_qkv after)
        ck_x2x, cv_x2x = self.x_2_x_attn_in(k_x, v_x, m_vv)
        ck_x2y, cv_x2y = self.x_2_y_attn_in(k_y, v_y, m_vi)
        if not self.oneside:
            m_ii, m_iv = attn_map["img_to_img_attn"], attn_map["img_to_vol_attn"]
            ck_y2y, cv_y2y = self.y_2_y_attn_in(k_y, v_y, m_ii)
            ck_y2x, cv_y2x = self.y_2_x_attn_in(k_x, v_x, m_iv)
            q_y = self._norm(self.q_proj_y(y), Hq)
            ck_y2y, ck_y2x = self._norm(ck_y2y, Hkv), self._norm(ck_y2x, Hkv)
        q_x, k_x, ck_x2x = self._norm(q_x, Hq), self._norm(k_x, Hkv), self._norm(ck_x2x, Hkv)
        k_y, ck_x2y = self._norm(k_y, Hkv), self._norm(ck_x2y, Hkv)

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
                 use_sequence_parallel=False, no_checkpoint_all_gather=False, *, oneside=False):
        super().__init__()
        hidden = int(dim * mlp_ratio)
        self.oneside = oneside
        self.norm = norm_layer(dim, elementwise_affine=False)
        self.crs_attn = CrossAttention(dim, num_q_heads=num_q_heads, num_kv_heads=num_kv_heads, qkv_bias=qkv_bias,
                                       use_weight_norm=use_weight_norm, oneside=oneside, topk_volume=topk_volume,
                                       topk_multiimage=topk_multiimage, use_sequence_parallel=use_sequence_parallel,
                                       no_checkpoint_all_gather=no_checkpoint_all_gather)
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
                 use_sequence_parallel=False, no_checkpoint_all_gather=False):
        super().__init__(dim, num_q_heads, num_kv_heads, mlp_ratio, qkv_bias, act_layer, norm_layer, use_weight_norm,
                         topk_volume, topk_multiimage, use_sequence_parallel, no_checkpoint_all_gather,
                         oneside=True)
