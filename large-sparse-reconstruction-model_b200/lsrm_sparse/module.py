"""The reference's nn.Module API (``sparse.module`` / ``sparse``), same
constructor arguments, forward signatures, return values and parameter names
(so reference checkpoints load):

* ``SparseResBlock``            — sparse/module/residual_block.py:16-34
* ``SpatialSparseAttentionIn``  — sparse/module/spatial_sparse_attention.py:16-67
* ``SpatialSparseAttentionMid`` — :70-193
* ``SpatialSparseAttentionOut`` — :196-270

Keyword-only extensions (off by default, i.e. reference behaviour):
``compression="mean"`` (block mean without the ResBlock), per-query-block
selection (``attn_map["cu_query_blocks"]``, ``attn_map["force_self_block"]``),
``window=W`` (sliding band instead of the intra-block window) and
``gate="per_head"``.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import api
from . import functional as F


class LayerNorm32(nn.LayerNorm):
    """residual_block.py:11-13: LayerNorm evaluated in fp32, cast back.  An
    affine one also evaluates its weight and bias in fp32, so a module cast to
    bf16 as a whole (``.to(torch.bfloat16)``) still runs (the reference's
    fp32 LayerNorm rejects bf16 parameters); with fp32 parameters the result
    is the reference's."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = None if self.weight is None else self.weight.float()
        b = None if self.bias is None else self.bias.float()
        return nn.functional.layer_norm(x.float(), self.normalized_shape, w, b, self.eps).type(x.dtype)


class SparseResBlock(nn.Module):
    """LN_fp32(x + W2·SiLU(W1·x + b1) + b2), non-affine LayerNorm."""

    def __init__(self, channels: int):
        super().__init__()
        self.channels = channels
        self.act_layers = nn.Sequential(
            nn.Linear(self.channels, self.channels),
            nn.SiLU(),
            nn.Linear(self.channels, self.channels),
        )
        self.norm = LayerNorm32(self.channels, elementwise_affine=False)

    def forward(self, x):
        h = self.act_layers(x)
        return self.norm(x + h)

    def forward_block_mean(self, x, cu_block_include_tokens):
        """block_mean(forward(x)) with the residual, LayerNorm and mean fused
        into one CUDA pass (the two Linear layers run as cuBLAS GEMMs)."""
        h = self.act_layers(x)
        return F.resnorm_mean(x, h, cu_block_include_tokens, self.norm.eps)


class SpatialSparseAttentionIn(torch.nn.Module):
    def __init__(self, head_dim: int, num_kv_heads: int, *, compression: str = "resblock"):
        super().__init__()
        assert compression in ("resblock", "mean")
        self.compression = compression
        if compression == "resblock":
            self.compression_key = SparseResBlock(num_kv_heads * head_dim)
            self.compression_value = SparseResBlock(num_kv_heads * head_dim)

    def sparse3d_compression(self, x, cu_block_include_tokens):
        return F.block_mean(x, cu_block_include_tokens)

    def forward(self, k, v, attn_map):
        cu = attn_map.get("local_cu_block_include_tokens", attn_map["cu_block_include_tokens"])
        if self.compression == "mean":
            return self.sparse3d_compression(k, cu), self.sparse3d_compression(v, cu)
        return (self.compression_key.forward_block_mean(k, cu), self.compression_value.forward_block_mean(v, cu))


class SpatialSparseAttentionMid(torch.nn.Module):
    def __init__(self, hidden_dim: int, num_q_heads: int, num_kv_heads: int, is_window_attn=False):
        super().__init__()
        self.is_window_attn = is_window_attn
        self.hidden_dim = hidden_dim
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = hidden_dim // num_q_heads

    def forward(self, q, cu_seqlens_q, k, compressed_k, v, compressed_v, topk: int, attn_map,
                return_sparse_info=False):
        q = q.view(-1, self.num_q_heads, self.head_dim)
        k = k.view(-1, self.num_kv_heads, self.head_dim)
        v = v.view(-1, self.num_kv_heads, self.head_dim)
        compressed_k = compressed_k.view(-1, self.num_kv_heads, self.head_dim)
        compressed_v = compressed_v.view(-1, self.num_kv_heads, self.head_dim)

        compressed_cu_seqlens = attn_map["cu_seqblocks"]
        cu_seqblocks = attn_map["cu_seqblocks"]
        cu_block_include_tokens = attn_map["cu_block_include_tokens"]
        cu_seqlens_k = cu_block_include_tokens[cu_seqblocks.long()]
        cu_query_blocks = attn_map.get("cu_query_blocks")

        need_lse = attn_map["block_topk"] is None
        compressed_attn_output, lse = api.compressed_attention(
            q, compressed_k, compressed_v, cu_seqlens_q, compressed_cu_seqlens, return_lse=True)

        sparse_info = {}
        if attn_map["block_topk"] is not None:
            block_topk = attn_map["block_topk"]
        else:
            block_topk = api.get_block_score(
                q.detach(), compressed_k.detach(), lse, topk, cu_seqlens_q, compressed_cu_seqlens,
                cu_query_blocks=cu_query_blocks, force_self_block=bool(attn_map.get("force_self_block", False)))
            if return_sparse_info:
                sparse_info["block_topk"] = block_topk
                sparse_info["cu_seqblocks"] = cu_seqblocks
                sparse_info["cu_block_include_tokens"] = cu_block_include_tokens
        del need_lse

        selection_attn_output = api.native_sparse_attend(
            q, k, v, block_topk, cu_seqblocks, cu_block_include_tokens, cu_seqlens_q, cu_seqlens_k,
            cu_query_blocks=cu_query_blocks)

        attn_output = {
            "selection_attn": selection_attn_output.reshape(selection_attn_output.shape[0], -1),
            "compressed_attn": compressed_attn_output.reshape(compressed_attn_output.shape[0], -1),
        }
        return attn_output, sparse_info


class SpatialSparseAttentionOut(torch.nn.Module):
    def __init__(self, hidden_dim: int, num_q_heads: int, num_kv_heads: int, is_window_attn=False, *,
                 window: Optional[int] = None, gate: str = "per_channel"):
        super().__init__()
        assert gate in ("per_channel", "per_head")
        self.hidden_dim = hidden_dim
        self.is_window_attn = is_window_attn
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = hidden_dim // num_q_heads
        self.window = window
        self.gate_mode = gate
        n = 3 if is_window_attn else 2
        width = n * hidden_dim if gate == "per_channel" else n * num_q_heads
        self.gate = torch.nn.Sequential(nn.Linear(hidden_dim, width, bias=False), nn.Sigmoid())

    def forward(self, x, q, k, v, attn_map, attn_output):
        q = q.view(-1, self.num_q_heads, self.head_dim)
        k = k.view(-1, self.num_kv_heads, self.head_dim)
        v = v.view(-1, self.num_kv_heads, self.head_dim)
        branches = [attn_output["compressed_attn"], attn_output["selection_attn"]]
        if self.is_window_attn:
            if self.window is None:
                cu = attn_map.get("local_cu_block_include_tokens", attn_map["cu_block_include_tokens"])
                w = api.sparse_window_attention(q, k, v, cu)
            else:
                w = api.sliding_window_attention(q, k, v, attn_map["cu_seqlens"], self.window)
            branches.append(w.reshape(w.shape[0], -1))
        # gate logits by a cuBLAS GEMM; sigmoid and the weighted sum fused in CUDA
        z = torch.nn.functional.linear(x, self.gate[0].weight)
        return F.gate_merge(z, branches, per_head=self.gate_mode == "per_head", head_dim=self.head_dim)


class CrossSelfGate(torch.nn.Module):
    """The closing step of CrossAttention for one token set
    (models_sparse/utils.py:131-132, 559-570):
    ``proj_x(x_cross * g[:, :dim] + x_self * g[:, dim:])`` with
    ``g = sigmoid(gate_x(x))``.  The sigmoid and the two-way merge run as one
    fused pass (``lsrm_gate_merge_fwd/bwd`` with two per-channel branches, fp32
    inside); the two Linears are library GEMMs.  Parameter names follow the
    reference (``gate_x.0``, ``proj_x``) so its state dict loads unchanged;
    ``gate_x`` holds only the Linear because its Sigmoid is fused."""

    def __init__(self, dim: int):
        super().__init__()
        self.dim = dim
        self.gate_x = nn.Sequential(nn.Linear(dim, 2 * dim))
        self.proj_x = nn.Linear(dim, dim)

    def forward(self, x: torch.Tensor, x_cross: torch.Tensor, x_self: torch.Tensor) -> torch.Tensor:
        logits = self.gate_x(x)
        return self.proj_x(F.gate_merge(logits, [x_cross, x_self]))
