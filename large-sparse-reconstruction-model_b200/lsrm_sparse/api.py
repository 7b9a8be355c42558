"""The reference's op-level API (``sparse.ops``), same names, argument order
and return conventions, backed by the sm_100a kernels.

* ``get_block_score``            — sparse/ops/block_score.py:16-98
* ``spatial_selection_attention`` — sparse/ops/triton_native_sparse_attention.py:17-41
* ``native_sparse_attend``       — sparse/ops/triton_native_sparse_attention_impl_kvcentric.py:1382-1435
* ``set_variant``                — kvcentric.py:1275 (accepted, no effect)
* ``sparse_window_attention``    — sparse/ops/block_window_attention.py:14-31
* ``compressed_attention``       — the flash_attn_varlen_func call of the
                                   compressed branch (spatial_sparse_attention.py:121-143)

Differences from the reference, all documented in the repository's design
notes: ties in top-k go to the lowest block id; a block listed twice for one
query raises (the reference attends it twice); selection entries outside
``[0, blocks_in_sequence)`` are skipped wherever they appear.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import functional as F
from . import ops

_LSE_CHECK = False


def _raise_on_device_errors():
    if _LSE_CHECK:
        e = ops.read_errors()
        if e:
            raise ops._lib.LsrmError(f"device error bits 0x{e:x}")


def get_block_score(q, compressed_k, lse, topk, cu_seqlens_q, compressed_cu_seqlens, seqlens_q=None,
                    compressed_seqlens=None, sm_scale=None, *, cu_query_blocks=None, force_self_block=False):
    """Top-k compressed blocks per query token ([Hkv, Nq, topk] int32,
    ascending, -1 padded).  With ``cu_query_blocks`` (extension) one selection
    per query block: [Hkv, n_query_blocks, topk]."""
    nb = compressed_k.shape[0]
    dummy_blocks = torch.arange(nb + 1, dtype=torch.int32, device=q.device)
    meta = ops.Meta(cu_seqlens_q, cu_seqlens_q, compressed_cu_seqlens, dummy_blocks)
    with torch.no_grad():
        return ops.block_topk(q, compressed_k, lse, int(topk), meta, cu_query_blocks=cu_query_blocks,
                              force_self=force_self_block, sm_scale=sm_scale)


def native_sparse_attend(q, k, v, topk_idx, cu_seqblocks, cu_block_include_tokens, cu_seqlens_q, cu_seqlens_k,
                         softmax_scale: Optional[float] = None, return_lse: bool = False, *, cu_query_blocks=None):
    """Variable-block selected attention; LSE (optional) is log2-based
    [Hq, Nq] fp32 as in the reference."""
    assert q.dtype in (torch.float16, torch.bfloat16), "Only fp16/bf16 supported"
    assert q.dtype == k.dtype == v.dtype
    assert topk_idx.dtype == torch.int32
    assert cu_seqlens_q.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    meta = ops.Meta(cu_seqlens_q, cu_seqlens_k, cu_seqblocks, cu_block_include_tokens)
    out, lse = F.select_attention(q, k, v, topk_idx, meta, softmax_scale, cu_query_blocks)
    _raise_on_device_errors()
    return (out, lse) if return_lse else out


def spatial_selection_attention(q, k, v, block_topk, cu_seqblocks, cu_block_include_tokens, cu_seqlens_q,
                                cu_seqlens_k, seqlens_q=None, seqlens_k=None, softmax_scale=None):
    """Drop-in replacement with the original function signature."""
    return native_sparse_attend(q, k, v, block_topk, cu_seqblocks, cu_block_include_tokens, cu_seqlens_q,
                                cu_seqlens_k, softmax_scale=softmax_scale)


def set_variant(variant: str):
    """Accepted for compatibility; the backward has a single deterministic
    implementation."""
    return None


def sparse_window_attention(q, k, v, cu_block_include_tokens, softmax_scale=None):
    """Self-attention independently within each block."""
    n = q.shape[0]
    two = torch.arange(2, dtype=torch.int32, device=q.device)  # built on the device: no host synchronisation
    cu_seq = two * n
    cu_sb = two * (cu_block_include_tokens.numel() - 1)
    meta = ops.Meta(cu_seq, cu_seq, cu_sb, cu_block_include_tokens)
    out, _ = F.dense_attention(q.contiguous(), k.contiguous(), v.contiguous(), meta, ops.DENSE_INTRA_BLOCK, 0,
                               softmax_scale)
    return out


def sliding_window_attention(q, k, v, cu_seqlens, window: int, softmax_scale=None):
    """Extension: band attention |i - j| <= window // 2 inside each sequence."""
    nb = cu_seqlens.numel() - 1
    cu_blocks = cu_seqlens
    cu_sb = torch.arange(nb + 1, dtype=torch.int32, device=q.device)
    meta = ops.Meta(cu_seqlens, cu_seqlens, cu_sb, cu_blocks)
    out, _ = F.dense_attention(q.contiguous(), k.contiguous(), v.contiguous(), meta, ops.DENSE_SLIDING, int(window),
                               softmax_scale)
    return out


def compressed_attention(q, compressed_k, compressed_v, cu_seqlens_q, compressed_cu_seqlens, return_lse=False,
                         softmax_scale=None):
    """Every query attends to all compressed blocks of its sequence; LSE is
    natural-log [Hq, Nq] (flash-attn's convention)."""
    nb = compressed_k.shape[0]
    dummy_blocks = torch.arange(nb + 1, dtype=torch.int32, device=q.device)
    meta = ops.Meta(cu_seqlens_q, cu_seqlens_q, compressed_cu_seqlens, dummy_blocks)
    out, lse = F.dense_attention(q.contiguous(), compressed_k.contiguous(), compressed_v.contiguous(), meta,
                                 ops.DENSE_COMPRESSED, 0, softmax_scale)
    return (out, lse) if return_lse else out
