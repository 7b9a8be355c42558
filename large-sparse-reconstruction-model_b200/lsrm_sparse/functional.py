"""Autograd functions over the CUDA ops (every forward and backward runs in
liblsrm_sparse.so; torch supplies memory, streams and the Linear GEMMs)."""

from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import ops


def _meta(cu_seqlens_q, cu_seqlens_k, cu_seqblocks, cu_block_include_tokens):
    return ops.Meta(cu_seqlens_q, cu_seqlens_k, cu_seqblocks, cu_block_include_tokens)


class SelectAttnFn(torch.autograd.Function):
    """Selected-block attention (native_sparse_attend, kvcentric.py:1281-1371)."""

    @staticmethod
    def forward(ctx, q, k, v, block_topk, meta, softmax_scale, cu_query_blocks):
        out, lse, ws = ops.select_attn_fwd(q, k, v, block_topk, meta, softmax_scale, cu_query_blocks)
        ctx.save_for_backward(q, k, v, out, lse, block_topk)
        ctx.meta = meta
        ctx.scale = softmax_scale
        ctx.cqb = cu_query_blocks
        ctx.ws = ws
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, dout, _dlse):
        q, k, v, out, lse, block_topk = ctx.saved_tensors
        dq, dk, dv = ops.select_attn_bwd(q, k, v, out, lse, dout, block_topk, ctx.meta, ctx.scale, ctx.cqb,
                                         workspace=ctx.ws)
        ctx.ws = None
        return dq, dk, dv, None, None, None, None


class DenseAttnFn(torch.autograd.Function):
    """Compressed / intra-block / sliding-window attention."""

    @staticmethod
    def forward(ctx, q, k, v, meta, mode, window, softmax_scale):
        out, lse = ops.dense_attn_fwd(q, k, v, meta, mode, window, softmax_scale)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.meta, ctx.mode, ctx.window, ctx.scale = meta, mode, window, softmax_scale
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, dout, _dlse):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = ops.dense_attn_bwd(q, k, v, out, lse, dout, ctx.meta, ctx.mode, ctx.window, ctx.scale)
        return dq, dk, dv, None, None, None, None


class BlockMeanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cu_block_include_tokens):
        ctx.save_for_backward(cu_block_include_tokens)
        ctx.n = x.shape[0]
        return ops.block_mean_fwd(x, cu_block_include_tokens)

    @staticmethod
    def backward(ctx, dout):
        (cu,) = ctx.saved_tensors
        return ops.block_mean_bwd(dout, cu, ctx.n), None


class ResNormMeanFn(torch.autograd.Function):
    """block_mean(LayerNorm_fp32(x + h)) — the SparseResBlock epilogue fused
    with the compression mean.  Gradient flows to x and h equally."""

    @staticmethod
    def forward(ctx, x, h, cu_block_include_tokens, eps):
        out, _, mean, rstd = ops.resnorm_mean_fwd(x, h, cu_block_include_tokens, eps)
        ctx.save_for_backward(x, h, cu_block_include_tokens, mean, rstd)
        return out

    @staticmethod
    def backward(ctx, dout):
        x, h, cu, mean, rstd = ctx.saved_tensors
        dr = ops.resnorm_mean_bwd(x, h, cu, mean, rstd, dout)
        return dr, dr, None, None


class GateMergeFn(torch.autograd.Function):
    """sum_i sigmoid(z_i) * branch_i (per channel or per head)."""

    @staticmethod
    def forward(ctx, z, per_head, head_dim, *branches):
        ctx.save_for_backward(z, *branches)
        ctx.per_head, ctx.head_dim = per_head, head_dim
        return ops.gate_merge_fwd(z, branches, per_head, head_dim)

    @staticmethod
    def backward(ctx, dout):
        z, *branches = ctx.saved_tensors
        dz, dbr = ops.gate_merge_bwd(z, branches, dout, ctx.per_head, ctx.head_dim)
        return (dz, None, None, *dbr)


def select_attention(q, k, v, block_topk, meta, softmax_scale=None, cu_query_blocks=None):
    return SelectAttnFn.apply(q, k, v, block_topk, meta, softmax_scale, cu_query_blocks)


def dense_attention(q, k, v, meta, mode, window=0, softmax_scale=None):
    return DenseAttnFn.apply(q, k, v, meta, mode, window, softmax_scale)


def block_mean(x, cu_block_include_tokens):
    return BlockMeanFn.apply(x, cu_block_include_tokens)


def resnorm_mean(x, h, cu_block_include_tokens, eps=1e-5):
    return ResNormMeanFn.apply(x, h, cu_block_include_tokens, eps)


def gate_merge(z, branches: Sequence[torch.Tensor], per_head=False, head_dim=0):
    return GateMergeFn.apply(z, per_head, head_dim, *branches)


def three_branch_attention(q, k, v, cu_blk, topk: int, window: int, gate_logits, *, compress=None,
                           per_head: bool = True, softmax_scale=None, capture=None):
    """The full native-sparse-attention op on one whole sequence, as
    SpatialSparseAttentionIn / Mid / Out run it (spatial_sparse_attention.py:
    16-270) with the BASELINE extensions on: compression of K/V per block,
    compressed attention (natural-log LSE), per-query-block top-k selection
    with the query block's own block forced (block_score.py:16-98 summed over
    the query block's tokens), selected-block attention, sliding-window
    attention (|i - j| <= window // 2) and the sigmoid-gated merge.

    q [N, H, D], k/v [N, Hkv, D] (one sequence, blocks given by ``cu_blk``,
    which are also the query blocks); ``gate_logits`` is a tensor [N, 3*H]
    (per head) or [N, 3*H*D] (per channel), or a callable returning it (it is
    called after the attention branches are enqueued, so a caller can wait for
    the gate input there).  ``compress(k2d, v2d, cu_blk) -> (ck, cv)`` replaces
    the block mean (e.g. the ResBlock compression); it returns [nb, Hkv*D].
    Returns the merged output [N, H*D].  Metadata is built on the device, so
    the call never synchronises the host.  ``capture`` (a dict) receives the
    selection, the compressed keys / values, the compressed LSE, the merged
    output and, after the backward, the gradients of the compressed keys /
    values (``dck``, ``dcv``)."""
    N, H, D = q.shape
    Hkv = k.shape[1]
    nb = cu_blk.numel() - 1
    dev = q.device
    two = torch.arange(2, dtype=torch.int32, device=dev)
    cu_seq = two * N
    meta = ops.Meta(cu_seq, cu_seq, two * nb, cu_blk)
    meta_c = ops.Meta(cu_seq, cu_seq, two * nb, torch.arange(nb + 1, dtype=torch.int32, device=dev))
    k2, v2 = k.reshape(N, Hkv * D), v.reshape(N, Hkv * D)
    if compress is None:
        ck, cv = block_mean(k2, cu_blk), block_mean(v2, cu_blk)
    else:
        ck, cv = compress(k2, v2, cu_blk)
    ck, cv = ck.view(nb, Hkv, D), cv.view(nb, Hkv, D)
    if capture is not None and ck.requires_grad:  # the gradients reaching the compression
        ck.register_hook(lambda g: capture.__setitem__("dck", g))
        cv.register_hook(lambda g: capture.__setitem__("dcv", g))
    o_c, lse = dense_attention(q, ck, cv, meta_c, ops.DENSE_COMPRESSED, 0, softmax_scale)
    with torch.no_grad():
        bt = ops.block_topk(q, ck, lse, topk, meta_c, cu_query_blocks=cu_blk, force_self=True,
                            sm_scale=softmax_scale)
    o_s, _ = select_attention(q, k, v, bt, meta, softmax_scale, cu_blk)
    o_w, _ = dense_attention(q, k, v, meta, ops.DENSE_SLIDING, window, softmax_scale)
    z = gate_logits() if callable(gate_logits) else gate_logits
    out = gate_merge(z, [o_c.view(N, -1), o_s.view(N, -1), o_w.view(N, -1)], per_head=per_head, head_dim=D)
    if capture is not None:
        capture.update(block_topk=bt, ck=ck.detach(), cv=cv.detach(), lse=lse, out=out.detach())
    return out


class QkvNormFn(torch.autograd.Function):
    """Stacked projections with the per-head LayerNorm32 in the GEMM's
    epilogue (lsrm_qkv_norm_fwd); the backward turns the outputs' gradients
    into the pre-norm gradient (lsrm_qkv_norm_bwd), then two GEMMs give the
    input and weight gradients."""

    @staticmethod
    def forward(ctx, x2, w, b, spec, head_dim, eps):
        ctx.set_materialize_grads(False)
        outs, rstd = ops.qkv_norm_fwd(x2, w, b, spec, head_dim, eps)
        norms = [on for _, on in outs if on is not None]
        ctx.spec, ctx.head_dim, ctx.has_b = spec, head_dim, b is not None
        ctx.save_for_backward(x2, w, rstd, *norms)
        return tuple(t for pair in outs for t in pair if t is not None)

    @staticmethod
    def backward(ctx, *grads):
        x2, w, rstd, *norms = ctx.saved_tensors
        g_it, n_it = iter(grads), iter(norms)
        segs = []
        for cols, raw, norm in ctx.spec:
            go = next(g_it) if raw else None
            gn = next(g_it) if norm else None
            on = next(n_it) if norm else None
            segs.append((cols, on, go, gn))
        dpre = ops.qkv_norm_bwd(x2.shape[0], w.shape[0], ctx.head_dim, segs, rstd, x2.device, x2.dtype)
        dx = dpre @ w if ctx.needs_input_grad[0] else None
        dw = dpre.t() @ x2 if ctx.needs_input_grad[1] else None
        db = dpre.float().sum(0).to(w.dtype) if ctx.has_b and ctx.needs_input_grad[2] else None
        return dx, dw, db, None, None, None


def qkv_norm(x, linears, outputs, head_dim: int, eps: float = 1e-5):
    """The Linears of ``linears`` (all over x's last dim, bf16) as one GEMM
    with the per-head LayerNorm32 of their outputs fused in its epilogue.
    ``outputs`` gives per Linear (raw, norm): whether its plain output and /
    or its per-head LayerNorm (non-affine over ``head_dim``) is wanted.
    Returns per Linear a (raw, norm) pair with None for what was not asked.
    The Linears must all have biases or none."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    w = torch.cat([lin.weight for lin in linears], 0)
    biases = [lin.bias for lin in linears]
    if any(b is not None for b in biases) and not all(b is not None for b in biases):
        raise ValueError("qkv_norm: the Linears must all have biases or none")
    b = torch.cat(biases) if biases[0] is not None else None
    spec = tuple((lin.weight.shape[0], bool(raw), bool(norm)) for lin, (raw, norm) in zip(linears, outputs))
    flat = iter(QkvNormFn.apply(x2, w, b, spec, int(head_dim), float(eps)))
    res = []
    for cols, raw, norm in spec:
        r = next(flat).reshape(*lead, cols) if raw else None
        n = next(flat).reshape(*lead, cols) if norm else None
        res.append((r, n))
    return res
