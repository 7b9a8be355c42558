"""Seeded random problem generators shared by the tests."""

from __future__ import annotations

import numpy as np
import torch


def cu(lengths):
    return torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32)


def random_problem(seed, seq_block_lens, Hq, Hkv, D, topk, dtype=torch.bfloat16, pad_frac=0.0, qblock=False,
                   scale=1.0):
    """Random q/k/v + per-token (or per-query-block) unique selections.

    seq_block_lens: list (per sequence) of block lengths.  Query blocks, when
    used, are the KV blocks themselves (self attention).
    """
    g = torch.Generator().manual_seed(seed)
    lens = [l for s in seq_block_lens for l in s]
    cu_blk = cu(lens)
    cu_seqblocks = cu([len(s) for s in seq_block_lens])
    cu_seqlens = cu([sum(s) for s in seq_block_lens])
    N = int(cu_seqlens[-1])
    q = (torch.randn(N, Hq, D, generator=g) * scale).to(dtype)
    k = (torch.randn(N, Hkv, D, generator=g) * scale).to(dtype)
    v = torch.randn(N, Hkv, D, generator=g).to(dtype)
    rows = len(lens) if qblock else N
    topk_t = torch.full((Hkv, rows, topk), -1, dtype=torch.int32)
    for b, blocks in enumerate(seq_block_lens):
        nb = len(blocks)
        if qblock:
            r0, r1 = int(cu_seqblocks[b]), int(cu_seqblocks[b + 1])
        else:
            r0, r1 = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        kk = min(topk, nb)
        for h in range(Hkv):
            for r in range(r0, r1):
                sel = torch.randperm(nb, generator=g)[:kk].sort().values.to(torch.int32)
                if pad_frac > 0 and kk > 1 and torch.rand(1, generator=g).item() < pad_frac:
                    sel = sel[: kk - 1]
                topk_t[h, r, : sel.numel()] = sel
    return dict(q=q, k=k, v=v, block_topk=topk_t, cu_blk=cu_blk, cu_seqblocks=cu_seqblocks, cu_seqlens=cu_seqlens,
                N=N)


def expand_qblock_selection(block_topk_qb, cu_blk):
    """[Hkv, nqb, k] per-query-block selection -> [Hkv, N, k] per token."""
    lens = (cu_blk[1:] - cu_blk[:-1]).long()
    idx = torch.repeat_interleave(torch.arange(lens.numel()), lens)
    return block_topk_qb[:, idx]


def coherent_selection(seed, cu_seqlens, cu_seqblocks, Hkv, topk, jitter=2):
    """Per-token selections that mostly agree inside runs of tokens (as the
    geometric selection of the reference does): each token picks the blocks
    nearest (in block order) to its own position, with a few swaps."""
    g = torch.Generator().manual_seed(seed)
    N = int(cu_seqlens[-1])
    out = torch.full((Hkv, N, topk), -1, dtype=torch.int32)
    for b in range(cu_seqlens.numel() - 1):
        s, e = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        nb = int(cu_seqblocks[b + 1] - cu_seqblocks[b])
        kk = min(topk, nb)
        for h in range(Hkv):
            for i in range(s, e):
                c = (i - s) * nb // max(e - s, 1)
                cand = torch.arange(max(0, c - kk), min(nb, c + kk + jitter))
                perm = torch.randperm(cand.numel(), generator=g)[:kk]
                out[h, i, :kk] = cand[perm].sort().values.to(torch.int32)
    return out


def by_value(obj):
    """Tensors (nested in tuples, lists, dicts) as numpy arrays: a spawned
    worker's results then travel through a multiprocessing queue by value,
    not as shared-memory handles that break when the worker exits before the
    parent has read them."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu().numpy().copy()
    if isinstance(obj, dict):
        return {k: by_value(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(by_value(v) for v in obj)
    return obj


def as_tensors(obj):
    """The inverse of by_value (numpy arrays back to tensors)."""
    import numpy as np

    if isinstance(obj, np.ndarray):
        return torch.from_numpy(obj)
    if isinstance(obj, dict):
        return {k: as_tensors(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(as_tensors(v) for v in obj)
    return obj
