"""Ulysses sequence parallelism for the three-branch sparse attention.

The voxel sequence is split across the W ranks of a process group into
contiguous runs of whole blocks (Morton order), balanced by token count with
the same greedy rule as the reference (models_sparse/seqparallel_utils.py:
547-601), so a caller that already holds the reference's shards keeps them.

Every branch of the op (compression, scoring, top-k, selected, sliding and
compressed attention, per-head gates) factors over heads, so one exchange
each way suffices: ``seq_to_head`` moves every rank's tokens of the heads
that rank computes (one ``all_to_all_single``; the CUDA pack kernel lays the
slices out rank-major and the received buffer is already token-major), the
rank runs the whole-sequence op for its H/W heads, and ``head_to_seq`` brings
the merged output back.  The backward is the same exchange in reverse.  The
reference instead all-gathers all K/V tokens on every rank
(models_sparse/utils.py:326-474); for H = Hkv the Ulysses exchange moves about
a quarter of those bytes.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import ops

__all__ = ["shard_blocks", "ShardPlan", "seq_to_head", "head_to_seq", "exchange_gate_logits",
           "three_branch_attention", "time_exchanges", "ExchangeTimer", "RowPlan", "DecoderShards",
           "seq_parallel_token_blocks"]


def shard_blocks(cu_block_include_tokens: Sequence[int], world: int) -> List[Tuple[int, int]]:
    """Per rank ``(first_block, end_block)``: contiguous runs of whole blocks
    with balanced token counts.

    Restates the greedy of seqparallel_utils.py:547-601: rank r aims at
    (tokens left) / (ranks left), takes at least one block, and keeps taking
    the next block while that brings its count at least as close to the aim;
    the last rank takes what remains."""
    cu = [int(x) for x in cu_block_include_tokens]
    nb = len(cu) - 1
    if world < 1:
        raise ValueError("world size must be >= 1")
    out = []
    b = 0
    for r in range(world):
        if r == world - 1:
            out.append((b, nb))
            break
        aim = (cu[nb] - cu[b]) / (world - r)
        start, count = b, 0
        while b < nb:
            ln = cu[b + 1] - cu[b]
            if b == start or abs(count + ln - aim) <= abs(count - aim):
                count += ln
                b += 1
            else:
                break
        out.append((start, b))
    return out


class ShardPlan:
    """Token ranges of every rank (host ints) and the split sizes of the
    exchange."""

    def __init__(self, cu_block_include_tokens: Sequence[int], world: int, rank: int):
        cu = [int(x) for x in cu_block_include_tokens]
        self.world, self.rank = world, rank
        self.blocks = shard_blocks(cu, world)
        self.tokens = [(cu[a], cu[b]) for a, b in self.blocks]
        self.counts = [e - s for s, e in self.tokens]
        self.total = cu[-1]

    @property
    def local(self) -> Tuple[int, int]:
        return self.tokens[self.rank]

    def heads_of(self, num_heads: int) -> Tuple[int, int]:
        """Head range this rank computes (H >= W), or its replicated head."""
        if num_heads >= self.world:
            hp = num_heads // self.world
            return self.rank * hp, (self.rank + 1) * hp
        h = self.rank // (self.world // num_heads)
        return h, h + 1


class ExchangeTimer:
    """Device timing of the exchanges, off unless enabled: CUDA events on the
    current stream around every ``all_to_all_single`` of this module (the
    collective waits for the stream's earlier work and the stream waits for
    it), and the bytes each one sends to and receives from other ranks (a
    rank's own slice is a local copy and is not counted)."""

    def __init__(self):
        self.records = []

    def stats(self) -> dict:
        """Totals since the timer was enabled: ``ms``, ``calls``,
        ``bytes_out`` / ``bytes_in`` (crossing the links).  Synchronises."""
        if not self.records:
            return {"ms": 0.0, "calls": 0, "bytes_out": 0, "bytes_in": 0}
        torch.cuda.synchronize()
        return {"ms": sum(a.elapsed_time(b) for a, b, _, _ in self.records), "calls": len(self.records),
                "bytes_out": sum(r[2] for r in self.records), "bytes_in": sum(r[3] for r in self.records)}


_timer: Optional[ExchangeTimer] = None


def time_exchanges(on: bool = True) -> Optional[ExchangeTimer]:
    """Start (a fresh timer) or stop timing the exchanges; returns the timer."""
    global _timer
    _timer = ExchangeTimer() if on else None
    return _timer


def _host_staged(t: torch.Tensor, group) -> bool:
    """Device tensors exchanged over a gloo group go through host memory
    (gloo's all-to-all and all-gather take host tensors only): ranks that share
    one GPU, or a machine without NCCL, still run the sequence-parallel path."""
    return t.is_cuda and dist.get_backend(group) == "gloo"


def _all_to_all(recv, send, out_splits, in_splits, group):
    if _host_staged(recv, group):
        r = torch.empty(recv.shape, dtype=recv.dtype)
        dist.all_to_all_single(r, send.cpu(), out_splits, in_splits, group=group)
        recv.copy_(r)
        return
    dist.all_to_all_single(recv, send, out_splits, in_splits, group=group)


def _a2a(recv: torch.Tensor, send: torch.Tensor, out_splits, in_splits, group, rank: int):
    t = _timer
    if t is None or not recv.is_cuda:
        _all_to_all(recv, send, out_splits, in_splits, group)
        return
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    _all_to_all(recv, send, out_splits, in_splits, group)
    e1.record()
    el = recv.element_size()
    t.records.append((e0, e1, (sum(in_splits) - in_splits[rank]) * el, (sum(out_splits) - out_splits[rank]) * el))


def _check_heads(H: int, W: int):
    if H % W and W % H:
        raise ValueError(f"heads ({H}) and world size ({W}) must divide one another")


class _SeqToHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, plan: ShardPlan, group, pack: Callable, unpack: Callable):
        n, H, D = x.shape
        W = plan.world
        _check_heads(H, W)
        hp = H // W if H >= W else 1
        send = pack(x, W)  # [W, n, hp, D]
        recv = torch.empty(plan.total, hp, D, dtype=x.dtype, device=x.device)
        row = hp * D
        _a2a(recv.view(-1), send.view(-1), [c * row for c in plan.counts], [n * row] * W, group, plan.rank)
        ctx.plan, ctx.group, ctx.unpack, ctx.H = plan, group, unpack, H
        return recv

    @staticmethod
    def backward(ctx, g):
        plan = ctx.plan
        N, hp, D = g.shape
        n = plan.counts[plan.rank]
        back = torch.empty(plan.world, n, hp, D, dtype=g.dtype, device=g.device)
        row = hp * D
        _a2a(back.view(-1), g.contiguous().view(-1), [n * row] * plan.world, [c * row for c in plan.counts],
             ctx.group, plan.rank)
        return ctx.unpack(back, ctx.H), None, None, None, None


class _HeadToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, plan: ShardPlan, num_heads: int, group, pack: Callable, unpack: Callable):
        N, hp, D = y.shape
        if num_heads < plan.world:
            raise ValueError("head_to_seq needs at least one head per rank")
        n = plan.counts[plan.rank]
        back = torch.empty(plan.world, n, hp, D, dtype=y.dtype, device=y.device)
        row = hp * D
        _a2a(back.view(-1), y.contiguous().view(-1), [n * row] * plan.world, [c * row for c in plan.counts], group,
             plan.rank)
        ctx.plan, ctx.group, ctx.pack = plan, group, pack
        return unpack(back, num_heads)

    @staticmethod
    def backward(ctx, g):
        plan = ctx.plan
        n, H, D = g.shape
        hp = H // plan.world
        send = ctx.pack(g, plan.world)
        recv = torch.empty(plan.total, hp, D, dtype=g.dtype, device=g.device)
        row = hp * D
        _a2a(recv.view(-1), send.view(-1), [c * row for c in plan.counts], [n * row] * plan.world, ctx.group,
             plan.rank)
        return recv, None, None, None, None, None


def seq_to_head(x: torch.Tensor, plan: ShardPlan, group=None, pack: Callable = ops.ulysses_pack,
                unpack: Callable = ops.ulysses_unpack, normalize: bool = False, eps: float = 1e-5) -> torch.Tensor:
    """[n_local, H, D] (this rank's tokens, all heads) -> [N, hp, D] (all
    tokens, this rank's heads).  Differentiable.  ``normalize`` applies the
    reference's per-head LayerNorm32 (non-affine, over D; models_sparse/utils.py:
    239-270) in the same pass that packs the send buffer (H % W == 0)."""
    if normalize:
        pack = lambda t, W: ops.head_layernorm_pack(t, W, eps)  # noqa: E731
        unpack = lambda back, H: ops.head_layernorm_pack_bwd(x, back, eps)  # noqa: E731
    return _SeqToHead.apply(x, plan, group, pack, unpack)


class _HeadLayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, eps):
        ctx.save_for_backward(x)
        ctx.eps = eps
        return ops.head_layernorm_pack(x, 1, eps)[0]

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return ops.head_layernorm_pack_bwd(x, g.unsqueeze(0), ctx.eps), None


def head_layernorm(x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Per-head LayerNorm32 of x [n, H, D] (non-affine, fp32, cast back) on
    one GPU, differentiable: the W = 1 case of the fused pack."""
    return _HeadLayerNorm.apply(x, eps)


def head_to_seq(y: torch.Tensor, plan: ShardPlan, num_heads: int, group=None, pack: Callable = ops.ulysses_pack,
                unpack: Callable = ops.ulysses_unpack) -> torch.Tensor:
    """[N, hp, D] -> [n_local, H, D].  Differentiable."""
    return _HeadToSeq.apply(y, plan, num_heads, group, pack, unpack)


def _pack_small(x: torch.Tensor, world: int) -> torch.Tensor:
    # [n, B, H] -> [W, n, B, hp]: gate logits are a few bytes per head, below
    # the 16-byte slices of the CUDA pack; a strided torch copy moves them.
    n, B, H = x.shape
    return x.view(n, B, world, H // world).permute(2, 0, 1, 3).contiguous()


def _unpack_small(y: torch.Tensor, B: int, H: int) -> torch.Tensor:
    W, n, _, hp = y.shape
    return y.permute(1, 2, 0, 3).reshape(n, B, H)


class _GateExchange(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, plan: ShardPlan, n_branch: int, group):
        n, C = z.shape
        H = C // n_branch
        W = plan.world
        if H % W:
            raise ValueError("per-head gates need the heads to split evenly across ranks")
        send = _pack_small(z.view(n, n_branch, H), W)
        hp = H // W
        recv = torch.empty(plan.total, n_branch, hp, dtype=z.dtype, device=z.device)
        row = n_branch * hp
        _a2a(recv.view(-1), send.view(-1), [c * row for c in plan.counts], [n * row] * W, group, plan.rank)
        ctx.plan, ctx.group, ctx.B, ctx.H = plan, group, n_branch, H
        return recv.view(plan.total, n_branch * hp)

    @staticmethod
    def backward(ctx, g):
        plan = ctx.plan
        W, B, H = plan.world, ctx.B, ctx.H
        hp = H // W
        n = plan.counts[plan.rank]
        back = torch.empty(W, n, B, hp, dtype=g.dtype, device=g.device)
        row = B * hp
        _a2a(back.view(-1), g.contiguous().view(-1), [n * row] * W, [c * row for c in plan.counts], ctx.group,
             plan.rank)
        return _unpack_small(back, B, H).reshape(n, B * H), None, None, None


def exchange_gate_logits(z: torch.Tensor, plan: ShardPlan, n_branch: int, group=None) -> torch.Tensor:
    """Per-head gate logits [n_local, n_branch*H] (column ``b*H + h``) ->
    [N, n_branch*hp] for this rank's heads, same column rule.  Differentiable."""
    return _GateExchange.apply(z, plan, n_branch, group)


def three_branch_attention(q, k, v, z, plan: ShardPlan, cu_block_include_tokens: torch.Tensor, topk: int,
                           window: int, group=None, branch_fn: Optional[Callable] = None,
                           pack: Callable = ops.ulysses_pack, unpack: Callable = ops.ulysses_unpack,
                           softmax_scale=None):
    """Sequence-parallel compressed + selected + sliding-window attention with
    per-head gates.

    q [n_local, Hq, D], k/v [n_local, Hkv, D], z [n_local, 3*Hq] per-head gate
    logits, all for this rank's tokens; ``cu_block_include_tokens`` is the
    whole sequence's block table (every rank holds it).  Returns the merged
    output [n_local, Hq, D].  ``branch_fn(q, k, v, z, cu_blk, topk, window,
    scale)`` computes the merged output of the whole sequence for the heads it
    is given; the default is :func:`whole_sequence_branches` (CUDA)."""
    Hq, Hkv = q.shape[1], k.shape[1]
    if Hkv % plan.world:
        # the block score of a kv head sums over all q heads of its group
        # (block_score.py:47-96); a group split across ranks would select
        # differently, so every rank must own whole groups
        raise ValueError(f"Ulysses needs the kv heads ({Hkv}) to split evenly over {plan.world} ranks")
    fn = branch_fn or whole_sequence_branches
    qh = seq_to_head(q, plan, group, pack, unpack)
    kh = seq_to_head(k, plan, group, pack, unpack)
    vh = seq_to_head(v, plan, group, pack, unpack)
    zh = exchange_gate_logits(z, plan, 3, group)
    oh = fn(qh, kh, vh, zh, cu_block_include_tokens, topk, window, softmax_scale)
    return head_to_seq(oh, plan, Hq, group, pack, unpack)


def whole_sequence_branches(q, k, v, z, cu_blk, topk: int, window: int, softmax_scale=None, capture=None):
    """The single-rank op on one whole sequence: block-mean compression,
    compressed attention, per-query-block top-k (own block forced), selected
    and sliding-window attention, per-head sigmoid gates.  q [N, H, D],
    k/v [N, Hkv, D], z [N, 3*H]."""
    from . import functional as F

    N, H, D = q.shape
    out = F.three_branch_attention(q, k, v, cu_blk, topk, window, z, per_head=True, softmax_scale=softmax_scale,
                                   capture=capture)
    return out.view(N, H, D)


# ---------------------------------------------------------------------------
# Token distribution of the sequence-parallel decoder
# ---------------------------------------------------------------------------


class RowPlan:
    """Split sizes of an exchange over rows of any kind (tokens or blocks):
    rank r holds ``counts[r]`` consecutive rows of ``total``.  Has the fields
    the exchanges read (``world``, ``rank``, ``counts``, ``total``)."""

    def __init__(self, counts: Sequence[int], rank: int):
        self.counts = [int(c) for c in counts]
        self.world, self.rank = len(self.counts), rank
        self.total = sum(self.counts)
        self.start = sum(self.counts[:rank])

    @property
    def local(self) -> Tuple[int, int]:
        return self.start, self.start + self.counts[self.rank]


class DecoderShards:
    """Where this rank's volume and image tokens and blocks lie, for the
    exchanges of ``CrossAttention(use_sequence_parallel=True)``: token plans
    (``vol``, ``img``: whole blocks, token-balanced) and the matching block
    plans (``vol_blocks``, ``img_blocks``) for the compressed keys."""

    def __init__(self, cu_vol: Sequence[int], cu_img: Sequence[int], world: int, rank: int, group=None):
        self.group, self.world, self.rank = group, world, rank
        self.vol = ShardPlan(cu_vol, world, rank)
        self.img = ShardPlan(cu_img, world, rank)
        self.vol_blocks = RowPlan([b - a for a, b in self.vol.blocks], rank)
        self.img_blocks = RowPlan([b - a for a, b in self.img.blocks], rank)


_VOL_KEYED = ("vol_to_vol_attn", "img_to_vol_attn")  # maps whose keys are volume tokens
_IMG_KEYED = ("img_to_img_attn", "vol_to_img_attn")


def _local_blocks(cu: torch.Tensor, plan: ShardPlan) -> torch.Tensor:
    b0, b1 = plan.blocks[plan.rank]
    return (cu[b0:b1 + 1] - cu[b0]).to(torch.int32)


class _Collect(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, plan: ShardPlan, group):
        n_max = max(plan.counts)
        pad = x.new_zeros((n_max,) + tuple(x.shape[1:]))
        pad[: x.shape[0]] = x
        full = x.new_empty((plan.world * n_max,) + tuple(x.shape[1:]))
        if _host_staged(x, group):
            f = torch.empty(full.shape, dtype=full.dtype)
            dist.all_gather_into_tensor(f, pad.cpu(), group=group)
            full.copy_(f)
        else:
            dist.all_gather_into_tensor(full, pad.contiguous(), group=group)
        ctx.plan = plan
        return torch.cat([full[r * n_max: r * n_max + c] for r, c in enumerate(plan.counts)])

    @staticmethod
    def backward(ctx, g):
        s, e = ctx.plan.local
        return g[s:e], None, None


def seq_parallel_token_blocks(vol_token_arr, img_token_arr, attn_map, mode: str = "distribute", group=None):
    """The token distribution of the sequence-parallel decoder, with the
    reference's call shape (models_sparse/seqparallel_utils.py:948-1169) for
    one sequence.

    ``mode="distribute"``: every rank holds all tokens; each tensor of
    ``vol_token_arr`` / ``img_token_arr`` ([N, C]) is cut to this rank's run of
    whole blocks (token-balanced, :func:`shard_blocks`; volume blocks from
    ``attn_map["vol_to_vol_attn"]``, image blocks from ``"img_to_img_attn"``).
    Every map gets ``local_cu_block_include_tokens`` (this rank's blocks of its
    key tokens, local offsets) and ``attn_map["sp"]`` the :class:`DecoderShards`;
    the maps' global tables stay as they are (the attention cores run on the
    whole sequence for this rank's heads).  Returns ``(vol_tokens, img_tokens,
    cu_seqlens_volume, cu_seqlens_image, attn_map)`` with local cu_seqlens.

    ``mode="collect"``: all-gathers the volume tensors back to all tokens
    (differentiable: the backward keeps this rank's rows, i.e. every rank is
    expected to compute the same loss on the collected tensor).
    """
    if mode not in ("distribute", "collect"):
        raise ValueError("mode must be 'distribute' or 'collect'")
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if mode == "collect":
        sp = attn_map["sp"]
        return [_Collect.apply(t, sp.vol, group) for t in vol_token_arr], [], None, None, attn_map
    cu_vol_t = attn_map["vol_to_vol_attn"]["cu_block_include_tokens"]
    cu_img_t = attn_map["img_to_img_attn"]["cu_block_include_tokens"]
    for keyed, ref in ((_VOL_KEYED, cu_vol_t), (_IMG_KEYED, cu_img_t)):
        for name in keyed:
            if name in attn_map and not torch.equal(attn_map[name]["cu_block_include_tokens"], ref):
                raise ValueError(f"{name} must use the same key blocks as {keyed[0]} under sequence parallelism")
    sp = DecoderShards(cu_vol_t.tolist(), cu_img_t.tolist(), world, rank, group)
    out = dict(attn_map)
    for keyed, plan, cu in ((_VOL_KEYED, sp.vol, cu_vol_t), (_IMG_KEYED, sp.img, cu_img_t)):
        loc = _local_blocks(cu, plan)
        for name in keyed:
            if name in out:
                out[name] = dict(out[name], local_cu_block_include_tokens=loc)
    out["sp"] = sp
    (vs, ve), (is_, ie) = sp.vol.local, sp.img.local
    dev = cu_vol_t.device
    cu_v = torch.tensor([0, ve - vs], dtype=torch.int32, device=dev)
    cu_i = torch.tensor([0, ie - is_], dtype=torch.int32, device=dev)
    return [t[vs:ve] for t in vol_token_arr], [t[is_:ie] for t in img_token_arr], cu_v, cu_i, out
