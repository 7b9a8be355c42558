"""CPU restatement of LSRM's variable-block native sparse attention.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): never imported by the
shipped package.  Floating-point math runs in float64 torch on the CPU unless
a function says otherwise; the block scorer runs in numpy float32 with a fixed
operation order so that its indices can be compared bit for bit with the CUDA
scorer.

Every function cites the reference lines it restates (paths are relative to
the root of chenxiex/Large-Sparse-Reconstruction-Model).

Selection semantics shared by every function here and by the CUDA kernels:

* ``block_topk[h, i, :]`` holds sequence-local block ids.  An entry is valid
  when ``0 <= id < blocks_in_sequence``; other entries (the reference pads with
  ``-1`` at the tail) are ignored.  For tail padding this is exactly the
  reference's ``valid_sel_count`` rule
  (sparse/ops/triton_native_sparse_attention_impl_kvcentric.py:151-166).
* A block listed twice is attended twice (multiplicity weight), as the
  reference's loops do (kvcentric.py:166-226 forward, :494-572 reverse map).
* A query with no valid block gets a NaN output row and ``-inf`` LSE
  (0/0 at kvcentric.py:229).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

LOG2E = 1.44269504  # the constant the reference uses (block_score.py:59-60)

__all__ = [
    "LOG2E",
    "segment_mean",
    "res_block",
    "compress_kv",
    "selection_attention",
    "compressed_attention",
    "window_attention_intra_block",
    "sliding_window_attention",
    "gate_merge",
    "exp2_fixed",
    "token_block_scores_exact",
    "get_block_score_exact",
    "get_block_score_qblock_exact",
    "block_score_reference_formula",
    "build_query_tiles",
    "build_tile_unions",
    "selection_flops",
    "dense_attention_flops",
    "three_branch_sample_step",
    "qblock_selection_exact",
    "three_branch_masked_dense",
    "three_branch_sampled",
    "compress_vjp",
    "compress_forward",
    "volume_sort_keys",
    "block_separation",
    "prepare_volume_output",
    "volume_block_topk",
]


def _i(x) -> List[int]:
    return [int(v) for v in torch.as_tensor(x).reshape(-1).tolist()]


# ---------------------------------------------------------------------------
# Compression (SpatialSparseAttentionIn)
# ---------------------------------------------------------------------------


def segment_mean(x: torch.Tensor, cu: torch.Tensor) -> torch.Tensor:
    """Mean of ``x`` rows over each segment ``[cu[b], cu[b+1])``.

    Restates ``torch.segment_reduce(reduce="mean")`` as used at
    sparse/module/spatial_sparse_attention.py:27-37.  Empty segments give NaN,
    as ``segment_reduce`` does.
    """
    xs = x.to(torch.float64)
    offs = _i(cu)
    out = torch.empty((len(offs) - 1,) + tuple(xs.shape[1:]), dtype=torch.float64)
    for b in range(len(offs) - 1):
        s, e = offs[b], offs[b + 1]
        out[b] = xs[s:e].mean(dim=0) if e > s else float("nan")
    return out


def res_block(x, w1, b1, w2, b2, eps: float = 1e-5) -> torch.Tensor:
    """``SparseResBlock``: LN_fp32(x + W2·SiLU(W1·x + b1) + b2), no affine.

    Restates sparse/module/residual_block.py:11-34 (LayerNorm32 with
    ``elementwise_affine=False`` and the default eps 1e-5).
    """
    xd = x.to(torch.float64)
    h = torch.nn.functional.linear(xd, w1.double(), b1.double())
    h = torch.nn.functional.silu(h)
    h = torch.nn.functional.linear(h, w2.double(), b2.double())
    y = xd + h
    return torch.nn.functional.layer_norm(y, (y.shape[-1],), eps=eps)


def compress_kv(x, cu_block_include_tokens, weights=None) -> torch.Tensor:
    """One branch of ``SpatialSparseAttentionIn.forward``.

    spatial_sparse_attention.py:46-66: the ResBlock runs token-wise, then the
    block mean.  ``weights=None`` is the pure block-mean compression.
    """
    if weights is not None:
        x = res_block(x, *weights)
    return segment_mean(x, cu_block_include_tokens)


# ---------------------------------------------------------------------------
# Attention branches
# ---------------------------------------------------------------------------


def _block_counts(block_topk_h: torch.Tensor, nb: int) -> torch.Tensor:
    """[nq, k] sequence-local ids -> [nq, nb] multiplicity counts (valid ids)."""
    sel = block_topk_h.long()
    valid = (sel >= 0) & (sel < nb)
    counts = torch.zeros(sel.shape[0], max(nb, 1), dtype=torch.float64)
    if nb > 0:
        counts.scatter_add_(1, sel.clamp(0, nb - 1), valid.to(torch.float64))
    return counts[:, :nb]


def _masked_softmax_attend(qh, kh, vh, log_weight, scale):
    """o = softmax(scale·q·kᵀ + log_weight)·v, lse (natural log)."""
    logits = (qh @ kh.transpose(0, 1)) * scale + log_weight
    lse = torch.logsumexp(logits, dim=-1)
    p = torch.softmax(logits, dim=-1)
    return p @ vh, lse


def selection_attention(
    q,
    k,
    v,
    block_topk,
    cu_seqblocks,
    cu_block_include_tokens,
    cu_seqlens_q,
    cu_seqlens_k,
    softmax_scale: Optional[float] = None,
    dtype=torch.float64,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Selected-block attention forward; returns ``(o, lse_log2)``.

    Restates ``forward_kernel_varblock``
    (sparse/ops/triton_native_sparse_attention_impl_kvcentric.py:55-247):
    query ``i`` of sequence ``b`` attends to the union (with multiplicity) of
    the token ranges ``cu_block_include_tokens[cu_seqblocks[b] + id]`` of its
    valid selected blocks, keys restricted to ``[cu_seqlens_k[b],
    cu_seqlens_k[b+1])`` (the ``c + tile + offs_n < seqlen_k`` mask, :181).
    LSE is returned in log2 units, ``[Hq, Nq]`` (:240-245).  Differentiable
    when the inputs require grad (the backward of the same formula is what
    kvcentric.py:262-478 and :687-923 compute).
    """
    Nq, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    qd, kd, vd = q.to(dtype), k.to(dtype), v.to(dtype)
    cq, ck, cs, cb = _i(cu_seqlens_q), _i(cu_seqlens_k), _i(cu_seqblocks), _i(cu_block_include_tokens)
    outs = []
    lses = []
    for b in range(len(cq) - 1):
        qs, qe, ks, ke = cq[b], cq[b + 1], ck[b], ck[b + 1]
        bs, be = cs[b], cs[b + 1]
        nb = be - bs
        # key token -> sequence-local block id (tokens outside any block: -1)
        key_block = torch.full((ke - ks,), -1, dtype=torch.long)
        for j in range(nb):
            t0, t1 = cb[bs + j], cb[bs + j + 1]
            lo, hi = max(t0, ks), min(t1, ke)
            if hi > lo:
                key_block[lo - ks : hi - ks] = j
        o_seq = []
        l_seq = []
        for hq in range(Hq):
            h = hq // G
            cnt = _block_counts(block_topk[h, qs:qe], nb)  # [nq, nb]
            if ke > ks:
                w = torch.zeros(qe - qs, ke - ks, dtype=torch.float64)
                inb = key_block >= 0
                w[:, inb] = cnt[:, key_block[inb]]
            else:
                w = torch.zeros(qe - qs, 0, dtype=torch.float64)
            logw = torch.where(w > 0, w.log(), torch.full_like(w, -math.inf)).to(dtype)
            empty = (w > 0).sum(dim=1) == 0  # rows with no attended key
            logw = torch.where(empty[:, None], torch.zeros_like(logw), logw)
            o_h, lse_h = _masked_softmax_attend(
                qd[qs:qe, hq], kd[ks:ke, h], vd[ks:ke, h], logw, scale
            )
            # 0/0 in the reference: NaN output, -inf LSE, no gradient path
            o_h = torch.where(empty[:, None], torch.full_like(o_h, math.nan), o_h)
            lse_h = torch.where(empty, torch.full_like(lse_h, -math.inf), lse_h)
            if ke == ks:
                o_h = torch.full((qe - qs, D), math.nan, dtype=dtype)
                lse_h = torch.full((qe - qs,), -math.inf, dtype=dtype)
            o_seq.append(o_h)
            l_seq.append(lse_h / math.log(2.0))
        if qe > qs:
            outs.append(torch.stack(o_seq, dim=1))
            lses.append(torch.stack(l_seq, dim=0))
    o = torch.cat(outs, 0) if outs else torch.zeros(0, Hq, D, dtype=dtype)
    lse = torch.cat(lses, 1) if lses else torch.zeros(Hq, 0, dtype=dtype)
    return o, lse


def compressed_attention(
    q, ck, cv, cu_seqlens_q, cu_seqblocks, softmax_scale=None, dtype=torch.float64
):
    """Compressed branch: every query attends to all compressed blocks of its
    sequence.  Returns ``(o, lse_ln)`` with the natural-log LSE ``[Hq, Nq]``.

    Restates the ``flash_attn_varlen_func(q, compressed_k, compressed_v,
    cu_seqlens_q, compressed_cu_seqlens, ..., causal=False,
    return_attn_probs=True)`` call at spatial_sparse_attention.py:121-143.
    """
    Nq, Hq, D = q.shape
    Hkv = ck.shape[1]
    G = Hq // Hkv
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    qd, kd, vd = q.to(dtype), ck.to(dtype), cv.to(dtype)
    cq, cs = _i(cu_seqlens_q), _i(cu_seqblocks)
    outs, lses = [], []
    for b in range(len(cq) - 1):
        qs, qe, ks, ke = cq[b], cq[b + 1], cs[b], cs[b + 1]
        if qe == qs:
            continue
        o_seq, l_seq = [], []
        for hq in range(Hq):
            h = hq // G
            zero = torch.zeros(qe - qs, ke - ks, dtype=dtype)
            o_h, l_h = _masked_softmax_attend(qd[qs:qe, hq], kd[ks:ke, h], vd[ks:ke, h], zero, scale)
            o_seq.append(o_h)
            l_seq.append(l_h)
        outs.append(torch.stack(o_seq, 1))
        lses.append(torch.stack(l_seq, 0))
    o = torch.cat(outs, 0) if outs else torch.zeros(0, Hq, D, dtype=dtype)
    lse = torch.cat(lses, 1) if lses else torch.zeros(Hq, 0, dtype=dtype)
    return o, lse


def _dense_segments_attention(q, k, v, segments, scale, band=None, dtype=torch.float64):
    Nq, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    qd, kd, vd = q.to(dtype), k.to(dtype), v.to(dtype)
    out = torch.zeros(Nq, Hq, D, dtype=dtype)
    rows = []
    for (s, e) in segments:
        if e <= s:
            continue
        idx = torch.arange(s, e)
        logw = torch.zeros(e - s, e - s, dtype=dtype)
        if band is not None:
            dist = (idx[:, None] - idx[None, :]).abs()
            logw = torch.where(dist <= band, logw, torch.full_like(logw, -math.inf))
        o_seg = []
        for hq in range(Hq):
            h = hq // G
            o_h, _ = _masked_softmax_attend(qd[s:e, hq], kd[s:e, h], vd[s:e, h], logw, scale)
            o_seg.append(o_h)
        rows.append((s, e, torch.stack(o_seg, 1)))
    for s, e, o in rows:
        out = out.index_copy(0, torch.arange(s, e), o)
    return out


def window_attention_intra_block(q, k, v, cu_block_include_tokens, softmax_scale=None, dtype=torch.float64):
    """Reference window branch: full attention inside each variable block.

    Restates ``sparse_window_attention`` (sparse/ops/block_window_attention.py:
    14-31), i.e. ``flash_attn_varlen_func`` with ``cu_seqlens_q = cu_seqlens_k
    = cu_block_include_tokens`` and the default scale 1/sqrt(d).
    """
    D = q.shape[-1]
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    cb = _i(cu_block_include_tokens)
    return _dense_segments_attention(q, k, v, list(zip(cb[:-1], cb[1:])), scale, dtype=dtype)


def sliding_window_attention(q, k, v, cu_seqlens, window: int, softmax_scale=None, dtype=torch.float64):
    """Extension (not in the reference): band attention ``|i - j| <= window // 2``
    inside each sequence, in token (Morton) order."""
    D = q.shape[-1]
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    cs = _i(cu_seqlens)
    return _dense_segments_attention(q, k, v, list(zip(cs[:-1], cs[1:])), scale, band=window // 2, dtype=dtype)


def gate_merge(x, gate_weight, branches: Sequence[torch.Tensor], mode: str = "per_channel", num_heads: int = 1):
    """Sigmoid-gated merge of the attention branches.

    ``per_channel`` restates ``SpatialSparseAttentionOut.forward``
    (spatial_sparse_attention.py:215-224, 257-269): ``g = sigmoid(x·Wgᵀ)`` with
    ``Wg`` of shape ``[n·C, C]`` and ``out = Σ g[:, i·C:(i+1)·C] ⊙ branch_i``
    (branch order: compressed, selection, window).  ``per_head`` is the
    extension where ``Wg`` is ``[n·H, hidden]`` and each gate value is
    broadcast over the ``head_dim`` channels of its head.
    """
    g = torch.sigmoid(x.double() @ gate_weight.double().t())
    out = 0
    n = len(branches)
    C = branches[0].shape[-1]
    for i, br in enumerate(branches):
        if mode == "per_channel":
            gi = g[:, i * C : (i + 1) * C]
        else:
            d = C // num_heads
            gi = g[:, i * num_heads : (i + 1) * num_heads].repeat_interleave(d, dim=1)
        out = out + gi * br.double()
    assert g.shape[1] == (n * C if mode == "per_channel" else n * num_heads)
    return out


# ---------------------------------------------------------------------------
# Block scoring + top-k with a fixed float32 operation order (bit-exact)
# ---------------------------------------------------------------------------

_F32 = np.float32
# Taylor coefficients ln(2)^i / i! of 2^f = exp(f·ln2) around 0, rounded to
# float32; stored as bit patterns so the CUDA scorer uses identical values.
_EXP2_COEF_BITS = [0x3F800000, 0x3F317218, 0x3E75FDF0, 0x3D635847, 0x3C1D955B, 0x3AAEC3FF, 0x39218489, 0x377FE5FE]
_EXP2_COEF = [np.array(b, dtype=np.uint32).view(_F32)[()] for b in _EXP2_COEF_BITS]
assert all(abs(float(c) - math.log(2.0) ** i / math.factorial(i)) < 1e-7 for i, c in enumerate(_EXP2_COEF))


def exp2_fixed(t: np.ndarray) -> np.ndarray:
    """2^t in float32 with a fixed, portable operation order.

    Range reduction ``n = rint(t)``, ``f = t - n`` (exact), degree-7 Taylor
    polynomial of ``exp(f ln 2)`` by Horner's rule with separately rounded
    multiplies and adds, then an exact scale by ``2^n``.  ``t < -125.5`` flushes
    to 0 (no subnormals), ``t >= 127.5`` gives inf.  The CUDA scorer evaluates
    the same sequence with ``__fmul_rn``/``__fadd_rn``, so both sides agree bit
    for bit.
    """
    t = np.asarray(t, dtype=_F32)
    n = np.rint(t)
    f = (t - n).astype(_F32)
    r = np.full_like(f, _EXP2_COEF[7])
    for c in _EXP2_COEF[6::-1]:
        r = (r * f).astype(_F32)
        r = (r + c).astype(_F32)
    n_cl = np.clip(n, -125, 127).astype(np.int32)
    scale = ((n_cl + 127).astype(np.uint32) << np.uint32(23)).view(_F32)
    with np.errstate(over="ignore"):
        out = (r * scale).astype(_F32)
    out = np.where(n < -125, _F32(0.0), out)
    out = np.where(n > 127, _F32(np.inf), out)
    return out.astype(_F32)


def _to_f32_np(x) -> np.ndarray:
    return torch.as_tensor(x).detach().to(torch.float32).cpu().numpy()


def token_block_scores_exact(q, ck, lse_ln, cu_seqlens_q, compressed_cu_seqlens, sm_scale=None):
    """Per-token block scores in fixed-order float32.

    score[h, i, b] = Σ_{g<G} exp2_fixed(dot(q[i, hG+g], ck[b, h]) · qk_scale
    − lse[hG+g, i]·1.44269504), where ``dot`` accumulates the products in
    ascending channel order with separately rounded multiply and add, and
    ``qk_scale = float32(sm_scale · 1.44269504)``.  This is the arithmetic of
    ``get_block_score`` (sparse/ops/block_score.py:57-92) with its summation
    order fixed.  Returns a list (one entry per sequence) of ``[Hkv, nq, nb]``
    float32 arrays.
    """
    qn = _to_f32_np(q)
    cn = _to_f32_np(ck)
    ln = _to_f32_np(lse_ln)
    Nq, Hq, D = qn.shape
    Hkv = cn.shape[1]
    G = Hq // Hkv
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    qk_scale = _F32(sm_scale * LOG2E)
    lse2 = (ln * _F32(LOG2E)).astype(_F32)
    cq, cc = _i(cu_seqlens_q), _i(compressed_cu_seqlens)
    res = []
    for b in range(len(cq) - 1):
        qs, qe, ks, ke = cq[b], cq[b + 1], cc[b], cc[b + 1]
        sc = np.zeros((Hkv, qe - qs, ke - ks), dtype=_F32)
        for h in range(Hkv):
            for g in range(G):
                hq = h * G + g
                qh = qn[qs:qe, hq, :]
                kh = cn[ks:ke, h, :]
                acc = np.zeros((qe - qs, ke - ks), dtype=_F32)
                for j in range(D):
                    acc = (acc + (qh[:, j : j + 1] * kh[None, :, j]).astype(_F32)).astype(_F32)
                t = ((acc * qk_scale).astype(_F32) - lse2[hq, qs:qe, None]).astype(_F32)
                sc[h] = (sc[h] + exp2_fixed(t)).astype(_F32)
        res.append(sc)
    return res


def _topk_lowest_id(scores: np.ndarray, k: int, force: Optional[np.ndarray] = None) -> np.ndarray:
    """Rows of ``scores`` [n, nb] -> ascending ids of the k best blocks.

    Order: larger score first, ties broken by the lower block id; then the
    chosen ids are sorted ascending and padded with -1 (block_score.py:85-96).
    ``force[i]`` (optional) is a block id that is always selected first.
    """
    n, nb = scores.shape
    out = np.full((n, k), -1, dtype=np.int32)
    kk = min(k, nb)
    if kk == 0:
        return out
    ids = np.arange(nb)
    for i in range(n):
        s = scores[i].astype(np.float64)
        chosen = []
        if force is not None and 0 <= force[i] < nb:
            chosen.append(int(force[i]))
        order = np.lexsort((ids, -s))  # primary: -score, secondary: id
        for b in order:
            if len(chosen) >= kk:
                break
            if force is not None and b == force[i]:
                continue
            chosen.append(int(b))
        out[i, :kk] = np.sort(np.array(chosen, dtype=np.int32))
    return out


def get_block_score_exact(q, compressed_k, lse, topk, cu_seqlens_q, compressed_cu_seqlens, sm_scale=None):
    """Bit-exact restatement of ``get_block_score`` (block_score.py:16-98).

    Returns ``[Hkv, Nq, topk]`` int32 of sequence-local block ids, ascending,
    ``-1``-padded when a sequence has fewer than ``topk`` blocks.  Ties go to
    the lowest block id.
    """
    Hkv = compressed_k.shape[1]
    Nq = q.shape[0]
    out = np.full((Hkv, Nq, topk), -1, dtype=np.int32)
    scores = token_block_scores_exact(q, compressed_k, lse, cu_seqlens_q, compressed_cu_seqlens, sm_scale)
    cq = _i(cu_seqlens_q)
    for b, sc in enumerate(scores):
        for h in range(Hkv):
            out[h, cq[b] : cq[b + 1]] = _topk_lowest_id(sc[h], topk)
    return torch.from_numpy(out)


def get_block_score_qblock_exact(
    q, compressed_k, lse, topk, cu_seqlens_q, compressed_cu_seqlens, cu_qblocks, sm_scale=None, force_self=False
):
    """Extension: one selection per query block.

    The score of block ``b`` for query block ``Q`` is the float32 sum, in
    ascending token order, of the per-token scores of
    ``token_block_scores_exact``.  ``cu_qblocks`` are global token offsets of
    the query blocks (each lies inside one sequence).  With ``force_self`` the
    query block's own index (sequence-local, query block ``j`` of a sequence
    maps to KV block ``j``) is always selected.  Returns ``[Hkv, n_qblocks,
    topk]`` int32.
    """
    Hkv = compressed_k.shape[1]
    cqb = _i(cu_qblocks)
    nqb = len(cqb) - 1
    out = np.full((Hkv, nqb, topk), -1, dtype=np.int32)
    scores = token_block_scores_exact(q, compressed_k, lse, cu_seqlens_q, compressed_cu_seqlens, sm_scale)
    cq = _i(cu_seqlens_q)
    qb = 0
    for b, sc in enumerate(scores):
        qs, qe = cq[b], cq[b + 1]
        first = qb
        rows = []
        while qb < nqb and cqb[qb] < qe:
            rows.append((cqb[qb] - qs, cqb[qb + 1] - qs))
            qb += 1
        for h in range(Hkv):
            agg = np.zeros((len(rows), sc.shape[2]), dtype=_F32)
            for r, (s, e) in enumerate(rows):
                acc = np.zeros(sc.shape[2], dtype=_F32)
                for t in range(s, e):
                    acc = (acc + sc[h, t]).astype(_F32)
                agg[r] = acc
            force = np.arange(len(rows)) if force_self else None
            out[h, first : first + len(rows)] = _topk_lowest_id(agg, topk, force)
    return torch.from_numpy(out)


def block_score_reference_formula(q, compressed_k, lse, cu_seqlens_q, compressed_cu_seqlens, sm_scale=None):
    """float64 scores of block_score.py:57-92 (for tolerance checks only)."""
    Nq, Hq, D = q.shape
    Hkv = compressed_k.shape[1]
    G = Hq // Hkv
    sm_scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    cq, cc = _i(cu_seqlens_q), _i(compressed_cu_seqlens)
    res = []
    for b in range(len(cq) - 1):
        qs, qe, ks, ke = cq[b], cq[b + 1], cc[b], cc[b + 1]
        sc = torch.zeros(Hkv, qe - qs, ke - ks, dtype=torch.float64)
        for h in range(Hkv):
            ckh = compressed_k[ks:ke, h].double()
            for g in range(G):
                hq = h * G + g
                qk = (q[qs:qe, hq].double() @ ckh.t()) * sm_scale * LOG2E
                sc[h] += torch.exp2(qk - lse[hq, qs:qe, None].double() * LOG2E)
        res.append(sc)
    return res


# ---------------------------------------------------------------------------
# Work decomposition (restated so that the CUDA builders can be checked)
# ---------------------------------------------------------------------------


@dataclass
class QueryTile:
    seq: int
    q_start: int  # global query index of the first query
    n_q: int  # queries in the tile (<= rows // G)


def build_query_tiles(cu_seqlens_q, queries_per_tile: int, cu_qblocks=None) -> List[QueryTile]:
    """Split each sequence's queries into tiles of ``queries_per_tile``.

    With ``cu_qblocks`` (global offsets of query blocks) no tile straddles a
    query-block boundary.
    """
    cq = _i(cu_seqlens_q)
    cuts = set(_i(cu_qblocks)) if cu_qblocks is not None else set()
    tiles = []
    for b in range(len(cq) - 1):
        s, e = cq[b], cq[b + 1]
        i = s
        while i < e:
            j = min(i + queries_per_tile, e)
            if cuts:
                nxt = [c for c in cuts if i < c < j]
                if nxt:
                    j = min(nxt)
            tiles.append(QueryTile(b, i, j - i))
            i = j
    return tiles


def build_tile_unions(block_topk_h: torch.Tensor, tiles: List[QueryTile], cu_seqblocks) -> List[Tuple[List[int], List[int]]]:
    """For each tile: ascending unique valid sequence-local block ids and,
    per id, the bitmask of tile queries that selected it."""
    cs = _i(cu_seqblocks)
    out = []
    for t in tiles:
        nb = cs[t.seq + 1] - cs[t.seq]
        masks = {}
        for r in range(t.n_q):
            for e in _i(block_topk_h[t.q_start + r]):
                if 0 <= e < nb:
                    masks[e] = masks.get(e, 0) | (1 << r)
        ids = sorted(masks)
        out.append((ids, [masks[i] for i in ids]))
    return out


# ---------------------------------------------------------------------------
# Algorithmic FLOP accounting (valid pairs only)
# ---------------------------------------------------------------------------


def selection_flops(block_topk, cu_seqblocks, cu_block_include_tokens, cu_seqlens_q, num_q_heads, head_dim) -> float:
    """4·d per (query head, attended key) for the forward pass.  Keys are
    counted with multiplicity, as the reference attends them."""
    G = num_q_heads // block_topk.shape[0]
    cs, cb, cq = _i(cu_seqblocks), _i(cu_block_include_tokens), _i(cu_seqlens_q)
    lens = np.diff(np.array(cb, dtype=np.int64))
    total = 0
    bt = block_topk.numpy() if isinstance(block_topk, torch.Tensor) else block_topk
    for b in range(len(cq) - 1):
        nb = cs[b + 1] - cs[b]
        sel = bt[:, cq[b] : cq[b + 1]].astype(np.int64)
        valid = (sel >= 0) & (sel < nb)
        seg = lens[cs[b] : cs[b + 1]]
        if nb:
            total += int(np.where(valid, seg[np.clip(sel, 0, nb - 1)], 0).sum())
    return 4.0 * head_dim * G * total


def dense_attention_flops(pairs: int, num_q_heads: int, head_dim: int) -> float:
    return 4.0 * head_dim * num_q_heads * pairs


# ---------------------------------------------------------------------------
# Bounded CPU sample of the three-branch op (the benchmark's CPU baseline)
# ---------------------------------------------------------------------------


def three_branch_sample_step(q, k, v, x, gate_w, g, cu_blk, qblock_ids, topk, window, per_head=True,
                             force_self=True):
    """float32 CPU forward + backward of the three-branch op for the query
    blocks ``qblock_ids`` of a single-sequence problem (keys gathered per
    query block), the restatement that the benchmark times on the host cores.

    Branches (gates in this order): compressed attention over the block means
    of K/V (spatial_sparse_attention.py:27-37, :121-143), selected blocks by
    the query-block score of ``get_block_score_qblock_exact`` with
    ``force_self`` (block_score.py:16-98 aggregated per query block), sliding
    window ``|i-j| <= window//2``; sigmoid-gated merge (:257-269, per head when
    ``per_head``).  Returns (loss, algorithmic flops of the attention
    branches, 14·d per attended (query head, key) pair).
    """
    N, H, D = q.shape
    nb = cu_blk.numel() - 1
    cb = _i(cu_blk)
    lens = torch.tensor(np.diff(np.array(cb)), dtype=torch.float32)
    qf = q.detach().float().requires_grad_()
    kf = k.detach().float().requires_grad_()
    vf = v.detach().float().requires_grad_()
    xf = x.detach().float().requires_grad_()
    wf = gate_w.detach().float().requires_grad_()
    blk_of = torch.repeat_interleave(torch.arange(nb), lens.long())
    ck = torch.zeros(nb, H, D).index_add(0, blk_of, kf) / lens[:, None, None]
    cv = torch.zeros(nb, H, D).index_add(0, blk_of, vf) / lens[:, None, None]
    scale = 1.0 / math.sqrt(D)
    half = window // 2
    loss = 0.0
    pairs = 0
    for qb in qblock_ids:
        r0, r1 = cb[qb], cb[qb + 1]
        L = r1 - r0
        qq = qf[r0:r1]  # [L, H, D]
        # compressed branch (natural-log LSE kept for scoring)
        sc = torch.einsum("lhd,bhd->hlb", qq, ck) * scale
        lse = torch.logsumexp(sc, -1)  # [H, L]
        o_c = torch.einsum("hlb,bhd->lhd", torch.softmax(sc, -1), cv)
        pairs += L * nb
        # scoring (bit-exact restatement) for this query block
        cq = torch.tensor([0, L], dtype=torch.int32)
        cc = torch.tensor([0, nb], dtype=torch.int32)
        cqb = torch.tensor([0, L], dtype=torch.int32)
        tok = token_block_scores_exact(qq.detach(), ck.detach(), lse.detach(), cq, cc)[0]  # [H, L, nb]
        fixed = []
        for h in range(H):
            agg = np.zeros(nb, dtype=_F32)
            for t in range(L):
                agg = (agg + tok[h, t]).astype(_F32)
            force = np.array([qb]) if force_self else None
            row = _topk_lowest_id(agg[None], topk, force)[0]
            fixed.append([int(t) for t in row if t >= 0])
        o_s = []
        for h in range(H):
            keys = torch.cat([torch.arange(cb[b], cb[b + 1]) for b in fixed[h]])
            s = (qq[:, h] @ kf[keys, h].t()) * scale
            o_s.append(torch.softmax(s, -1) @ vf[keys, h])
            pairs += L * keys.numel()
        o_s = torch.stack(o_s, 1)
        # sliding window
        k0, k1 = max(0, r0 - half), min(N, r1 + half)
        idx_q = torch.arange(r0, r1)[:, None]
        idx_k = torch.arange(k0, k1)[None, :]
        band = (idx_q - idx_k).abs() <= half
        s = torch.einsum("lhd,khd->hlk", qq, kf[k0:k1]) * scale
        s = s.masked_fill(~band[None], float("-inf"))
        o_w = torch.einsum("hlk,khd->lhd", torch.softmax(s, -1), vf[k0:k1])
        pairs += int(band.sum())
        # gated merge
        z = torch.sigmoid(xf[r0:r1] @ wf.t())
        branches = [o_c, o_s, o_w]
        out = 0
        for i, br in enumerate(branches):
            gi = z[:, i * H:(i + 1) * H, None] if per_head else z[:, i * H * D:(i + 1) * H * D].view(L, H, D)
            out = out + gi * br
        loss = loss + (out.reshape(L, -1) * g[r0:r1].float()).sum()
    loss.backward()
    return float(loss.detach()), 14.0 * D * H * pairs


# ---------------------------------------------------------------------------
# The whole three-branch step with its gradients (parity of the timed path)
# ---------------------------------------------------------------------------


def qblock_selection_exact(q_rows, ck, lse_rows, topk: int, force_block: Optional[int] = None, sm_scale=None):
    """Selection of ONE query block in the fixed float32 order of
    ``get_block_score_qblock_exact``: the per-token scores of
    ``token_block_scores_exact`` (block_score.py:57-92) summed over the block's
    tokens in ascending order, top-k with ties to the lower id, ``force_block``
    always chosen, ids ascending (block_score.py:85-96).  q_rows [L, Hq, D],
    ck [nb, Hkv, D], lse_rows [Hq, L] (natural log).  Returns [Hkv, topk]."""
    L = q_rows.shape[0]
    nb = ck.shape[0]
    cq = torch.tensor([0, L], dtype=torch.int32)
    cc = torch.tensor([0, nb], dtype=torch.int32)
    sc = token_block_scores_exact(q_rows, ck, lse_rows, cq, cc, sm_scale)[0]  # [Hkv, L, nb]
    out = np.full((sc.shape[0], topk), -1, dtype=np.int32)
    force = None if force_block is None else np.array([force_block])
    for h in range(sc.shape[0]):
        acc = np.zeros(nb, dtype=_F32)
        for t in range(L):
            acc = (acc + sc[h, t]).astype(_F32)
        out[h] = _topk_lowest_id(acc[None], topk, force)[0]
    return torch.from_numpy(out)


def _gate_slices(z, i, h, H, D, per_head):
    """Gate of branch ``i`` for head ``h``: per head one column ``i*H + h``
    broadcast over D; per channel the D columns of the head
    (spatial_sparse_attention.py:257-269)."""
    if per_head:
        return z[:, i * H + h : i * H + h + 1]
    C = H * D
    return z[:, i * C + h * D : i * C + (h + 1) * D]


def _res_block_tokens(x, w):
    """SparseResBlock on tokens (residual_block.py:16-34) in x's dtype."""
    w1, b1, w2, b2 = (t.to(x.dtype) for t in w)
    h = torch.nn.functional.linear(torch.nn.functional.silu(torch.nn.functional.linear(x, w1, b1)), w2, b2)
    y = x + h
    return torch.nn.functional.layer_norm(y, (y.shape[-1],), eps=1e-5)


def three_branch_masked_dense(q, k, v, x, gate_w, g, cu_blk, block_topk, window: int, per_head: bool = True,
                              compress=None, softmax_scale=None, dtype=torch.float64):
    """The three-branch op on one sequence as masked DENSE attention, forward
    and backward, with autograd in ``dtype`` (the BASELINE config-1 check).

    * compression: ``compress=None`` block mean of K/V
      (spatial_sparse_attention.py:27-37); else ``{"k": (w1, b1, w2, b2),
      "v": (...)}`` runs the token-wise ResBlock first (:46-66,
      residual_block.py:16-34);
    * compressed branch: softmax over every block of the sequence
      (spatial_sparse_attention.py:121-143), natural-log LSE kept;
    * selected branch: query i attends key j when block(j) is in
      ``block_topk[h_kv, block(i)]`` (per-query-block selection [Hkv, nb, k],
      ids of the one sequence; kvcentric.py:127-247);
    * sliding window: ``|i - j| <= window // 2``;
    * gates: ``sigmoid(x · gate_wᵀ)``, branches in the order compressed,
      selected, window (:257-269), per head or per channel.

    Loss = Σ out ⊙ g.  Returns a dict with ``out`` [N, H*D], ``lse_c`` [H, N],
    ``ck``/``cv`` [nb, Hkv, D] and the gradients ``q, k, v, x, gate_w``,
    ``dck``/``dcv`` (and ``compress_k`` / ``compress_v`` weight-gradient
    tuples).  Each head's dense
    [N, N] work is checkpointed, so memory stays at one head's matrices."""
    from torch.utils.checkpoint import checkpoint

    N, H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    cb = _i(cu_blk)
    nb = len(cb) - 1
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    lens = torch.tensor(np.diff(np.array(cb)), dtype=dtype)
    blk_of = torch.repeat_interleave(torch.arange(nb), lens.long())
    leaf = lambda t: t.detach().to(dtype).requires_grad_()  # noqa: E731
    qd, kd, vd, xd, wd = leaf(q), leaf(k), leaf(v), leaf(x), leaf(gate_w)
    cw = None
    if compress is not None:
        cw = {s: tuple(leaf(t) for t in compress[s]) for s in ("k", "v")}
        kc = _res_block_tokens(kd.reshape(N, -1), cw["k"]).view(N, Hkv, D)
        vc = _res_block_tokens(vd.reshape(N, -1), cw["v"]).view(N, Hkv, D)
    else:
        kc, vc = kd, vd
    ck = torch.zeros(nb, Hkv, D, dtype=dtype).index_add(0, blk_of, kc) / lens[:, None, None]
    cv = torch.zeros(nb, Hkv, D, dtype=dtype).index_add(0, blk_of, vc) / lens[:, None, None]
    ck.retain_grad()
    cv.retain_grad()
    z = torch.sigmoid(xd @ wd.t())
    bt = torch.as_tensor(block_topk).long()
    idx = torch.arange(N)
    band = (idx[:, None] - idx[None, :]).abs() <= window // 2
    allowed = []
    for hk in range(Hkv):
        a = torch.zeros(nb, nb, dtype=torch.bool)
        sel = bt[hk]
        valid = (sel >= 0) & (sel < nb)
        rows = torch.arange(nb)[:, None].expand_as(sel)
        a[rows[valid], sel[valid]] = True
        allowed.append(a)

    def head(h, qh, kh, vh, ckh, cvh, zz):
        sc = (qh @ ckh.t()) * scale
        lse = torch.logsumexp(sc, -1)
        o_c = torch.softmax(sc, -1) @ cvh
        s = (qh @ kh.t()) * scale
        m_sel = allowed[h // G][blk_of][:, blk_of]
        o_s = torch.softmax(s.masked_fill(~m_sel, -math.inf), -1) @ vh
        o_w = torch.softmax(s.masked_fill(~band, -math.inf), -1) @ vh
        out = sum(_gate_slices(zz, i, h, H, D, per_head) * o for i, o in enumerate((o_c, o_s, o_w)))
        return out, lse

    outs, lses = [], []
    for h in range(H):
        hk = h // G
        o, l = checkpoint(head, h, qd[:, h], kd[:, hk], vd[:, hk], ck[:, hk], cv[:, hk], z, use_reentrant=False)
        outs.append(o)
        lses.append(l)
    out = torch.stack(outs, 1).reshape(N, H * D)
    loss = (out * torch.as_tensor(g).to(dtype)).sum()
    loss.backward()
    res = dict(out=out.detach(), lse_c=torch.stack(lses).detach(), ck=ck.detach(), cv=cv.detach(), q=qd.grad,
               k=kd.grad, v=vd.grad, x=xd.grad, gate_w=wd.grad, dck=ck.grad, dcv=cv.grad)
    if cw is not None:
        res["compress_k"] = tuple(t.grad for t in cw["k"])
        res["compress_v"] = tuple(t.grad for t in cw["v"])
    return res


def three_branch_sampled(q, k, v, x, gate_w, g, cu_blk, block_topk, qblock_ids, window: int, ck, cv,
                         per_head: bool = True, softmax_scale=None, dtype=torch.float32):
    """Forward and backward of the three-branch op for the query blocks
    ``qblock_ids`` only (loss = Σ over their rows of out ⊙ g), keys gathered
    per query block and head, autograd in ``dtype``.  Same branches and gate
    rule as :func:`three_branch_masked_dense`; the compressed keys/values
    ``ck``/``cv`` [nb, Hkv, D] are inputs (their gradients are returned, so a
    caller maps them back through its compression), ``block_topk`` [Hkv, nb,
    k] the per-query-block selection.

    Returns a dict: ``rows`` (token ids of the sampled blocks, block order),
    ``out`` [R, H*D], ``q`` [R, H, D] and ``x`` [R, hidden] (gradients of those
    rows; every other row's gradient is zero), ``gate_w``, ``ck``/``cv``
    (gradients [nb, Hkv, D]), ``k_direct``/``v_direct`` [N, Hkv, D] (the
    gradients through the selected and window branches, without the
    compression path), ``lse_c`` [H, R]."""
    N, H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    cb = _i(cu_blk)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    half = window // 2
    bt = torch.as_tensor(block_topk).long()
    ckl = ck.detach().to(dtype).requires_grad_()
    cvl = cv.detach().to(dtype).requires_grad_()
    wl = gate_w.detach().to(dtype).requires_grad_()
    gt = torch.as_tensor(g)
    kd_direct = torch.zeros(N, Hkv, D, dtype=dtype)
    vd_direct = torch.zeros(N, Hkv, D, dtype=dtype)
    rows, outs, dqs, dxs, lses = [], [], [], [], []
    for qb in qblock_ids:
        r0, r1 = cb[qb], cb[qb + 1]
        L = r1 - r0
        qq = q[r0:r1].detach().to(dtype).requires_grad_()
        xx = x[r0:r1].detach().to(dtype).requires_grad_()
        z = torch.sigmoid(xx @ wl.t())
        k0, k1 = max(0, r0 - half), min(N, r1 + half)
        ii = torch.arange(r0, r1)[:, None]
        jj = torch.arange(k0, k1)[None, :]
        band = (ii - jj).abs() <= half
        leaves = []
        out = torch.zeros(L, H * D, dtype=dtype)
        lse_b = []
        for hk in range(Hkv):
            sel = [int(b) for b in bt[hk, qb] if 0 <= int(b) < len(cb) - 1]
            keys = torch.cat([torch.arange(cb[b], cb[b + 1]) for b in sel]) if sel else torch.zeros(0, dtype=torch.long)
            ks = k[keys, hk].detach().to(dtype).requires_grad_()
            vs = v[keys, hk].detach().to(dtype).requires_grad_()
            kw = k[k0:k1, hk].detach().to(dtype).requires_grad_()
            vw = v[k0:k1, hk].detach().to(dtype).requires_grad_()
            leaves.append((keys, ks, vs, kw, vw, hk))
            for h in range(hk * G, (hk + 1) * G):
                qh = qq[:, h]
                sc = (qh @ ckl[:, hk].t()) * scale
                lse_b.append(torch.logsumexp(sc, -1))
                o_c = torch.softmax(sc, -1) @ cvl[:, hk]
                o_s = torch.softmax((qh @ ks.t()) * scale, -1) @ vs
                sw = ((qh @ kw.t()) * scale).masked_fill(~band, -math.inf)
                o_w = torch.softmax(sw, -1) @ vw
                o_h = sum(_gate_slices(z, i, h, H, D, per_head) * o for i, o in enumerate((o_c, o_s, o_w)))
                out = out.index_copy(1, torch.arange(h * D, (h + 1) * D), o_h)
        loss = (out * gt[r0:r1].to(dtype)).sum()
        loss.backward()
        for keys, ks, vs, kw, vw, hk in leaves:
            kd_direct[:, hk].index_add_(0, keys, ks.grad)
            vd_direct[:, hk].index_add_(0, keys, vs.grad)
            kd_direct[k0:k1, hk] += kw.grad
            vd_direct[k0:k1, hk] += vw.grad
        rows.append(torch.arange(r0, r1))
        outs.append(out.detach())
        dqs.append(qq.grad)
        dxs.append(xx.grad)
        lses.append(torch.stack(lse_b).detach())
    return dict(rows=torch.cat(rows), out=torch.cat(outs), q=torch.cat(dqs), x=torch.cat(dxs), gate_w=wl.grad,
                ck=ckl.grad, cv=cvl.grad, k_direct=kd_direct, v_direct=vd_direct, lse_c=torch.cat(lses, 1))


def compress_vjp(x_rows, dy_rows, weights=None, dtype=torch.float32):
    """Gradient of the token-wise compression input for some token rows:
    identity for the block mean (``weights=None``); the ResBlock's vector-
    Jacobian product (residual_block.py:16-34) otherwise.  ``dy_rows`` is the
    gradient of the compressed per-token values (for the block mean of block b
    that is dck[b] / L_b on each of b's tokens).  Returns (dx_rows, weight
    gradients or None)."""
    if weights is None:
        return dy_rows.to(dtype), None
    xl = x_rows.detach().to(dtype).requires_grad_()
    wl = tuple(t.detach().to(dtype).requires_grad_() for t in weights)
    y = _res_block_tokens(xl, wl)
    y.backward(dy_rows.to(dtype))
    return xl.grad, tuple(t.grad for t in wl)


def compress_forward(x_rows, weights=None, dtype=torch.float32):
    """Token-wise compression values (before the block mean): x itself, or
    the ResBlock output."""
    xr = x_rows.detach().to(dtype)
    return xr if weights is None else _res_block_tokens(xr, tuple(t.to(dtype) for t in weights))


# ---------------------------------------------------------------------------
# block metadata
# ---------------------------------------------------------------------------


def volume_sort_keys(coords, volume_res: int, block_size: int) -> np.ndarray:
    """Key of ``sort_volume_blocks`` (misc/sparse_utils.py:126-152): batch,
    block cell (z, y, x) and position inside the cell, most significant
    first; int64."""
    c = np.asarray(coords, dtype=np.int64)
    r, b = int(volume_res), int(block_size)
    blk, inb = c[:, 1:] // b, c[:, 1:] % b
    return (r ** 3 * c[:, 0] + r * r * b * blk[:, 0] + r * b * b * blk[:, 1] + b ** 3 * blk[:, 2]
            + b * b * inb[:, 0] + b * inb[:, 1] + inb[:, 2])


def block_separation(coords, dim: int, block_size, batch: int, resolution):
    """``compute_block_separation`` (misc/sparse_utils.py:592-641): per batch
    element, the token count of every non-empty cell (histogram over
    [0, cells), flattened with the first coordinate most significant; ids
    outside the range are not counted, as torch.histc ignores them).
    Returns ``(cu_seqblocks, cu_block_include_tokens)`` int32."""
    c = np.asarray(coords, dtype=np.int64)
    cells_per = [int(resolution[d]) // int(block_size[d]) for d in range(dim)]
    cells = int(np.prod(cells_per))
    mult = [int(np.prod(cells_per[d + 1:])) for d in range(dim)]
    counts, seqblocks = [], []
    for b in range(batch):
        cb = c[c[:, 0] == b]
        flat = np.zeros(cb.shape[0], dtype=np.int64)
        for d in range(dim):
            flat += (cb[:, 1 + d] // int(block_size[d])) * mult[d]
        flat = flat[(flat >= 0) & (flat < cells)]
        h = np.bincount(flat, minlength=cells)
        nz = h[h > 0]
        counts.append(nz)
        seqblocks.append(len(nz))
    cu_sb = np.concatenate([[0], np.cumsum(seqblocks)]).astype(np.int32)
    allc = np.concatenate(counts) if counts else np.zeros(0, np.int64)
    cu_blk = np.concatenate([[0], np.cumsum(allc)]).astype(np.int32)
    return cu_sb, cu_blk


def prepare_volume_output(volume, volume_index, output_dim: int, upsample_scale: int, vol_res: int,
                          batch_size: Optional[int] = None):
    """``VolTransformer.prepare_volume_output`` (models_sparse/voldecoder.py:
    196-268), restated in numpy with explicit loops over tokens and
    sub-voxels.  ``volume`` [N, C * u^3] (token i's features channel-major,
    element c * u^3 + s), ``volume_index`` [N, 4] (batch, z, y, x) grouped by
    batch.  Sub-voxel s = (dz * u + dy) * u + dx (:210-230, meshgrid "ij").
    Returns ``(sparse_feat [N * u^3, C], cu_seqlens, seqlens,
    index_volume [B, R*u, R*u, R*u])``; batch boundaries are where the batch
    id changes (:232-241), scaled by u^3 (:242); the index volume holds the
    sub-voxel's row inside its sequence, -1 elsewhere (:246-259)."""
    vol = np.asarray(volume)
    vi = np.asarray(volume_index).astype(np.int64)
    n = vi.shape[0]
    u = int(upsample_scale)
    S = u ** 3
    C = int(output_dim)
    B = int(vi[:, 0].max()) + 1 if batch_size is None else int(batch_size)
    feat = vol.reshape(n, C, S).transpose(0, 2, 1).reshape(n * S, C).copy()
    starts = [0] + [i for i in range(1, n) if vi[i, 0] != vi[i - 1, 0]] + [n]
    cu = np.array(starts, dtype=np.int64) * S
    cu = cu.astype(np.int32)
    seqlens = (cu[1:] - cu[:-1]).astype(np.int32)
    R = int(vol_res) * u
    index_volume = np.full((B, R, R, R), -1, dtype=np.int32)
    for b in range(B):
        t0, t1 = int(cu[b]) // S, int(cu[b + 1]) // S
        for i in range(t0, t1):
            for s in range(S):
                dz, dy, dx = s // (u * u), (s // u) % u, s % u
                index_volume[b, vi[i, 1] * u + dz, vi[i, 2] * u + dy, vi[i, 3] * u + dx] = (i - t0) * S + s
    return feat, cu, seqlens, index_volume


def volume_block_topk(coords, cu_seqblocks, cu_block_include_tokens, batch: int, volume_res: int,
                      bbox_radius: float, topk: int, return_geometry: bool = False, rows=None):
    """The geometric block selection of ``build_volume_to_volume_attn`` with
    ``use_3d_aware_attn`` (misc/sparse_utils.py:1203-1279), one row per token
    (the reference stacks the result twice, :1270).  ``coords`` [n, 4]
    (batch, z, y, x) sorted by block (the separation's order).  In fp32, in the
    reference's order: point = 2 * (c / (res - 1) - 0.5) * r with
    r = bbox_radius * 1.05 and (x, y, z) from columns 3, 2, 1 (:644-650);
    block centre = sequential sum of its points / count (segment_reduce mean,
    :1238-1243); d^2 = (dx^2 + dy^2) + dz^2 (:1245-1249).  Blocks are ranked
    by d^2, ties to the lower id (the reference ranks sqrt(d^2) with
    torch.topk), the first ``topk`` ids sorted ascending, -1 padding (:1250-1266).
    ``return_geometry`` also returns the points and block centres; ``rows``
    (token indices) evaluates only those tokens (centres still from all)."""
    c = np.asarray(coords).astype(np.int64)
    cu_sb = np.asarray(cu_seqblocks).astype(np.int64)
    cu_blk = np.asarray(cu_block_include_tokens).astype(np.int64)
    f32 = np.float32
    r = f32(bbox_radius * 1.05)
    den = f32(volume_res - 1)

    def pt(v):
        return (f32(2.0) * ((v.astype(f32) / den).astype(f32) - f32(0.5))).astype(f32) * r

    pts = np.stack([pt(c[:, 3]), pt(c[:, 2]), pt(c[:, 1])], 1).astype(f32)
    nb_all = int(cu_sb[batch])
    cent = np.zeros((nb_all, 3), f32)
    for j in range(nb_all):
        acc = np.zeros(3, f32)
        for t in range(int(cu_blk[j]), int(cu_blk[j + 1])):
            acc = (acc + pts[t]).astype(f32)
        cent[j] = (acc / f32(cu_blk[j + 1] - cu_blk[j])).astype(f32)
    rows = range(c.shape[0]) if rows is None else [int(x) for x in rows]
    out = np.full((len(rows), topk), -1, dtype=np.int32)
    for o, t in enumerate(rows):
        b = int(c[t, 0])
        b0, b1 = int(cu_sb[b]), int(cu_sb[b + 1])
        d = (pts[t][None, :] - cent[b0:b1]).astype(f32)
        sq = (d * d).astype(f32)
        d2 = ((sq[:, 0] + sq[:, 1]).astype(f32) + sq[:, 2]).astype(f32)
        order = np.lexsort((np.arange(b1 - b0), d2))[:topk]
        sel = np.sort(order)
        out[o, : sel.size] = sel
    return (out, pts, cent) if return_geometry else out
