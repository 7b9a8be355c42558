"""Backward of the selected-block and dense-branch attention on the GPU vs the
reference fixtures and the float64 oracle (autograd)."""

import zlib

import pytest
import torch

import oracle
from tests.cases import coherent_selection, cu, expand_qblock_selection, random_problem
from tests.golden.make_golden import selection_cases

pytestmark = pytest.mark.gpu

ATOL_BF16 = 2e-2  # max-abs, gradients in bf16 (dO ~ N(0, 0.1))
COS_MIN = 0.9995


def _cos(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def _oracle_grads(p, bt_tok, do):
    q = p["q"].double().requires_grad_()
    k = p["k"].double().requires_grad_()
    v = p["v"].double().requires_grad_()
    o, _ = oracle.selection_attention(q, k, v, bt_tok, p["cu_seqblocks"], p["cu_blk"], p["cu_seqlens"],
                                      p["cu_seqlens"])
    ok = ~torch.isnan(o).any(-1)
    (o[ok] * do.double()[ok]).sum().backward()
    return q.grad, k.grad, v.grad


def _check(got, ref, what):
    got = got.float().cpu()
    err = (got - ref.float()).abs().max().item()
    assert err < ATOL_BF16, f"{what}: max-abs {err}"
    assert _cos(got, ref) >= COS_MIN, f"{what}: cosine {_cos(got, ref)}"


@pytest.mark.parametrize("name", [c[0] for c in selection_cases() if c[0] != "sel_dup_and_empty"])
def test_select_bwd_matches_reference_fixture(golden, name):
    from lsrm_sparse import ops

    g = golden(name)
    dev = "cuda"
    q, k, v, do = (torch.from_numpy(g[n]).half().to(dev) for n in ("q", "k", "v", "do"))
    cus = [torch.from_numpy(g[n]).to(dev) for n in ("cu_seqlens", "cu_seqlens", "cu_seqblocks",
                                                     "cu_block_include_tokens")]
    meta = ops.Meta(*cus)
    bt = torch.from_numpy(g["block_topk"]).to(dev)
    out, lse, ws = ops.select_attn_fwd(q, k, v, bt, meta)
    dq, dk, dv = ops.select_attn_bwd(q, k, v, out, lse, do, bt, meta, workspace=ws)
    assert ops.read_errors() == 0
    for nm, t in (("dq", dq), ("dk", dk), ("dv", dv)):
        ref = torch.from_numpy(g[nm])
        assert (t.float().cpu() - ref).abs().max() < 3e-3, nm


CASES = [
    # name, seq_block_lens, Hq, Hkv, D, topk, qblock, pad
    ("mha_d64", [[40, 70, 33, 90, 64, 21, 128, 55]], 2, 2, 64, 3, False, 0.0),
    ("gqa16_d32_small_blocks", [[5, 8, 3, 7, 8, 2, 6, 8, 8, 1, 4, 8] * 3], 32, 2, 32, 6, False, 0.2),
    ("g4_d64_two_seqs", [[100, 150, 30], [64, 64, 200, 17, 90]], 8, 2, 64, 2, False, 0.3),
    ("qblock_mha_d64", [[64, 256, 100, 130, 77, 190, 64]], 2, 2, 64, 3, True, 0.0),
    ("g2_d32_long_blocks", [[300, 129, 7, 260]], 4, 2, 32, 2, False, 0.0),
    ("mha_d64_many_tiles", [[96] * 24], 1, 1, 64, 4, False, 0.0),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_select_bwd_vs_oracle(case):
    from lsrm_sparse import ops

    name, sbl, Hq, Hkv, D, topk, qblock, pad = case
    p = random_problem(zlib.crc32(name.encode()) % 1000, sbl, Hq, Hkv, D, topk, pad_frac=pad, qblock=qblock)
    gen = torch.Generator().manual_seed(5)
    do = (torch.randn(p["q"].shape, generator=gen) * 0.1).bfloat16()
    dev = "cuda"
    meta = ops.Meta(p["cu_seqlens"].to(dev), p["cu_seqlens"].to(dev), p["cu_seqblocks"].to(dev), p["cu_blk"].to(dev))
    bt = p["block_topk"]
    cqb = p["cu_blk"].to(dev) if qblock else None
    q, k, v = p["q"].to(dev), p["k"].to(dev), p["v"].to(dev)
    out, lse, ws = ops.select_attn_fwd(q, k, v, bt.to(dev), meta, cu_query_blocks=cqb)
    dq, dk, dv = ops.select_attn_bwd(q, k, v, out, lse, do.to(dev), bt.to(dev), meta, cu_query_blocks=cqb,
                                     workspace=ws)
    assert ops.read_errors() == 0
    bt_tok = expand_qblock_selection(bt, p["cu_blk"]) if qblock else bt
    rq, rk, rv = _oracle_grads(p, bt_tok, do)
    _check(dq, rq, "dq")
    _check(dk, rk, "dk")
    _check(dv, rv, "dv")


def test_select_bwd_is_deterministic():
    from lsrm_sparse import ops

    p = random_problem(11, [[64, 33, 128, 90, 17, 200] * 3], 4, 1, 64, 5)
    dev = "cuda"
    bt = coherent_selection(12, p["cu_seqlens"], p["cu_seqblocks"], 1, 5)
    meta = ops.Meta(p["cu_seqlens"].to(dev), p["cu_seqlens"].to(dev), p["cu_seqblocks"].to(dev), p["cu_blk"].to(dev))
    q, k, v = p["q"].to(dev), p["k"].to(dev), p["v"].to(dev)
    do = (torch.randn(q.shape, device=dev) * 0.1).bfloat16()
    out, lse, ws = ops.select_attn_fwd(q, k, v, bt.to(dev), meta)
    g1 = ops.select_attn_bwd(q, k, v, out, lse, do, bt.to(dev), meta, workspace=ws)
    g2 = ops.select_attn_bwd(q, k, v, out, lse, do, bt.to(dev), meta)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def _dense_oracle(fn, q, k, v, do, *args):
    qd, kd, vd = (t.double().requires_grad_() for t in (q, k, v))
    o = fn(qd, kd, vd, *args)
    if isinstance(o, tuple):
        o = o[0]
    (o * do.double()).sum().backward()
    return qd.grad, kd.grad, vd.grad


@pytest.mark.parametrize("D,Hq,Hkv", [(64, 4, 4), (32, 8, 2)])
def test_compressed_bwd_vs_oracle(D, Hq, Hkv):
    from lsrm_sparse import ops

    g = torch.Generator().manual_seed(D + Hq)
    seq_q = [3000, 17, 5200]
    seq_nb = [40, 3, 150]
    cq, cb = cu(seq_q), cu(seq_nb)
    q = torch.randn(sum(seq_q), Hq, D, generator=g).bfloat16()
    ck = torch.randn(sum(seq_nb), Hkv, D, generator=g).bfloat16()
    cv = torch.randn(sum(seq_nb), Hkv, D, generator=g).bfloat16()
    do = (torch.randn(q.shape, generator=g) * 0.1).bfloat16()
    dev = "cuda"
    meta = ops.Meta(cq.to(dev), cq.to(dev), cb.to(dev), torch.arange(sum(seq_nb) + 1, dtype=torch.int32).to(dev))
    out, lse = ops.dense_attn_fwd(q.to(dev), ck.to(dev), cv.to(dev), meta, ops.DENSE_COMPRESSED)
    dq, dk, dv = ops.dense_attn_bwd(q.to(dev), ck.to(dev), cv.to(dev), out, lse, do.to(dev), meta,
                                    ops.DENSE_COMPRESSED)
    assert ops.read_errors() == 0
    rq, rk, rv = _dense_oracle(oracle.compressed_attention, q, ck, cv, do, cq, cb)
    _check(dq, rq, "dq")
    # compressed keys collect thousands of queries: compare with a relative bound
    for nm, got, ref in (("dk", dk, rk), ("dv", dv, rv)):
        scale = ref.abs().max().item()
        assert (got.float().cpu() - ref).abs().max().item() < max(ATOL_BF16, 1e-2 * scale), nm
        assert _cos(got.float().cpu(), ref) >= COS_MIN, nm


def test_intra_block_window_bwd_vs_oracle():
    from lsrm_sparse import ops

    p = random_problem(3, [[5, 130, 64, 1, 200, 90], [12, 300]], 4, 2, 64, 1)
    gen = torch.Generator().manual_seed(9)
    do = (torch.randn(p["q"].shape, generator=gen) * 0.1).bfloat16()
    dev = "cuda"
    meta = ops.Meta(p["cu_seqlens"].to(dev), p["cu_seqlens"].to(dev), p["cu_seqblocks"].to(dev), p["cu_blk"].to(dev))
    q, k, v = p["q"].to(dev), p["k"].to(dev), p["v"].to(dev)
    out, lse = ops.dense_attn_fwd(q, k, v, meta, ops.DENSE_INTRA_BLOCK)
    dq, dk, dv = ops.dense_attn_bwd(q, k, v, out, lse, do.to(dev), meta, ops.DENSE_INTRA_BLOCK)
    assert ops.read_errors() == 0
    rq, rk, rv = _dense_oracle(oracle.window_attention_intra_block, p["q"], p["k"], p["v"], do, p["cu_blk"])
    _check(dq, rq, "dq")
    _check(dk, rk, "dk")
    _check(dv, rv, "dv")


@pytest.mark.parametrize("window", [128, 512])
def test_sliding_window_bwd_vs_oracle(window):
    from lsrm_sparse import ops

    p = random_problem(4, [[100] * 9, [50, 77]], 2, 2, 64, 1)
    gen = torch.Generator().manual_seed(10)
    do = (torch.randn(p["q"].shape, generator=gen) * 0.1).bfloat16()
    dev = "cuda"
    meta = ops.Meta(p["cu_seqlens"].to(dev), p["cu_seqlens"].to(dev), p["cu_seqblocks"].to(dev), p["cu_blk"].to(dev))
    q, k, v = p["q"].to(dev), p["k"].to(dev), p["v"].to(dev)
    out, lse = ops.dense_attn_fwd(q, k, v, meta, ops.DENSE_SLIDING, window)
    dq, dk, dv = ops.dense_attn_bwd(q, k, v, out, lse, do.to(dev), meta, ops.DENSE_SLIDING, window)
    assert ops.read_errors() == 0
    rq, rk, rv = _dense_oracle(oracle.sliding_window_attention, p["q"], p["k"], p["v"], do, p["cu_seqlens"], window)
    _check(dq, rq, "dq")
    _check(dk, rk, "dk")
    _check(dv, rv, "dv")
