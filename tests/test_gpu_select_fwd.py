"""Selected-block and dense-branch attention forward on the GPU vs the
reference fixtures and the CPU oracle."""

import math
import zlib

import numpy as np
import pytest
import torch

import oracle
from tests.cases import coherent_selection, cu, expand_qblock_selection, random_problem
from tests.golden.make_golden import selection_cases

pytestmark = pytest.mark.gpu

# BASELINE tolerances: bf16 outputs within 2e-2 max-abs and cosine >= 0.9995
ATOL_BF16 = 2e-2
COS_MIN = 0.9995


def _cos(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def _meta(p, ops):
    return ops.Meta(p["cu_seqlens"], p["cu_seqlens"], p["cu_seqblocks"], p["cu_blk"])


@pytest.mark.parametrize("name", [c[0] for c in selection_cases() if c[0] != "sel_dup_and_empty"])
def test_select_fwd_matches_reference_fixture(golden, name):
    from lsrm_sparse import ops

    g = golden(name)
    dev = "cuda"
    q = torch.from_numpy(g["q"]).half().to(dev)
    k = torch.from_numpy(g["k"]).half().to(dev)
    v = torch.from_numpy(g["v"]).half().to(dev)
    meta = ops.Meta(*(torch.from_numpy(g[n]).to(dev) for n in ("cu_seqlens", "cu_seqlens", "cu_seqblocks",
                                                             "cu_block_include_tokens")))
    bt = torch.from_numpy(g["block_topk"]).to(dev)
    out, lse, _ = ops.select_attn_fwd(q, k, v, bt, meta)
    assert ops.read_errors() == 0
    ref_o = torch.from_numpy(g["o"])
    ref_l = torch.from_numpy(g["lse_log2"])
    assert (out.float().cpu() - ref_o).abs().max() < 2e-3
    assert (lse.cpu() - ref_l).abs().max() < 2e-3


def test_select_fwd_duplicate_block_is_rejected(golden):
    from lsrm_sparse import ops

    g = golden("sel_dup_and_empty")
    dev = "cuda"
    q = torch.from_numpy(g["q"]).half().to(dev)
    k = torch.from_numpy(g["k"]).half().to(dev)
    v = torch.from_numpy(g["v"]).half().to(dev)
    meta = ops.Meta(*(torch.from_numpy(g[n]).to(dev) for n in ("cu_seqlens", "cu_seqlens", "cu_seqblocks",
                                                             "cu_block_include_tokens")))
    ops.read_errors()
    ops.select_attn_fwd(q, k, v, torch.from_numpy(g["block_topk"]).to(dev), meta)
    assert ops.read_errors() & 0x2  # LSRM_ERR_DUPLICATE_BLOCK


def test_select_fwd_empty_selection_row_is_nan(golden):
    from lsrm_sparse import ops

    g = golden("sel_dup_and_empty")
    bt = torch.from_numpy(g["block_topk"]).clone()
    bt[0, 3] = torch.tensor([2, 4, -1])  # remove the duplicates, keep the empty row 7
    bt[0, 5] = torch.tensor([1, 3, -1])
    dev = "cuda"
    q, k, v = (torch.from_numpy(g[n]).half().to(dev) for n in ("q", "k", "v"))
    cus = [torch.from_numpy(g[n]) for n in ("cu_seqlens", "cu_seqlens", "cu_seqblocks", "cu_block_include_tokens")]
    meta = ops.Meta(*(c.to(dev) for c in cus))
    out, lse, _ = ops.select_attn_fwd(q, k, v, bt.to(dev), meta)
    assert ops.read_errors() == 0
    ref_o, ref_l = oracle.selection_attention(q.cpu(), k.cpu(), v.cpu(), bt, cus[2], cus[3], cus[0], cus[1])
    nan_ref = torch.isnan(ref_o).any(-1)
    nan_got = torch.isnan(out.float().cpu()).any(-1)
    assert torch.equal(nan_ref, nan_got) and nan_ref.any()
    assert torch.equal(torch.isneginf(ref_l), torch.isneginf(lse.cpu()))
    ok = ~nan_ref
    assert (out.float().cpu()[ok] - ref_o[ok]).abs().max() < 2e-3


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
def test_select_fwd_vs_oracle(case):
    from lsrm_sparse import ops

    name, sbl, Hq, Hkv, D, topk, qblock, pad = case
    p = random_problem(zlib.crc32(name.encode()) % 1000, sbl, Hq, Hkv, D, topk, pad_frac=pad, qblock=qblock)
    dev = "cuda"
    meta = _meta({k: v.to(dev) for k, v in p.items() if torch.is_tensor(v)}, ops)
    bt = p["block_topk"]
    cqb = p["cu_blk"].to(dev) if qblock else None
    out, lse, _ = ops.select_attn_fwd(p["q"].to(dev), p["k"].to(dev), p["v"].to(dev), bt.to(dev), meta,
                                      cu_query_blocks=cqb)
    assert ops.read_errors() == 0
    bt_tok = expand_qblock_selection(bt, p["cu_blk"]) if qblock else bt
    ref_o, ref_l = oracle.selection_attention(p["q"], p["k"], p["v"], bt_tok, p["cu_seqblocks"], p["cu_blk"],
                                              p["cu_seqlens"], p["cu_seqlens"])
    got = out.float().cpu()
    assert (got - ref_o).abs().max() < ATOL_BF16, (got - ref_o).abs().max()
    assert _cos(got, ref_o) >= COS_MIN
    assert (lse.cpu() - ref_l).abs().max() < 1e-2


def test_select_fwd_coherent_selection_gqa():
    from lsrm_sparse import ops

    sbl = [[37, 64, 12, 80, 45, 9, 120, 33, 70, 51]]
    p = random_problem(7, sbl, 16, 1, 64, 4)
    bt = coherent_selection(8, p["cu_seqlens"], p["cu_seqblocks"], 1, 4)
    dev = "cuda"
    meta = _meta({k: v.to(dev) for k, v in p.items() if torch.is_tensor(v)}, ops)
    out, lse, _ = ops.select_attn_fwd(p["q"].to(dev), p["k"].to(dev), p["v"].to(dev), bt.to(dev), meta)
    assert ops.read_errors() == 0
    ref_o, _ = oracle.selection_attention(p["q"], p["k"], p["v"], bt, p["cu_seqblocks"], p["cu_blk"], p["cu_seqlens"],
                                          p["cu_seqlens"])
    got = out.float().cpu()
    assert (got - ref_o).abs().max() < ATOL_BF16
    assert _cos(got, ref_o) >= COS_MIN


@pytest.mark.parametrize("D,Hq,Hkv", [(64, 4, 4), (32, 8, 2)])
def test_compressed_fwd_vs_oracle(D, Hq, Hkv):
    from lsrm_sparse import ops

    g = torch.Generator().manual_seed(D + Hq)
    seq_q = [300, 17, 520]
    seq_nb = [40, 3, 150]
    cq, cb = cu(seq_q), cu(seq_nb)
    q = torch.randn(sum(seq_q), Hq, D, generator=g).bfloat16()
    ck = torch.randn(sum(seq_nb), Hkv, D, generator=g).bfloat16()
    cv = torch.randn(sum(seq_nb), Hkv, D, generator=g).bfloat16()
    dev = "cuda"
    cu_blk_dummy = torch.arange(sum(seq_nb) + 1, dtype=torch.int32)
    meta = ops.Meta(cq.to(dev), cq.to(dev), cb.to(dev), cu_blk_dummy.to(dev))
    out, lse = ops.dense_attn_fwd(q.to(dev), ck.to(dev), cv.to(dev), meta, ops.DENSE_COMPRESSED)
    assert ops.read_errors() == 0
    ref_o, ref_l = oracle.compressed_attention(q, ck, cv, cq, cb)
    assert (out.float().cpu() - ref_o).abs().max() < ATOL_BF16
    assert (lse.cpu() - ref_l).abs().max() < 1e-2


def test_intra_block_window_fwd_vs_oracle():
    from lsrm_sparse import ops

    sbl = [[5, 130, 64, 1, 200, 90], [12, 300]]
    p = random_problem(3, sbl, 4, 2, 64, 1)
    dev = "cuda"
    meta = _meta({k: v.to(dev) for k, v in p.items() if torch.is_tensor(v)}, ops)
    out, _ = ops.dense_attn_fwd(p["q"].to(dev), p["k"].to(dev), p["v"].to(dev), meta, ops.DENSE_INTRA_BLOCK)
    assert ops.read_errors() == 0
    ref = oracle.window_attention_intra_block(p["q"], p["k"], p["v"], p["cu_blk"])
    assert (out.float().cpu() - ref).abs().max() < ATOL_BF16


@pytest.mark.parametrize("window", [128, 512])
def test_sliding_window_fwd_vs_oracle(window):
    from lsrm_sparse import ops

    sbl = [[100] * 9, [50, 77]]
    p = random_problem(4, sbl, 2, 2, 64, 1)
    dev = "cuda"
    meta = _meta({k: v.to(dev) for k, v in p.items() if torch.is_tensor(v)}, ops)
    out, _ = ops.dense_attn_fwd(p["q"].to(dev), p["k"].to(dev), p["v"].to(dev), meta, ops.DENSE_SLIDING, window)
    assert ops.read_errors() == 0
    ref = oracle.sliding_window_attention(p["q"], p["k"], p["v"], p["cu_seqlens"], window)
    assert (out.float().cpu() - ref).abs().max() < ATOL_BF16
