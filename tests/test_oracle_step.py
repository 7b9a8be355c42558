"""CPU checks of the oracle's whole-step restatements: the masked-dense form
(used for BASELINE config 1 in full) and the gathered, sampled form (used
for configs 2 and 3) agree with each other and with the per-branch oracles
that the reference fixtures pin (selection, compressed, sliding window,
gate), forward and backward, with block-mean and ResBlock compression."""

import math

import numpy as np
import pytest
import torch

import oracle
from tests.cases import cu


def _problem(seed, lens, H, Hkv, D, topk, window, per_head, resblock):
    g = torch.Generator().manual_seed(seed)
    N = sum(lens)
    nb = len(lens)
    cu_blk = cu(lens)
    q = torch.randn(N, H, D, generator=g).double()
    k = torch.randn(N, Hkv, D, generator=g).double()
    v = torch.randn(N, Hkv, D, generator=g).double()
    hidden = H * D
    x = torch.randn(N, hidden, generator=g).double()
    n_gate = 3 * H if per_head else 3 * hidden
    gw = torch.randn(n_gate, hidden, generator=g).double() / math.sqrt(hidden)
    gout = 0.1 * torch.randn(N, hidden, generator=g).double()
    bt = torch.full((Hkv, nb, topk), -1, dtype=torch.int32)
    for h in range(Hkv):
        for b in range(nb):
            others = [i for i in torch.randperm(nb, generator=g).tolist() if i != b][: topk - 1]
            bt[h, b, : len(others) + 1] = torch.tensor(sorted(others + [b]), dtype=torch.int32)
    comp = None
    if resblock:
        C = Hkv * D
        comp = {s: (torch.randn(C, C, generator=g).double() / math.sqrt(C), 0.1 * torch.randn(C, generator=g).double(),
                    torch.randn(C, C, generator=g).double() / math.sqrt(C), 0.1 * torch.randn(C, generator=g).double())
                for s in ("k", "v")}
    return dict(q=q, k=k, v=v, x=x, gw=gw, g=gout, cu_blk=cu_blk, bt=bt, comp=comp, N=N, nb=nb, H=H, Hkv=Hkv, D=D,
                window=window, per_head=per_head)


CASES = [
    dict(seed=1, lens=[40, 70, 33, 90, 64, 21, 55, 47], H=4, Hkv=2, D=16, topk=3, window=64, per_head=True,
         resblock=False),
    dict(seed=2, lens=[30, 17, 64, 45, 8, 90, 33], H=2, Hkv=2, D=16, topk=4, window=32, per_head=False,
         resblock=True),
]


@pytest.mark.parametrize("case", CASES)
def test_masked_dense_step_matches_per_branch_oracles(case):
    p = _problem(**case)
    r = oracle.three_branch_masked_dense(p["q"], p["k"], p["v"], p["x"], p["gw"], p["g"], p["cu_blk"], p["bt"],
                                         p["window"], p["per_head"], p["comp"])
    N, H, D, nb = p["N"], p["H"], p["D"], p["nb"]
    cb = p["cu_blk"]
    ck = oracle.compress_kv(p["k"].reshape(N, -1), cb, p["comp"]["k"] if p["comp"] else None).view(nb, p["Hkv"], D)
    cv = oracle.compress_kv(p["v"].reshape(N, -1), cb, p["comp"]["v"] if p["comp"] else None).view(nb, p["Hkv"], D)
    assert torch.allclose(r["ck"], ck, atol=1e-12) and torch.allclose(r["cv"], cv, atol=1e-12)
    cq = torch.tensor([0, N], dtype=torch.int32)
    cs = torch.tensor([0, nb], dtype=torch.int32)
    o_c, lse = oracle.compressed_attention(p["q"], ck, cv, cq, cs)
    assert torch.allclose(r["lse_c"], lse, atol=1e-10)
    per_tok = p["bt"][:, torch.repeat_interleave(torch.arange(nb), (cb[1:] - cb[:-1]).long())]
    o_s, _ = oracle.selection_attention(p["q"], p["k"], p["v"], per_tok, cs, cb, cq, cq)
    o_w = oracle.sliding_window_attention(p["q"], p["k"], p["v"], cq, p["window"])
    mode = "per_head" if p["per_head"] else "per_channel"
    ref = oracle.gate_merge(p["x"], p["gw"], [o.reshape(N, -1) for o in (o_c, o_s, o_w)], mode, H)
    assert torch.allclose(r["out"], ref, atol=1e-10)


@pytest.mark.parametrize("case", CASES)
def test_sampled_step_equals_masked_dense_on_all_blocks(case):
    p = _problem(**case)
    N, nb, D = p["N"], p["nb"], p["D"]
    dense = oracle.three_branch_masked_dense(p["q"], p["k"], p["v"], p["x"], p["gw"], p["g"], p["cu_blk"], p["bt"],
                                             p["window"], p["per_head"], p["comp"])
    s = oracle.three_branch_sampled(p["q"], p["k"], p["v"], p["x"], p["gw"], p["g"], p["cu_blk"], p["bt"],
                                    list(range(nb)), p["window"], dense["ck"], dense["cv"], p["per_head"],
                                    dtype=torch.float64)
    assert torch.equal(s["rows"], torch.arange(N))
    assert torch.allclose(s["out"], dense["out"], atol=1e-10)
    assert torch.allclose(s["lse_c"], dense["lse_c"], atol=1e-10)
    for name in ("q", "x", "gate_w"):
        assert torch.allclose(s[name], dense[name], atol=1e-9), name
    lens = (p["cu_blk"][1:] - p["cu_blk"][:-1]).double()
    blk_of = torch.repeat_interleave(torch.arange(nb), lens.long())
    for name, dc in (("k", s["ck"]), ("v", s["cv"])):
        dy = (dc / lens[:, None, None])[blk_of].reshape(N, -1)
        w = p["comp"][name] if p["comp"] else None
        dx, dw = oracle.compress_vjp(p[name].reshape(N, -1), dy, w, dtype=torch.float64)
        full = s[name + "_direct"] + dx.view_as(s[name + "_direct"])
        assert torch.allclose(full, dense[name], atol=1e-9), name
        if w is not None:
            for a, b in zip(dw, dense["compress_" + name]):
                assert torch.allclose(a, b, atol=1e-9)


def test_sampled_step_on_a_subset_only_counts_its_rows():
    p = _problem(**CASES[0])
    N, nb = p["N"], p["nb"]
    subset = [1, 4, 6]
    mask = torch.zeros(N, 1, dtype=torch.float64)
    cb = p["cu_blk"]
    for b in subset:
        mask[cb[b]:cb[b + 1]] = 1
    dense = oracle.three_branch_masked_dense(p["q"], p["k"], p["v"], p["x"], p["gw"], p["g"] * mask, cb, p["bt"],
                                             p["window"], p["per_head"])
    s = oracle.three_branch_sampled(p["q"], p["k"], p["v"], p["x"], p["gw"], p["g"], cb, p["bt"], subset,
                                    p["window"], dense["ck"], dense["cv"], p["per_head"], dtype=torch.float64)
    assert torch.allclose(s["out"], dense["out"][s["rows"]], atol=1e-10)
    assert torch.allclose(s["q"], dense["q"][s["rows"]], atol=1e-10)
    others = torch.ones(N, dtype=torch.bool)
    others[s["rows"]] = False
    assert dense["q"][others].abs().max() == 0
    assert torch.allclose(s["gate_w"], dense["gate_w"], atol=1e-9)


def test_single_block_selection_equals_the_sequence_scorer():
    """qblock_selection_exact on one query block is the per-query-block exact
    scorer's row for that block (same fixed float32 order)."""
    g = torch.Generator().manual_seed(5)
    lens = [20, 33, 12, 9, 40, 16, 25]
    N, nb, Hq, Hkv, D = sum(lens), len(lens), 4, 2, 32
    cb = cu(lens)
    q = torch.randn(N, Hq, D, generator=g).bfloat16()
    ck = torch.randn(nb, Hkv, D, generator=g).bfloat16()
    lse = torch.randn(Hq, N, generator=g).float() + 3
    cq = torch.tensor([0, N], dtype=torch.int32)
    cs = torch.tensor([0, nb], dtype=torch.int32)
    full = oracle.get_block_score_qblock_exact(q, ck, lse, 3, cq, cs, cb, force_self=True)
    for b in (0, 3, 6):
        one = oracle.qblock_selection_exact(q[cb[b]:cb[b + 1]], ck, lse[:, cb[b]:cb[b + 1]], 3, force_block=b)
        assert torch.equal(one, full[:, b]), b
    assert np.all(full.numpy() >= 0)
