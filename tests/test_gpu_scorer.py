"""Per-query-block selection: the tensor-core scorer with exact refinement
must return exactly the indices of the fixed-order exact scorer."""

import os

import numpy as np
import pytest
import torch

import oracle
from tests.cases import cu

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(seed, qb_lens, Hq, Hkv, D, dup_blocks=0):
    g = torch.Generator().manual_seed(seed)
    N = sum(qb_lens)
    nb = len(qb_lens)
    cq = torch.tensor([0, N], dtype=torch.int32)
    cc = torch.tensor([0, nb], dtype=torch.int32)
    cqb = cu(qb_lens)
    q = torch.randn(N, Hq, D, generator=g).bfloat16()
    ck = torch.randn(nb, Hkv, D, generator=g).bfloat16()
    if dup_blocks:
        ck[1:1 + dup_blocks] = ck[0:1]  # identical compressed keys: exact score ties
    _, lse = oracle.compressed_attention(q, ck, ck, cq, cc)
    return q, ck, lse.float(), cq, cc, cqb


def _gpu(q, ck, lse, topk, cq, cc, cqb, force_self):
    from lsrm_sparse import api, ops

    out = api.get_block_score(q.to(DEV), ck.to(DEV), lse.to(DEV), topk, cq.to(DEV), cc.to(DEV),
                              cu_query_blocks=cqb.to(DEV), force_self_block=force_self)
    assert ops.read_errors() == 0
    return out.cpu()


CASES = [
    # seed, qb lens, Hq, Hkv, D, topk, force_self, dup
    (1, [17, 300, 3, 64, 25, 129, 256, 257, 90], 4, 2, 64, 4, True, 0),
    (2, list(np.random.default_rng(0).integers(1, 200, 150)), 2, 2, 64, 8, True, 0),
    (3, list(np.random.default_rng(1).integers(1, 120, 140)), 8, 1, 32, 16, False, 0),
    (4, [40] * 20, 2, 1, 64, 6, True, 9),
    (5, [30, 0, 12, 33, 41], 2, 2, 16, 3, True, 0),
]


@pytest.mark.parametrize("case", CASES, ids=[f"case{c[0]}" for c in CASES])
def test_fast_qblock_scorer_bit_exact_vs_oracle(case):
    seed, lens, Hq, Hkv, D, topk, force, dup = case
    lens = [int(x) for x in lens]
    q, ck, lse, cq, cc, cqb = _inputs(seed, lens, Hq, Hkv, D, dup)
    got = _gpu(q, ck, lse, topk, cq, cc, cqb, force)
    ref = oracle.get_block_score_qblock_exact(q, ck, lse, topk, cq, cc, cqb, force_self=force)
    assert torch.equal(got, ref)


def test_fast_qblock_scorer_matches_exact_kernel_large():
    from lsrm_sparse import ops

    rng = np.random.default_rng(7)
    lens = [int(x) for x in rng.integers(32, 256, 700)]
    q, ck, lse, cq, cc, cqb = _inputs(9, lens, 4, 4, 64)
    fast = _gpu(q, ck, lse, 16, cq, cc, cqb, True)
    os.environ["LSRM_SCORER"] = "exact"
    try:
        exact = _gpu(q, ck, lse, 16, cq, cc, cqb, True)
    finally:
        del os.environ["LSRM_SCORER"]
    assert torch.equal(fast, exact)
