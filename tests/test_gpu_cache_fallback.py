"""Selected-block attention on problems whose lists overflow the kernels'
shared-memory caches:

* a query tile whose union of selected blocks has more than 512 entries
  (the forward and dQ producers walk it from global memory),
* KV blocks selected by more than 1024 query tiles (the dK/dV reverse map
  streams through its cache in segments of 1024 entries): 1250 tiles, 5000
  tiles (five segments, 8 query heads per kv head) and 1094 tiles of 128
  queries on two kv heads,
* a KV block with more than 4096 8-row query windows (dK/dV window list) but
  few enough reverse entries for one cache segment,
* a KV block selected by 10000 query tiles (16 query heads per kv head: 8
  queries per tile), beyond the 2048 entries of the reverse map's small sort
  and the 8192 of its former capacity.

Checked against a gather-based fp32 torch reference of the same op (each query
attends the tokens of its selected blocks), forward and backward."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL_BF16 = 2e-2
COS_MIN = 0.9995


def _cos(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def _problem(N, L, Hq, Hkv, D, picks, seed, popular):
    """One sequence of N tokens in blocks of L; every query selects `picks`
    distinct blocks (block 0 always when `popular`)."""
    g = torch.Generator().manual_seed(seed)
    nb = N // L
    q = torch.randn(N, Hq, D, generator=g).bfloat16()
    k = torch.randn(N, Hkv, D, generator=g).bfloat16()
    v = torch.randn(N, Hkv, D, generator=g).bfloat16()
    n_rand = picks - 1 if popular else picks
    stride = (nb - 1) // n_rand
    r = torch.randint(0, nb - 1, (Hkv, N, 1), generator=g)
    sel = 1 + (r + torch.arange(n_rand) * stride) % (nb - 1)  # distinct, never block 0
    if popular:
        sel = torch.cat([torch.zeros(Hkv, N, 1, dtype=sel.dtype), sel], -1)
    sel = sel.sort(-1).values.to(torch.int32)
    cu_blk = (torch.arange(nb + 1) * L).to(torch.int32)
    cu_seqblocks = torch.tensor([0, nb], dtype=torch.int32)
    cu_seqlens = torch.tensor([0, N], dtype=torch.int32)
    return q, k, v, sel, cu_blk, cu_seqblocks, cu_seqlens


def _reference(q, k, v, sel, L, do):
    qf, kf, vf = (t.float().requires_grad_() for t in (q, k, v))
    N, Hq, D = q.shape
    G = Hq // k.shape[1]
    idx = (sel.long()[..., None] * L + torch.arange(L, device=sel.device)).reshape(sel.shape[0], N, -1)
    outs = []
    for h in range(Hq):
        kh = kf[:, h // G][idx[h // G]]  # [N, picks*L, D]
        vh = vf[:, h // G][idx[h // G]]
        s = (qf[:, h, None, :] * kh).sum(-1) / math.sqrt(D)
        outs.append((s.softmax(-1)[..., None] * vh).sum(1))
    o = torch.stack(outs, 1)
    (o * do.float()).sum().backward()
    return o.detach(), qf.grad, kf.grad, vf.grad


def _check(got, ref, what, rel=False):
    got = got.float()
    bound = max(ATOL_BF16, 1e-2 * ref.abs().max().item()) if rel else ATOL_BF16
    err = (got - ref).abs().max().item()
    assert err < bound, f"{what}: max-abs {err} (bound {bound})"
    assert _cos(got, ref) >= COS_MIN, f"{what}: cosine {_cos(got, ref)}"


CASES = [
    # name, N, L, Hq, Hkv, D, picks, popular
    ("union_over_512", 4096, 4, 1, 1, 64, 8, False),        # ~645 blocks per 128-query tile
    ("reverse_over_1024", 20000, 4, 8, 1, 64, 4, True),     # block 0 in all 1250 16-query tiles
    ("windows_over_4096", 40000, 4, 1, 1, 64, 4, True),     # block 0: 313 tiles, ~5000 8-query windows
    ("reverse_five_segments", 80000, 4, 8, 1, 64, 4, True),  # block 0 in all 5000 16-query tiles
    ("reverse_two_heads_g1", 140000, 4, 2, 2, 64, 4, True),  # block 0 in all 1094 128-query tiles, per head
    ("reverse_over_8192_g16", 80000, 4, 16, 1, 32, 4, True),  # block 0 in all 10000 8-query tiles (wide sort)
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_cache_overflow_paths(case):
    from lsrm_sparse import ops

    name, N, L, Hq, Hkv, D, picks, popular = case
    q, k, v, sel, cu_blk, cu_sb, cu_sl = (t.cuda() for t in _problem(N, L, Hq, Hkv, D, picks, 17, popular))
    do = (torch.randn(q.shape, generator=torch.Generator().manual_seed(18)) * 0.1).bfloat16().cuda()
    meta = ops.Meta(cu_sl, cu_sl, cu_sb, cu_blk)
    out, lse, ws = ops.select_attn_fwd(q, k, v, sel, meta)
    dq, dk, dv = ops.select_attn_bwd(q, k, v, out, lse, do, sel, meta, workspace=ws)
    torch.cuda.synchronize()
    assert ops.read_errors() == 0
    ro, rq, rk, rv = _reference(q, k, v, sel, L, do)
    _check(out, ro, "out")
    _check(dq, rq, "dq")
    _check(dk, rk, "dk", rel=popular)
    _check(dv, rv, "dv", rel=popular)
