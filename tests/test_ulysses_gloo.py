"""Sequence-parallel (Ulysses) host logic on CPU gloo ranks.

The exchange, the shard plan and the orchestration run as they do on GPUs;
the two things that need a device are replaced by test doubles: the pack /
unpack layouts by their torch restatement (checked against the CUDA kernels
in test_gpu_ulysses.py) and the per-head branch compute by the fp64 oracle.
The result on every rank must equal the single-process oracle on the whole
sequence, forward and backward."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tests.cases import as_tensors, by_value, cu, expand_qblock_selection


def pack_ref(x, world):
    n, H, D = x.shape
    hp = H // world if H >= world else 1
    rep = 1 if H >= world else world // H
    return torch.stack([x[:, (p // rep) * hp:(p // rep) * hp + hp] for p in range(world)]).contiguous()


def unpack_ref(y, H):
    world, n, hp, D = y.shape
    rep = 1 if H >= world else world // H
    groups = world // rep
    acc_t = torch.promote_types(y.dtype, torch.float32)  # fp32 for bf16/fp16, as the kernel
    parts = []
    for g in range(groups):
        acc = y[g * rep].to(acc_t)
        for j in range(1, rep):
            acc = acc + y[g * rep + j].to(acc_t)
        parts.append(acc.to(y.dtype))
    return torch.cat(parts, 1)


def oracle_branches(q, k, v, z, cu_blk, topk, window, scale=None):
    """Whole-sequence three-branch op in fp64 (heads given), per-head gates."""
    N, H, D = q.shape
    nb = cu_blk.numel() - 1
    cq = torch.tensor([0, N], dtype=torch.int32)
    cs = torch.tensor([0, nb], dtype=torch.int32)
    Hkv = k.shape[1]
    ck = oracle.segment_mean(k.reshape(N, -1), cu_blk).view(nb, Hkv, D)
    cv = oracle.segment_mean(v.reshape(N, -1), cu_blk).view(nb, Hkv, D)
    o_c, lse = oracle.compressed_attention(q, ck, cv, cq, cs, scale)
    bt = oracle.get_block_score_qblock_exact(q.detach().float(), ck.detach().float(), lse.detach().float(), topk, cq,
                                             cs, cu_blk, force_self=True)
    o_s, _ = oracle.selection_attention(q, k, v, expand_qblock_selection(bt, cu_blk), cs, cu_blk, cq, cq, scale)
    o_w = oracle.sliding_window_attention(q, k, v, cq, window, scale)
    g = torch.sigmoid(z.double()).view(N, 3, H, 1)
    return g[:, 0] * o_c + g[:, 1] * o_s + g[:, 2] * o_w


def _problem(Hq, Hkv, D, lens, seed=3):
    g = torch.Generator().manual_seed(seed)
    N = sum(lens)
    q = torch.randn(N, Hq, D, generator=g, dtype=torch.float64)
    k = torch.randn(N, Hkv, D, generator=g, dtype=torch.float64)
    v = torch.randn(N, Hkv, D, generator=g, dtype=torch.float64)
    z = torch.randn(N, 3 * Hq, generator=g, dtype=torch.float64)
    dout = torch.randn(N, Hq, D, generator=g, dtype=torch.float64)
    return q, k, v, z, dout, cu(lens)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, Hq, Hkv, D, lens, topk, window, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from lsrm_sparse import ulysses

        q, k, v, z, dout, cu_blk = _problem(Hq, Hkv, D, lens)
        plan = ulysses.ShardPlan(cu_blk.tolist(), world, rank)
        s, e = plan.local
        ql, kl, vl, zl = (t[s:e].clone().requires_grad_(True) for t in (q, k, v, z))
        out = ulysses.three_branch_attention(ql, kl, vl, zl, plan, cu_blk, topk, window, branch_fn=oracle_branches,
                                             pack=pack_ref, unpack=unpack_ref)
        out.backward(dout[s:e])
        q_out.put(by_value((rank, s, e, out.detach(), ql.grad, kl.grad, vl.grad, zl.grad)))
    finally:
        dist.destroy_process_group()


def _run(world, Hq, Hkv, D, lens, topk=3, window=16):
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, Hq, Hkv, D, lens, topk, window, qq))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [as_tensors(qq.get(timeout=240)) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # single-process reference on the whole sequence
    q, k, v, z, dout, cu_blk = _problem(Hq, Hkv, D, lens)
    q, k, v, z = (t.clone().requires_grad_(True) for t in (q, k, v, z))
    ref = oracle_branches(q, k, v, z, cu_blk, topk, window)
    ref.backward(dout)
    for rank, s, e, o, dq, dk, dv, dz in res:
        torch.testing.assert_close(o, ref[s:e].detach(), rtol=1e-9, atol=1e-9)
        torch.testing.assert_close(dq, q.grad[s:e], rtol=1e-9, atol=1e-9)
        torch.testing.assert_close(dk, k.grad[s:e], rtol=1e-9, atol=1e-9)
        torch.testing.assert_close(dv, v.grad[s:e], rtol=1e-9, atol=1e-9)
        torch.testing.assert_close(dz, z.grad[s:e], rtol=1e-9, atol=1e-9)


LENS = [17, 30, 8, 25, 40, 12, 33, 21, 9, 28]


def test_ulysses_two_ranks_matches_whole_sequence_oracle():
    _run(2, Hq=4, Hkv=2, D=8, lens=LENS)


def test_ulysses_two_ranks_gqa_groups():
    # G = 4 q heads per kv head; each rank owns one whole group
    _run(2, Hq=8, Hkv=2, D=8, lens=LENS)


def test_ulysses_rejects_split_kv_groups():
    from lsrm_sparse import ulysses

    plan = ulysses.ShardPlan(cu(LENS).tolist(), 2, 0)
    q = torch.zeros(plan.counts[0], 2, 8)
    k = torch.zeros(plan.counts[0], 1, 8)
    with pytest.raises(ValueError, match="kv heads"):
        ulysses.three_branch_attention(q, k, k, torch.zeros(plan.counts[0], 6), plan, cu(LENS), 3, 16,
                                       branch_fn=oracle_branches, pack=pack_ref, unpack=unpack_ref)


def test_shard_blocks_balances_whole_blocks():
    from lsrm_sparse import ulysses

    lens = [17, 30, 8, 25, 40, 12, 33, 21, 9, 28]
    cu_blk = [0]
    for l in lens:
        cu_blk.append(cu_blk[-1] + l)
    for world in (1, 2, 3, 4, 8):
        sh = ulysses.shard_blocks(cu_blk, world)
        assert len(sh) == world
        assert sh[0][0] == 0 and sh[-1][1] == len(lens)
        assert all(a[1] == b[0] for a, b in zip(sh, sh[1:]))
        if world <= len(lens):
            assert all(b > a for a, b in sh)  # every rank owns at least one block
    # the greedy aims at (tokens left) / (ranks left) and stops at the closer side
    sh = ulysses.shard_blocks([0, 10, 20, 30, 40], 2)
    assert sh == [(0, 2), (2, 4)]
    sh = ulysses.shard_blocks([0, 10, 25, 30, 40], 2)
    assert sh == [(0, 2), (2, 4)]  # 25 vs target 20: |25-20| <= |10-20|


def test_pack_unpack_reference_round_trip():
    x = torch.randn(11, 8, 4)
    for world in (1, 2, 4, 8):
        y = pack_ref(x, world)
        assert torch.equal(unpack_ref(y, 8), x)
    # replicated heads: unpack sums the replicas
    x = torch.randn(5, 2, 4)
    y = pack_ref(x, 8)
    assert y.shape == (8, 5, 1, 4)
    torch.testing.assert_close(unpack_ref(y, 2), 4 * x)
