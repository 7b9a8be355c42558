"""Token distribution of the sequence-parallel decoder on CPU gloo ranks
(``ulysses.seq_parallel_token_blocks``): each rank gets a run of whole blocks
of both token sets, every map gets its keys' local block table, ``collect``
gives back all volume tokens in order (forward and backward), and maps whose
key blocks disagree are refused."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.cases import as_tensors, by_value, cu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _maps(vol_lens, img_lens):
    cv, ci = cu(vol_lens), cu(img_lens)
    two = torch.tensor([0, 1], dtype=torch.int32)
    mk = lambda c: {"block_topk": None, "cu_seqblocks": two * (c.numel() - 1), "cu_block_include_tokens": c}  # noqa
    return {"vol_to_vol_attn": mk(cv), "img_to_vol_attn": mk(cv.clone()), "img_to_img_attn": mk(ci),
            "vol_to_img_attn": mk(ci.clone())}


def _worker(rank, world, port, vol_lens, img_lens, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from lsrm_sparse import ulysses

        nx, ny = sum(vol_lens), sum(img_lens)
        x = torch.arange(nx * 3, dtype=torch.float32).view(nx, 3)
        y = -torch.arange(ny * 2, dtype=torch.float32).view(ny, 2)
        (xl,), (yl,), cxl, cyl, m = ulysses.seq_parallel_token_blocks([x], [y], _maps(vol_lens, img_lens))
        sp = m["sp"]
        res = {"x": xl, "y": yl, "cx": cxl, "cy": cyl, "vol": sp.vol.local, "img": sp.img.local,
               "vb": sp.vol_blocks.counts, "ib": sp.img_blocks.counts,
               "loc": {k: v["local_cu_block_include_tokens"] for k, v in m.items() if k != "sp"}}
        xg = xl.clone().requires_grad_()
        (full,), _, _, _, _ = ulysses.seq_parallel_token_blocks([xg], [], m, "collect")
        full.sum().backward()
        res["full"], res["grad"] = full.detach(), xg.grad
        q.put((rank, by_value(res)))
    finally:
        dist.destroy_process_group()


def _run(world, vol_lens, img_lens):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, vol_lens, img_lens, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {r: as_tensors(res) for r, res in (q.get(timeout=120) for _ in ps)}
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    return out


def test_distribute_and_collect_whole_blocks():
    from lsrm_sparse import ulysses

    vol_lens, img_lens = [40, 70, 33, 90, 64, 21, 55], [16, 16, 32, 16, 48]
    out = _run(2, vol_lens, img_lens)
    cv, ci = cu(vol_lens), cu(img_lens)
    nx, ny = int(cv[-1]), int(ci[-1])
    x = torch.arange(nx * 3, dtype=torch.float32).view(nx, 3)
    y = -torch.arange(ny * 2, dtype=torch.float32).view(ny, 2)
    vb = ulysses.shard_blocks(cv.tolist(), 2)
    ib = ulysses.shard_blocks(ci.tolist(), 2)
    for r in range(2):
        o = out[r]
        (a, b), (c, d) = vb[r], ib[r]
        s, e = int(cv[a]), int(cv[b])
        assert o["vol"] == (s, e) and torch.equal(o["x"], x[s:e])
        assert torch.equal(o["cx"], torch.tensor([0, e - s], dtype=torch.int32))
        si, ei = int(ci[c]), int(ci[d])
        assert o["img"] == (si, ei) and torch.equal(o["y"], y[si:ei])
        assert o["vb"] == [bb - aa for aa, bb in vb] and o["ib"] == [bb - aa for aa, bb in ib]
        for k in ("vol_to_vol_attn", "img_to_vol_attn"):
            assert torch.equal(o["loc"][k], (cv[a:b + 1] - cv[a]).int())
        for k in ("img_to_img_attn", "vol_to_img_attn"):
            assert torch.equal(o["loc"][k], (ci[c:d + 1] - ci[c]).int())
        assert torch.equal(o["full"], x)  # collect: all volume tokens, in order
        assert torch.equal(o["grad"], torch.ones(e - s, 3))  # backward keeps this rank's rows


def test_distribute_refuses_mismatched_key_blocks():
    import torch.distributed as d

    from lsrm_sparse import ulysses

    if not d.is_available():
        pytest.skip("torch.distributed unavailable")
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(_free_port())
    d.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=30))
    try:
        m = _maps([10, 20], [8, 8])
        m["img_to_vol_attn"]["cu_block_include_tokens"] = cu([15, 15])
        with pytest.raises(ValueError, match="same key blocks"):
            ulysses.seq_parallel_token_blocks([torch.zeros(30, 2)], [torch.zeros(16, 2)], m)
    finally:
        d.destroy_process_group()
