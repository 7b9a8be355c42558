"""VolTransformer's sequence-parallel orchestration on two CPU gloo ranks:
with ``use_sequence_parallel=True`` every rank embeds all voxel tokens, keeps
its run of whole blocks of both token sets (``seq_parallel_token_blocks``
distribute, models_sparse/voldecoder.py:305-316), runs the layer loop and the
skip blocks on them, and collects the upsampled volume back (:417-421) before
the output formatting.  With token-local stub blocks (the real blocks need
the GPU and are checked on it) the collected output, the index volume and
every parameter gradient summed over the ranks equal the single-process
model's (fp32, 1e-5).  (The image tokens' routing through the skip links is
pinned by the reference fixtures in test_voltransformer_orchestration.py.)"""

import datetime
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tests.cases import as_tensors, by_value, cu

VOL_LENS, IMG_LENS = [23, 40, 17, 31, 9, 28], [12, 12, 20, 12]
KW = dict(vol_res=8, upsample_scale=2, embed_dim=32, output_dim=4, depth=3, num_q_heads=2, num_kv_heads=2,
          skip_links=(1, 0), use_decomposed_embed=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class LocalStub(torch.nn.Module):
    """A token-local stand-in for BlockMix / BlockMixOneside (their call
    signature and return shape): every token changes by a function of itself,
    so a sequence-parallel run must reproduce the single-process one exactly."""

    def __init__(self, dim, seed, oneside):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.wx = torch.nn.Parameter(torch.randn(dim, dim, generator=g) / dim ** 0.5)
        self.wy = torch.nn.Parameter(torch.randn(dim, dim, generator=g) / dim ** 0.5)
        self.oneside = oneside

    def forward(self, x, cu_seqlens_x, y, cu_seqlens_y, attn_map, im_num):
        x = x + torch.tanh(x @ self.wx)
        if self.oneside:
            return x, {}
        return x, y + torch.tanh(y @ self.wy), {}


def _model(sp):
    from lsrm_sparse.decoder import VolTransformer

    torch.manual_seed(7)
    m = VolTransformer(**KW, use_sequence_parallel=sp)
    m.cross_blocks = torch.nn.ModuleList(LocalStub(KW["embed_dim"], 10 + i, False) for i in range(KW["depth"]))
    m.skip_blocks = torch.nn.ModuleList(LocalStub(KW["embed_dim"], 20 + i, True)
                                        for i in range(len(KW["skip_links"])))

    def prep(volume, volume_index, prior_volume):  # the output formatting, CPU restatement
        u, od = m.upsample_scale, m.output_dim
        feat = volume.reshape(-1, od, u, u, u).permute(0, 2, 3, 4, 1).reshape(-1, od)
        _, c, sl, iv = oracle.prepare_volume_output(volume.detach().numpy(), volume_index.numpy(), od, u, m.vol_res)
        return {"sparse_feat": feat, "dense_feat": prior_volume, "cu_seqlens": torch.from_numpy(c),
                "seqlens": torch.from_numpy(sl), "index_volume": torch.from_numpy(iv)}

    m.prepare_volume_output = prep
    return m


def _inputs():
    g = torch.Generator().manual_seed(3)
    R, C = KW["vol_res"], KW["embed_dim"]
    nx, ny = sum(VOL_LENS), sum(IMG_LENS)
    flat = torch.randperm(R ** 3, generator=g)[:nx]
    vi = torch.stack([torch.zeros_like(flat), flat // (R * R), (flat // R) % R, flat % R], 1).long()
    ii = torch.zeros(ny, 4, dtype=torch.long)
    two = torch.tensor([0, 1], dtype=torch.int32)
    mk = lambda c: {"block_topk": None, "cu_seqblocks": two * (c.numel() - 1), "cu_block_include_tokens": c}  # noqa
    cv, ci = cu(VOL_LENS), cu(IMG_LENS)
    maps = {"vol_to_vol_attn": mk(cv), "img_to_vol_attn": mk(cv.clone()), "img_to_img_attn": mk(ci),
            "vol_to_img_attn": mk(ci.clone())}
    return dict(y=torch.randn(ny, C, generator=g), prior_im=torch.randn(ny, C, generator=g),
                prior_vol=torch.randn(nx, C, generator=g), vi=vi, ii=ii, maps=maps,
                w=torch.randn(nx * KW["upsample_scale"] ** 3, KW["output_dim"], generator=g))


def _step(m, inp):
    y = inp["y"].clone().requires_grad_()
    out, _ = m(y, [inp["prior_im"]], inp["ii"], inp["prior_vol"], None, inp["vi"], torch.zeros(1), None,
               inp["maps"], 4)
    (out["sparse_feat"] * inp["w"]).sum().backward()
    grads = {k: p.grad.clone() for k, p in m.named_parameters() if p.grad is not None}
    return out, y.grad, grads


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        out, gy, grads = _step(_model(True), _inputs())
        for t in [gy] + list(grads.values()):  # each rank's share: summed over the ranks
            if t is not None:
                dist.all_reduce(t)
        q.put((rank, by_value({"feat": out["sparse_feat"], "cu": out["cu_seqlens"], "iv": out["index_volume"],
                               "gy": gy, "grads": grads})))
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_voltransformer_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r: as_tensors(v) for r, v in (q.get(timeout=120) for _ in ps)}
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    out, gy, grads = _step(_model(False), _inputs())
    for r in range(2):
        got = res[r]
        np.testing.assert_allclose(got["feat"].numpy(), out["sparse_feat"].detach().numpy(), rtol=1e-5, atol=1e-5)
        assert torch.equal(got["cu"], out["cu_seqlens"]) and torch.equal(got["iv"], out["index_volume"])
        # the stub blocks are token-local, so the image tokens do not reach the volume output
        assert gy is None and got["gy"] is None
        assert set(got["grads"]) == set(grads)
        for k, g in grads.items():
            np.testing.assert_allclose(got["grads"][k].numpy(), g.numpy(), rtol=1e-5, atol=1e-5, err_msg=k)
