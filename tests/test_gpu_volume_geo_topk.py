"""Geometric volume-to-volume block selection on the GPU
(lsrm_volume_block_topk via lsrm_sparse.blocks) vs the reference fixture and
the oracle: the selected block ids must agree exactly."""

import types

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _sorted_case(seed, counts, res, bs):
    from lsrm_sparse import blocks

    g = torch.Generator().manual_seed(seed)
    parts = []
    for b, n in enumerate(counts):
        flat = torch.randperm(res ** 3, generator=g)[:n]
        z, y, x = flat // (res * res), (flat // res) % res, flat % res
        parts.append(torch.stack([torch.full_like(z, b), z, y, x], 1))
    coords = torch.cat(parts).to(torch.int32).cuda()
    keys = blocks.volume_sort_keys(coords, res, bs)
    return coords[torch.argsort(keys, stable=True)].contiguous()


def test_geo_topk_matches_reference_fixture(golden):
    from lsrm_sparse import blocks, ops

    g = golden("volume_geo_topk")
    args = types.SimpleNamespace(block_size=int(g["block_size"]), volume_res=int(g["volume_res"]),
                                 use_3d_aware_attn=True, topk_volume=int(g["topk"]), bbox_radius=float(g["bbox_radius"]))
    out = blocks.build_volume_to_volume_attn(torch.from_numpy(g["coords"]).cuda(), args)
    assert ops.read_errors() == 0
    assert np.array_equal(out["cu_seqblocks"].cpu().numpy(), g["cu_seqblocks"])
    assert np.array_equal(out["cu_block_include_tokens"].cpu().numpy(), g["cu_block_include_tokens"])
    assert np.array_equal(out["block_topk"].cpu().numpy(), g["block_topk"])


@pytest.mark.parametrize("counts,res,bs,k", [([3000, 1200, 5], 48, 8, 8), ([2500], 32, 4, 20), ([700, 50], 16, 8, 64)])
def test_geo_topk_vs_oracle(counts, res, bs, k):
    from lsrm_sparse import blocks, ops

    coords = _sorted_case(11 + k, counts, res, bs)
    B = len(counts)
    cu_sb, cu_blk, _ = blocks.block_separation(coords, 3, [bs] * 3, B, [res] * 3)
    got = blocks.volume_block_topk(coords, cu_sb, cu_blk, B, res, 0.5, k)
    torch.cuda.synchronize()
    assert ops.read_errors() == 0
    ref = oracle.volume_block_topk(coords.cpu().numpy(), cu_sb.cpu().numpy(), cu_blk.cpu().numpy(), B, res, 0.5, k)
    assert np.array_equal(got.cpu().numpy(), ref)
