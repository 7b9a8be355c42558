"""Block metadata on the device vs the reference's own outputs (fixtures made
by running sort_volume_blocks / compute_block_separation) and vs the oracle
on larger random inputs; bit-exact."""

import types

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_block_metadata_matches_reference_fixture(golden):
    from lsrm_sparse import blocks, ops

    g = golden("block_metadata")
    coords = torch.from_numpy(g["coords"]).cuda()
    feats = torch.arange(coords.shape[0], dtype=torch.float32, device="cuda")[:, None]
    args = types.SimpleNamespace(block_size=int(g["block_size"]), volume_res=int(g["volume_res"]))
    f2, c2, idx = blocks.sort_volume_blocks(feats, coords, args)
    assert np.array_equal(idx.cpu().numpy(), g["sort_idx"])
    assert torch.equal(f2[:, 0].long().cpu(), torch.from_numpy(g["sort_idx"]))
    bs = int(g["block_size"])
    cu_sb, cu_blk = blocks.compute_block_separation(c2, 3, [bs] * 3, int(g["batch"]), [int(g["volume_res"])] * 3)
    assert np.array_equal(cu_sb.cpu().numpy(), g["cu_seqblocks"])
    assert np.array_equal(cu_blk.cpu().numpy(), g["cu_block_include_tokens"])
    img = torch.from_numpy(g["img_coords"]).cuda()
    cu_sb, cu_blk = blocks.compute_block_separation(img, 3, [1, 4, 4], 2, [3, 8, 8])
    assert np.array_equal(cu_sb.cpu().numpy(), g["img_cu_seqblocks"])
    assert np.array_equal(cu_blk.cpu().numpy(), g["img_cu_block_include_tokens"])
    assert ops.read_errors() == 0


@pytest.mark.parametrize("res,bs,batch,n", [(64, 8, 2, 20000), (128, 16, 1, 300000), (32, 4, 5, 3000), (16, 16, 3, 100)])
def test_block_separation_random_vs_oracle(res, bs, batch, n):
    from lsrm_sparse import blocks, ops

    rng = np.random.default_rng(res + bs + batch)
    per = [rng.choice(res ** 3, size=min(n, res ** 3), replace=False) for _ in range(batch)]
    coords = np.concatenate([np.stack([np.full(len(f), b), f // (res * res), (f // res) % res, f % res], 1)
                             for b, f in enumerate(per)]).astype(np.int32)
    keys = oracle.volume_sort_keys(coords, res, bs)
    order = np.argsort(keys, kind="stable")
    ct = torch.from_numpy(coords).cuda()
    got_keys = blocks.volume_sort_keys(ct, res, bs).cpu().numpy()
    assert np.array_equal(got_keys, keys)
    sc = coords[order]
    cu_sb, cu_blk, cu_seq = blocks.block_separation(torch.from_numpy(sc).cuda(), 3, [bs] * 3, batch, [res] * 3)
    ref_sb, ref_blk = oracle.block_separation(sc, 3, [bs] * 3, batch, [res] * 3)
    assert np.array_equal(cu_sb.cpu().numpy(), ref_sb)
    assert np.array_equal(cu_blk.cpu().numpy(), ref_blk)
    assert np.array_equal(cu_seq.cpu().numpy(), np.concatenate([[0], np.cumsum([len(f) for f in per])]))
    assert ops.read_errors() == 0


def test_block_separation_ignores_cells_outside_the_grid():
    from lsrm_sparse import blocks

    coords = np.array([[0, 0, 0, 0], [0, 0, 0, 9], [0, -1, 0, 0], [0, 3, 3, 3], [0, 40, 0, 0]], dtype=np.int32)
    cu_sb, cu_blk, _ = blocks.block_separation(torch.from_numpy(coords).cuda(), 3, [4, 4, 4], 1, [8, 8, 8])
    ref_sb, ref_blk = oracle.block_separation(coords, 3, [4, 4, 4], 1, [8, 8, 8])
    assert np.array_equal(cu_sb.cpu().numpy(), ref_sb)
    assert np.array_equal(cu_blk.cpu().numpy(), ref_blk)


def test_block_separation_bad_batch_id_sets_error_bit():
    from lsrm_sparse import _lib, blocks, ops

    coords = np.array([[0, 0, 0, 0], [3, 1, 1, 1]], dtype=np.int32)
    blocks.block_separation(torch.from_numpy(coords).cuda(), 3, [2, 2, 2], 2, [4, 4, 4])
    assert ops.read_errors() & _lib.LSRM_ERR_BAD_INDEX


def test_sort_image_blocks_matches_reference_fixture(golden):
    """lsrm_image_sort_keys + argsort (sort_image_blocks) vs the reference's
    own output on shuffled image tokens."""
    import types

    from lsrm_sparse import blocks

    g = golden("image_sort")
    coords = torch.from_numpy(g["coords"]).cuda()
    args = types.SimpleNamespace(block_size=int(g["block_size"]), patch_size=int(g["patch_size"]),
                                 input_image_res=[int(g["image_res"]) // 2, int(g["image_res"])])
    feats = torch.arange(coords.shape[0], dtype=torch.float32, device="cuda")[:, None]
    f, c, idx = blocks.sort_image_blocks(feats, coords, args)
    assert np.array_equal(idx.cpu().numpy(), g["sort_idx"])
    assert np.array_equal(c.cpu().numpy(), g["sorted_coords"])
    assert np.array_equal(f[:, 0].long().cpu().numpy(), g["sort_idx"])
