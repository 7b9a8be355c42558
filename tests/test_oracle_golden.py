"""Pin the CPU oracle to fixtures produced by the reference's own code."""

import math

import numpy as np
import pytest
import torch

import oracle
from tests.golden.make_golden import selection_cases

SEL_CASES = [c[0] for c in selection_cases()]


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.asarray(a)).to(dtype)


@pytest.mark.parametrize("name", SEL_CASES)
def test_selection_forward_backward_matches_reference(golden, name):
    g = golden(name)
    q = _t(g["q"]).double().requires_grad_()
    k = _t(g["k"]).double().requires_grad_()
    v = _t(g["v"]).double().requires_grad_()
    topk = torch.from_numpy(g["block_topk"])
    o, lse = oracle.selection_attention(
        q, k, v, topk, _t(g["cu_seqblocks"], torch.int32), _t(g["cu_block_include_tokens"], torch.int32),
        _t(g["cu_seqlens"], torch.int32), _t(g["cu_seqlens"], torch.int32),
    )
    ref_o, ref_lse = g["o"], g["lse_log2"]
    nan_rows = np.isnan(ref_o).any(axis=-1)
    # rows with no valid block: NaN output and -inf LSE in both
    assert np.array_equal(nan_rows, np.isnan(o.detach().numpy()).any(axis=-1))
    assert np.array_equal(np.isneginf(ref_lse), np.isneginf(lse.detach().numpy()))
    ok = ~nan_rows
    # reference ran in fp16: compare with fp16-level tolerance
    assert np.abs(o.detach().numpy()[ok] - ref_o[ok]).max() < 2e-3
    fin = np.isfinite(ref_lse)
    assert np.abs(lse.detach().numpy()[fin] - ref_lse[fin]).max() < 2e-3
    # gradients (rows with NaN output excluded from the loss)
    do = _t(g["do"]).double()
    okt = torch.from_numpy(ok)
    (o[okt] * do[okt]).sum().backward()
    for name_g, t in (("dq", q), ("dk", k), ("dv", v)):
        ref = g[name_g]
        got = t.grad.numpy()
        if name_g == "dq":
            got, ref = got[ok], ref[ok]
        if np.isnan(ref).any():
            # the reference's NaN rows leak into dK/dV; compare the finite part
            m = np.isfinite(ref)
            got, ref = got[m], ref[m]
        assert np.abs(got - ref).max() < 3e-3, name_g


@pytest.mark.parametrize("name", ["score_g1", "score_g4", "score_few_blocks"])
def test_block_score_matches_reference(golden, name):
    g = golden(name)
    args = (_t(g["q"]), _t(g["ck"]), _t(g["lse"]), int(g["topk"]),
            _t(g["cu_seqlens_q"], torch.int32), _t(g["compressed_cu_seqlens"], torch.int32))
    got = oracle.get_block_score_exact(*args).numpy()
    ref = g["block_topk"]
    assert got.shape == ref.shape
    assert np.array_equal(got < 0, ref < 0)
    if not np.array_equal(got, ref):
        # allowed only where the float64 scores of the differing blocks tie
        scores = oracle.block_score_reference_formula(args[0], args[1], args[2], args[4], args[5])
        cq = g["cu_seqlens_q"]
        for h, i in zip(*np.nonzero((got != ref).any(-1))):
            b = np.searchsorted(cq, i, side="right") - 1
            s = scores[b][h, i - cq[b]].numpy()
            a = set(got[h, i]) - set(ref[h, i])
            r = set(ref[h, i]) - set(got[h, i])
            for x, y in zip(sorted(a), sorted(r)):
                assert abs(s[x] - s[y]) <= 1e-6 * s.max()


def test_exp2_fixed_accuracy():
    t = np.linspace(-125, 20, 200001, dtype=np.float32)
    got = oracle.exp2_fixed(t).astype(np.float64)
    ref = np.exp2(t.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 4e-7
    assert oracle.exp2_fixed(np.float32(-130.0)) == 0.0


def test_compression_matches_reference(golden):
    g = golden("compress_resblock")
    for which, out in (("key", "ck"), ("value", "cv")):
        w = [torch.from_numpy(g[f"w:compression_{which}.act_layers.{i}.{p}"]) for i, p in
             ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias"))]
        x = torch.from_numpy(g["k" if which == "key" else "v"])
        got = oracle.compress_kv(x, torch.from_numpy(g["cu_block_include_tokens"]), weights=w)
        assert np.abs(got.numpy() - g[out]).max() < 1e-5


@pytest.mark.parametrize("window", [False, True])
def test_gate_merge_matches_reference(golden, window):
    g = golden("gate_window" if window else "gate_nowindow")
    branches = [torch.from_numpy(g["compressed"]), torch.from_numpy(g["selection"])]
    if window:
        Hq, Hkv = 4, 2
        D = g["x"].shape[1] // Hq
        q = torch.from_numpy(g["q"]).view(-1, Hq, D)
        k = torch.from_numpy(g["k"]).view(-1, Hkv, D)
        v = torch.from_numpy(g["v"]).view(-1, Hkv, D)
        w = oracle.window_attention_intra_block(q, k, v, torch.from_numpy(g["cu_block_include_tokens"]))
        branches.append(w.reshape(w.shape[0], -1))
    got = oracle.gate_merge(torch.from_numpy(g["x"]), torch.from_numpy(g["gate_weight"]), branches)
    assert np.abs(got.numpy() - g["out"]).max() < 1e-5


def test_block_score_tie_goes_to_lowest_id():
    # identical compressed keys -> identical scores -> lowest ids win
    q = torch.randn(6, 2, 16)
    ck = torch.randn(1, 1, 16).repeat(5, 1, 1)
    lse = torch.zeros(2, 6)
    cu = torch.tensor([0, 6], dtype=torch.int32)
    cc = torch.tensor([0, 5], dtype=torch.int32)
    out = oracle.get_block_score_exact(q, ck, lse, 3, cu, cc)
    assert (out[0] == torch.tensor([0, 1, 2], dtype=torch.int32)).all()


def test_qblock_scoring_force_self():
    torch.manual_seed(0)
    q = torch.randn(12, 2, 16)
    ck = torch.randn(4, 1, 16)
    lse = torch.zeros(2, 12)
    cu = torch.tensor([0, 12], dtype=torch.int32)
    cc = torch.tensor([0, 4], dtype=torch.int32)
    cqb = torch.tensor([0, 3, 6, 9, 12], dtype=torch.int32)
    out = oracle.get_block_score_qblock_exact(q, ck, lse, 2, cu, cc, cqb, force_self=True)
    for qb in range(4):
        assert qb in out[0, qb].tolist()
    # query-block score = sum of token scores
    tok = oracle.token_block_scores_exact(q, ck, lse, cu, cc)[0][0]
    agg = tok[0:3].sum(0)
    best = [i for i in np.argsort(-agg, kind="stable") if i != 0][:1]
    assert sorted([0] + best) == out[0, 0].tolist()


def test_tiles_and_unions():
    cu = torch.tensor([0, 10, 25], dtype=torch.int32)
    tiles = oracle.build_query_tiles(cu, 4)
    assert [(t.seq, t.q_start, t.n_q) for t in tiles] == [
        (0, 0, 4), (0, 4, 4), (0, 8, 2), (1, 10, 4), (1, 14, 4), (1, 18, 4), (1, 22, 3)]
    tiles = oracle.build_query_tiles(cu, 4, cu_qblocks=torch.tensor([0, 3, 10, 17, 25]))
    assert [(t.q_start, t.n_q) for t in tiles] == [(0, 3), (3, 4), (7, 3), (10, 4), (14, 3), (17, 4), (21, 4)]
    bt = torch.tensor([[1, 3, -1], [3, 0, 9], [2, 2, 1]], dtype=torch.int32)
    un = oracle.build_tile_unions(bt, [oracle.nsa_oracle.QueryTile(0, 0, 3)], torch.tensor([0, 4]))
    assert un[0] == ([0, 1, 2, 3], [0b010, 0b101, 0b100, 0b011])


def test_block_metadata_matches_reference(golden):
    g = golden("block_metadata")
    keys = oracle.volume_sort_keys(g["coords"], int(g["volume_res"]), int(g["block_size"]))
    assert np.array_equal(np.argsort(keys, kind="stable"), g["sort_idx"])
    sorted_coords = g["coords"][g["sort_idx"]]
    bs = int(g["block_size"])
    cu_sb, cu_blk = oracle.block_separation(sorted_coords, 3, [bs] * 3, int(g["batch"]), [int(g["volume_res"])] * 3)
    assert np.array_equal(cu_sb, g["cu_seqblocks"])
    assert np.array_equal(cu_blk, g["cu_block_include_tokens"])
    cu_sb, cu_blk = oracle.block_separation(g["img_coords"], 3, [1, 4, 4], 2, [3, 8, 8])
    assert np.array_equal(cu_sb, g["img_cu_seqblocks"])
    assert np.array_equal(cu_blk, g["img_cu_block_include_tokens"])


def test_volume_output_matches_reference(golden):
    """prepare_volume_output restated in the oracle vs the reference method's
    own outputs (models_sparse/voldecoder.py:196-268), bit for bit."""
    g = golden("volume_output")
    feat, cu, seqlens, iv = oracle.prepare_volume_output(g["volume"], g["volume_index"], int(g["output_dim"]),
                                                         int(g["upsample_scale"]), int(g["vol_res"]))
    assert np.array_equal(feat, g["sparse_feat"])
    assert np.array_equal(cu, g["cu_seqlens"])
    assert np.array_equal(seqlens, g["seqlens"])
    assert np.array_equal(iv, g["index_volume"])


def test_volume_geo_topk_matches_reference(golden):
    """The geometric block selection restated in the oracle vs
    build_volume_to_volume_attn's own output (misc/sparse_utils.py:1203-1279)."""
    g = golden("volume_geo_topk")
    out = oracle.volume_block_topk(g["coords"], g["cu_seqblocks"], g["cu_block_include_tokens"], int(g["batch"]),
                                   int(g["volume_res"]), float(g["bbox_radius"]), int(g["topk"]))
    assert np.array_equal(out, g["block_topk"][0])
    assert np.array_equal(g["block_topk"][0], g["block_topk"][1])


def _image_case(g):
    B, M = g["scene_cameras"].shape[:2]
    w2c, th, crop = oracle.camera_terms(g["scene_cameras"], g.get("scene_crop_input"), g.get("scene_origin_size"))
    ps, bs, H = int(g["patch_size"]), int(g["block_size"]), int(g["image_res"])
    return dict(B=B, M=M, w2c=w2c, th=th, crop=crop, ps=ps, bs=bs, H=H, win=int(g["attn_winsize"]) ** 2,
                topk=int(g["topk_multiimage"]) * M, max_dist=2 * float(g["bbox_radius"]))


@pytest.mark.parametrize("name", ["image_maps", "image_maps_crop"])
def test_image_maps_match_reference(golden, name):
    """The image-side maps restated in the oracle vs the reference's own
    build_image_to_image_attn / build_image_to_volume_attn /
    build_volume_to_image_attn and from_imcoords_to_points
    (misc/sparse_utils.py:653-1200), with and without cropped views.  Token
    points and the image-to-volume map are equal; the view maps are equal
    except where torch.topk resolved a tie, and those rows must be valid for
    some resolution of the ties (``view_rows_equivalent``).  A planted
    mistake (a block outside every window) must be caught."""
    g = golden(name)
    c = _image_case(g)
    impts = oracle.image_token_points(g["imcoords"], g["scene_surface_points"], g["scene_surface_masks"],
                                      c["H"] // c["ps"])
    assert np.array_equal(impts, g["impoints"])
    i2v = oracle.image_volume_block_topk(impts, g["imcoords"][:, 0], g["volcoords"], g["i2v_cu_seqblocks"],
                                         g["i2v_cu_block_include_tokens"], c["B"], int(g["volume_res"]),
                                         float(g["bbox_radius"]), int(g["topk_volume"]))
    assert np.array_equal(i2v, g["i2v_block_topk"][0])
    volpts = oracle.voxel_points(g["volcoords"], int(g["volume_res"]), float(g["bbox_radius"]))
    mi = g["scene_mask_input"][:, :, 0]
    equal_rows = 0
    for key, pts, bid in (("i2i", impts, g["imcoords"][:, 0]), ("v2i", volpts, g["volcoords"][:, 0])):
        out, det = oracle.view_block_topk(pts, bid, mi, g["scene_surface_points"], g["scene_surface_masks"],
                                          c["w2c"], c["th"], c["ps"], c["bs"], c["win"], c["topk"], c["max_dist"],
                                          crop=c["crop"], return_values=True)
        ref = g[f"{key}_block_topk"]
        assert np.array_equal(ref[0], ref[1])
        assert oracle.view_rows_equivalent(out, ref[0], det, c["win"]) == []
        equal_rows += int((out == ref[0]).all(1).sum())
        if key == "v2i":
            assert np.array_equal(out, ref[0])  # no ties on these points
            planted = ref[0].copy()
            row = int(np.nonzero((planted >= 0).sum(1) == planted.shape[1])[0][0])
            far = [x for x in range(int(g["v2i_cu_seqblocks"][1])) if x not in planted[row]]
            planted[row, 0] = far[-1]
            assert row in oracle.view_rows_equivalent(out, planted, det, c["win"])
    assert equal_rows > 0.8 * (g["imcoords"].shape[0] + g["volcoords"].shape[0])


def test_image_sort_matches_reference(golden):
    """sort_image_blocks' key restated in the oracle gives the reference's
    order (misc/sparse_utils.py:95-124)."""
    g = golden("image_sort")
    c = g["coords"]
    keys = oracle.image_sort_keys(c, int(c[:, 1].max()) + 1, int(g["image_res"]) // int(g["patch_size"]),
                                  int(g["block_size"]))
    idx = np.argsort(keys, kind="stable")
    assert np.array_equal(idx, g["sort_idx"])
    assert np.array_equal(c[idx], g["sorted_coords"])
