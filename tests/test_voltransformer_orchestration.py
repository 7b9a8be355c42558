"""VolTransformer's orchestration against the reference's own forward
(models_sparse/voldecoder.py:270-424), on the CPU: the fixtures
(tests/golden/voltransformer_fwd_*.npz, written by ``make_golden.py --only
voltransformer``) ran the reference's VolTransformer with its decoder blocks
replaced by seeded stubs (the real blocks need the GPU; they are pinned by
their own tests).  Here the same stubs go into this package's VolTransformer,
the reference's weights are loaded strictly, and the output formatting runs
as the CPU restatement (its GPU kernel is pinned separately): position
embedding (per-axis tables, or the full table through the voxel mask and
token order), device-side batch offsets, the layer loop with its skip links
and one-sided skip blocks, the final LayerNorm and the upsampler must give
the reference's sub-voxel features, offsets and index volume, and the same
gradients of the image tokens and of every parameter (fp32, 1e-5)."""

import os

import numpy as np
import pytest
import torch

import oracle
from tests.golden import make_golden

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _prepare_cpu(m):
    def prep(volume, volume_index, prior_volume):
        u, od = m.upsample_scale, m.output_dim
        feat = volume.reshape(-1, od, u, u, u).permute(0, 2, 3, 4, 1).reshape(-1, od)
        _, cu, seqlens, iv = oracle.prepare_volume_output(volume.detach().numpy(), volume_index.numpy(), od, u,
                                                          m.vol_res)
        return {"sparse_feat": feat, "dense_feat": prior_volume, "cu_seqlens": torch.from_numpy(cu),
                "seqlens": torch.from_numpy(seqlens), "index_volume": torch.from_numpy(iv)}
    return prep


@pytest.mark.parametrize("name,kw", make_golden.VOLT_FWD_CASES, ids=[c[0] for c in make_golden.VOLT_FWD_CASES])
def test_voltransformer_orchestration_matches_reference(name, kw):
    from lsrm_sparse.decoder import VolTransformer

    fx = np.load(os.path.join(HERE, name + ".npz"))
    m = make_golden.stub_blocks(VolTransformer(**kw), kw["embed_dim"])
    sd = {k[3:]: torch.from_numpy(fx[k]) for k in fx.files if k.startswith("sd_")}
    m.load_state_dict(sd, strict=True)
    m.prepare_volume_output = _prepare_cpu(m)
    inp = {k[3:]: torch.from_numpy(fx[k]) for k in fx.files if k.startswith("in_")}
    y = inp["y"].clone().requires_grad_()
    out, info = m(y, [inp["prior_imfeat"]], inp["image_index"], inp["prior_volfeat"], inp["mask_volume"],
                  inp["volume_index"], torch.zeros(1), inp["volume_coords_idx"], {}, 4)
    assert len(info) == kw["depth"] + len(kw["skip_links"])
    (out["sparse_feat"] * inp["grad_w"]).sum().backward()
    np.testing.assert_allclose(out["sparse_feat"].detach().numpy(), fx["out_sparse_feat"], rtol=1e-5, atol=1e-5)
    assert np.array_equal(out["cu_seqlens"].numpy(), fx["out_cu_seqlens"])
    assert np.array_equal(out["index_volume"].numpy(), fx["out_index_volume"])
    np.testing.assert_allclose(y.grad.numpy(), fx["grad_y"], rtol=1e-5, atol=1e-5)
    grads = {k[5:]: fx[k] for k in fx.files if k.startswith("grad_") and k != "grad_y" and k != "grad_w"}
    ours = {k: p.grad for k, p in m.named_parameters() if p.grad is not None}
    assert set(ours) == set(grads), set(ours) ^ set(grads)
    for k, g in grads.items():
        np.testing.assert_allclose(ours[k].numpy(), g, rtol=1e-5, atol=1e-5, err_msg=k)
