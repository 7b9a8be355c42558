"""The decoder blocks keep the reference's parameter layout, so a reference
checkpoint loads with ``strict=True``: names and shapes of every parameter of
``BlockMix`` / ``BlockMixOneside`` (models_sparse/utils.py:575-705, holding
``CrossAttention`` with its optional weight norm at :228-236 and ``Mlp``)
against ``tests/golden/module_keys.json``, which ``make_golden.py --only
modules`` wrote from the reference modules themselves.  CPU only."""

import json
import os

import pytest
import torch

from tests.golden import make_golden

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("name,kw", make_golden.MODULE_CASES, ids=[c[0] for c in make_golden.MODULE_CASES])
def test_blockmix_state_dict_matches_reference_layout(name, kw):
    from lsrm_sparse import decoder

    with open(os.path.join(HERE, "module_keys.json")) as f:
        ref = json.load(f)[name]
    kw = dict(kw)
    cls = decoder.BlockMixOneside if kw.pop("oneside", False) else decoder.BlockMix
    m = cls(**kw)
    ours = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert ours == ref
    g = torch.Generator().manual_seed(0)
    sd = {k: torch.randn(*shape, generator=g) for k, shape in ref.items()}
    m.load_state_dict(sd, strict=True)
    for k, v in m.state_dict().items():
        assert torch.equal(v, sd[k]), k


@pytest.mark.parametrize("name,kw", make_golden.VOLT_CASES, ids=[c[0] for c in make_golden.VOLT_CASES])
def test_voltransformer_state_dict_matches_reference_layout(name, kw):
    """``VolTransformer`` (models_sparse/voldecoder.py:39-194): the position
    tables, the 24 + skip blocks, the skip and fuse Linears, the final norm and
    the upsampler keep the reference's names and shapes, and a reference
    state dict loads strictly."""
    from lsrm_sparse import decoder

    with open(os.path.join(HERE, "module_keys.json")) as f:
        ref = json.load(f)[name]
    m = decoder.VolTransformer(**kw)
    ours = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert ours == ref
    g = torch.Generator().manual_seed(1)
    sd = {k: torch.randn(*shape, generator=g) for k, shape in ref.items()}
    m.load_state_dict(sd, strict=True)
    for k, v in m.state_dict().items():
        assert torch.equal(v, sd[k]), k


def test_voltransformer_init_rule():
    """Linear weights truncated-normal with std 0.02 inside [-2, 2] and zero
    biases, LayerNorm weight 1 and bias 0 (voldecoder.py:183-193)."""
    from lsrm_sparse import decoder

    torch.manual_seed(0)
    m = decoder.VolTransformer(vol_res=4, upsample_scale=2, embed_dim=64, output_dim=4, depth=2, num_q_heads=4,
                               num_kv_heads=2, skip_links=(0,))
    w = m.upsampler.dconv3d.weight
    assert abs(float(w.std()) - 0.02) < 4e-3 and float(w.abs().max()) <= 2.0
    assert torch.count_nonzero(m.upsampler.dconv3d.bias) == 0
    assert torch.equal(m.norm.weight, torch.ones(64)) and torch.count_nonzero(m.norm.bias) == 0


def test_batch_cu_seqlens_matches_the_reference_gap_walk():
    """Batch offsets from ascending batch ids, on the device in the library
    (searchsorted), against the reference's gap walk (voldecoder.py:318-327)."""
    from lsrm_sparse import decoder

    ids = torch.tensor([0] * 5 + [1] * 3 + [2] * 7 + [3], dtype=torch.int32)
    gap = ids[1:] - ids[:-1]
    seq = torch.nonzero(gap) + 1
    want = [0] + [int(seq[n]) for n in range(3)] + [ids.shape[0]]
    assert decoder.batch_cu_seqlens(ids, 4).tolist() == want
