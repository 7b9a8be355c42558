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
