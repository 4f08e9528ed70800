"""SliceGPT: the unsliced rotation reproduces the model, principal components beat a random basis at equal width,
and the saved basis re-slices without calibration."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.runtime.cache import StepBatch
from economize_b200.techniques.slicegpt import SliceGPTConfig, SliceGPTTechnique

from .helpers import prompts, tiny_model

CAL = torch.randint(0, 1024, (4, 64), generator=torch.Generator().manual_seed(1))


def _logits(model, tokens):
    b, s = tokens.shape
    cache = model.new_cache(b, 128)
    h, _ = model.forward_step(tokens, StepBatch.prefill(torch.full((b,), s, dtype=torch.int32), s), cache)
    return model.logits(h).float()


def test_identity_width_is_exact():
    plain = eco.apply(tiny_model()).decode(prompts((20,))[0], 12, decoding=eco.DecodeConfig(cycle_length=1)).tokens
    m = tiny_model()
    out = eco.apply(m, SliceGPTConfig(sparsity=0.0, round_to=64), calibration=CAL).decode(
        prompts((20,))[0], 12, decoding=eco.DecodeConfig(cycle_length=1)).tokens
    assert torch.equal(plain, out)


def test_pca_beats_random_basis():
    ref = _logits(tiny_model(), CAL)
    m = tiny_model()
    eco.apply(m, SliceGPTConfig(sparsity=0.25, round_to=64), calibration=CAL)
    assert m.config.hidden_size == 192 and m.layers[0].wqkv.shape[1] == 192
    err_pca = (_logits(m, CAL) - ref).norm()
    r = tiny_model()
    tech = SliceGPTTechnique(SliceGPTConfig(sparsity=0.25, round_to=64), r)
    q, _ = torch.linalg.qr(torch.randn(256, 256, generator=torch.Generator().manual_seed(0)))
    tech.basis = q[:, :192].contiguous()
    tech.attach()
    err_rand = (_logits(r, CAL) - ref).norm()
    assert err_pca < 0.8 * err_rand, (float(err_pca), float(err_rand))


def test_saved_basis_reslices(tmp_path):
    m = tiny_model()
    em = eco.apply(m, SliceGPTConfig(sparsity=0.25, round_to=64), calibration=CAL)
    em.save_pretrained(tmp_path)
    again = eco.load(tiny_model(), tmp_path)
    assert again.model.config.hidden_size == 192
    torch.testing.assert_close(_logits(again.model, CAL[:1]), _logits(m, CAL[:1]))


def test_per_block_is_refused():
    with pytest.raises(eco.ConfigError, match="global"):
        SliceGPTConfig(rotation="per_block")
