"""Composed drafters: ``hybrid`` (prompt lookup over a model drafter) and ``draft_with`` (other techniques on the
draft path only) stay lossless under greedy verification and leave the target untouched."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.ops.act_sparse import TealWeight
from economize_b200.techniques.draft_model import DraftModelConfig
from economize_b200.techniques.draft_with import DraftWith, DraftWithConfig
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.hybrid import HybridConfig
from economize_b200.techniques.quant import QuantConfig
from economize_b200.techniques.sparsity import TealConfig

from .helpers import prompts, tiny_model

CAL = torch.randint(0, 1024, (2, 48), generator=torch.Generator().manual_seed(3))
TREE = {"depth": 4, "topk": 4, "total_tokens": 16}


def _repetitive(n=40, seed=1):
    g = torch.Generator().manual_seed(seed)
    base = torch.randint(0, 1024, (10,), generator=g)
    return torch.cat([base, base, base, base])[:n]


@pytest.fixture(scope="module")
def model():
    return tiny_model()


@pytest.mark.parametrize("fallback,decoding", [
    (lambda m: DraftModelConfig(model=tiny_model(num_layers=2)), eco.DecodeConfig(cycle_length=5)),
    (lambda m: Eagle3Config(), eco.DecodeConfig(cycle_length=5, draft_policy="dynamic_tree",
                                                draft_policy_options=TREE)),
])
def test_hybrid_is_lossless_and_copies(model, fallback, decoding):
    ps = [_repetitive(), prompts((23,))[0]]
    plain = eco.apply(model).decode_batch(ps, 24, decoding=eco.DecodeConfig(cycle_length=1))
    em = eco.apply(model, HybridConfig(fallback=fallback(model)))
    out = em.decode_batch(ps, 24, decoding=decoding)
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens)


def test_hybrid_config_roundtrip(tmp_path, model):
    em = eco.apply(model, HybridConfig(fallback=Eagle3Config(), max_ngram=4))
    em.save_pretrained(tmp_path)
    again = eco.load(tiny_model(), tmp_path)
    cfg = again.techniques["hybrid"].config
    assert cfg.max_ngram == 4 and cfg.fallback.technique == "eagle3"
    a = em.techniques["hybrid"].fallback.state_dict()
    b = again.techniques["hybrid"].fallback.state_dict()
    assert all(torch.equal(a[k].cpu(), b[k].cpu()) for k in a)


def test_hybrid_refuses_bad_roles():
    with pytest.raises(eco.ConfigError):
        HybridConfig(fallback=TealConfig())
    with pytest.raises(eco.ConfigError):
        HybridConfig(fallback=Eagle3Config(), primary=Eagle3Config(), max_ngram=5)


@pytest.mark.parametrize("inner", [
    lambda: TealConfig(sparsity=0.5, allocation="uniform", backend="dense"),
    lambda: QuantConfig(format="int8", method="rtn", symmetric=True, backend="fake"),
])
def test_draft_with_is_lossless_and_leaves_target(model, inner):
    before = {k: v.clone() for k, v in model.state_dict().items()}
    plain = eco.apply(model).decode_batch(prompts(), 20, decoding=eco.DecodeConfig(cycle_length=1))
    em = eco.apply(model, DraftWith(inner()), calibration=CAL)
    out = em.decode_batch(prompts(), 20, decoding=eco.DecodeConfig(cycle_length=4))
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens)
    assert sum(r.accepted for r in out) > 0
    for k, v in model.state_dict().items():
        assert torch.equal(v, before[k]), k
    view = em.techniques["draft_with"].view
    assert not isinstance(model.layers[0].wqkv, TealWeight)
    assert view.layers[0].wqkv is not model.layers[0].wqkv


def test_draft_with_config_checks():
    with pytest.raises(eco.ConfigError):
        DraftWithConfig(techniques=())
    with pytest.raises(eco.ConfigError):
        DraftWith(Eagle3Config())
    cfg = DraftWithConfig.from_dict(DraftWith(TealConfig(sparsity=0.3)).to_dict())
    assert cfg.techniques[0].sparsity == 0.3
