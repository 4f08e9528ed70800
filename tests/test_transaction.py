"""Transactional attach: when a technique fails part way through ``apply``, the techniques attached before it are
undone and the engine model is restored (economize ``core/recipe.py:207-227``, ``_weights/transaction.py``)."""

from dataclasses import dataclass
from typing import ClassVar

import pytest
import torch

import economize_b200 as eco
from economize_b200.core.technique import Capability, Technique, TechniqueConfig, register_technique
from economize_b200.techniques.prune import DepthPruneConfig, PruneConfig

from .helpers import tiny_model


@dataclass(frozen=True)
class _FailingConfig(TechniqueConfig):
    technique: ClassVar[str] = "_test_failing_attach"


@register_technique
class _FailingTechnique(Technique):
    """Installs a hook and then raises inside its own attach."""

    config_class = _FailingConfig
    capabilities = Capability.DRAFTER
    detached = 0

    def attach(self) -> None:
        self.model.layers[0].attn_input_hook = lambda x: None
        raise RuntimeError("attach failed on purpose")

    def detach(self) -> None:
        type(self).detached += 1
        self.model.layers[0].attn_input_hook = None


def _state(model):
    return {k: v.detach().clone() for k, v in model.state_dict().items()}


def test_failed_apply_restores_weights_and_structure():
    model = tiny_model()
    before = _state(model)
    layers = len(model.layers)
    with pytest.raises(RuntimeError, match="on purpose") as info:
        eco.apply(model, DepthPruneConfig(num_blocks=1, method="shortgpt"),
                  PruneConfig(method="magnitude", sparsity=0.5), _FailingConfig(),
                  calibration=torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(0)))
    assert len(model.layers) == layers and model.config.num_layers == layers
    after = _state(model)
    assert after.keys() == before.keys()
    assert all(torch.equal(before[k], after[k]) for k in before)
    assert getattr(model.layers[0], "attn_input_hook", None) is None
    assert any("restored" in note for note in getattr(info.value, "__notes__", []))
    # the restored model works: plain decoding equals a fresh model's
    fresh = eco.apply(tiny_model()).decode_batch([torch.arange(9)], 6, decoding=eco.DecodeConfig(cycle_length=1))
    again = eco.apply(model).decode_batch([torch.arange(9)], 6, decoding=eco.DecodeConfig(cycle_length=1))
    assert torch.equal(fresh[0].tokens, again[0].tokens)


def test_successful_apply_is_unchanged():
    model = tiny_model()
    em = eco.apply(model, PruneConfig(method="magnitude", sparsity=0.5))
    w = em.model.layers[0].wo
    assert float((w == 0).float().mean()) >= 0.45


def test_depth_prune_changes_the_model_it_is_rolled_back_from():
    model = tiny_model()
    layers = len(model.layers)
    em = eco.apply(model, DepthPruneConfig(num_blocks=1, method="shortgpt"),
                   calibration=torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(0)))
    assert len(em.model.layers) == layers - 1  # the transform the failing apply above had to undo
