"""Sparse KV views: self-speculation on sink+window / retrieved-chunk views (MagicDec, TriForce), DuoAttention
streaming heads, Quest page selection, and the placed draft model."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.techniques.duo_attention import DuoAttentionConfig
from economize_b200.techniques.placed_draft import PlacedDraftModelConfig
from economize_b200.techniques.quest import QuestConfig
from economize_b200.techniques.sparse_kv_draft import MagicDecConfig, TriForceConfig

from .helpers import micro_model, prompts, reference_greedy, tiny_model


@pytest.mark.parametrize("config", [MagicDecConfig(sink=4, window=16),
                                    TriForceConfig(sink=4, window=16, chunk=32, chunks=1)])
def test_self_speculation_on_sparse_views_is_lossless(config):
    model = tiny_model()
    eff = eco.apply(model, config, decoding=eco.DecodeConfig(cycle_length=4))
    p = prompts((100,))[0]
    out = eff.decode(p, 10)
    assert torch.equal(out.tokens, reference_greedy(model, p, 10))
    assert out.mean_accepted < 3.0  # the view really drafts from less context


def test_duo_attention_heads_and_decoding():
    cal = torch.randint(0, 1024, (1, 96), generator=torch.Generator().manual_seed(0))
    eff = eco.apply(tiny_model(), DuoAttentionConfig(streaming_ratio=0.5, sink=4, window=16), calibration=cal)
    tech = eff.techniques["duo_attention"]
    assert int(tech.streaming.sum()) == tech.streaming.numel() // 2
    p = prompts((80,))[0]
    spec = eco.DecodeConfig(cycle_length=1)
    assert torch.equal(eff.decode(p, 8, decoding=spec).tokens, eff.decode(p, 8, decoding=spec).tokens)


def test_quest_selects_pages():
    eff = eco.apply(tiny_model(), QuestConfig(page=16, pages=2))
    p = prompts((100,))[0]
    base = eco.EfficientModel(tiny_model(), [], eco.DecodeConfig())
    out = eff.decode(p, 6).tokens
    assert out.numel() == 6
    tech = eff.techniques["quest"]
    assert tech.kmin[0] is not None and tech.kmin[0].shape[2] == 128 // 16
    del base


def test_placed_draft_on_cpu():
    model = tiny_model()
    draft = micro_model(vocab=1024)
    eff = eco.apply(model, PlacedDraftModelConfig(model=draft, device="cpu"))
    p = prompts((15,))[0]
    assert torch.equal(eff.decode(p, 8).tokens, reference_greedy(model, p, 8))
