"""LayerRunner (economize ``runtime/runner.py``): layer ranges, overrides and captures against the full pass."""

import pytest
import torch

from economize_b200.errors import ConfigError
from economize_b200.runtime.cache import StepBatch
from economize_b200.runtime.runner import LayerRunner

from .helpers import tiny_model


def _batch(T):
    return StepBatch.prefill(torch.tensor([T, T - 3], dtype=torch.int32), T)


def test_ranges_compose_to_the_exact_pass():
    model = tiny_model()
    runner = LayerRunner(model)
    tokens = torch.randint(0, 1024, (2, 12), generator=torch.Generator().manual_seed(0))
    exact = runner.forward(tokens, _batch(12), runner.new_cache(2, 128), capture=(2, -2))
    h = runner.embed(tokens)
    cache = runner.new_cache(2, 128)
    mid, aux = runner.run(h, _batch(12), cache, 1, 2, capture=(2,))
    end, _ = runner.run(mid, _batch(12), cache, 3, 4)
    torch.testing.assert_close(aux[2], exact.hidden[2])
    torch.testing.assert_close(end, exact.hidden[-2])


def test_overrides_replace_layers():
    model = tiny_model()
    runner = LayerRunner(model)
    tokens = torch.randint(0, 1024, (2, 9), generator=torch.Generator().manual_seed(1))
    h = runner.embed(tokens)
    skipped, _ = runner.run(h, _batch(9), runner.new_cache(2, 64), 1, 4, overrides={2: lambda x, b, c: x})
    a, _ = runner.run(h, _batch(9), runner.new_cache(2, 64), 1, 1)
    b, _ = runner.run(a, _batch(9), runner.new_cache(2, 64), 3, 4)
    # the override passes layer 2's input through; layer 3's cache slots start fresh in both runs
    torch.testing.assert_close(skipped, b)
    with pytest.raises(ConfigError):
        runner.run(h, _batch(9), runner.new_cache(2, 64), 2, 3, overrides={4: lambda x, b, c: x})


def test_replay_rebuilds_the_cache():
    model = tiny_model()
    runner = LayerRunner(model)
    tokens = torch.randint(0, 1024, (1, 10), generator=torch.Generator().manual_seed(2))
    cache = runner.new_cache(1, 64)
    first = runner.forward(tokens, StepBatch.prefill(torch.tensor([10], dtype=torch.int32), 10), cache)
    data = cache.data.clone()
    cache.reset()
    again = runner.replay(tokens, cache, torch.tensor([10]))
    assert torch.equal(runner.logits(again.final).argmax(-1), runner.logits(first.final).argmax(-1))
    torch.testing.assert_close(again.final, first.final)
    torch.testing.assert_close(cache.data, data)


def test_attention_usage_traces_paths():
    import economize_b200 as eco
    from economize_b200 import ops

    ops.attention_usage(reset=True)
    eco.apply(tiny_model()).decode_batch([torch.arange(12)], 4, decoding=eco.DecodeConfig(cycle_length=1))
    usage = ops.attention_usage()
    assert usage.get(("cpu", "float32", 12, "causal"), 0) == 4  # the prefill, one call per layer
    assert usage.get(("cpu", "float32", 1, "masked+exact_tail"), 0) == 4 * 3  # three decode steps
    assert ops.attention_usage(reset=True) and not ops.attention_usage()
