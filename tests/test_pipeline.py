"""Pipeline placement: layers split over devices in stages (two stages on the CPU here; the same code moves the
stream between GPUs). Decoding with a split model equals decoding with the whole model, plain and speculative."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.errors import ConfigError
from economize_b200.parallel.pipeline import pipeline_split, stage_sizes
from economize_b200.runtime.cache import SplitKVCache
from economize_b200.techniques.eagle3 import Eagle3Config

from .helpers import tiny_model


def test_stage_sizes():
    assert stage_sizes(10, 3) == [4, 3, 3]
    with pytest.raises(ConfigError):
        stage_sizes(2, 3)


@pytest.mark.parametrize("decoding", [dict(cycle_length=1), dict(cycle_length=7, draft_policy="dynamic_tree",
                                                                 draft_policy_options={"depth": 6, "topk": 10,
                                                                                       "total_tokens": 60})])
def test_split_model_decodes_like_the_whole(decoding):
    model = tiny_model()
    em = eco.apply(model, Eagle3Config())
    prompts = [torch.randint(0, 1024, (n,), generator=torch.Generator().manual_seed(n)) for n in (30, 9)]
    want = em.decode_batch(prompts, 12, decoding=eco.DecodeConfig(**decoding))
    split = eco.apply(tiny_model(), Eagle3Config())
    split.techniques["eagle3"].load_state_dict(em.techniques["eagle3"].state_dict())
    target = split.model
    pipeline_split(split, ["cpu", "cpu"], balance=[1, 3])
    target.placement = [torch.device("cpu")] * 1 + [torch.device("cpu", 0)] * 3  # two stages on one host
    cache = target.new_cache(2, 256)
    assert isinstance(cache, SplitKVCache) and [len(r) for r, _ in cache.parts] == [1, 3]
    got = split.decode_batch(prompts, 12, decoding=eco.DecodeConfig(**decoding))
    for a, b in zip(want, got):
        assert torch.equal(a.tokens, b.tokens)
