"""The lm-eval model (economize ``tests/integrations/test_lm_eval.py``): scores equal a direct log-softmax of the
model's logits, rolling windows add up, and generations are the engine's greedy continuations cut at the stop
string. lm-eval itself is not needed: requests are plain objects with ``args``."""

from types import SimpleNamespace

import pytest
import torch

import economize_b200 as eco
from economize_b200.integrations.lm_eval import EconomizeLM

from .helpers import reference_greedy, tiny_model


class CharTokenizer:
    """Token id = character code (ids below the tiny model's vocabulary of 1024)."""

    bos_token_id = 1

    def encode(self, text, add_special_tokens=False):
        return [ord(ch) for ch in text]

    def decode(self, ids):
        return "".join(chr(i) for i in ids)


@pytest.fixture(scope="module")
def lm():
    return EconomizeLM(eco.apply(tiny_model()), CharTokenizer(), decoding=eco.DecodeConfig(cycle_length=1),
                       max_length=64)


def test_loglikelihood_matches_direct_scores(lm):
    req = SimpleNamespace(args=("hello ", "world"))
    (score, greedy), = lm.loglikelihood([req])
    ids = torch.tensor([ord(c) for c in "hello world"])
    with torch.no_grad():
        logp = torch.log_softmax(lm.model(ids[None])[0].float(), -1)
    ref = sum(float(logp[i - 1, ids[i]]) for i in range(6, 11))
    assert score == pytest.approx(ref, rel=1e-5)
    assert greedy == all(int(logp[i - 1].argmax()) == int(ids[i]) for i in range(6, 11))


def test_rolling_equals_one_window_when_it_fits(lm):
    text = "abcdefghij"
    rolled, = lm.loglikelihood_rolling([SimpleNamespace(args=(text,))])
    whole, _ = lm.loglikelihood([SimpleNamespace(args=(text[0], text[1:]))])[0]
    assert rolled == pytest.approx(whole, rel=1e-5)
    long_text = "the quick brown fox jumps over the lazy dog " * 3  # 132 characters: three windows of 64
    assert lm.loglikelihood_rolling([SimpleNamespace(args=(long_text,))])[0] < 0


def test_generate_until_cuts_at_stop(lm):
    prompt = "abc"
    ids = torch.tensor([ord(c) for c in prompt])
    full = reference_greedy(lm.model.model, ids, 12)
    text = "".join(chr(int(t)) for t in full)
    out, = lm.generate_until([SimpleNamespace(args=(prompt, {"max_gen_toks": 12}))])
    assert out == text
    stop = text[5]
    cut, = lm.generate_until([SimpleNamespace(args=(prompt, {"max_gen_toks": 12, "until": [stop]}))])
    assert cut == text[:text.find(stop)]
