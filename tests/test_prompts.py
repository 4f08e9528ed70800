"""Benchmark prompt sets: synthetic ids, the built-in smoke prompts, and local JSON-lines files in the Spec-Bench,
GSM8K and HumanEval layouts."""

import json

import pytest
import torch

from economize_b200.bench.prompts import SMOKE_PROMPTS, load_prompts
from economize_b200.errors import ConfigError


class Chars:
    def encode(self, text, add_special_tokens=False):
        return [ord(c) % 1024 for c in text]


def test_synthetic_and_smoke():
    a = load_prompts("synthetic", 3, length=17, vocab_size=1024, seed=1)
    b = load_prompts("synthetic", 3, length=17, vocab_size=1024, seed=1)
    assert all(torch.equal(x, y) and x.shape == (17,) for x, y in zip(a, b))
    smoke = load_prompts("smoke", 5, tokenizer=Chars())
    assert len(smoke) == 5 and smoke[4].tolist() == Chars().encode(SMOKE_PROMPTS[0])
    with pytest.raises(ConfigError, match="vocab_size"):
        load_prompts("synthetic", 2)


@pytest.mark.parametrize("record,text", [({"turns": ["first turn", "second"]}, "first turn"),
                                         ({"question": "2 + 2?"}, "2 + 2?"), ({"prompt": "def f():"}, "def f():")])
def test_jsonl_layouts(tmp_path, record, text):
    path = tmp_path / "p.jsonl"
    path.write_text(json.dumps(record) + "\n")
    (ids,) = load_prompts(path, 1, tokenizer=Chars())
    assert ids.tolist() == Chars().encode(text)
    bad = tmp_path / "bad.jsonl"
    bad.write_text(json.dumps({"x": 1}) + "\n")
    with pytest.raises(ConfigError, match="one of"):
        load_prompts(bad, 1, tokenizer=Chars())
