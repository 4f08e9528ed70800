"""Hub persistence (economize ``tests/core/test_hub.py``): the model card names the techniques and the base model,
a saved folder loads back with identical drafts, and push/pull go through the Hub API (replaced here by fakes: no
network in the tests)."""

import shutil

import pytest
import torch

import economize_b200 as eco
from economize_b200.core.hub import from_pretrained, model_card, push_to_hub, save_pretrained
from economize_b200.errors import CheckpointFormatError
from economize_b200.techniques.eagle3 import Eagle3Config

from .helpers import prompts, tiny_model


def _model():
    em = eco.apply(tiny_model(), Eagle3Config(), decoding=eco.DecodeConfig(cycle_length=4))
    em.techniques["eagle3"].reset_parameters(seed=5)
    return em


def test_card_and_local_roundtrip(tmp_path):
    em = _model()
    card = model_card(em, "user/tiny-eagle3", base_model="org/tiny")
    assert card.startswith("---\nlibrary_name: economize_b200") and "base_model: org/tiny" in card
    assert "`eagle3`" in card and "cycle_length" in card
    out = save_pretrained(em, tmp_path / "ckpt", repo_id="user/tiny-eagle3", base_model="org/tiny")
    assert (out / "README.md").is_file() and (out / "economize_config.json").is_file()
    back = from_pretrained(out, tiny_model())
    dc = eco.DecodeConfig(cycle_length=4)
    for a, b in zip(em.decode_batch(prompts(), 12, decoding=dc), back.decode_batch(prompts(), 12, decoding=dc)):
        assert torch.equal(a.tokens, b.tokens) and a.accepted == b.accepted


class FakeApi:
    def __init__(self, store):
        self.store, self.calls = store, []

    def create_repo(self, repo_id, private=False, exist_ok=True):
        self.calls.append(("create", repo_id, private))

    def upload_folder(self, repo_id, folder_path, commit_message):
        shutil.copytree(folder_path, self.store / repo_id.replace("/", "--"))
        self.calls.append(("upload", repo_id, commit_message))
        return "commit-1"


def test_push_and_pull_through_the_hub_api(tmp_path):
    em = _model()
    api = FakeApi(tmp_path)
    assert push_to_hub(em, "user/tiny", private=True, api=api) == "commit-1"
    assert api.calls[0] == ("create", "user/tiny", True) and api.calls[1][0] == "upload"
    assert (tmp_path / "user--tiny" / "README.md").is_file()

    def download(repo_id, revision=None):
        return str(tmp_path / repo_id.replace("/", "--"))

    back = from_pretrained("user/tiny", tiny_model(), download=download)
    assert torch.equal(back.techniques["eagle3"].fc, em.techniques["eagle3"].fc)

    def offline(repo_id, revision=None):
        raise OSError("no network")

    with pytest.raises(CheckpointFormatError, match="cannot fetch"):
        from_pretrained("user/missing", tiny_model(), download=offline)
