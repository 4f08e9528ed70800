"""Host-side retrieval drafters: n-gram index trees, suffix decoding, REST, lookahead pools and their union."""

import torch

import economize_b200 as eco
from economize_b200.decoding.ngram_index import NGramIndex
from economize_b200.techniques.lookahead import LookaheadConfig
from economize_b200.techniques.rest import RestConfig
from economize_b200.techniques.suffix_decoding import SuffixDecodingConfig
from economize_b200.techniques.union import UnionConfig, merge_trees

from .helpers import reference_greedy, tiny_model


def test_index_tree_follows_the_longest_match():
    idx = NGramIndex(4)
    idx.add([1, 2, 3, 4, 5, 1, 2, 3, 9])
    tokens, parents = idx.draft_tree([7, 1, 2, 3], budget=4, depth=3, branch=2)
    assert tokens[0] in (4, 9) and parents[0] == -1
    assert set(tokens[:2]) == {4, 9}


def test_merge_trees_shares_prefixes():
    t, p = merge_trees([([5, 6], [-1, 0]), ([5, 7], [-1, 0])], 8)
    assert t == [5, 6, 7] and p == [-1, 0, 0]


def _repetitive_prompt():
    base = torch.randint(0, 1024, (12,), generator=torch.Generator().manual_seed(9))
    return torch.cat([base, base, base[:6]])


def test_retrieval_drafters_are_lossless_and_accept():
    model = tiny_model()
    p = _repetitive_prompt()
    ref = reference_greedy(model, p, 16)
    corpus = torch.stack([torch.cat([p, ref])] * 2)
    for cfg in (SuffixDecodingConfig(), RestConfig(corpus=corpus), LookaheadConfig(), UnionConfig(corpus=corpus)):
        eff = eco.apply(model, cfg)
        out = eff.decode(p, 16)
        assert torch.equal(out.tokens, ref), cfg.technique
        if cfg.technique in ("rest", "union"):  # the corpus holds the exact continuation
            assert out.mean_accepted > 1.0, cfg.technique


def test_suffix_global_index():
    model = tiny_model()
    p = _repetitive_prompt()
    ref = reference_greedy(model, p, 12)
    eff = eco.apply(model, SuffixDecodingConfig())
    eff.techniques["suffix_decoding"].add_corpus([torch.cat([p, ref]).tolist()])
    out = eff.decode(p, 12)
    assert torch.equal(out.tokens, ref) and out.mean_accepted > 1.0
