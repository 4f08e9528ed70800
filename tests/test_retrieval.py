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


def test_jacobi_window_fills_and_makes_ngrams():
    from economize_b200.techniques.lookahead import JacobiWindow

    w = JacobiWindow([10, 11, 12, 13, 14], depth=3)  # W + N - 3 = 5 tokens: W = 4, N = 4
    toks, pars, last = w.nodes(0)
    assert toks == [10, 11, 12, 13, 14] and pars == [-1, 0, 1, 2, 3] and last == [0, 1, 2, 3, 4]
    assert w.step([20, 21, 22, 23, 24], root=1) == []
    toks, pars, last = w.nodes(2)  # after two verification-branch nodes
    assert toks == [11, 12, 13, 14, 20, 21, 22, 23, 24]
    # level 1 column j below the first block's column j: the root, then level 0's tokens
    assert pars == [-1, 2, 3, 4, -1, 2, 3, 4, 5] and last == [6, 7, 8, 9, 10]
    assert w.step([30, 31, 32, 33, 34], root=2) == []
    assert w.full and [len(lv) for lv in w.levels] == [3, 4, 4]  # W - 1, W, W
    grams = w.step([40, 41, 42, 43], root=3)
    # one N-gram per column: the first block's column j, then the column down the levels, then the prediction
    assert grams == [(3, (21, 31, 40)), (12, (22, 32, 41)), (13, (23, 33, 42)), (14, (24, 34, 43))]
    assert [len(lv) for lv in w.levels] == [3, 4, 4]


def test_lookahead_pool_learns_from_the_window_and_accepts():
    """A model whose greedy output repeats: the Jacobi window converges on the cycle, its n-grams reach the pool and
    the verification branch accepts them; the output equals plain greedy decoding."""
    model = tiny_model()
    p = _repetitive_prompt()
    ref = reference_greedy(model, p, 40)
    eff = eco.apply(model, LookaheadConfig(window=5, ngram=4, guesses=5))
    out = eff.decode(p, 40)
    assert torch.equal(out.tokens, ref)
    assert out.mean_accepted > 1.2  # n-grams from the window are accepted
    assert eff.techniques["lookahead"].config.budget <= 63


def test_lookahead_refuses_trees_beyond_the_pass():
    import pytest

    from economize_b200.errors import ConfigError

    with pytest.raises(ConfigError, match="nodes"):
        LookaheadConfig(window=15, ngram=5, guesses=15)


def test_suffix_index_orders_suffixes_and_counts_continuations(tmp_path):
    import numpy as np

    from economize_b200.techniques.retrieval import SuffixIndex, suffix_array

    toks = np.array([3, 1, 2, 3, 1, 2, 4, -1, 3, 1, 5, -1], dtype=np.int64)
    sa = suffix_array(toks, depth=64)
    keys = [tuple(toks[i:i + 6].tolist()) for i in sa]
    assert keys == sorted(keys)  # sorted by their first tokens (separators lowest)
    idx = SuffixIndex.build([[3, 1, 2, 3, 1, 2, 4], [3, 1, 5]])
    lo, hi = idx.find([3, 1])
    assert hi - lo == 3
    tokens, parents = idx.draft_tree([9, 3, 1], budget=4, max_depth=2, branch=2, min_match=1)
    assert tokens[0] == 2 and parents[0] == -1  # "3 1" is followed by 2 twice and by 5 once
    idx.save(tmp_path / "store")
    again = SuffixIndex.load(tmp_path / "store", mmap=True)
    assert again.draft_tree([9, 3, 1], 4, 2, 2, 1) == (tokens, parents)


def test_rest_with_a_persistent_datastore_and_cli(tmp_path):
    import numpy as np

    from economize_b200.techniques.retrieval.__main__ import main

    model = tiny_model()
    p = _repetitive_prompt()
    ref = reference_greedy(model, p, 16)
    flat = torch.cat([p, ref]).numpy().astype(np.uint32)
    flat.tofile(tmp_path / "corpus.bin")
    main(["build", str(tmp_path / "store"), "--tokens", str(tmp_path / "corpus.bin"), "--depth", "32"])
    eff = eco.apply(model, RestConfig(datastore=str(tmp_path / "store")))
    out = eff.decode(p, 16)
    assert torch.equal(out.tokens, ref) and out.mean_accepted > 1.0
